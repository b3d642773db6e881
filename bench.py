"""Benchmark of the quantized-weight hot path on B200.

Default workload (one JSON line): the decode Q-GEMV sweep -- Q5_0 [4864 x 896],
Q6_K [896 x 4864] and Q4_K [896 x 4864] at batch 1, 4 and 16 with fp32
activations ~ N(0,1).  One step runs every (type, batch) case once over each
of `copies` device copies of its weight, so each step streams more than three
times the 126 MB L2 from HBM (inputs larger than L2; no flush needed).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 (torchrun, one rank per GPU): every rank runs the same sweep on its own
GPU (weak scaling, no collective in the data path); the time is the max over
ranks and `value` sums all ranks' bytes.

Metric: algorithmic GB/s = (packed weight bytes + fp32 x bytes + fp32 y bytes)
/ time.  `e2e` runs the same sweep through the reference-facing host-buffer
call (hd_qgemv_host: x copied in, y copied out, per call).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [ROOT, os.path.join(ROOT, "hace-fem-hacedle_b200", "python")]

from hacedle_cuda import synth as S  # noqa: E402

METRIC = "Q-GEMV GB/s vs 8 TB/s HBM; prefill TFLOP/s; decode tokens/s (0.5B-shape)"
CASES = [(S.GGML_Q5_0, 4864, 896), (S.GGML_Q6_K, 896, 4864), (S.GGML_Q4_K, 896, 4864)]
BATCHES = [1, 4, 16]
FALLBACK_HBM_GBS = 6650.0


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return FALLBACK_HBM_GBS, 1590.0, "fallback"


def case_bytes(t, N, K, B):
    return S.nbytes(t, N, K) + 4 * B * K + 4 * B * N


class Clocks:
    """nvidia-smi samples during the timed region."""

    def __init__(self, index: int):
        self.index, self.proc, self.lines = index, None, []

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_init():
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        import datetime

        import torch
        import torch.distributed as dist

        lr = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(lr)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        return dist.get_rank(), dist.get_world_size(), lr
    return 0, 1, 0


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# ------------------------------------------------------------------ our arm
def run_ours(args, rank, world, local):
    import torch

    import hacedle_cuda as hc

    torch.cuda.set_device(local)
    ctx = hc.Context(local)
    if args.only:
        fns = {"prefill": lambda: prefill_workload(ctx, args), "dequant": lambda: dequant_workload(ctx),
               "decode": lambda: decode_workload(ctx, args, rank, world),
               "layer7b": lambda: layer7b_workload(ctx, args, rank, world),
               "gemv_large": lambda: gemv_large_workload(ctx)}
        r = fns[args.only]()
        if rank == 0:
            print(json.dumps({"workload": args.only, "n_gpus": world, "result": r}), flush=True)
        ctx.close()
        return
    hbm, _, peak_kind = peaks()
    l2 = torch.cuda.get_device_properties(local).L2_cache_size
    # Weights: `copies` device copies per type, together > 3x L2 per case.
    weights, raws = {}, {}
    for (t, N, K) in CASES:
        raw = S.gen_weight(t, N, K, seed=2 + t)
        raws[t] = raw
        nb = S.nbytes(t, N, K)
        copies = max(args.copies, int(np.ceil(3 * l2 / nb)))
        weights[t] = [ctx.weight(t, raw, N, K) for _ in range(copies)]
    xs = {(t, B): torch.from_numpy(S.gen_activations(B, K, 100 + B)).cuda() for (t, N, K) in CASES for B in BATCHES}
    ys = {(t, B): torch.empty(B, N, device="cuda") for (t, N, K) in CASES for B in BATCHES}

    def segment(t, B):
        for w in weights[t]:
            ctx.qgemv(w, xs[(t, B)], ys[(t, B)])

    # One warm pass allocates the split-K workspace; then capture each
    # (type, batch) segment as a CUDA graph (PDL edges between launches).
    for (t, N, K) in CASES:
        for B in BATCHES:
            segment(t, B)
    torch.cuda.synchronize()
    graphs, launches_per_step = {}, 0
    cap_stream = torch.cuda.Stream()
    for (t, N, K) in CASES:
        for B in BATCHES:
            g = torch.cuda.CUDAGraph()
            n0 = ctx.launches
            with torch.cuda.graph(g, stream=cap_stream):
                ctx.set_stream(torch.cuda.current_stream().cuda_stream)
                segment(t, B)
            launches_per_step += ctx.launches - n0
            graphs[(t, B)] = g
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()

    step_bytes = sum(case_bytes(t, N, K, B) * len(weights[t]) for (t, N, K) in CASES for B in BATCHES)
    ev = {k: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for k in graphs}
    case_ms = {k: 0.0 for k in graphs}

    for _ in range(args.warmup):
        for g in graphs.values():
            g.replay()
    torch.cuda.synchronize()
    barrier(world)
    with Clocks(local) as clk:
        torch.cuda.synchronize()
        barrier(world)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            for k, g in graphs.items():
                ev[k][0].record()
                g.replay()
                ev[k][1].record()
            torch.cuda.synchronize()
            for k in graphs:
                case_ms[k] += ev[k][0].elapsed_time(ev[k][1])
        end.record()
        torch.cuda.synchronize()
        barrier(world)
    total_ms = start.elapsed_time(end)
    kernel_ms = sum(case_ms.values())
    ms_all = max_over_ranks(kernel_ms, world)
    value = step_bytes * args.steps * world / (ms_all * 1e-3) / 1e9

    # Per-case breakdown (rank-local), and the dominant kernel's roofline:
    # every launch in the timed region is the Q-GEMV kernel.
    breakdown = {}
    for (t, N, K) in CASES:
        for B in BATCHES:
            n = len(weights[t]) * args.steps
            per = case_ms[(t, B)] / n
            breakdown[f"{S.TYPE_NAME[t]}_B{B}"] = {
                "gbs": round(case_bytes(t, N, K, B) / (per * 1e-3) / 1e9, 1), "us_per_launch": round(per * 1e3, 3)}
    launches = launches_per_step * args.steps
    achieved = step_bytes * args.steps / (kernel_ms * 1e-3) / 1e9
    # Batch 1 and 4 run the small-matrix tensor-core k_qgemv_sm (mma.sync),
    # batch 16 the tcgen05 k_qgemv_tc (hd_qgemv picks by batch and size):
    # their shares of the step's time.
    tc_ms = sum(case_ms[(t, B)] for (t, N, K) in CASES for B in BATCHES if B >= 5)
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(achieved / hbm, 4), "traffic": None, "peak_kind": peak_kind,
                "kernel": "k_qgemv_sm", "algorithmic_bytes_per_step": step_bytes,
                "kernel_time_share": {"k_qgemv_sm (B=1,4)": round(1 - tc_ms / kernel_ms, 3),
                                      "k_qgemv_tc (B=16)": round(tc_ms / kernel_ms, 3)}}
    # DRAM bytes of one captured launch (ncu --set full, Q5_0 batch 1), with its
    # algorithmic bytes: profiles/qgemv_sm_q5_0_b1_ncu.md.
    # (not measured in this run: copied from that committed capture)
    trf = os.path.join(ROOT, "profiles", "qgemv_sm_q5_0_b1_ncu.md")
    if os.path.exists(trf):
        kv = dict(ln.split(":", 1) for ln in open(trf) if ln.startswith(("dram_bytes_per_launch", "algorithmic_bytes")))
        if kv:
            roofline["traffic"] = int(kv["dram_bytes_per_launch"])
            roofline["traffic_kernel"] = "k_qgemv_sm<Q5_0,B=1> on 4864x896"
            roofline["traffic_algorithmic_bytes"] = int(kv["algorithmic_bytes_per_launch"])
            roofline["traffic_source"] = "copied from profiles/qgemv_sm_q5_0_b1_ncu.md (one ncu capture), not this run"

    # End to end through the host-buffer C-ABI call.
    e2e = None
    if not args.no_e2e:
        e2e = e2e_host(ctx, weights, args)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline_sample(raws, budget_s=args.cpu_seconds)

    # Secondary workloads (outside the timed region of the headline).
    extra = {}
    if not args.no_extra:
        for name, fn in (("gemv_large", lambda: gemv_large_workload(ctx)),
                         ("prefill_qgemm", lambda: prefill_workload(ctx, args)),
                         ("dequant_q8_0", lambda: dequant_workload(ctx)),
                         ("decode_q05b", lambda: decode_workload(ctx, args, rank, world)),
                         ("layer7b_sharded", lambda: layer7b_workload(ctx, args, rank, world))):
            try:
                extra[name] = fn()
            except Exception as e:  # report, keep the headline
                extra[name] = {"error": f"{type(e).__name__}: {e}"}

    res = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_all / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32-accumulate (Q5_0/Q6_K/Q4_K weights)",
        "data": "synthetic (seeded PCG64, BASELINE generators)",
        "config": {"workload": "decode Q-GEMV sweep: Q5_0 4864x896, Q6_K 896x4864, Q4_K 896x4864 at B=1,4,16",
                   "copies_per_type": {S.TYPE_NAME[t]: len(weights[t]) for t in weights},
                   "l2_policy": "inputs larger than L2 (rotating weight copies, > 3x L2 per case)",
                   "graph": "CUDA graph per case, programmatic dependent launch"},
        "roofline": roofline, "breakdown": breakdown, "gpu_launches": launches,
        "e2e": e2e, "cpu_baseline": cpu, "clocks": clk.summary(),
        "wall_ms_timed_region": round(total_ms, 3),
        "workloads": extra,
    }
    # The multi-GPU figures at the top level: the row-sharded 7B-shaped layer
    # (exchange over NVLink included, strong scaling) and the 256-sequence
    # decode (replicas, sequences sharded over the ranks).
    l7 = extra.get("layer7b_sharded", {})
    # (the 256 sequences run as seqs{256 / ranks} per rank)
    dq = next((v for k, v in extra.get("decode_q05b", {}).items()
               if k.startswith("seqs") and k != "seqs1" and isinstance(v, dict)), {})
    if "B1" in l7:
        res["layer7b_B1_gbs"] = l7["B1"].get("gbs")
        res["layer7b_B1_exchange_ms"] = l7["B1"].get("exchange_ms")
    if "B512" in l7:
        res["layer7b_B512_tflops"] = l7["B512"].get("tflops")
        res["layer7b_B512_exchange_ms"] = l7["B512"].get("exchange_ms")
    if dq:
        res["decode_256seq_tokens_per_s"] = dq.get("tokens_per_s_all_gpus")
    if rank == 0:
        print(json.dumps(res), flush=True)
    ctx.close()


def _median(v):
    return float(np.median(np.array(v)))


def prefill_workload(ctx, args, reps=3):
    """Prefill Q-GEMM, Q5_0 [4864 x 896] and Q4_K [896 x 4864] times
    X [T x K] for T = 128, 512, 2048.  A timed batch runs the GEMM once on each
    of `nrot` weight copies and activation buffers (more than 256 MB of inputs
    in all, so that no call finds its inputs in the 126 MB L2), back to back
    on the stream behind a device-side spin that covers the host's enqueue
    time, so the events measure device time only; ms per call = batch time /
    nrot, median of `reps` batches."""
    import torch

    _, bf16, kind = peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    out = {"unit": "TFLOP/s", "peak_bf16_tflops": bf16, "peak_kind": kind,
           "l2_policy": "inputs rotated over > 256 MB per timed batch, 256 MB flush before each batch"}
    for (t, N, K) in [(S.GGML_Q5_0, 4864, 896), (S.GGML_Q4_K, 896, 4864)]:
        raw = S.gen_weight(t, N, K, seed=2 + t)
        for T in (128, 512, 2048):
            nrot = max(4, -(-(256 << 20) // (S.nbytes(t, N, K) + T * K * 4)))
            ws = [ctx.weight(t, raw, N, K) for _ in range(nrot)]
            X0 = torch.from_numpy(S.gen_activations(T, K, 7)).cuda()
            Xs = [X0.clone() for _ in range(nrot)]
            Y = torch.empty(T, N, device="cuda")
            row = {"calls_per_batch": nrot}
            for prec, nm in ((1, "bf16_tc"), (0, "fp32")):
                for i in range(nrot):
                    ctx.qgemm(ws[i], Xs[i], Y, precision=prec)
                ts = []
                for _ in range(reps):
                    flush.zero_()
                    torch.cuda._sleep(int(4e6 + nrot * 1e5))
                    e0.record()
                    for i in range(nrot):
                        ctx.qgemm(ws[i], Xs[i], Y, precision=prec)
                    e1.record()
                    torch.cuda.synchronize()
                    ts.append(e0.elapsed_time(e1) / nrot)
                ms = _median(ts)
                tf = 2.0 * T * N * K / (ms * 1e-3) / 1e12
                row[nm] = {"ms": round(ms, 4), "tflops": round(tf, 2)}
                if prec == 1:
                    row[nm]["frac_of_bf16_peak"] = round(tf / bf16, 4)
            ctx.check_device_errors()
            out[f"{S.TYPE_NAME[t]}_{N}x{K}_T{T}"] = row
            for w in ws:
                w.free()
            del Xs
    return out


def dequant_workload(ctx, copies=160):
    """Q8_0 [896 x 896] full dequant (bit-exact f32 out) and its B=1
    GEMV, rotating over `copies` weights and outputs (> L2)."""
    import torch

    hbm, _, kind = peaks()
    t, N, K = S.GGML_Q8_0, 896, 896
    raw = S.gen_weight(t, N, K, seed=1)
    ws = [ctx.weight(t, raw, N, K) for _ in range(copies)]
    outs = [torch.empty(N * K, device="cuda") for _ in range(copies)]
    x = torch.from_numpy(S.gen_activations(1, K, 11)).cuda()
    y = torch.empty(1, N, device="cuda")
    res = {}
    for nm, fn, byts in (("dequant", lambda i: ctx.dequantize(ws[i], outs[i]), S.nbytes(t, N, K) + 4 * N * K),
                         ("gemv_b1", lambda i: ctx.qgemv(ws[i], x, y), S.nbytes(t, N, K) + 4 * K + 4 * N)):
        for i in range(copies):
            fn(i)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        with torch.cuda.graph(g, stream=s):
            ctx.set_stream(torch.cuda.current_stream().cuda_stream)
            for i in range(copies):
                fn(i)
        ctx.set_stream(torch.cuda.current_stream().cuda_stream)
        for _ in range(3):
            g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(10):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (10 * copies)
        res[nm] = {"us_per_launch": round(us, 3), "gbs": round(byts / (us * 1e-6) / 1e9, 1),
                   "frac_of_hbm": round(byts / (us * 1e-6) / 1e9 / hbm, 4), "bytes_per_launch": byts}
    for w in ws:
        w.free()
    res["peak_kind"] = kind
    return res


def decode_workload(ctx, args, rank, world):
    """Qwen2.5-0.5B-shaped decoder with random weights -- prefill 512
    ids, greedy 128 tokens -- at batch 1, and 256 sequences split over the
    ranks (replicated weights, no collective)."""
    import hacedle_cuda as hc

    hbm, _, kind = peaks()
    model = S.gen_decoder(S.QWEN05B, seed=4)
    n_prompt, n_gen = 512, 128
    res = {"unit": "tokens/s", "n_prompt": n_prompt, "n_gen": n_gen, "peak_kind": kind}
    w_bytes = 386_849_280  # packed weights + f32 bias/norm vectors read per decode step
    seqs_list = [1] + ([max(1, args.decode_batch // world)] if args.decode_batch > 0 else [])
    dec = hc.Decoder(ctx, model, max_ctx=n_prompt + n_gen, max_seqs=max(seqs_list))
    for S_ in seqs_list:
        prompts = np.stack([S.gen_prompt(n_prompt, S.QWEN05B["vocab"], seed=4 + s) for s in range(S_)])
        # fp32-accuracy prefill (exact weights, tensor cores): its greedy tokens
        # are the oracle's, so sequence 0 can be checked against the golden
        prec = hc.PREC_FP32
        toks, dms, pms = dec.generate(prompts, n_gen, precision=prec)
        step_ms = dms / (n_gen - 1)
        tps = S_ * (n_gen - 1) / (dms * 1e-3)
        ent = {"seqs_per_gpu": S_, "decode_ms": round(dms, 3), "ms_per_step": round(step_ms, 4),
               "tokens_per_s_per_gpu": round(tps, 1), "tokens_per_s_all_gpus": round(tps * world, 1),
               "prefill_ms": round(pms, 3), "prefill_precision": "fp32" if prec == hc.PREC_FP32 else "bf16_tc",
               "weight_gbs_per_step": round(w_bytes / (step_ms * 1e-3) / 1e9, 1),
               "frac_of_hbm": round(w_bytes / (step_ms * 1e-3) / 1e9 / hbm, 4)}
        # sequence 0's prompt is the golden's (gen_prompt(512, seed=4)): its
        # greedy tokens must be the oracle's on either prefill precision
        gold = os.path.join(ROOT, "tests", "golden", "decoder_q05b_tokens.json")
        if os.path.exists(gold):
            ref = json.load(open(gold))["tokens"]
            ent["greedy_tokens_match_oracle"] = toks[0].tolist() == ref
            ent["greedy_tokens_checked"] = "sequence 0 (the golden prompt), all 128 tokens"
        res[f"seqs{S_}"] = ent
    dec.free()
    return res


def layer7b_workload(ctx, args, rank, world, reps=5):
    """The seven projections of a Qwen2.5-7B-shaped layer (q/k/v/o and
    gate/up Q4_K, down Q6_K), output rows sharded over the ranks.  Each rank
    computes its rows (GEMV at B=1, tcgen05 GEMM at B=64 and 512), then the
    outputs are exchanged over NVLink: by default one launch of our own kernel
    writes all seven slices into every rank's full outputs and completes with
    one handshake (hd_push_columns_multi, IPC-mapped buffers);
    HACEDLE_EXCHANGE=push1 pushes output by output (seven handshakes),
    HACEDLE_EXCHANGE=nccl uses an NCCL all-gather plus hd_gather_columns.
    Total work is fixed (strong scaling); times are device times (the work is
    queued behind a device-side spin), max over ranks, after a 256 MB L2 flush
    before every rep."""
    import torch

    import hacedle_cuda as hc
    from hacedle_cuda import shard

    hbm, bf16, kind = peaks()
    H, F, nq, nkv = 3584, 18944, 28 * 128, 4 * 128
    mats = [("q", S.GGML_Q4_K, nq, H), ("k", S.GGML_Q4_K, nkv, H), ("v", S.GGML_Q4_K, nkv, H),
            ("o", S.GGML_Q4_K, H, nq), ("gate", S.GGML_Q4_K, F, H), ("up", S.GGML_Q4_K, F, H),
            ("down", S.GGML_Q6_K, H, F)]
    ws = []
    for i, (nm, t, N, K) in enumerate(mats):
        raw = S.gen_weight(t, N, K, seed=50 + i)
        ws.append((nm, t, N, K, ctx.weight(t, shard.row_slice(raw, t, N, K, rank, world), N // world, K)))
    w_total = sum(S.nbytes(t, N, K) for _, t, N, K in mats)
    flops_per_tok = sum(2 * N * K for _, t, N, K in mats)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    use_nccl = os.environ.get("HACEDLE_EXCHANGE", "") == "nccl"
    one_by_one = os.environ.get("HACEDLE_EXCHANGE", "") == "push1"
    peer = None
    if world > 1 and not use_nccl:
        import torch.distributed as dist

        def ago(obj):
            out = [None] * world
            dist.all_gather_object(out, obj)
            return out
        peer = shard.PeerExchange(ctx, world, rank, [(512, N) for _, _, N, _ in mats], ago)
    res = {"scaling": "strong", "ranks": world, "weight_bytes_layer": w_total, "peak_kind": kind,
           "exchange": ("none" if world == 1 else
                        "NCCL all_gather_into_tensor (torch.distributed) + hd_gather_columns" if use_nccl else
                        "hd_push_columns per output: P2P stores over NVLink into IPC-mapped outputs, "
                        "one epoch handshake each" if one_by_one else
                        "hd_push_columns_multi: P2P stores over NVLink into IPC-mapped outputs, all seven "
                        "outputs in one launch with one epoch handshake")}
    for B in (1, 64, 512):
        xs = {K: torch.from_numpy(S.gen_activations(B, K, 60)).cuda() for K in (H, F)}
        ys = [torch.empty(B, N // world, device="cuda") for _, _, N, _, _ in ws]
        gath = ([torch.empty(world, B, N // world, device="cuda") for _, _, N, _, _ in ws] if world > 1 and not peer
                else [None] * len(ws))
        full = ([peer.full(i, B) for i in range(len(ws))] if peer else
                [torch.empty(B, N, device="cuda") for _, _, N, _, _ in ws])

        def compute():
            for (nm, t, N, K, w), y in zip(ws, ys):
                if B <= 16:
                    ctx.qgemv(w, xs[K], y)
                else:
                    ctx.qgemm(w, xs[K], y, precision=hc.PREC_BF16_TC)

        def exchange():
            import torch.distributed as dist
            if peer and not one_by_one:
                peer.push_all([(i, y, N // world) for i, ((nm, t, N, K, w), y) in enumerate(zip(ws, ys))], B)
                return
            for i, ((nm, t, N, K, w), y, g, f) in enumerate(zip(ws, ys, gath, full)):
                if peer:
                    peer.push(i, y, B, N // world)
                elif world > 1:
                    dist.all_gather_into_tensor(g.view(-1), y.view(-1))
                    ctx.gather_columns(g, f, world, B, N // world)
                else:
                    f.copy_(y)

        for _ in range(2):
            compute()
            exchange()
        torch.cuda.synchronize()
        c_ms, t_ms = [], []
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        for _ in range(reps):
            flush.zero_()
            barrier(world)
            torch.cuda._sleep(int(3e6))  # covers the host's enqueue time: the events see device time
            ev[0].record()
            compute()
            ev[1].record()
            exchange()
            ev[2].record()
            torch.cuda.synchronize()
            c_ms.append(ev[0].elapsed_time(ev[1]))
            t_ms.append(ev[0].elapsed_time(ev[2]))
        ctx.check_device_errors()
        cm = max_over_ranks(_median(c_ms), world)
        tm = max_over_ranks(_median(t_ms), world)
        ent = {"compute_ms": round(cm, 4), "exchange_ms": round(tm - cm, 4), "total_ms": round(tm, 4),
               "allgather_bytes": int(4 * B * sum(N for _, _, N, _ in mats) * (world - 1) // world)}
        if B == 1:
            ent["gbs"] = round(w_total / (tm * 1e-3) / 1e9, 1)
            ent["compute_gbs_per_gpu"] = round(w_total / world / (cm * 1e-3) / 1e9, 1)
            ent["frac_of_hbm_compute"] = round(w_total / world / (cm * 1e-3) / 1e9 / hbm, 4)
        else:
            ent["tflops"] = round(flops_per_tok * B / (tm * 1e-3) / 1e12, 2)
            ent["compute_tflops_per_gpu"] = round(flops_per_tok * B / world / (cm * 1e-3) / 1e12, 2)
        res[f"B{B}"] = ent
    if peer:
        barrier(world)
        peer.close()
    for *_, w in ws:
        w.free()
    return res


LARGE_CASES = [(S.GGML_Q5_0, 18944, 3584), (S.GGML_Q4_K, 18944, 3584), (S.GGML_Q6_K, 3584, 18944),
               (S.GGML_Q8_0, 151936, 896)]


def gemv_large_workload(ctx, batches=(1, 4), reps=5):
    """Decode Q-GEMV on matrices large enough to stream at HBM bandwidth:
    Q5_0 and Q4_K [18944 x 3584] (the 7B-shaped gate/up), Q6_K
    [3584 x 18944] (down) and the Q8_0 [151936 x 896] tied LM head, at batch 1
    and 4.  Each case is one CUDA graph of back-to-back GEMVs (PDL edges) over
    weight copies that together exceed 3x L2, so every launch streams its
    weight from HBM; us per launch = graph time / launches, median of `reps`
    replays."""
    import torch

    hbm, _, kind = peaks()
    l2 = torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size
    res = {"unit": "GB/s", "peak_hbm_gbs": hbm, "peak_kind": kind,
           "l2_policy": "weight copies > 3x L2 per graph, rotated"}
    for (t, N, K) in LARGE_CASES:
        nb = S.nbytes(t, N, K)
        raw = S.gen_weight(t, N, K, seed=2 + t)
        ws = [ctx.weight(t, raw, N, K) for _ in range(max(4, int(np.ceil(3 * l2 / nb))))]
        for B in batches:
            x = torch.from_numpy(S.gen_activations(B, K, 5)).cuda()
            y = torch.empty(B, N, device="cuda")
            for w in ws:
                ctx.qgemv(w, x, y)
            torch.cuda.synchronize()
            g, st = torch.cuda.CUDAGraph(), torch.cuda.Stream()
            with torch.cuda.graph(g, stream=st):
                ctx.set_stream(torch.cuda.current_stream().cuda_stream)
                for w in ws:
                    ctx.qgemv(w, x, y)
            ctx.set_stream(torch.cuda.current_stream().cuda_stream)
            for _ in range(3):
                g.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ts = []
            for _ in range(reps):
                e0.record()
                g.replay()
                e1.record()
                torch.cuda.synchronize()
                ts.append(e0.elapsed_time(e1) * 1e3 / len(ws))
            us = _median(ts)
            byts = case_bytes(t, N, K, B)
            gbs = byts / (us * 1e-6) / 1e9
            res[f"{S.TYPE_NAME[t]}_{N}x{K}_B{B}"] = {
                "us_per_launch": round(us, 3), "gbs": round(gbs, 1),
                "frac_of_hbm": round(gbs / hbm, 4), "bytes_per_launch": byts, "launches_per_graph": len(ws)}
            del g
        ctx.check_device_errors()
        for w in ws:
            w.free()
    return res


def e2e_host(ctx, weights, args):
    """Same sweep through hd_qgemv_host with host buffers (one weight copy per
    case is enough: x and y cross PCIe every call, weights are device-resident)."""
    import torch

    reps = 8

    def pinned(shape):
        return torch.empty(shape, dtype=torch.float32, pin_memory=True).numpy()

    # x and y live in pinned host memory (page-locked: the copies are DMA)
    xs, ys = {}, {}
    for (t, N, K) in CASES:
        for B in BATCHES:
            xs[(t, B)] = pinned((B, K))
            xs[(t, B)][:] = S.gen_activations(B, K, 100 + B)
            ys[(t, B)] = pinned((B, N))
    for (t, N, K) in CASES:
        for B in BATCHES:
            ctx.qgemv_host(weights[t][0], xs[(t, B)], out=ys[(t, B)])
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    byts = h2d = d2h = 0
    for _ in range(reps):
        for (t, N, K) in CASES:
            for i, B in enumerate(BATCHES):
                w = weights[t][(_ * 3 + i) % len(weights[t])]
                ctx.qgemv_host(w, xs[(t, B)], out=ys[(t, B)])
                byts += case_bytes(t, N, K, B)
                h2d += 4 * B * K
                d2h += 4 * B * N
    dt = time.perf_counter() - t0
    return {"value": round(byts / dt / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d // reps,
            "d2h_bytes_per_step": d2h // reps, "calls_per_step": len(CASES) * len(BATCHES),
            "api": "hd_qgemv_host (pinned host x in, pinned host y out, sync per call)"}


def cpu_baseline_sample(raws, budget_s=10.0, threads=1):
    """The reference's CPU path (oracle port: whole-tensor dequant + sequential
    GEMV, as NativeBackend / block.rs do) on a bounded sample of the sweep."""
    from oracle import oracle as O

    xs = {(K, B): S.gen_activations(B, K, 100 + B) for (t, N, K) in CASES for B in BATCHES}
    t0 = time.perf_counter()
    byts, n = 0, 0
    while True:
        for (t, N, K) in CASES:
            for B in BATCHES:
                O.qgemv(t, raws[t], N, K, xs[(K, B)], threads=threads)
                byts += case_bytes(t, N, K, B)
                n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": round(byts / dt / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} GEMVs ({n // 9} passes of the 9-case sweep), whole-tensor dequant per call",
            "seconds": round(dt, 2)}


# ------------------------------------------------------------ reference arm
def run_reference(args, rank, world):
    """The reference's CPU implementation of the path (the oracle port; the
    Rust crate has no toolchain here and does not build), all host threads."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    raws = {t: S.gen_weight(t, N, K, seed=2 + t) for (t, N, K) in CASES}
    from oracle import oracle as O

    O.lib()
    for _ in range(max(1, args.warmup)):
        for (t, N, K) in CASES:
            O.qgemv(t, raws[t], N, K, S.gen_activations(1, K, 101), threads=threads)
    xs = {(K, B): S.gen_activations(B, K, 100 + B) for (t, N, K) in CASES for B in BATCHES}  # outside the timing
    byts, t_total = 0, 0.0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        for (t, N, K) in CASES:
            for B in BATCHES:
                O.qgemv(t, raws[t], N, K, xs[(K, B)], threads=threads)
                byts += case_bytes(t, N, K, B)
        t_total += time.perf_counter() - t0
    value = byts / t_total / 1e9
    res = {"metric": METRIC, "value": round(value, 4), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(t_total / args.steps * 1e3, 3), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded PCG64)",
           "config": {"workload": "decode Q-GEMV sweep: Q5_0 4864x896, Q6_K 896x4864, Q4_K 896x4864 at B=1,4,16"},
           "impl": "reference",
           "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                            "sample": "one pass of the 9-case sweep per step (whole-tensor dequant per call)"},
           "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(res), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--copies", type=int, default=8)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="headline GEMV sweep only")
    ap.add_argument("--only", choices=["prefill", "dequant", "decode", "layer7b", "gemv_large"],
                    help="run one secondary workload")
    ap.add_argument("--decode-batch", type=int, default=256,
                    help="sequences decoded together, split over the ranks (0: batch 1 only)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, rank, int(os.environ.get("WORLD_SIZE", "1")))
        return
    rank, world, local = dist_init()
    try:
        run_ours(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
