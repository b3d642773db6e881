"""GGUF v2/v3 files through the library's reader (hd_gguf_* in
include/hacedle_cuda.h): metadata, tensor index and bytes, device upload, and
the model dict of a Qwen2-architecture GGUF in the form `Decoder` and the
oracle take.

Replaces GgufLoader (src/x/loader/gguf/loader.rs:64-141) and the tensor-name
projection of tensor_projection.rs for the qwen2 architecture (llama.cpp
tensor names: token_embd, blk.N.attn_{norm,q,k,v,output}, blk.N.ffn_{norm,
gate,up,down}, output_norm).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import HdError, Weight, lib

VALUE_TYPES = {0: "u8", 1: "i8", 2: "u16", 3: "i16", 4: "u32", 5: "i32", 6: "f32", 7: "bool", 8: "str",
               9: "array", 10: "u64", 11: "i64", 12: "f64"}
_NUMPY = {0: np.uint8, 1: np.int8, 2: np.uint16, 3: np.int16, 4: np.uint32, 5: np.int32, 6: np.float32,
          7: np.uint8, 10: np.uint64, 11: np.int64, 12: np.float64}
TYPE_F32 = 0


class _TensorInfo(C.Structure):
    _fields_ = [("name", C.c_char_p), ("ggml_type", C.c_int32), ("n_dims", C.c_int32), ("dims", C.c_int64 * 4),
                ("offset", C.c_uint64), ("nbytes", C.c_uint64), ("data", C.c_void_p)]


def _raise(rc: int):
    if rc:
        raise HdError(rc, lib().hd_gguf_error().decode(errors="replace"))


class GGUF:
    """A parsed GGUF file (`path`, mapped read-only) or byte string (`data`).

    tensors: list of {name, type, dims (ggml order, dims[0] contiguous),
    offset, nbytes}; kv: {key: value} with ints, floats, bools, str, numpy
    arrays or lists of str."""

    def __init__(self, path: str | None = None, data: bytes | None = None):
        h = C.c_void_p()
        if path is not None:
            rc = lib().hd_gguf_open(os.fsencode(path), C.byref(h))
        else:
            buf = np.frombuffer(data, np.uint8)
            rc = lib().hd_gguf_open_memory(buf.ctypes.data, buf.size, C.byref(h))
        _raise(rc)
        self.h = h
        ver, nt, nk, al = C.c_uint32(), C.c_int64(), C.c_int64(), C.c_uint64()
        _raise(lib().hd_gguf_counts(h, C.byref(ver), C.byref(nt), C.byref(nk), C.byref(al)))
        self.version, self.alignment = ver.value, al.value
        self.tensors = [self._tensor(i) for i in range(nt.value)]
        self._by_name = {t["name"]: i for i, t in enumerate(self.tensors)}
        self.kv = {}
        self.kv_types = {}
        for i in range(nk.value):
            key, vt, at, n = C.c_char_p(), C.c_int32(), C.c_int32(), C.c_uint64()
            _raise(lib().hd_gguf_kv(h, i, C.byref(key), C.byref(vt), C.byref(at), C.byref(n)))
            k = key.value.decode(errors="replace")
            self.kv_types[k] = (VALUE_TYPES.get(vt.value, vt.value), VALUE_TYPES.get(at.value, at.value))
            self.kv[k] = self._value(i, vt.value, at.value, n.value)

    def _tensor(self, i: int) -> dict:
        info = _TensorInfo()
        _raise(lib().hd_gguf_tensor(self.h, i, C.byref(info)))
        return {"name": info.name.decode(errors="replace"), "type": info.ggml_type,
                "dims": tuple(info.dims[d] for d in range(info.n_dims)), "offset": info.offset,
                "nbytes": info.nbytes, "_data": info.data}

    def _string(self, i: int, j: int) -> str:
        s, n = C.c_void_p(), C.c_uint64()
        _raise(lib().hd_gguf_kv_string(self.h, i, j, C.byref(s), C.byref(n)))
        return C.string_at(s.value, n.value).decode(errors="replace") if n.value else ""

    def _value(self, i: int, vt: int, at: int, n: int):
        if vt == 8:
            return self._string(i, 0)
        if vt == 9:
            if at == 8:
                return [self._string(i, j) for j in range(n)]
            p, cnt = C.c_void_p(), C.c_uint64()
            _raise(lib().hd_gguf_kv_array(self.h, i, C.byref(p), C.byref(cnt)))
            dt = np.dtype(_NUMPY[at])
            raw = C.string_at(p.value, cnt.value * dt.itemsize) if cnt.value else b""
            arr = np.frombuffer(raw, dt).copy()
            return arr.astype(bool) if at == 7 else arr
        if vt == 10:  # u64: the full range, from the raw value
            p, cnt = C.c_void_p(), C.c_uint64()
            _raise(lib().hd_gguf_kv_array(self.h, i, C.byref(p), C.byref(cnt)))
            return int(np.frombuffer(C.string_at(p.value, 8), np.uint64)[0])
        if vt in (6, 12):
            v = C.c_double()
            _raise(lib().hd_gguf_kv_float(self.h, i, C.byref(v)))
            return v.value
        v = C.c_int64()
        _raise(lib().hd_gguf_kv_int(self.h, i, C.byref(v)))
        return bool(v.value) if vt == 7 else v.value

    def tensor(self, name: str) -> dict:
        idx = C.c_int64()
        _raise(lib().hd_gguf_find_tensor(self.h, name.encode(), C.byref(idx)))
        return self.tensors[idx.value]

    def has(self, name: str) -> bool:
        return name in self._by_name

    def tensor_bytes(self, name: str) -> np.ndarray:
        """A copy of the tensor's bytes (GgufLoader::tensor_bytes, loader.rs:117-141)."""
        t = self.tensor(name)
        if t["nbytes"] == 0:
            raise HdError(3, f"gguf: size of ggml type {t['type']} of '{name}' is not known")
        return np.frombuffer(C.string_at(t["_data"], t["nbytes"]), np.uint8).copy()

    def f32(self, name: str) -> np.ndarray:
        t = self.tensor(name)
        if t["type"] != TYPE_F32:
            raise HdError(3, f"gguf: '{name}' has ggml type {t['type']}, not F32")
        return self.tensor_bytes(name).view(np.float32).reshape(tuple(reversed(t["dims"])))

    def matrix(self, name: str) -> tuple:
        """(ggml_type, raw bytes, rows, cols) of a 2-D tensor (dims {cols, rows})."""
        t = self.tensor(name)
        return (t["type"], self.tensor_bytes(name), int(t["dims"][1]), int(t["dims"][0]))

    def upload(self, ctx, name: str) -> Weight:
        """hd_gguf_upload: the named quantized matrix as a device weight."""
        h = C.c_void_p()
        ctx._check(lib().hd_gguf_upload(ctx.h, self.h, name.encode(), C.byref(h)))
        t = self.tensor(name)
        return Weight.from_handle(ctx, h, t["type"], int(t["dims"][1]), int(t["dims"][0]), int(t["nbytes"]))

    def close(self):
        if getattr(self, "h", None):
            lib().hd_gguf_close(self.h)
        self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def qwen2_model(g: GGUF) -> dict:
    """The Decoder / oracle model dict of a qwen2-architecture GGUF: config from
    the qwen2.* metadata, quantized matrices as (type, bytes, rows, cols), f32
    biases and norm weights.  The LM head must be tied to token_embd (no
    output.weight), as in Qwen2.5-0.5B."""
    arch = g.kv.get("general.architecture")
    if arch != "qwen2":
        raise HdError(8, f"gguf: architecture {arch!r} (qwen2 is read)")
    if g.has("output.weight"):
        raise HdError(8, "gguf: untied LM head (output.weight): the decoder reads the tied token_embd")
    kv = g.kv
    H = int(kv["qwen2.embedding_length"])
    nh = int(kv["qwen2.attention.head_count"])
    cfg = {"hidden": H, "n_layers": int(kv["qwen2.block_count"]), "n_heads": nh,
           "n_kv": int(kv.get("qwen2.attention.head_count_kv", nh)),
           "head_dim": int(kv.get("qwen2.attention.key_length", H // nh)),
           "ffn": int(kv["qwen2.feed_forward_length"]), "vocab": int(g.tensor("token_embd.weight")["dims"][1]),
           "eps": float(kv.get("qwen2.attention.layer_norm_rms_epsilon", 1e-6)),
           "theta": float(kv.get("qwen2.rope.freq_base", 1e6))}
    layers = []
    for i in range(cfg["n_layers"]):
        b = f"blk.{i}."
        L = {"wq": g.matrix(b + "attn_q.weight"), "wk": g.matrix(b + "attn_k.weight"),
             "wv": g.matrix(b + "attn_v.weight"), "wo": g.matrix(b + "attn_output.weight"),
             "wg": g.matrix(b + "ffn_gate.weight"), "wu": g.matrix(b + "ffn_up.weight"),
             "wd": g.matrix(b + "ffn_down.weight"),
             "bq": g.f32(b + "attn_q.bias"), "bk": g.f32(b + "attn_k.bias"), "bv": g.f32(b + "attn_v.bias"),
             "attn_norm": g.f32(b + "attn_norm.weight"), "ffn_norm": g.f32(b + "ffn_norm.weight")}
        layers.append(L)
    return {"cfg": cfg, "layers": layers, "out_norm": g.f32("output_norm.weight"),
            "embed": g.matrix("token_embd.weight")}
