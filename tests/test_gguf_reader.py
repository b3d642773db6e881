"""The GGUF v2/v3 reader (hd_gguf_*), host only: against gguf-py's own reader
on the committed fixtures (tests/golden/make_gguf_fixtures.py writes them with
GGUFWriter), against the synthetic model the fixture was made from, every
metadata value type, a non-default alignment, and malformed files (truncated
anywhere, corrupted bytes, bad magic, other versions) failing with an error
code instead of reading out of range."""
import os

import numpy as np
import pytest

import hacedle_cuda as hc
from hacedle_cuda import gguf as G
from hacedle_cuda import synth as S

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TINY_PATH = os.path.join(GOLD, "qwen2_tiny.gguf")
ALIGN_PATH = os.path.join(GOLD, "align64.gguf")
TINY = dict(hidden=64, n_layers=3, n_heads=2, n_kv=1, head_dim=32, ffn=256, vocab=256, eps=1e-6, theta=1e6)


def _bytes(path):
    with open(path, "rb") as f:
        return f.read()


@pytest.mark.parametrize("path", [TINY_PATH, ALIGN_PATH])
def test_reader_matches_gguf_py(path):
    gguf = pytest.importorskip("gguf")
    ref = gguf.GGUFReader(path)
    g = G.GGUF(path)
    assert [t["name"] for t in g.tensors] == [t.name for t in ref.tensors]
    for t, r in zip(g.tensors, ref.tensors):
        assert t["type"] == int(r.tensor_type)
        assert t["dims"] == tuple(int(d) for d in r.shape)
        assert t["offset"] == r.data_offset
        assert t["nbytes"] == r.n_bytes
        assert g.tensor_bytes(t["name"]).tobytes() == np.asarray(r.data).tobytes()
    keys = [k for k in ref.fields if not k.startswith("GGUF.")]
    assert sorted(keys) == sorted(g.kv)
    for k in keys:
        f = ref.fields[k]
        want = f.contents()
        got = g.kv[k]
        if isinstance(got, np.ndarray):
            assert got.tolist() == list(want)
        elif isinstance(got, float):
            assert got == pytest.approx(want, rel=1e-7)
        else:
            assert got == want, k


def test_tiny_model_is_the_synthetic_decoder():
    g = G.GGUF(TINY_PATH)
    m = G.qwen2_model(g)
    ref = S.gen_decoder(TINY, seed=21)
    assert m["cfg"]["hidden"] == 64 and m["cfg"]["n_layers"] == 3 and m["cfg"]["vocab"] == 256
    assert m["cfg"]["n_heads"] == 2 and m["cfg"]["n_kv"] == 1 and m["cfg"]["head_dim"] == 32
    assert m["cfg"]["eps"] == pytest.approx(1e-6) and m["cfg"]["theta"] == 1e6
    for L, R in zip(m["layers"], ref["layers"]):
        for k in ("wq", "wk", "wv", "wo", "wg", "wu", "wd"):
            assert L[k][0] == R[k][0] and L[k][2:] == R[k][2:], k
            assert L[k][1].tobytes() == np.asarray(R[k][1], np.uint8).tobytes(), k
        for k in ("bq", "bk", "bv", "attn_norm", "ffn_norm"):
            assert np.array_equal(L[k], R[k]), k
    assert np.array_equal(m["out_norm"], ref["out_norm"])
    assert m["embed"][1].tobytes() == np.asarray(ref["embed"][1], np.uint8).tobytes()


def test_every_value_type():
    kv = G.GGUF(TINY_PATH).kv
    assert kv["test.u8"] == 200 and kv["test.i8"] == -100
    assert kv["test.u16"] == 60000 and kv["test.i16"] == -30000
    assert kv["test.u32"] == 4000000000 and kv["test.i32"] == -2000000000
    assert kv["test.u64"] == 2 ** 63 + 5 and kv["test.i64"] == -(2 ** 62)
    assert kv["test.f32"] == 0.15625 and kv["test.f64"] == 2.718281828459045
    assert kv["test.bool"] is True and kv["test.str"] == "héllo gguf"
    assert kv["test.arr_i32"].tolist() == [1, -2, 3, -4]
    assert kv["test.arr_f32"].tolist() == [0.5, -1.25]
    assert kv["tokenizer.ggml.tokens"] == [f"tok{i}" for i in range(12)] + ["", "é"]


def test_alignment_64():
    g = G.GGUF(ALIGN_PATH)
    assert g.alignment == 64
    assert all(t["offset"] % 64 == 0 for t in g.tensors)
    assert g.f32("a").tolist() == [0.0, 1.0, 2.0]
    t, raw, rows, cols = g.matrix("b")
    assert (t, rows, cols) == (S.GGML_Q8_0, 2, 64)
    assert raw.tobytes() == np.asarray(S.gen_weight(S.GGML_Q8_0, 2, 64, 9), np.uint8).tobytes()


def test_open_memory_equals_open_file():
    a, b = G.GGUF(TINY_PATH), G.GGUF(data=_bytes(TINY_PATH))
    assert [(t["name"], t["type"], t["dims"], t["offset"], t["nbytes"]) for t in a.tensors] == \
           [(t["name"], t["type"], t["dims"], t["offset"], t["nbytes"]) for t in b.tensors]
    assert a.tensor_bytes("blk.2.ffn_down.weight").tobytes() == b.tensor_bytes("blk.2.ffn_down.weight").tobytes()


def test_missing_names_and_files():
    g = G.GGUF(TINY_PATH)
    with pytest.raises(hc.HdError) as e:
        g.tensor("no.such.tensor")
    assert e.value.code == hc.HD_E_ARG and "no.such.tensor" in str(e.value)
    with pytest.raises(hc.HdError) as e:
        G.GGUF(os.path.join(GOLD, "does_not_exist.gguf"))
    assert e.value.code == hc.HD_E_ARG
    with pytest.raises(hc.HdError):
        g.f32("token_embd.weight")             # Q8_0, not F32
    assert hc.lib().hd_gguf_upload(None, g.h, b"token_embd.weight", None) == hc.HD_E_ARG


def test_truncated_anywhere_fails_cleanly():
    """Every prefix that cuts the header, metadata, tensor index or tensor data
    is rejected with HD_E_ARG (the reader checks bounds before every read)."""
    raw = _bytes(TINY_PATH)
    g = G.GGUF(TINY_PATH)
    end_of_index = min(t["offset"] for t in g.tensors)
    cuts = sorted(set(list(range(0, end_of_index, 5)) + [end_of_index - 1, len(raw) - 1,
                                                          g.tensors[-1]["offset"] + 3]))
    for n in cuts:
        with pytest.raises(hc.HdError) as e:
            G.GGUF(data=raw[:n] if n >= 1 else b"\0")
        assert e.value.code == hc.HD_E_ARG, n


def test_corrupted_bytes_never_read_out_of_range():
    """Seeded random corruption of the header and index region: each file
    either parses (and every tensor lies inside it) or fails with an error."""
    raw = bytearray(_bytes(TINY_PATH))
    end_of_index = min(t["offset"] for t in G.GGUF(TINY_PATH).tensors)
    rng = np.random.default_rng(5)
    ok = 0
    for _ in range(400):
        b = bytearray(raw)
        for _ in range(int(rng.integers(1, 4))):
            b[int(rng.integers(4, end_of_index))] = int(rng.integers(0, 256))
        try:
            g = G.GGUF(data=bytes(b))
        except hc.HdError as e:
            assert e.code in (hc.HD_E_ARG, hc.HD_E_UNSUPPORTED)
            continue
        ok += 1
        for t in g.tensors:
            assert t["offset"] + t["nbytes"] <= len(b)
    assert ok < 400


def test_magic_and_version():
    raw = bytearray(_bytes(ALIGN_PATH))
    bad = bytearray(raw)
    bad[0:4] = b"GGUX"
    with pytest.raises(hc.HdError) as e:
        G.GGUF(data=bytes(bad))
    assert e.value.code == hc.HD_E_ARG
    for v in (1, 4, 0x03000000):          # v1 (u32 counts), unknown, byte-swapped (big-endian file)
        bad = bytearray(raw)
        bad[4:8] = int(v).to_bytes(4, "little")
        with pytest.raises(hc.HdError) as e:
            G.GGUF(data=bytes(bad))
        assert e.value.code == hc.HD_E_UNSUPPORTED
    v2 = bytearray(raw)                    # v2 has the v3 layout
    v2[4:8] = (2).to_bytes(4, "little")
    assert G.GGUF(data=bytes(v2)).version == 2
