"""The C-ABI library: it loads, exports every symbol include/hacedle_cuda.h
declares, and rejects bad arguments before touching a GPU (CPU only)."""
import ctypes as C
import os
import re

import pytest

import hacedle_cuda as hc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = []
    for fn in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if fn.endswith(".h"):
            txt = open(os.path.join(ROOT, "include", fn)).read()
            names += re.findall(r"^(?:int|const char \*|uint64_t)\s*\**\s*(hd_\w+)\s*\(", txt, re.M)
    return names


def test_library_built_in_tree():
    assert os.path.exists(hc.LIB_PATH), "run __graft_entry__.build() first"


def test_exports_every_declared_symbol():
    L = hc.lib()
    declared = _declared()
    assert len(declared) >= 30
    assert set(declared) == set(hc.EXPORTS), set(declared) ^ set(hc.EXPORTS)
    for name in declared:
        assert hasattr(L, name), name


def test_version_string():
    assert b"sm_100a" in hc.lib().hd_version()


def test_null_arguments_are_rejected_without_a_gpu():
    L = hc.lib()
    assert L.hd_qgemv(None, None, None, None, 1, None, None) == hc.HD_E_ARG
    assert L.hd_weight_upload(None, None, 0, 8, 1, 32, None) == hc.HD_E_ARG
    assert L.hd_dequantize(None, None, None, 0) == hc.HD_E_ARG
    assert L.hd_rmsnorm(None, None, None, None, None, 1, 1, C.c_float(1e-6)) == hc.HD_E_ARG
    assert L.hd_ctx_create(0, None) == hc.HD_E_ARG
    assert L.hd_ctx_destroy(None) == hc.HD_E_ARG
    assert L.hd_last_error(None) == b"null context"
    # NVLink exchange entry points
    assert L.hd_xbuf_alloc(None, 1024, None) == hc.HD_E_ARG
    assert L.hd_xbuf_free(None, None) == hc.HD_E_ARG
    assert L.hd_ipc_handle(None, None, None) == hc.HD_E_ARG
    assert L.hd_ipc_open(None, None, None) == hc.HD_E_ARG
    assert L.hd_ipc_close(None, None) == hc.HD_E_ARG
    assert L.hd_push_columns(None, None, None, None, 2, 0, 1, 4, 1) == hc.HD_E_ARG


def test_context_creation_fails_cleanly_without_device():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = C.c_void_p()
    assert hc.lib().hd_ctx_create(0, C.byref(h)) == hc.HD_E_CUDA
    assert not h.value
