"""hd_argmax_rows_noalloc, the argmax entry point for callers that cannot let
a library allocate device memory (runtimes that own every byte of HBM through
their own pool, or latency-critical paths that cannot take cudaMalloc's
synchronization).  It is called here through the C ABI and must give exactly
the indices of hd_argmax_rows, on two calls in a row that share its static
scratch array.  This file is collected last so that a stop-at-first-failure
run has already run every other test."""
import ctypes as C

import numpy as np
import pytest

import hacedle_cuda as hc
from hacedle_cuda import synth as S
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream or hc.CUDA_STREAM_LEGACY


def _noalloc(x, rows, n):
    import torch
    idx = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
    rc = hc.lib().hd_argmax_rows_noalloc(x.data_ptr(), rows, n, idx.data_ptr(), _stream())
    assert rc == hc.HD_OK, rc
    torch.cuda.synchronize()
    return idx.cpu().numpy()


def _reference(ctx, x, rows):
    import torch
    idx = torch.empty(rows, dtype=torch.int32, device="cuda")
    ctx.argmax_rows(x, idx)
    torch.cuda.synchronize()
    return idx.cpu().numpy()


# (1000, 140000): 16384 partials allow 16 chunks per row, so each of the 18
# chunks of 8192 values is widened to 8750.
@pytest.mark.parametrize("rows,n", [(1, 151936), (3, 2_000_000), (64, 100_000), (300, 8193), (5, 7),
                                    (1000, 140_000)])
def test_noalloc_argmax_matches_existing_entry_point_twice(ctx, rows, n):
    import torch
    for call in range(2):
        x = S.rng(1000 * call + rows).standard_normal((rows, n), dtype=np.float32)
        if n > 10:
            x[0, [3, n - 1]] = 50.0 + call      # tie: the lower index wins
            x[-1, 0] = np.nan                   # NaN at index 0 gives 0
        xd = torch.from_numpy(x).cuda()
        got = _noalloc(xd, rows, n)
        exp = _reference(ctx, xd, rows)
        assert np.array_equal(got, exp), (call, got[:8], exp[:8])
        # and directly against the oracle's ArgMaxSampler::sample
        assert [int(v) for v in got] == [O.argmax(x[r]) for r in range(rows)]
        del xd


def test_noalloc_rejects_rows_beyond_its_scratch():
    import torch
    x = torch.zeros(4097, 16, device="cuda")
    idx = torch.zeros(4097, dtype=torch.int32, device="cuda")
    rc = hc.lib().hd_argmax_rows_noalloc(x.data_ptr(), 4097, 16, idx.data_ptr(), _stream())
    assert rc == hc.HD_E_SHAPE
    # indices are int32: rows of 2^31 values or more are refused before any access
    assert hc.lib().hd_argmax_rows_noalloc(x.data_ptr(), 1, 1 << 31, idx.data_ptr(), _stream()) == hc.HD_E_SHAPE
    assert hc.lib().hd_argmax_rows_noalloc(None, 1, 16, None, None) == hc.HD_E_ARG
