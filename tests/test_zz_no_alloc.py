"""GPU: q6w_linear_argmax_noalloc, the vocab projection + argmax entry point
that allocates nothing (its argmax scratch is a library-owned device array),
for callers that cannot allocate device memory: FFI hosts without a CUDA
allocator of their own, and serving loops under a fixed memory budget.

Checked through the C ABI against q6w_linear_argmax (caller scratch) on two
calls in a row -- the second smaller than the first, so stale keys left in
the shared array by the first call would show -- with the FP32 linear
tolerance the other linear tests use.  Kept in its own file, collected last.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import codec
from q6w_b200 import _lib

pytestmark = pytest.mark.gpu
MAX_ROWS = 32768
TOL = 1e-4  # max |logit difference|, as tests/test_gpu_linear.py against torch FP32


def _weights(rows, cols, seed):
    rng = np.random.default_rng(seed)
    q = rng.integers(-32, 32, size=(rows, cols))
    s = rng.uniform(0.001, 0.05, size=rows).astype(np.float32)
    packed = torch.frombuffer(bytearray(codec.pack_int6(q, allow_minus32=True)), dtype=torch.uint8).cuda()
    return packed, torch.from_numpy(s).cuda()


def _with_scratch(lib, packed, scales, x, rows, cols):
    n = x.shape[0]
    am = torch.empty(n, dtype=torch.int32, device="cuda")
    lg = torch.empty((n, rows), device="cuda")
    scratch = torch.empty(n, dtype=torch.int64, device="cuda")
    _lib.check(lib.q6w_linear_argmax(packed.data_ptr(), scales.data_ptr(), x.data_ptr(), lg.data_ptr(),
                                     am.data_ptr(), scratch.data_ptr(), n * 8, rows, cols, n, _lib.stream_handle()))
    return am, lg


def _no_alloc(lib, packed, scales, x, rows, cols):
    n = x.shape[0]
    am = torch.empty(n, dtype=torch.int32, device="cuda")
    lg = torch.empty((n, rows), device="cuda")
    _lib.check(lib.q6w_linear_argmax_noalloc(packed.data_ptr(), scales.data_ptr(), x.data_ptr(), lg.data_ptr(),
                                             am.data_ptr(), rows, cols, n, _lib.stream_handle()))
    return am, lg


def test_no_alloc_matches_scratch_entry_point_twice():
    lib = _lib.load()
    rows, cols = 4096, 128
    packed, scales = _weights(rows, cols, 21)
    g = torch.Generator().manual_seed(5)
    for n in (300, 7):  # two calls in a row, the second smaller
        x = torch.randn(n, cols, generator=g).cuda()
        am_ref, lg_ref = _with_scratch(lib, packed, scales, x, rows, cols)
        am, lg = _no_alloc(lib, packed, scales, x, rows, cols)
        torch.cuda.synchronize()
        assert torch.equal(am, am_ref)
        assert float((lg - lg_ref).abs().max()) <= TOL
        assert torch.equal(am.long(), lg.argmax(dim=1))


def test_no_alloc_rejects_oversize_batch():
    lib = _lib.load()
    rc = lib.q6w_linear_argmax_noalloc(None, None, None, None, None, 4096, 128, MAX_ROWS + 1, ctypes.c_void_p(0))
    assert rc == _lib.Q6W_ERR_ARG
    assert b"exceeds the built-in maximum" in lib.q6w_last_error()
