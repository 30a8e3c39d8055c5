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
import json
import os
import subprocess
import sys
import textwrap
from pathlib import Path

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


def test_no_alloc_full_array_and_empty_batch():
    """n == MAX_ROWS fills the whole shared array; n == 0 returns at once."""
    lib = _lib.load()
    rows, cols = 64, 16
    packed, scales = _weights(rows, cols, 33)
    x = torch.randn(MAX_ROWS, cols, generator=torch.Generator().manual_seed(9)).cuda()
    am_ref, lg_ref = _with_scratch(lib, packed, scales, x, rows, cols)
    am, lg = _no_alloc(lib, packed, scales, x, rows, cols)
    torch.cuda.synchronize()
    assert torch.equal(am, am_ref)
    assert float((lg - lg_ref).abs().max()) <= TOL
    rc = lib.q6w_linear_argmax_noalloc(packed.data_ptr(), scales.data_ptr(), x.data_ptr(), None, None, rows, cols, 0,
                                       _lib.stream_handle())
    assert rc == _lib.Q6W_OK


# Child process: raw CUDA runtime through ctypes (no torch, whose memory a
# device reset would invalidate).  Calls both entry points, resets the
# device (a new primary context), and calls them again.
_RESET_CHILD = textwrap.dedent("""
    import ctypes, json, sys
    import numpy as np
    lib = ctypes.CDLL(sys.argv[1])
    rt = ctypes.CDLL("libcudart.so.12")
    V, P = ctypes.c_void_p, ctypes.c_int64
    lib.q6w_linear_argmax.argtypes = [V, V, V, V, V, V, ctypes.c_size_t, P, P, P, V]
    lib.q6w_linear_argmax_noalloc.argtypes = [V, V, V, V, V, P, P, P, V]
    rows, cols, n = 256, 32, 40
    rng = np.random.default_rng(3)
    packed = rng.integers(0, 256, rows * cols * 3 // 4).astype(np.uint8)
    scales = rng.uniform(0.001, 0.05, rows).astype(np.float32)
    x = rng.standard_normal((n, cols)).astype(np.float32)

    def dev(arr):
        p = V()
        assert rt.cudaMalloc(ctypes.byref(p), ctypes.c_size_t(arr.nbytes)) == 0
        assert rt.cudaMemcpy(p, arr.ctypes.data_as(V), ctypes.c_size_t(arr.nbytes), 1) == 0
        return p

    def host(p, shape, dt):
        out = np.empty(shape, dt)
        assert rt.cudaMemcpy(out.ctypes.data_as(V), p, ctypes.c_size_t(out.nbytes), 2) == 0
        return out

    def run():
        pk, sc, xx = dev(packed), dev(scales), dev(x)
        lg0, lg1 = dev(np.zeros((n, rows), np.float32)), dev(np.zeros((n, rows), np.float32))
        am0, am1 = dev(np.zeros(n, np.int32)), dev(np.zeros(n, np.int32))
        scratch = dev(np.zeros(n, np.int64))
        rc0 = lib.q6w_linear_argmax(pk, sc, xx, lg0, am0, scratch, n * 8, rows, cols, n, None)
        rc1 = lib.q6w_linear_argmax_noalloc(pk, sc, xx, lg1, am1, rows, cols, n, None)
        assert rt.cudaDeviceSynchronize() == 0
        a0, a1 = host(am0, n, np.int32), host(am1, n, np.int32)
        l0, l1 = host(lg0, (n, rows), np.float32), host(lg1, (n, rows), np.float32)
        return {"rc": [rc0, rc1], "argmax_equal": bool((a0 == a1).all()),
                "max_logit_diff": float(np.abs(l0 - l1).max()), "argmax_is_logit_max": bool((a1 == l1.argmax(1)).all())}

    first = run()
    reset = rt.cudaDeviceReset()
    second = run()
    print(json.dumps({"first": first, "reset": reset, "second": second}))
""")


def test_no_alloc_after_device_reset():
    """The library-owned array's address is looked up again in a new context."""
    env = dict(os.environ)
    r = subprocess.run([sys.executable, "-c", _RESET_CHILD, str(_lib.LIB_PATH)], capture_output=True, text=True,
                       timeout=300, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["reset"] == 0
    for part in ("first", "second"):
        res = out[part]
        assert res["rc"] == [0, 0], res
        assert res["argmax_equal"] and res["argmax_is_logit_max"], res
        assert res["max_logit_diff"] <= TOL, res
