"""GPU: failure detection without a GPU fault.  A device-side wait that
nothing completes must end after its bound with an error status the host
reads, and leave the context usable (the bounded waits of the tensor-core
and streaming pipelines all go through the routine exercised here)."""

import time

import numpy as np
import pytest
import torch

from oracle import codec
from q6w_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_reports():
    lib = _lib.load()
    ws = torch.zeros(64, dtype=torch.int32, device="cuda")
    h = _lib.stream_handle()
    t0 = time.perf_counter()
    _lib.check(lib.q6w_selftest_wait_timeout(ws.data_ptr(), 4_000_000, h))  # ~2 ms of SM clock
    rc = lib.q6w_workspace_status(ws.data_ptr(), h)  # synchronises
    elapsed = time.perf_counter() - t0
    assert rc == _lib.Q6W_ERR_DEVICE
    assert b"ran out of time" in lib.q6w_last_error()
    assert elapsed < 5.0
    # the status was cleared, and the context still runs kernels correctly
    assert lib.q6w_workspace_status(ws.data_ptr(), h) == _lib.Q6W_OK
    rng = np.random.default_rng(1)
    q = rng.integers(-32, 32, size=(8, 64))
    s = rng.uniform(0.01, 0.05, size=8).astype(np.float32)
    packed = torch.frombuffer(bytearray(codec.pack_int6(q, allow_minus32=True)), dtype=torch.uint8).cuda()
    got = ops.dequantize_rows(packed, torch.from_numpy(s).cuda(), 8, 64).cpu().numpy()
    assert np.array_equal(got, codec.dequantize(q, s))


def test_bounded_wait_argument_checks():
    lib = _lib.load()
    ws = torch.zeros(4, dtype=torch.int32, device="cuda")
    assert lib.q6w_selftest_wait_timeout(ws.data_ptr(), 0, _lib.stream_handle()) == _lib.Q6W_ERR_ARG
    assert lib.q6w_selftest_wait_timeout(None, 100, _lib.stream_handle()) == _lib.Q6W_ERR_ARG
