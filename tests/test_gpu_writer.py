"""GPU: the Q6W writer's quantization + packing on the device
(q6w_quantize_rows), against the reference and the host writer.

Bit-exact: codes, packed bytes and scales equal the reference's
``quantize_rows`` + ``pack_signed_int6`` (quantization/q6w_format.py:52-98)
on the recorded golden matrix (all-zero row, exact .5 ties), equal the host
writer's on larger seeded matrices, and a tiny synthetic model written with
the device quantizer has the SHA-256 the reference-loaded golden model has.
The error statistics (FP64 sums here, FP32 torch reductions there) agree to
a relative 1e-5.
"""

import hashlib

import numpy as np
import pytest
import torch

from q6w_b200 import format as fmt
from q6w_b200 import ops

pytestmark = pytest.mark.gpu


def _stats_close(a, b):
    for k in ("max_abs_error", "mean_abs_error", "rmse"):
        assert abs(a[k] - b[k]) <= 1e-5 * max(abs(b[k]), 1e-30), (k, a[k], b[k])


def test_device_quantizer_matches_reference_golden(golden_codec):
    case = golden_codec["quantize"][0]
    w = torch.tensor(case["weights"], dtype=torch.float32)
    packed, scales, stats = ops.quantize_rows(w)
    want_q = np.array(case["q"], dtype=np.int64)
    assert packed.cpu().numpy().tobytes() == fmt.pack_signed_int6(want_q)
    got_s = scales.cpu().numpy().astype(np.float32)
    assert np.array_equal(got_s.view(np.uint32), np.array(case["scales"], dtype=np.float32).view(np.uint32))
    _stats_close(stats, case["stats"])


@pytest.mark.parametrize("rows,cols,seed", [(384, 128, 1), (1000, 352, 2), (3, 4, 3), (2048, 5632, 4)])
def test_device_quantizer_matches_host_writer(rows, cols, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.empty(rows, cols).normal_(0.0, 0.02, generator=g)
    w[0] = 0.0                                   # all-zero row: scale 1.0
    if rows > 2:
        w[1, :4] = torch.tensor([0.5, -0.5, 1.5, 31.0]) * (w[1].abs().max() / 31.0)  # ties after the scale
    packed, scales, stats = ops.quantize_rows(w)
    q, s, st = fmt.quantize_rows(w)
    assert packed.cpu().numpy().tobytes() == fmt.pack_signed_int6(q)
    assert np.array_equal(scales.cpu().numpy().view(np.uint32), s.view(np.uint32))
    _stats_close(stats, st)


def test_device_writer_reproduces_golden_tiny_binary(tmp_path, golden_tiny):
    b, m = tmp_path / "tiny.bin", tmp_path / "tiny.json"
    man = fmt.write_synthetic(fmt.TINY_ARGS, golden_tiny["seed"], b, m, device="cuda")
    assert hashlib.sha256(b.read_bytes()).hexdigest() == golden_tiny["binary_sha256"]
    assert man["binary_sha256"] == golden_tiny["binary_sha256"]
    fmt.Q6WImage(b, m)  # header + SHA + offsets check of the loader


def test_device_quantizer_rejects_bad_width():
    with pytest.raises(ValueError, match="divisible by four"):
        ops.quantize_rows(torch.zeros(2, 6))
