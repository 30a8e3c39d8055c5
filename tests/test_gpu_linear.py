"""GPU: the Q6W linear (isolated sweep on the tiny model's shapes) against an
FP64 dequant-then-matmul reference and torch FP32.

Tolerance (FP32 path): |y - y64| <= 1e-5 * sum_k |w_k x_k| + 1e-30 per
element, i.e. FP32 summation error relative to the magnitude of the terms.
Batches of 16+ rows at widths that are multiples of 128 run on the tcgen05
tensor cores (three bf16 parts of x, exact products, FP32 accumulation in
tensor memory in the tensor core's order): the stated, looser tolerance
there is 1e-4 * sum_k |w_k x_k| per element, plus a relative RMS error
below 1e-5 over the whole output.
"""

import numpy as np
import pytest
import torch

from oracle import codec
from q6w_b200 import ops

pytestmark = pytest.mark.gpu

SHAPES = [(128, 128), (64, 128), (384, 128), (128, 384), (4096, 128)]
BATCHES = [1, 8, 64, 512, 4096]
REL = 1e-5
REL_TC = 1e-4
RMS_TC = 1e-5


def make(rows, cols, n, seed):
    rng = np.random.default_rng(seed)
    q = rng.integers(-32, 32, size=(rows, cols))
    s = rng.uniform(0.001, 0.05, size=rows).astype(np.float32)
    x = rng.standard_normal((n, cols)).astype(np.float32)
    packed = torch.frombuffer(bytearray(codec.pack_int6(q, allow_minus32=True)), dtype=torch.uint8).cuda()
    return q, s, x, packed


def check(y, q, s, x, rel=REL, rms=None):
    w = codec.dequantize(q, s).astype(np.float64)
    y64 = x.astype(np.float64) @ w.T
    mag = np.abs(x.astype(np.float64)) @ np.abs(w).T
    err = np.abs(y.astype(np.float64) - y64)
    assert (err <= rel * mag + 1e-30).all(), float((err / (mag + 1e-30)).max())
    if rms is not None:
        assert np.sqrt((err ** 2).mean() / max((y64 ** 2).mean(), 1e-300)) <= rms
    return float((err / (mag + 1e-30)).max())


def uses_tensor_cores(rows, cols, n):
    return ops.linear_workspace_bytes(rows, cols, n) > 0


@pytest.mark.parametrize("rows,cols", SHAPES)
@pytest.mark.parametrize("n", BATCHES)
def test_linear_sweep(rows, cols, n):
    """The public op on every sweep point: FP32 kernels for n <= 8, tensor cores for n >= 64."""
    q, s, x, packed = make(rows, cols, n, rows * 7 + cols * 3 + n)
    tc = uses_tensor_cores(rows, cols, n)
    assert tc == (n >= 64)
    y = ops.q6w_linear(torch.from_numpy(x).cuda(), packed, torch.from_numpy(s).cuda(), rows, cols)
    torch.cuda.synchronize()
    y = y.cpu().numpy()
    check(y, q, s, x, REL_TC if tc else REL, RMS_TC if tc else None)
    # against torch's own FP32 matmul, whose rounding is of the same order as ours:
    # 2e-5 of sum |w x| per element (torch alone sits ~1e-6 of it from FP64)
    w32 = torch.from_numpy(codec.dequantize(q, s))
    ref32 = (torch.from_numpy(x) @ w32.T).numpy()
    mag = (torch.from_numpy(np.abs(x)) @ w32.abs().T).numpy()
    assert (np.abs(y - ref32) <= 2e-5 * mag + 1e-30).all()


@pytest.mark.parametrize("rows,cols", SHAPES)
@pytest.mark.parametrize("n", [64, 512])
def test_linear_sweep_fp32_kernels(rows, cols, n):
    """The FP32 SIMT GEMM on the batched sweep points (tensor cores off) keeps the FP32 tolerance."""
    q, s, x, packed = make(rows, cols, n, rows * 5 + cols + n)
    y = ops.q6w_linear(torch.from_numpy(x).cuda(), packed, torch.from_numpy(s).cuda(), rows, cols,
                       tensor_cores=False).cpu().numpy()
    check(y, q, s, x)


@pytest.mark.parametrize("rows,cols,n", [(64, 256, 16), (200, 128, 17), (130, 1024, 100), (2048, 5632, 64),
                                         (256, 2048, 300), (32000, 2048, 64), (6, 128, 1000)])
def test_linear_tensor_core_shapes(rows, cols, n):
    """tcgen05 linear on partial weight tiles (rows not a multiple of 128),
    partial activation tiles, long K (split across clusters) and the
    1.1B-shape matrices, against FP64."""
    assert uses_tensor_cores(rows, cols, n)
    q, s, x, packed = make(rows, cols, n, rows + 3 * cols + 7 * n)
    y = ops.q6w_linear(torch.from_numpy(x).cuda(), packed, torch.from_numpy(s).cuda(), rows, cols).cpu().numpy()
    worst = check(y, q, s, x, REL_TC, RMS_TC)
    print(f"tensor-core linear {rows}x{cols} n={n}: max |err| / sum|w x| = {worst:.2e}")


# One activation row at K a multiple of 512 takes the HBM-streaming kernel
# (bulk-copied tiles, factored row scale, 2^-p pre-scaled inputs): the
# 1.1B-shape matrices and the extremes of its warp layout (K 512 / 4096).
STREAM_SHAPES = [(2048, 2048), (256, 2048), (5632, 2048), (2048, 5632), (512, 512), (1024, 4096), (6016, 2048)]


@pytest.mark.parametrize("rows,cols", STREAM_SHAPES)
def test_linear_stream_one_row(rows, cols):
    q, s, x, packed = make(rows, cols, 1, rows + 5 * cols)
    y = ops.q6w_linear(torch.from_numpy(x).cuda(), packed, torch.from_numpy(s).cuda(), rows, cols).cpu().numpy()
    check(y, q, s, x)


def test_linear_stream_argmax():
    q, s, x, packed = make(4096, 2048, 1, 4242)
    am, lg = ops.linear_argmax(torch.from_numpy(x).cuda(), packed, torch.from_numpy(s).cuda(), 4096, 2048, True)
    lg = lg.cpu().numpy()
    check(lg, q, s, x)
    assert np.array_equal(am.cpu().numpy(), lg.argmax(axis=1))


@pytest.mark.parametrize("rows,cols,n", [(63, 128, 3), (6, 20, 9), (10, 36, 1), (2, 4, 1), (4096, 128, 2)])
def test_linear_general_shapes(rows, cols, n):
    q, s, x, packed = make(rows, cols, n, 11 + rows + cols + n)
    y = ops.q6w_linear(torch.from_numpy(x).cuda(), packed, torch.from_numpy(s).cuda(), rows, cols).cpu().numpy()
    check(y, q, s, x)


def test_linear_unaligned_x_uses_general_path():
    q, s, x, packed = make(64, 128, 4, 5)
    buf = torch.zeros(4 * 128 + 1, device="cuda")
    xv = buf[1:].view(4, 128)
    xv.copy_(torch.from_numpy(x))
    y = ops.q6w_linear(xv, packed, torch.from_numpy(s).cuda(), 64, 128).cpu().numpy()
    check(y, q, s, x)


@pytest.mark.parametrize("rows,cols,n", [(4096, 128, 1), (4096, 128, 3), (4096, 128, 300), (32000, 256, 2)])
def test_linear_argmax(rows, cols, n):
    q, s, x, packed = make(rows, cols, n, 99 + n)
    am, lg = ops.linear_argmax(torch.from_numpy(x).cuda(), packed, torch.from_numpy(s).cuda(), rows, cols, True)
    lg = lg.cpu().numpy()
    check(lg, q, s, x)
    assert np.array_equal(am.cpu().numpy(), lg.argmax(axis=1))  # first maximum of the device logits


def test_linear_argmax_ties_pick_first():
    rows, cols = 64, 16
    q = np.zeros((rows, cols), dtype=np.int64)
    q[[5, 9, 40], 0] = 7  # three equal maxima
    s = np.full(rows, 0.01, dtype=np.float32)
    packed = torch.frombuffer(bytearray(codec.pack_int6(q)), dtype=torch.uint8).cuda()
    x = torch.zeros(2, cols, device="cuda")
    x[:, 0] = 1.0
    am, _ = ops.linear_argmax(x, packed, torch.from_numpy(s).cuda(), rows, cols)
    assert am.cpu().tolist() == [5, 5]


def test_rmsnorm_matches_reference_formula():
    torch.manual_seed(0)
    x = torch.randn(37, 128)
    w = torch.rand(128) + 0.5
    got = ops.rmsnorm(x.cuda(), w.cuda(), 1e-5).cpu()
    want = (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-5)) * w
    assert (got - want).abs().max() <= 2e-6
