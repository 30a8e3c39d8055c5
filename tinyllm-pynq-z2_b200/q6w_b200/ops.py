"""Device codec and linear ops over the C ABI (torch tensors as plumbing).

These mirror the reference's codec functions (quantization/q6w_format.py)
with the work done by the sm_100a kernels: same names, same argument
meaning, same ValueError messages for malformed input.  Results are CUDA
tensors on ``device``.
"""

import json
import math
from pathlib import Path

import numpy as np
import torch

from . import _lib
from .format import HEADER, MAGIC, VERSION, Q6WImage


def _dev(device):
    d = torch.device(device)
    if d.type != "cuda":
        raise ValueError("q6w_b200 ops run on CUDA devices only")
    return d


def _bytes_to_device(data, device):
    buf = torch.frombuffer(bytearray(data), dtype=torch.uint8) if len(data) else torch.empty(0, dtype=torch.uint8)
    return buf.to(device, non_blocking=False)


def unpack_signed_int6(data, rows, columns, device="cuda"):
    """Decode packed Q6 bytes to int8 codes [rows, columns] on the GPU.

    Same contract as quantization/q6w_format.py:67-81 (the result is a CUDA
    int8 tensor instead of a numpy array).  ``data`` is bytes-like or a
    CUDA uint8 tensor.
    """
    if columns % 4:
        raise ValueError("Q6 row width must be divisible by four")
    expected = rows * columns * 6 // 8
    device = _dev(device)
    packed = data if isinstance(data, torch.Tensor) else _bytes_to_device(data, device)
    if packed.numel() != expected:
        raise ValueError(f"Packed Q6 length mismatch: expected {expected}, got {packed.numel()}")
    out = torch.empty((rows, columns), dtype=torch.int8, device=device)
    lib = _lib.load()
    with torch.cuda.device(device):
        _lib.check(lib.q6w_unpack(packed.data_ptr(), out.data_ptr(), rows, columns, _lib.stream_handle()), "q6w_unpack")
    return out


def dequantize_rows(packed, scales, rows, columns):
    """``float32(q) * scale[row]`` on the GPU (quantization/q6w_format.py:257-259)."""
    out = torch.empty((rows, columns), dtype=torch.float32, device=packed.device)
    lib = _lib.load()
    with torch.cuda.device(packed.device):
        _lib.check(lib.q6w_dequant(packed.data_ptr(), scales.data_ptr(), out.data_ptr(), rows, columns,
                                   _lib.stream_handle()), "q6w_dequant")
    return out


def quantize_rows(tensor, device="cuda"):
    """Row-wise int6 quantization + packing on the GPU: the device half of the
    Q6W writer (quantization/q6w_format.py:84-98 and 52-64).

    Codes and scales are bit-identical to the reference's ``quantize_rows``
    (same FP32 division and round-half-even); the codes come back already
    packed.  Returns (packed uint8 [rows*cols*3/4], scales float32 [rows],
    stats dict) with packed/scales on ``device``; the stats are summed in
    FP64 and agree with the reference's FP32 reductions to their rounding.
    """
    device = _dev(device)
    w = tensor.detach().to(device=device, dtype=torch.float32).contiguous()
    if w.ndim != 2:
        raise ValueError("Per-output-row quantization requires a matrix")
    rows, cols = w.shape
    if cols % 4:
        raise ValueError("Q6 rows must be 2D and have a width divisible by four")
    packed = torch.empty(rows * cols * 3 // 4, dtype=torch.uint8, device=device)
    scales = torch.empty(rows, dtype=torch.float32, device=device)
    row_err = torch.empty((max(rows, 1), 3), dtype=torch.float64, device=device)
    stats = torch.zeros(3, dtype=torch.float64, device=device)
    lib = _lib.load()
    with torch.cuda.device(device):
        _lib.check(lib.q6w_quantize_rows(w.data_ptr(), rows, cols, packed.data_ptr(), scales.data_ptr(),
                                         row_err.data_ptr(), stats.data_ptr(), _lib.stream_handle()),
                   "q6w_quantize_rows")
    st = stats.tolist()
    return packed, scales, {"max_abs_error": st[0], "mean_abs_error": st[1], "rmse": st[2]}


_LINEAR_WS = {}  # device index -> cached workspace of the tensor-core linear


def _linear_workspace(device, nbytes):
    buf = _LINEAR_WS.get(device.index)
    if buf is None or buf.numel() < nbytes:
        raw = torch.zeros(nbytes + 256, dtype=torch.uint8, device=device)
        off = (-raw.data_ptr()) % 256
        buf = raw[off: off + nbytes]
        _LINEAR_WS[device.index] = buf
    return buf


def linear_workspace_bytes(rows, columns, n):
    """Workspace the tensor-core linear needs for this shape (0: FP32 kernels)."""
    return int(_lib.load().q6w_linear_workspace_bytes(rows, columns, n))


def q6w_linear(x, packed, scales, rows, columns, tensor_cores=True):
    """``x @ dequant(W).T`` for x [..., columns] FP32 on the GPU -> [..., rows].

    The ``nn.Linear`` of the cached step (torch_benchmark.py:105-107, 121,
    123, 125).  Batches of 16 or more rows whose width is a multiple of 128
    run on the tcgen05 tensor cores (q6w_linear_ex, a cached workspace per
    device; agreement with FP64 within 1e-4 * sum|w x| per element); other
    shapes, and ``tensor_cores=False``, run the FP32 kernels (1e-5).
    """
    if x.dtype != torch.float32 or x.shape[-1] != columns:
        raise ValueError("x must be float32 with last dimension == columns")
    xs = x.reshape(-1, columns).contiguous()
    n = xs.shape[0]
    y = torch.empty((n, rows), dtype=torch.float32, device=x.device)
    lib = _lib.load()
    need = linear_workspace_bytes(rows, columns, n) if tensor_cores else 0
    with torch.cuda.device(x.device):
        if need:
            ws = _linear_workspace(x.device, need)
            _lib.check(lib.q6w_linear_ex(packed.data_ptr(), scales.data_ptr(), xs.data_ptr(), y.data_ptr(), rows,
                                         columns, n, ws.data_ptr(), ws.numel(), _lib.stream_handle()),
                       "q6w_linear_ex")
        else:
            _lib.check(lib.q6w_linear(packed.data_ptr(), scales.data_ptr(), xs.data_ptr(), y.data_ptr(), rows,
                                      columns, n, _lib.stream_handle()), "q6w_linear")
    return y.reshape(*x.shape[:-1], rows)


class DeviceImage:
    """A verified Q6W file uploaded unchanged to one GPU.

    The device blob is the file's bytes (64-byte aligned sections, the
    allocation itself 256-byte aligned), so every tensor is addressed in
    place: ``qmat(name)`` returns (packed view, scales view, rows, cols).
    """

    def __init__(self, image, device):
        self.image = image
        self.device = _dev(device)
        self.blob = _bytes_to_device(image.blob, self.device)

    def _view(self, offset, nbytes):
        return self.blob[offset: offset + nbytes]

    def qmat(self, name):
        e = self.image.tensors[name]
        rows, cols = e["shape"]
        packed = self._view(e["data_offset"], e["data_bytes"])
        scales = self._view(e["scale_offset"], e["scale_bytes"]).view(torch.float32)
        return packed, scales, rows, cols

    def fp32(self, name):
        e = self.image.tensors[name]
        return self._view(e["data_offset"], e["data_bytes"]).view(torch.float32).view(*e["shape"])


def load_dequantized_state(binary_path, manifest_path, checkpoint_state=None, device="cuda"):
    """Q6W file -> dict of dequantized FP32 CUDA tensors, plus the manifest.

    Same checks and result keys as quantization/q6w_format.py:230-268 (SHA,
    header, offsets; ``output.weight`` aliases ``tok_embeddings.weight``), with
    the unpack and dequantization done on the GPU.  ``checkpoint_state``, when
    given, supplies extra non-file tensors and is copied to ``device``.
    """
    image = Q6WImage(binary_path, manifest_path)
    dimg = DeviceImage(image, device)
    result = {}
    if checkpoint_state:
        result = {k: v.detach().to(device=dimg.device, dtype=torch.float32).clone() for k, v in checkpoint_state.items()}
    for name, e in image.tensors.items():
        if e["dtype"] == "signed_int6_twos_complement":
            packed, scales, rows, cols = dimg.qmat(name)
            result[name] = dequantize_rows(packed, scales, rows, cols)
        else:
            result[name] = dimg.fp32(name).clone()
    result["output.weight"] = result["tok_embeddings.weight"]
    return result, image.manifest


def linear_argmax(x, packed, scales, rows, columns, want_logits=False):
    """Fused ``x @ dequant(W).T`` + first-maximum argmax per row.

    Returns (argmax int32 [n], logits [n, rows] or None).
    """
    xs = x.reshape(-1, columns).contiguous()
    n = xs.shape[0]
    am = torch.empty(n, dtype=torch.int32, device=x.device)
    lg = torch.empty((n, rows), dtype=torch.float32, device=x.device) if want_logits else None
    scratch = torch.empty(max(1, n), dtype=torch.int64, device=x.device)
    lib = _lib.load()
    with torch.cuda.device(x.device):
        _lib.check(lib.q6w_linear_argmax(packed.data_ptr(), scales.data_ptr(), xs.data_ptr(),
                                         lg.data_ptr() if lg is not None else None, am.data_ptr(),
                                         scratch.data_ptr(), scratch.numel() * 8, rows, columns, n,
                                         _lib.stream_handle()), "q6w_linear_argmax")
    return am, lg


def sample(logits, history, history_len, rng_state, temperature, top_p=0.9, repetition_penalty=1.0,
           no_repeat_ngram_size=0, stop_ids=(), min_new_tokens=0, stop_token_bias=0.0, stop_token_bias_after=None):
    """The reference's per-step sampling (torch_benchmark.py:272-285) on rows
    of logits, on the GPU: repetition penalty and n-gram blocking over each
    row's ``history`` (its first ``history_len`` tokens; history_len is also
    the decode index), stop-id masking / bias, then temperature / top-p
    sampling from each row's XorShift64 state.

    logits [n, V] float32; history [n, H] int32; history_len [n] int32;
    rng_state [n] int64 (the generator states, advanced in place).  Returns
    int32 tokens [n].
    """
    n, V = logits.shape
    lg = logits.contiguous()
    hist = history.to(torch.int32).contiguous()
    hl = history_len.to(torch.int32).contiguous()
    if rng_state.dtype != torch.int64 or not rng_state.is_contiguous():
        raise ValueError("rng_state must be a contiguous int64 tensor")
    out = torch.empty(n, dtype=torch.int32, device=logits.device)
    stop = sorted(set(int(t) for t in stop_ids))
    arr = (_lib.c_int32 * max(1, len(stop)))(*stop) if stop else None
    bias_after = min_new_tokens if stop_token_bias_after is None else stop_token_bias_after
    sa = _lib.SampleArgs(float(temperature), float(top_p), float(repetition_penalty), int(no_repeat_ngram_size),
                         float(stop_token_bias), int(bias_after), None)
    lib = _lib.load()
    with torch.cuda.device(logits.device):
        _lib.check(lib.q6w_sample(lg.data_ptr(), V, n, V, hist.data_ptr() if hist.numel() else None,
                                  hist.shape[1] if hist.dim() == 2 else 0, hl.data_ptr(), rng_state.data_ptr(), sa,
                                  arr, len(stop), int(min_new_tokens), out.data_ptr(), _lib.stream_handle()),
                   "q6w_sample")
    return out


def rmsnorm(x, weight, eps):
    """Row-wise RMSNorm of x [..., length] (torch_benchmark.py:22-24)."""
    xs = x.reshape(-1, x.shape[-1]).contiguous()
    out = torch.empty_like(xs)
    lib = _lib.load()
    with torch.cuda.device(x.device):
        _lib.check(lib.q6w_rmsnorm(xs.data_ptr(), weight.data_ptr(), out.data_ptr(), xs.shape[0], xs.shape[1],
                                   float(eps), _lib.stream_handle()), "q6w_rmsnorm")
    return out.view_as(x)


def gqa_attention(queries, keys, values, lengths, groups_per_kv):
    """Decode attention over per-sequence caches.

    queries [n, heads, hd]; keys/values [n, max_len, kv_heads, hd] (any
    sequence stride); lengths int32 [n] on the device.  Returns [n, heads, hd].
    """
    n, H, hd = queries.shape
    _, max_len, kv, _ = keys.shape
    q = queries.contiguous()
    out = torch.empty_like(q)
    if keys.stride()[1:] != (kv * hd, hd, 1) or values.stride() != keys.stride():
        raise ValueError("keys/values must be [n, max_len, kv_heads, head_dim] with contiguous rows")
    lib = _lib.load()
    with torch.cuda.device(q.device):
        _lib.check(lib.q6w_gqa_attention(q.data_ptr(), keys.data_ptr(), values.data_ptr(), out.data_ptr(),
                                         lengths.to(torch.int32).contiguous().data_ptr(), n, kv, groups_per_kv, hd,
                                         max_len, keys.stride(0), _lib.stream_handle()), "q6w_gqa_attention")
    return out
