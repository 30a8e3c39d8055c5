"""Oracle restatement of the Q6W codec (test infrastructure only).

The Q6W format stores signed int6 weights, four values per three bytes, as a
little-endian stream of 6-bit two's-complement fields: value ``i`` of a
3-byte group occupies bits ``6*i .. 6*i+5`` of the 24-bit integer
``b0 | b1 << 8 | b2 << 16``.  This is the bit layout written by the reference
packer ``quantization/q6w_format.py:59-64`` and read back by its unpacker
``quantization/q6w_format.py:73-81``; here it is restated as a 24-bit field
stream rather than per-byte masks.

Each function cites the reference lines whose behaviour it follows.
"""

import hashlib
import json
import math
import struct
from pathlib import Path

import numpy as np
import torch

# quantization/q6w_format.py:11-16
MAGIC = b"TLQ6ROW\0"
VERSION = 1
HEADER = struct.Struct("<8sIIII")
ALIGNMENT = 64
QMIN = -31
QMAX = 31


def pack_int6(values, allow_minus32=False):
    """Pack a [rows, cols] signed-int6 matrix row-major, 4 values -> 3 bytes.

    Follows ``pack_signed_int6`` (quantization/q6w_format.py:52-64), including
    its rejection of values outside [-31, 31].  ``allow_minus32`` widens the
    accepted range to the full 6-bit code space [-32, 31] (code 0x20), which
    the reference unpacker decodes (q6w_format.py:79-80) but its packer never
    emits; the isolated linear sweep draws from that full range.
    """
    q = np.asarray(values, dtype=np.int16)
    if q.ndim != 2 or q.shape[1] % 4:
        raise ValueError("Q6 rows must be 2D and have a width divisible by four")
    lo = -32 if allow_minus32 else QMIN
    if q.size and (q.min() < lo or q.max() > QMAX):
        raise ValueError(f"Q6 values must be in [{lo}, {QMAX}]")
    fields = (q.astype(np.int32) & 0x3F).reshape(q.shape[0], -1, 4)
    stream = fields[..., 0] | (fields[..., 1] << 6) | (fields[..., 2] << 12) | (fields[..., 3] << 18)
    out = np.empty(stream.shape + (3,), dtype=np.uint8)
    out[..., 0] = stream & 0xFF
    out[..., 1] = (stream >> 8) & 0xFF
    out[..., 2] = (stream >> 16) & 0xFF
    return out.tobytes(order="C")


def unpack_int6(data, rows, cols):
    """Decode packed Q6 bytes to an int8 [rows, cols] matrix.

    Follows ``unpack_signed_int6`` (quantization/q6w_format.py:67-81): the same
    length check and error text, 6-bit fields read low-bit-first, and codes
    >= 32 sign-extended (so 0x20 decodes to -32).
    """
    if cols % 4:
        raise ValueError("Q6 row width must be divisible by four")
    expected = rows * cols * 6 // 8
    if len(data) != expected:
        raise ValueError(f"Packed Q6 length mismatch: expected {expected}, got {len(data)}")
    b = np.frombuffer(data, dtype=np.uint8).reshape(rows, cols // 4, 3).astype(np.int32)
    stream = b[..., 0] | (b[..., 1] << 8) | (b[..., 2] << 16)
    fields = np.stack([(stream >> (6 * i)) & 0x3F for i in range(4)], axis=-1)
    signed = np.where(fields >= 32, fields - 64, fields).astype(np.int8)
    return signed.reshape(rows, cols)


def quantize_rows(tensor):
    """Symmetric per-output-row int6 quantization.

    Follows ``quantize_rows`` (quantization/q6w_format.py:84-98): scale =
    max|row| / 31 (1.0 for an all-zero row), q = clamp(round_half_even(w /
    scale), -31, 31), computed with torch FP32 CPU ops.
    Returns (q int8 numpy [rows, cols], scales little-endian f32 numpy [rows]).
    """
    w = tensor.detach().to(device="cpu", dtype=torch.float32).contiguous()
    if w.ndim != 2:
        raise ValueError("Per-output-row quantization requires a matrix")
    peak = w.abs().amax(dim=1)
    scale = torch.where(peak > 0, peak / QMAX, torch.ones_like(peak))
    q = torch.round(w / scale[:, None]).clamp(QMIN, QMAX).to(torch.int8)
    return q.numpy(), scale.numpy().astype("<f4", copy=False)


def dequantize(q, scales):
    """``float32(q) * scale[row]`` -- one rounded FP32 product per element.

    Follows quantization/q6w_format.py:257-259.
    """
    return np.asarray(q).astype(np.float32) * np.asarray(scales, dtype="<f4")[:, None]


def sha256_file(path):
    """quantization/q6w_format.py:44-49."""
    h = hashlib.sha256()
    with Path(path).open("rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def load_state(binary_path, manifest_path):
    """Read a Q6W binary + manifest into a dict of FP32 CPU tensors.

    Follows ``load_dequantized_state`` (quantization/q6w_format.py:230-268):
    SHA-256 check against the manifest, header check, per-entry unpack and
    dequantization driven by the manifest offsets, FP32 norm vectors read raw,
    and ``output.weight`` aliased to ``tok_embeddings.weight``.  Unlike the
    reference it needs no template checkpoint: every tensor comes from the
    file.  Returns (state, manifest).
    """
    binary_path = Path(binary_path)
    manifest = json.loads(Path(manifest_path).read_text(encoding="utf-8"))
    if sha256_file(binary_path) != manifest["binary_sha256"]:
        raise ValueError("Q6 binary SHA-256 does not match its manifest")
    blob = binary_path.read_bytes()
    head = HEADER.unpack(blob[: HEADER.size])
    if head != (MAGIC, VERSION, manifest["tensor_count"], 6, 1):
        raise ValueError("Q6 binary header does not match the supported format")
    state = {}
    for entry in manifest["tensors"]:
        shape = tuple(entry["shape"])
        lo, n = entry["data_offset"], entry["data_bytes"]
        data = blob[lo : lo + n]
        if len(data) != n:
            raise ValueError(f"Truncated Q6 data for {entry['name']}")
        if entry["dtype"] == "signed_int6_twos_complement":
            rows, cols = shape
            s_lo, s_n = entry["scale_offset"], entry["scale_bytes"]
            scales = np.frombuffer(blob[s_lo : s_lo + s_n], dtype="<f4")
            if len(scales) != rows or s_n != rows * 4:
                raise ValueError(f"Invalid scale array for {entry['name']}")
            w = dequantize(unpack_int6(data, rows, cols), scales)
            state[entry["name"]] = torch.from_numpy(np.ascontiguousarray(w))
        elif entry["dtype"] == "little_endian_float32":
            v = np.frombuffer(data, dtype="<f4")
            if v.size != math.prod(shape):
                raise ValueError(f"Invalid FP32 tensor size for {entry['name']}")
            state[entry["name"]] = torch.from_numpy(v.copy().reshape(shape))
        else:
            raise ValueError(f"Unsupported tensor dtype {entry['dtype']}")
    state["output.weight"] = state["tok_embeddings.weight"]
    return state, manifest
