"""Q6W file format: reader, writer and synthetic-model generator (host side).

The byte layout is the reference's ``TinyLLMStory-zh Q6W rowwise v1`` format
(quantization/q6w_format.py:11-16, 101-227): a 24-byte ``<8sIIII`` header,
then 64-byte-aligned sections -- for every quantized tensor its row scales
(little-endian f32) followed by its packed signed-int6 rows, then the FP32
norm vectors -- described by a JSON manifest carrying offsets, shapes and the
binary's SHA-256.  The layout is kept byte-identical because it is the
drop-in contract: files written here load in the reference and vice versa.

Differences from the reference, all additive:

* tensor names are generated for any ``n_layers`` (the reference hard-codes
  five layers at q6w_format.py:17-37);
* ``write_q6w`` takes an in-memory state dict (the reference exporter needs a
  checkpoint file, q6w_format.py:108-121);
* ``pack_signed_int6(..., allow_minus32=True)`` accepts the full 6-bit code
  space for synthetic linear tests; model weights never reach -32.

Nothing here touches the GPU; decoding and dequantization on the device are
in ``q6w_b200.ops``.
"""

import hashlib
import json
import struct
from pathlib import Path

import numpy as np
import torch

MAGIC = b"TLQ6ROW\0"
VERSION = 1
HEADER = struct.Struct("<8sIIII")
ALIGNMENT = 64
QMIN = -31
QMAX = 31
FORMAT_NAME = "TinyLLMStory-zh Q6W rowwise v1"

LAYER_QUANT = ("attention.wq", "attention.wk", "attention.wv", "attention.wo",
               "feed_forward.w1", "feed_forward.w2", "feed_forward.w3")
LAYER_NORMS = ("attention_norm", "ffn_norm")


def quant_keys(n_layers):
    """Quantized tensor names in file order (q6w_format.py:17-30 for n_layers=5)."""
    keys = ["tok_embeddings.weight"]
    for l in range(n_layers):
        keys += [f"layers.{l}.{name}.weight" for name in LAYER_QUANT]
    return keys


def norm_keys(n_layers):
    """FP32 norm tensor names in file order (q6w_format.py:31-37 for n_layers=5)."""
    keys = []
    for l in range(n_layers):
        keys += [f"layers.{l}.{name}.weight" for name in LAYER_NORMS]
    return keys + ["norm.weight"]


QUANT_KEYS = quant_keys(5)
NORM_KEYS = norm_keys(5)


def align_up(value, alignment=ALIGNMENT):
    return (value + alignment - 1) // alignment * alignment


def sha256_file(path):
    digest = hashlib.sha256()
    with Path(path).open("rb") as f:
        for block in iter(lambda: f.read(1 << 22), b""):
            digest.update(block)
    return digest.hexdigest()


def pack_signed_int6(values, allow_minus32=False):
    """Pack a [rows, cols] int matrix as Q6W rows (4 six-bit fields per 3 bytes).

    Same contract as the reference packer (q6w_format.py:52-64): 2-D input,
    width divisible by four, values in [-31, 31] (or [-32, 31] with
    ``allow_minus32``), ValueError otherwise.
    """
    q = np.asarray(values)
    if q.ndim != 2 or q.shape[1] % 4:
        raise ValueError("Q6 rows must be 2D and have a width divisible by four")
    lo = -32 if allow_minus32 else QMIN
    if q.size and (int(q.min()) < lo or int(q.max()) > QMAX):
        raise ValueError(f"Q6 values must be in [{lo}, {QMAX}]")
    if q.size == 0:
        return b""
    u = (q.astype(np.int32) & 0x3F).reshape(q.shape[0], -1, 4)
    word = u[..., 0] | (u[..., 1] << 6) | (u[..., 2] << 12) | (u[..., 3] << 18)
    return word.astype("<u4").view(np.uint8).reshape(word.shape + (4,))[..., :3].tobytes()


def quantize_rows(tensor):
    """Row-wise symmetric int6 quantization (q6w_format.py:84-98 semantics).

    scale = max|row| / 31 in FP32 (1.0 for an all-zero row); q =
    clamp(round-half-even(w / scale), -31, 31).  Returns (q int8 ndarray,
    scales '<f4' ndarray, error stats dict).
    """
    w = tensor.detach().to(device="cpu", dtype=torch.float32).contiguous()
    if w.ndim != 2:
        raise ValueError("Per-output-row quantization requires a matrix")
    peak = w.abs().amax(dim=1)
    scales = torch.where(peak > 0, peak / QMAX, torch.ones_like(peak))
    q = torch.round(w / scales[:, None]).clamp(QMIN, QMAX).to(torch.int8)
    err = q.float() * scales[:, None] - w
    stats = {
        "max_abs_error": float(err.abs().max()),
        "mean_abs_error": float(err.abs().mean()),
        "rmse": float(err.square().mean().sqrt()),
    }
    return q.numpy(), scales.numpy().astype("<f4", copy=False), stats


def _model_shapes(args):
    dim, hd = args["dim"], args["dim"] // args["n_heads"]
    kv = (args.get("n_kv_heads") or args["n_heads"]) * hd
    hidden = ffn_dim(args)
    per_layer = {
        "attention.wq": (dim, dim), "attention.wk": (kv, dim), "attention.wv": (kv, dim),
        "attention.wo": (dim, dim), "feed_forward.w1": (hidden, dim),
        "feed_forward.w2": (dim, hidden), "feed_forward.w3": (hidden, dim),
    }
    shapes = {"tok_embeddings.weight": (args["vocab_size"], dim)}
    for l in range(args["n_layers"]):
        for name, shp in per_layer.items():
            shapes[f"layers.{l}.{name}.weight"] = shp
    for key in norm_keys(args["n_layers"]):
        shapes[key] = (dim,)
    return shapes


def ffn_dim(args):
    """SwiGLU width: explicit ``hidden_dim`` or the rule of torch_benchmark.py:61-64."""
    if args.get("hidden_dim") is not None:
        return int(args["hidden_dim"])
    multiple = args.get("multiple_of", 256)
    h = int(2 * (4 * args["dim"]) / 3)
    return multiple * ((h + multiple - 1) // multiple)


def _quantize_on_device(t, device):
    """GPU quantize + pack of one matrix, with the writer's self-check done on
    the device: every code dequantizes to within half a scale step of its
    weight (the round-trip check of the host path, without a host unpack).
    The bound allows the FP32 roundings of w / scale (ratios up to 31, so up
    to 31 * 2^-24 of a step) and of q * scale."""
    from . import ops

    w = t.detach().to(device=device, dtype=torch.float32).contiguous()
    packed, scales, stats = ops.quantize_rows(w, device)
    rows, cols = w.shape
    deq = ops.dequantize_rows(packed, scales, rows, cols)
    if not bool(((deq - w).abs() <= scales[:, None] * (0.5 + 1e-5)).all()):
        raise AssertionError("Q6 device quantization self-check failed")
    return packed.cpu().numpy().tobytes(), scales.cpu().numpy().astype("<f4", copy=False), stats


def write_q6w(state, model_args, output_path, manifest_path, provenance=None, overwrite=False, device=None):
    """Write ``state`` (FP32 tensors by name) as a Q6W binary + manifest.

    Section order, alignment, header and manifest schema follow
    ``export_q6w`` (q6w_format.py:134-227).  Every quantized tensor is
    round-trip checked after packing.  With ``device`` a CUDA device, the
    quantization and packing run on that GPU (``ops.quantize_rows``: same
    codes, scales and bytes; error statistics summed in FP64).  Returns the
    manifest dict.
    """
    output_path, manifest_path = Path(output_path), Path(manifest_path)
    if not overwrite and (output_path.exists() or manifest_path.exists()):
        raise FileExistsError("Refusing to overwrite an existing Q6 artifact or manifest")
    n_layers = int(model_args["n_layers"])
    qkeys, nkeys = quant_keys(n_layers), norm_keys(n_layers)
    shapes = _model_shapes(model_args)
    missing = [k for k in qkeys + nkeys if k not in state]
    if missing:
        raise ValueError(f"State is missing tensors: {missing[:4]}")
    output_path.parent.mkdir(parents=True, exist_ok=True)
    entries = []
    with output_path.open("wb") as out:
        out.write(HEADER.pack(MAGIC, VERSION, len(qkeys) + len(nkeys), 6, 1))

        def put(data):
            out.write(b"\0" * (align_up(out.tell()) - out.tell()))
            off = out.tell()
            out.write(data)
            return off

        for key in qkeys:
            t = state[key]
            if tuple(t.shape) != shapes[key] or t.shape[1] % 4:
                raise ValueError(f"Unsupported quantized tensor shape for {key}: {tuple(t.shape)}")
            if not torch.isfinite(t).all():
                raise ValueError(f"Non-finite values found in {key}")
            if device is not None and torch.device(device).type == "cuda":
                packed, scales, stats = _quantize_on_device(t, device)
            else:
                q, scales, stats = quantize_rows(t)
                packed = pack_signed_int6(q)
                if not np.array_equal(_unpack_host(packed, *t.shape), q):
                    raise AssertionError(f"Q6 pack/unpack self-check failed for {key}")
            sb = scales.tobytes()
            s_off = put(sb)
            d_off = put(packed)
            entries.append({
                "name": key, "shape": list(t.shape), "dtype": "signed_int6_twos_complement",
                "layout": "row_major; each output row has one symmetric scale",
                "qmin": QMIN, "qmax": QMAX, "scale_dtype": "little_endian_float32",
                "scale_shape": [t.shape[0]], "scale_offset": s_off, "scale_bytes": len(sb),
                "data_offset": d_off, "data_bytes": len(packed), "values": int(t.numel()),
                "stats": stats,
            })
        for key in nkeys:
            t = state[key].detach().to(device="cpu", dtype=torch.float32).contiguous()
            if tuple(t.shape) != shapes[key]:
                raise ValueError(f"Unsupported norm shape for {key}: {tuple(t.shape)}")
            data = t.numpy().astype("<f4", copy=False).tobytes()
            off = put(data)
            entries.append({"name": key, "shape": list(t.shape), "dtype": "little_endian_float32",
                            "layout": "row_major", "data_offset": off, "data_bytes": len(data),
                            "values": int(t.numel())})
    q_count = sum(int(np.prod(shapes[k])) for k in qkeys)
    n_count = sum(int(np.prod(shapes[k])) for k in nkeys)
    manifest = {
        "format": FORMAT_NAME,
        "magic_ascii": MAGIC.rstrip(b"\0").decode("ascii"),
        "version": VERSION,
        "quantization": {
            "kind": "weight-only symmetric per-output-row int6",
            "integer_range": [QMIN, QMAX],
            "scale": "max(abs(row))/31; all-zero rows use 1.0",
            "rounding": "nearest via torch.round (ties-to-even)",
            "packing": "four signed 6-bit two's-complement values packed low-bit-first into 3 bytes",
            "activations": "FP32 reference; activation quantization is not included",
            "norm_parameters": "FP32",
            "tied_output": "output.weight aliases tok_embeddings.weight; stored once",
        },
        "model_args": dict(model_args),
        "unique_parameter_count": q_count + n_count,
        "q6_value_count": q_count,
        "fp32_norm_value_count": n_count,
        "tensor_count": len(entries),
        "header": {
            "struct": "<8sIIII", "bytes": HEADER.size,
            "fields": ["magic[8]", "version:uint32", "tensor_count:uint32", "weight_bits:uint32",
                       "scale_dtype:uint32 (1=FP32)"],
            "payload_alignment_bytes": ALIGNMENT,
        },
        "binary_file": output_path.name,
        "binary_bytes": output_path.stat().st_size,
        "binary_sha256": sha256_file(output_path),
        "fp32_unique_weight_bytes": (q_count + n_count) * 4,
        "tensors": entries,
    }
    if provenance:
        manifest.update(provenance)
    manifest_path.parent.mkdir(parents=True, exist_ok=True)
    with manifest_path.open("w", encoding="utf-8", newline="\n") as f:
        json.dump(manifest, f, ensure_ascii=False, indent=2)
        f.write("\n")
    return manifest


def export_q6w(checkpoint_path, output_path, manifest_path):
    """Checkpoint file -> Q6W (same contract as q6w_format.py:108-227)."""
    ckpt = torch.load(checkpoint_path, map_location="cpu", weights_only=True)
    state = ckpt["model"]
    if not torch.equal(state["tok_embeddings.weight"], state["output.weight"]):
        raise ValueError("This Q6W exporter expects tied input embeddings/output weights")
    n_layers = int(ckpt["model_args"]["n_layers"])
    if set(state) != set(quant_keys(n_layers) + norm_keys(n_layers) + ["output.weight"]):
        raise ValueError("Checkpoint tensor names do not match the documented TinyLLMStory-zh architecture")
    prov = {"source_checkpoint": Path(checkpoint_path).name,
            "source_step": int(ckpt.get("iter_num", 0)),
            "source_checkpoint_sha256": sha256_file(checkpoint_path)}
    return write_q6w(state, ckpt["model_args"], output_path, manifest_path, prov)


def _unpack_host(data, rows, cols):
    """Host decode used only for the writer's round-trip self-check."""
    b = np.frombuffer(data, dtype=np.uint8).reshape(rows, cols // 4, 3).astype(np.int32)
    word = b[..., 0] | (b[..., 1] << 8) | (b[..., 2] << 16)
    f = np.stack([(word >> (6 * i)) & 0x3F for i in range(4)], axis=-1)
    return np.where(f >= 32, f - 64, f).astype(np.int8).reshape(rows, cols)


class Q6WImage:
    """A verified Q6W binary held in host memory, plus its manifest.

    ``tensors`` maps name -> manifest entry.  Construction performs the
    checks of q6w_format.py:234-240 (SHA-256, header) and validates every
    entry's offsets, sizes and shapes against the blob, raising ValueError on
    any mismatch -- nothing is dequantized on the host.
    """

    def __init__(self, binary_path, manifest_path, check_sha=True):
        self.binary_path = Path(binary_path)
        self.manifest = json.loads(Path(manifest_path).read_text(encoding="utf-8"))
        self.blob = self.binary_path.read_bytes()
        if check_sha and hashlib.sha256(self.blob).hexdigest() != self.manifest["binary_sha256"]:
            raise ValueError("Q6 binary SHA-256 does not match its manifest")
        if len(self.blob) < HEADER.size:
            raise ValueError("Q6 binary is shorter than its header")
        head = HEADER.unpack(self.blob[: HEADER.size])
        if head != (MAGIC, VERSION, self.manifest["tensor_count"], 6, 1):
            raise ValueError("Q6 binary header does not match the supported format")
        self.tensors = {}
        for e in self.manifest["tensors"]:
            self._check_entry(e)
            self.tensors[e["name"]] = e
        self.model_args = dict(self.manifest["model_args"])
        n_layers = int(self.model_args["n_layers"])
        shapes = _model_shapes(self.model_args)
        for key in quant_keys(n_layers) + norm_keys(n_layers):
            if key not in self.tensors:
                raise ValueError(f"Manifest lacks tensor {key}")
            if tuple(self.tensors[key]["shape"]) != shapes[key]:
                raise ValueError(f"Tensor {key} has shape {self.tensors[key]['shape']}, expected {shapes[key]}")

    def _check_entry(self, e):
        n = len(self.blob)
        lo, size = e["data_offset"], e["data_bytes"]
        if lo < HEADER.size or lo + size > n:
            raise ValueError(f"Truncated Q6 data for {e['name']}")
        if e["dtype"] == "signed_int6_twos_complement":
            rows, cols = e["shape"]
            if cols % 4 or size != rows * cols * 3 // 4:
                raise ValueError(f"Packed Q6 length mismatch for {e['name']}")
            if e["scale_bytes"] != rows * 4 or e["scale_offset"] + e["scale_bytes"] > n:
                raise ValueError(f"Invalid scale array for {e['name']}")
            if e["scale_offset"] % 4:
                raise ValueError(f"Misaligned scale array for {e['name']}")
        elif e["dtype"] == "little_endian_float32":
            if size != 4 * int(np.prod(e["shape"])) or lo % 4:
                raise ValueError(f"Invalid FP32 tensor size for {e['name']}")
        else:
            raise ValueError(f"Unsupported tensor dtype {e['dtype']}")


# --- synthetic models -------------------------------------------------------

TINY_ARGS = {"dim": 128, "n_layers": 5, "n_heads": 8, "n_kv_heads": 4, "vocab_size": 4096,
             "hidden_dim": 384, "multiple_of": 32, "norm_eps": 1e-5, "max_seq_len": 256, "dropout": 0.0}
SCALED_ARGS = {"dim": 2048, "n_layers": 22, "n_heads": 32, "n_kv_heads": 4, "vocab_size": 32000,
               "hidden_dim": 5632, "multiple_of": 256, "norm_eps": 1e-5, "max_seq_len": 256, "dropout": 0.0}


def synthetic_state(model_args, seed, std=0.02):
    """Seeded FP32 weights: every quantized tensor ~ N(0, std), norms = 1.

    Tensors are drawn from one ``torch.Generator`` (CPU, ``manual_seed(seed)``)
    in file order, so a seed fully determines the model.
    """
    gen = torch.Generator().manual_seed(int(seed))
    shapes = _model_shapes(model_args)
    state = {}
    for key in quant_keys(int(model_args["n_layers"])):
        state[key] = torch.empty(shapes[key]).normal_(0.0, std, generator=gen)
    for key in norm_keys(int(model_args["n_layers"])):
        state[key] = torch.ones(shapes[key])
    return state


def write_synthetic(model_args, seed, output_path, manifest_path, std=0.02, overwrite=False, device=None):
    """Generate a seeded synthetic model and write it as Q6W; returns the manifest.

    The weights are always drawn on the host generator (the seed fixes the
    model); ``device`` moves the quantization and packing to that GPU.
    """
    state = synthetic_state(model_args, seed, std)
    prov = {"synthetic": {"seed": int(seed), "init": f"normal(0, {std}) per quantized tensor, "
                          "torch.Generator(cpu).manual_seed(seed), drawn in file order; norms = 1.0"}}
    return write_q6w(state, model_args, output_path, manifest_path, prov, overwrite=overwrite, device=device)


class RandomImage:
    """An in-memory Q6W image with uniformly random 6-bit codes (every byte
    pattern is a valid code stream) for throughput runs of models too large to
    quantize on the host quickly.

    Same layout as ``write_q6w`` (header, then per quantized tensor its scales
    and packed rows, then the norms, every section 64-byte aligned) and the
    attributes ``Q6WImage`` exposes (``blob``, ``tensors``, ``model_args``,
    ``manifest``).  Row scales are ``1 / (18 * sqrt(cols))`` times U(0.5, 1.5),
    so a matrix roughly preserves the magnitude of a normalised input; norms
    are 1.  Values differ from any trained model, costs do not.
    """

    def __init__(self, model_args, seed=0):
        self.model_args = dict(model_args)
        n_layers = int(self.model_args["n_layers"])
        shapes = _model_shapes(self.model_args)
        qkeys, nkeys = quant_keys(n_layers), norm_keys(n_layers)
        entries, off = [], HEADER.size
        for key in qkeys:
            rows, cols = shapes[key]
            s_off = align_up(off)
            d_off = align_up(s_off + 4 * rows)
            off = d_off + rows * cols * 3 // 4
            entries.append({"name": key, "shape": [rows, cols], "dtype": "signed_int6_twos_complement",
                            "scale_offset": s_off, "scale_bytes": 4 * rows, "data_offset": d_off,
                            "data_bytes": rows * cols * 3 // 4})
        for key in nkeys:
            d_off = align_up(off)
            off = d_off + 4 * shapes[key][0]
            entries.append({"name": key, "shape": list(shapes[key]), "dtype": "little_endian_float32",
                            "data_offset": d_off, "data_bytes": 4 * shapes[key][0]})
        rng = np.random.default_rng(int(seed))
        blob = np.zeros(off, dtype=np.uint8)
        blob[: HEADER.size] = np.frombuffer(HEADER.pack(MAGIC, VERSION, len(entries), 6, 1), dtype=np.uint8)
        for e in entries:
            lo, hi = e["data_offset"], e["data_offset"] + e["data_bytes"]
            if e["dtype"] == "signed_int6_twos_complement":
                rows, cols = e["shape"]
                blob[lo:hi] = rng.integers(0, 256, hi - lo, dtype=np.uint8)
                sc = (rng.uniform(0.5, 1.5, rows) / (18.0 * np.sqrt(cols))).astype("<f4")
                blob[e["scale_offset"]: e["scale_offset"] + 4 * rows] = np.frombuffer(sc.tobytes(), dtype=np.uint8)
            else:
                blob[lo:hi] = np.frombuffer(np.ones(e["shape"][0], dtype="<f4").tobytes(), dtype=np.uint8)
        self.blob = blob.tobytes()
        self.tensors = {e["name"]: e for e in entries}
        self.manifest = {"format": FORMAT_NAME, "model_args": self.model_args, "tensor_count": len(entries),
                         "tensors": entries, "synthetic": {"seed": int(seed), "codes": "uniform random bytes"}}
