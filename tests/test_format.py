"""CPU: Q6W file reader/writer (host logic) against the oracle codec."""

import json

import numpy as np
import pytest
import torch

from oracle import codec
from q6w_b200 import format as fmt


def test_pack_rejects_out_of_range_and_bad_width():
    with pytest.raises(ValueError, match="divisible by four"):
        fmt.pack_signed_int6(np.zeros((2, 6)))
    with pytest.raises(ValueError, match=r"\[-31, 31\]"):
        fmt.pack_signed_int6(np.full((1, 4), -32))
    with pytest.raises(ValueError):
        fmt.pack_signed_int6(np.full((1, 4), 32), allow_minus32=True)


def test_pack_full_code_space_round_trip():
    rng = np.random.default_rng(3)
    q = rng.integers(-32, 32, size=(17, 64))
    data = fmt.pack_signed_int6(q, allow_minus32=True)
    assert data == codec.pack_int6(q, allow_minus32=True)
    assert np.array_equal(codec.unpack_int6(data, 17, 64), q)


def test_empty_matrix():
    assert fmt.pack_signed_int6(np.zeros((0, 8), dtype=np.int64)) == b""
    assert codec.unpack_int6(b"", 0, 8).shape == (0, 8)


@pytest.mark.parametrize("n_layers", [1, 3, 7])
def test_writer_any_layer_count(tmp_path, n_layers):
    args = dict(fmt.TINY_ARGS, n_layers=n_layers, vocab_size=64, max_seq_len=16)
    man = fmt.write_synthetic(args, 5, tmp_path / "m.bin", tmp_path / "m.json")
    assert man["tensor_count"] == 7 * n_layers + 1 + 2 * n_layers + 1
    state, _ = codec.load_state(tmp_path / "m.bin", tmp_path / "m.json")
    src = fmt.synthetic_state(args, 5)
    for key in fmt.quant_keys(n_layers):
        q, s = codec.quantize_rows(src[key])
        assert torch.equal(state[key], torch.from_numpy(codec.dequantize(q, s)))
    for key in fmt.norm_keys(n_layers):
        assert torch.equal(state[key], src[key])
    img = fmt.Q6WImage(tmp_path / "m.bin", tmp_path / "m.json")
    for e in man["tensors"]:
        assert e["data_offset"] % 64 == 0
        if "scale_offset" in e:
            assert e["scale_offset"] % 64 == 0
    assert img.model_args["n_layers"] == n_layers


def test_writer_refuses_overwrite(tmp_path):
    args = dict(fmt.TINY_ARGS, n_layers=1, vocab_size=16, max_seq_len=8)
    fmt.write_synthetic(args, 1, tmp_path / "a.bin", tmp_path / "a.json")
    with pytest.raises(FileExistsError):
        fmt.write_synthetic(args, 1, tmp_path / "a.bin", tmp_path / "a.json")


@pytest.fixture()
def small(tmp_path):
    args = dict(fmt.TINY_ARGS, n_layers=1, vocab_size=32, max_seq_len=8)
    fmt.write_synthetic(args, 2, tmp_path / "s.bin", tmp_path / "s.json")
    return tmp_path / "s.bin", tmp_path / "s.json"


def test_reader_detects_sha_mismatch(small):
    b, m = small
    raw = bytearray(b.read_bytes())
    raw[100] ^= 1
    b.write_bytes(bytes(raw))
    with pytest.raises(ValueError, match="SHA-256"):
        fmt.Q6WImage(b, m)


def test_reader_detects_bad_header(small):
    b, m = small
    raw = bytearray(b.read_bytes())
    raw[0:8] = b"BADMAGIC"
    b.write_bytes(bytes(raw))
    man = json.loads(m.read_text())
    import hashlib

    man["binary_sha256"] = hashlib.sha256(bytes(raw)).hexdigest()
    m.write_text(json.dumps(man))
    with pytest.raises(ValueError, match="header"):
        fmt.Q6WImage(b, m)


def test_reader_detects_truncation(small):
    b, m = small
    raw = b.read_bytes()[:-100]
    b.write_bytes(raw)
    man = json.loads(m.read_text())
    import hashlib

    man["binary_sha256"] = hashlib.sha256(raw).hexdigest()
    m.write_text(json.dumps(man))
    with pytest.raises(ValueError, match="Truncated|Invalid"):
        fmt.Q6WImage(b, m)


def test_reader_detects_bad_shape(small):
    b, m = small
    man = json.loads(m.read_text())
    man["tensors"][1]["shape"] = [man["tensors"][1]["shape"][0], 64]
    m.write_text(json.dumps(man))
    with pytest.raises(ValueError):
        fmt.Q6WImage(b, m)


def test_reader_accepts_shipped_artifact(shipped_files):
    img = fmt.Q6WImage(*shipped_files)
    assert img.model_args["dim"] == 128 and len(img.tensors) == 47


def test_random_image_layout():
    """The random-code image used for large-model throughput runs has the
    writer's layout: header, 64-byte aligned sections, no overlaps, norms 1."""
    import numpy as np

    img = fmt.RandomImage(dict(fmt.TINY_ARGS), seed=3)
    head = fmt.HEADER.unpack(img.blob[: fmt.HEADER.size])
    assert head == (fmt.MAGIC, fmt.VERSION, len(img.tensors), 6, 1)
    spans = []
    for e in img.tensors.values():
        assert e["data_offset"] % fmt.ALIGNMENT == 0
        spans.append((e["data_offset"], e["data_offset"] + e["data_bytes"]))
        if "scale_offset" in e:
            assert e["scale_offset"] % fmt.ALIGNMENT == 0
            spans.append((e["scale_offset"], e["scale_offset"] + e["scale_bytes"]))
            rows, cols = e["shape"]
            assert e["data_bytes"] == rows * cols * 3 // 4
            sc = np.frombuffer(img.blob[e["scale_offset"]: e["scale_offset"] + e["scale_bytes"]], dtype="<f4")
            assert (sc > 0).all() and np.isfinite(sc).all()
        else:
            v = np.frombuffer(img.blob[e["data_offset"]: e["data_offset"] + e["data_bytes"]], dtype="<f4")
            assert (v == 1.0).all()
    spans.sort()
    assert spans[0][0] >= fmt.HEADER.size
    assert all(a[1] <= b[0] for a, b in zip(spans, spans[1:]))
    assert spans[-1][1] == len(img.blob)
