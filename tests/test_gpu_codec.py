"""GPU: Q6W decode and dequantization, bit-exact against the oracle codec."""

import numpy as np
import pytest
import torch

from oracle import codec
from q6w_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,cols", [(1, 4), (3, 16), (7, 12), (128, 128), (64, 384), (4096, 128), (33, 5632)])
def test_unpack_bit_exact(rows, cols):
    rng = np.random.default_rng(rows * 1000 + cols)
    q = rng.integers(-32, 32, size=(rows, cols))
    data = codec.pack_int6(q, allow_minus32=True)
    got = ops.unpack_signed_int6(data, rows, cols).cpu().numpy()
    assert np.array_equal(got, q)
    assert np.array_equal(got, codec.unpack_int6(data, rows, cols))


def test_unpack_golden(golden_codec):
    for case in golden_codec["pack"] + golden_codec["unpack_only"]:
        got = ops.unpack_signed_int6(bytes.fromhex(case["packed_hex"]), case["rows"], case["cols"])
        assert got.cpu().tolist() == case["unpacked"]


def test_unpack_unaligned_output_and_empty():
    q = np.arange(-32, 32).reshape(2, 32)
    data = torch.frombuffer(bytearray(codec.pack_int6(q, allow_minus32=True)), dtype=torch.uint8).cuda()
    buf = torch.zeros(2 * 32 + 1, dtype=torch.int8, device="cuda")
    from q6w_b200 import _lib

    lib = _lib.load()
    _lib.check(lib.q6w_unpack(data.data_ptr(), buf[1:].data_ptr(), 2, 32, _lib.stream_handle()))
    assert np.array_equal(buf[1:].cpu().numpy().reshape(2, 32), q)
    assert ops.unpack_signed_int6(b"", 0, 8).shape == (0, 8)


def test_unpack_errors():
    with pytest.raises(ValueError, match="divisible by four"):
        ops.unpack_signed_int6(b"\0" * 3, 1, 6)
    with pytest.raises(ValueError, match="length mismatch"):
        ops.unpack_signed_int6(b"\0" * 5, 1, 8)


@pytest.mark.parametrize("rows,cols", [(1, 4), (5, 20), (4096, 128), (384, 128), (32000, 2048)])
def test_dequant_bit_exact(rows, cols):
    rng = np.random.default_rng(rows + cols)
    q = rng.integers(-32, 32, size=(rows, cols))
    s = rng.uniform(0.001, 0.05, size=rows).astype(np.float32)
    packed = torch.frombuffer(bytearray(codec.pack_int6(q, allow_minus32=True)), dtype=torch.uint8).cuda()
    got = ops.dequantize_rows(packed, torch.from_numpy(s).cuda(), rows, cols).cpu().numpy()
    want = codec.dequantize(q, s)
    assert got.dtype == np.float32 and np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_load_dequantized_state_matches_oracle(tiny_files):
    state, manifest = ops.load_dequantized_state(*tiny_files)
    ref, _ = codec.load_state(*tiny_files)
    assert set(state) == set(ref)
    for k in ref:
        assert torch.equal(state[k].cpu(), ref[k]), k
    assert state["output.weight"].data_ptr() == state["tok_embeddings.weight"].data_ptr()
