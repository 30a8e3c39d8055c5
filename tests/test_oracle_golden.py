"""CPU: the oracle (and the product's host codec) pinned to the reference's
own outputs recorded in tests/golden/ by make_golden.py."""

import numpy as np
import pytest
import torch

from oracle import codec
from oracle.model import OracleModel, greedy_request
from q6w_b200 import format as fmt


def test_pack_matches_reference_bytes(golden_codec):
    for case in golden_codec["pack"]:
        q = np.array(case["codes"])
        assert codec.pack_int6(q).hex() == case["packed_hex"]
        assert fmt.pack_signed_int6(q).hex() == case["packed_hex"]


def test_unpack_matches_reference(golden_codec):
    for case in golden_codec["pack"] + golden_codec["unpack_only"]:
        got = codec.unpack_int6(bytes.fromhex(case["packed_hex"]), case["rows"], case["cols"])
        assert got.tolist() == case["unpacked"]


def test_unpack_covers_all_codes(golden_codec):
    case = golden_codec["unpack_only"][0]
    got = codec.unpack_int6(bytes.fromhex(case["packed_hex"]), 1, 64)
    assert sorted(got[0].tolist()) == list(range(-32, 32))


def test_quantize_rows_matches_reference(golden_codec):
    for case in golden_codec["quantize"]:
        w = torch.tensor(case["weights"], dtype=torch.float32)
        q, s = codec.quantize_rows(w)
        assert q.tolist() == case["q"]
        assert np.array_equal(s, np.array(case["scales"], dtype=np.float32))
        q2, s2, stats = fmt.quantize_rows(w)
        assert q2.tolist() == case["q"] and np.array_equal(s2, s)
        assert stats["max_abs_error"] == pytest.approx(case["stats"]["max_abs_error"], rel=1e-6)


def test_oracle_tiny_request_tokens(tiny_files, golden_tiny):
    m = OracleModel.from_q6w(*tiny_files)
    out = greedy_request(m, golden_tiny["prompt"], golden_tiny["new_tokens"])
    assert out["generated"] == golden_tiny["generated"]
    assert np.allclose(out["margins"], golden_tiny["margins"], atol=1e-6)


def test_oracle_tiny_logits(tiny_files, golden_tiny):
    ref = np.load(__import__("conftest").GOLDEN / "tiny_logits.npz")
    m = OracleModel.from_q6w(*tiny_files)
    out = greedy_request(m, golden_tiny["prompt"], 5, keep_logits=True)
    got = out["logits"].numpy()
    # bitwise on the machine that made the fixture; FP32-rounding close elsewhere
    assert np.abs(got[0] - ref["prompt_last"]).max() <= 1e-5
    assert np.abs(got[1:5] - ref["decode_1_4"]).max() <= 1e-5


def test_oracle_stop_contract(tiny_files, golden_tiny):
    case = golden_tiny["stop_case"]
    m = OracleModel.from_q6w(*tiny_files)
    out = greedy_request(m, golden_tiny["prompt"], golden_tiny["new_tokens"], case["stop_ids"], case["min_new_tokens"])
    assert out["sampled"] == case["sampled"]
    assert out["generated"] == case["generated"]
    assert out["stopped_on"] == case["stopped_on"]


def test_oracle_shipped_request(shipped_files, golden_shipped):
    m = OracleModel.from_q6w(*shipped_files)
    g = golden_shipped
    out = greedy_request(m, g["prompt"], g["new_tokens"], g["stop_ids"], g["min_new_tokens"])
    assert out["sampled"] == g["sampled"]
    assert out["generated"] == g["generated"]


def test_batch_scorer_agrees_with_step(tiny_files, golden_tiny):
    from oracle.model import BatchScorer

    m = OracleModel.from_q6w(*tiny_files)
    sc = BatchScorer(m)
    prompts = [golden_tiny["prompt"], golden_tiny["prompt"][:7]]
    outs = [greedy_request(m, p, 12) for p in prompts]
    summary = sc.verify_greedy(prompts, [o["sampled"] for o in outs], 12)
    assert summary["failures"] == [] and summary["picks"] == 24
    # a planted wrong pick is caught
    bad = [list(o["sampled"]) for o in outs]
    bad[1][3] = (bad[1][3] + 1) % 4096
    assert sc.verify_greedy(prompts, bad, 12)["failures"]


@pytest.fixture(scope="module")
def golden_sampling():
    import json

    from conftest import GOLDEN

    return json.loads((GOLDEN / "sampling.json").read_text())


def test_oracle_sampler_reproduces_reference_streams(tiny_files, golden_sampling):
    """XorShift64, temperature / top-p sampling and the repetition, n-gram and
    stop-bias processors of the oracle give the reference generate()'s tokens."""
    from oracle.sampler import sampled_request

    torch.set_num_threads(1)
    orc = OracleModel.from_q6w(*tiny_files)
    for case in golden_sampling["cases"]:
        kw = dict(case["kwargs"])
        if "stop_token" in kw:
            kw["stop_token"] = set(kw["stop_token"])
        got = sampled_request(orc, golden_sampling["prompt"], case["new_tokens"], **kw)
        assert got["generated"] == case["generated"], kw
        assert got["stopped"] == case["stopped"] and got["stop_reason"] == case["stop_reason"]


def test_xorshift_known_values():
    """The reference generator's first draws for seed 1 (torch_benchmark.py:133-144), restated by hand."""
    from oracle.sampler import XorShift64

    mask = (1 << 64) - 1
    s = 1
    want = []
    for _ in range(3):
        s ^= s >> 12
        s ^= (s << 25) & mask
        s ^= s >> 27
        want.append((((s * 0x2545F4914F6CDD1D) & mask) >> 40) / 16777216.0)
    r = XorShift64(1)
    assert [r.random_f32() for _ in range(3)] == want


def test_oracle_fp16_kv_matches_reference_wrapper(tiny_files):
    """OracleModel(kv_dtype=float16) against the reference's FP16KVTransformer
    (quantization/compare_kv_cache.py:15-72) on the golden request."""
    import json

    from conftest import GOLDEN

    doc = json.loads((GOLDEN / "fp16_kv.json").read_text())
    rows = np.load(GOLDEN / "fp16_kv_logits.npz")["rows"]
    torch.set_num_threads(1)
    orc = OracleModel.from_q6w(*tiny_files, kv_dtype=torch.float16)
    assert greedy_request(orc, doc["prompt"], 128)["generated"] == doc["generated"]
    k, v = orc.new_cache()
    got = []
    with torch.inference_mode():
        for pos, tok in enumerate(doc["prompt"] + doc["generated"][:4]):
            lg = orc.step(tok, pos, k, v)
            if pos >= len(doc["prompt"]) - 1:
                got.append(lg.numpy())
    assert np.array_equal(np.stack(got), rows)  # the same torch CPU operations: bit for bit


def test_oracle_forward_all_matches_reference_forward(tiny_files):
    """All-position logits and the masked loss of the reference's non-cached
    forward (training/model.py:249-269; attention by scaled_dot_product_attention
    there, by the cached step here: the same sums in another order)."""
    import json

    from conftest import GOLDEN
    from oracle.model import forward_all

    doc = json.loads((GOLDEN / "forward_all.json").read_text())
    rows = np.load(GOLDEN / "forward_all_logits.npz")["rows"]
    torch.set_num_threads(1)
    orc = OracleModel.from_q6w(*tiny_files)
    logits, loss = forward_all(orc, doc["tokens"], doc["targets"])
    got = np.stack([lg[::doc["rows_every"]].numpy() for lg in logits])
    assert np.abs(got - rows).max() <= 2e-5
    assert loss == pytest.approx(doc["loss"], rel=1e-6)
