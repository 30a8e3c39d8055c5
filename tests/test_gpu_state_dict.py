"""GPU: the drop-in class's ``load_state_dict`` (FP32 weights in, quantized
and packed on the device with the reference's row rule) and the batched
``decode_greedy_batch`` of the drop-in contract.

* FP32 weights loaded into a model built from another file give the model
  that the writer + ``from_q6w`` give for the same weights: bit-identical
  logits and tokens.
* The dequantized state of a Q6W file (``oracle.codec.load_state``, the
  reference's ``load_dequantized_state``) round-trips: the same greedy tokens,
  logits within 1e-5 (codes equal, scales within one rounding).
* Key checks as torch's: missing tensors always raise, unexpected ones raise
  under ``strict``; a tied head that differs from the embedding raises.
"""

import pytest
import torch

from conftest import small_model_files
from oracle.codec import load_state
from q6w_b200 import format as fmt
from q6w_b200.model import Q6WCudaTransformer

pytestmark = pytest.mark.gpu

ARGS = dict(fmt.TINY_ARGS, n_layers=2, max_seq_len=64)


def _prompts(n, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(3, 4096, (int(L),), generator=g).tolist()
            for L in torch.randint(2, 12, (n,), generator=g)]


@pytest.fixture(scope="module")
def pair(tmp_path_factory):
    a = small_model_files(tmp_path_factory, ARGS, 41, "sd_a")
    b = small_model_files(tmp_path_factory, ARGS, 42, "sd_b")
    return a, b


def test_fp32_state_equals_written_model(pair):
    (ab, am), (bb, bm) = pair
    ref = Q6WCudaTransformer.from_q6w(ab, am)
    other = Q6WCudaTransformer.from_q6w(bb, bm)
    out = other.load_state_dict(fmt.synthetic_state(ARGS, 41))
    assert out.missing_keys == [] and out.unexpected_keys == []
    k1, v1 = ref.new_cache()
    k2, v2 = other.new_cache()
    for pos, t in enumerate([5, 900, 31, 4000, 7]):
        assert torch.equal(ref.step(t, pos, k1, v1), other.step(t, pos, k2, v2)), pos
    prompts = _prompts(70, 3)
    assert other.decode_greedy_batch(prompts, 10) == ref.decode_greedy_batch(prompts, 10)


def test_dequantized_state_round_trips(pair):
    (ab, am), (bb, bm) = pair
    ref = Q6WCudaTransformer.from_q6w(ab, am)
    other = Q6WCudaTransformer.from_q6w(bb, bm)
    state, _ = load_state(ab, am)  # includes the tied output.weight
    other.load_state_dict(state)
    prompts = _prompts(12, 4)
    ra = ref.generate_greedy(prompts, 8, keep_logits=True)
    rb = other.generate_greedy(prompts, 8, keep_logits=True)
    assert ra.sampled == rb.sampled
    assert float((ra.logits - rb.logits).abs().max()) <= 1e-5


def test_decode_greedy_batch_contract(pair):
    (ab, am), _ = pair
    model = Q6WCudaTransformer.from_q6w(ab, am)
    prompts = _prompts(9, 5)
    first = model.generate_greedy(prompts, 6).sampled
    stop = first[0][2]
    ids, picks = model.decode_greedy_batch(prompts, 6, stop_ids=[stop])
    ref = model.generate_greedy(prompts, 6, stop_ids=(stop,))
    assert ids == ref.generated and picks == ref.sampled
    assert picks[0][-1] == stop and stop not in ids[0]


def test_key_checks(pair):
    (ab, am), _ = pair
    model = Q6WCudaTransformer.from_q6w(ab, am)
    state = fmt.synthetic_state(ARGS, 7)
    with pytest.raises(RuntimeError):
        model.load_state_dict({k: v for k, v in state.items() if k != "norm.weight"})
    extra = dict(state, **{"bogus.weight": torch.zeros(3)})
    with pytest.raises(RuntimeError):
        model.load_state_dict(extra)
    out = model.load_state_dict(extra, strict=False)
    assert out.unexpected_keys == ["bogus.weight"]
    bad = dict(state, **{"output.weight": state["tok_embeddings.weight"] + 1.0})
    with pytest.raises(ValueError):
        model.load_state_dict(bad)
