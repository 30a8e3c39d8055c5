"""GPU: the reference's sampler and logit processors on the device
(benchmarks/torch_benchmark.py:133-296) against the oracle restatement and
the reference's own sampled streams.

Parity.  The processors and the top-p bookkeeping reproduce the reference's
arithmetic exactly (FP32 shaping; exact FP64 sums of the kept
probabilities); the probabilities themselves come from CUDA's expf and a
different FP32 summation order of the softmax denominator (torch CPU sums
each of 8-16 vector lanes sequentially: up to ~2000 terms, a relative error
of up to ~1e-4 in the worst case, ~1e-6 typically).  So a pick may differ
from the reference only when its decision sat within 1e-4 of a boundary
(coin against a cumulative sum, or the nucleus sum against top_p) or inside
a group of equal probabilities; every other pick must be identical, at least
99% of all picks must be, and every stream must stop exactly where generate
stops.
"""

import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle.model import BatchScorer, OracleModel
from oracle.sampler import XorShift64, decision, process_logits, verify_sampled
from q6w_b200 import generate, ops
from q6w_b200.model import Q6WCudaTransformer

pytestmark = pytest.mark.gpu
MARGIN = 1e-4

SETTINGS = [
    dict(temperature=0.8, top_p=0.9),
    dict(temperature=1.0, top_p=1.0),
    dict(temperature=0.7, top_p=0.95, repetition_penalty=1.3, no_repeat_ngram_size=3),
    dict(temperature=0.9, top_p=0.9, stop_ids=(907, 12), min_new_tokens=6, stop_token_bias=2.5,
         stop_token_bias_after=8),
    dict(temperature=0.0, top_p=0.9, repetition_penalty=1.2, no_repeat_ngram_size=2),
    dict(temperature=1.2, top_p=0.5, no_repeat_ngram_size=1),
    dict(temperature=0.6, top_p=0.0, repetition_penalty=0.8),
]


@pytest.fixture(scope="module")
def golden_sampling():
    return json.loads((GOLDEN / "sampling.json").read_text())


@pytest.fixture(scope="module")
def tiny(tiny_files):
    return Q6WCudaTransformer.from_q6w(*tiny_files), OracleModel.from_q6w(*tiny_files)


def _rows(n, V, seed, spread):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(n, V, generator=g) * spread


def _histories(n, H, V, seed):
    """Histories with repeats, so the penalty and the n-gram bans engage."""
    rng = np.random.default_rng(seed)
    h = rng.integers(0, V, size=(n, H))
    for i in range(n):
        L = int(rng.integers(0, H + 1))
        if L >= 6:
            h[i, L - 3: L] = h[i, 1:4]  # the last trigram repeats an earlier one
        h[i, L:] = -1
    lens = np.array([int((row >= 0).sum()) for row in h])
    return torch.from_numpy(np.where(h < 0, 0, h).astype(np.int32)), torch.from_numpy(lens.astype(np.int32))


@pytest.mark.parametrize("V,spread", [(4096, 2.0), (4096, 0.3), (32000, 1.0)])
@pytest.mark.parametrize("k", range(len(SETTINGS)))
def test_sample_op_matches_oracle(V, spread, k):
    cfg = dict(SETTINGS[k])
    n, H = (96 if V > 4096 else 256), 40
    logits = _rows(n, V, 100 + k, spread)
    hist, lens = _histories(n, H, V, 200 + k)
    seeds = [int(s) for s in np.random.default_rng(300 + k).integers(1, 2 ** 63, size=n)]
    rng = torch.tensor(seeds, dtype=torch.int64).cuda()
    stop_ids = cfg.pop("stop_ids", ())
    min_new = cfg.pop("min_new_tokens", 0)
    bias = cfg.pop("stop_token_bias", 0.0)
    after = cfg.pop("stop_token_bias_after", None)
    got = ops.sample(logits.cuda(), hist.cuda(), lens.cuda(), rng, stop_ids=stop_ids, min_new_tokens=min_new,
                     stop_token_bias=bias, stop_token_bias_after=after, **cfg).cpu().tolist()
    states = rng.cpu().tolist()
    exact = boundary = 0
    for i in range(n):
        L = int(lens[i])
        history = hist[i, :L].tolist()
        shaped = process_logits(logits[i], history, L, tuple(stop_ids) if stop_ids else None, min_new,
                                min_new if after is None else after, bias, cfg.get("repetition_penalty", 1.0),
                                cfg.get("no_repeat_ngram_size", 0))
        r = XorShift64(seeds[i])
        d = decision(shaped, cfg["temperature"], cfg["top_p"], r)
        if got[i] == d["token"]:
            exact += 1
        else:
            assert d["margin"] <= MARGIN or d["tie"], (i, got[i], d)
            boundary += 1
        want_state = r.state - (1 << 64) if r.state >= (1 << 63) else r.state
        assert states[i] == want_state  # one coin drawn at temperature > 0, none at 0
    assert exact >= n - max(1, n // 50), (exact, boundary)


def test_generate_reproduces_reference_sampled_streams(tiny, golden_sampling):
    """The drop-in generate() with the reference's sampling arguments, against
    the reference's own streams (every pick exact, or a boundary case that
    teacher forcing through the oracle explains)."""
    cuda, orc = tiny
    prompt = golden_sampling["prompt"]
    for case in golden_sampling["cases"]:
        kw = dict(case["kwargs"])
        if "stop_token" in kw:
            kw["stop_token"] = set(kw["stop_token"])
        gen, pre_s, dec_s, stopped, reason = generate(cuda, prompt, case["new_tokens"], cuda.device, **kw)
        if gen == case["generated"]:
            assert stopped == case["stopped"] and reason == case["stop_reason"]
            continue
        stream = gen + ([reason] if stopped else [])
        vk = {k: v for k, v in kw.items() if k != "seed"}
        summary = verify_sampled(BatchScorer(orc), [prompt], [stream], [kw.get("seed", 1)], case["new_tokens"], **vk)
        assert summary["failures"] == [], (kw, summary)


@pytest.mark.parametrize("k", [0, 2, 3, 5])
def test_generate_sampled_batch_teacher_forced(tiny, k):
    """Many sequences at once (the batched step on the tensor-core path), each
    with its own seed, verified by teacher forcing through the oracle."""
    cuda, orc = tiny
    cfg = dict(SETTINGS[k])
    stop_ids = cfg.pop("stop_ids", ())
    g = torch.Generator().manual_seed(40 + k)
    n = 96
    prompts = [torch.randint(3, 4096, (int(L),), generator=g).tolist()
               for L in torch.randint(4, 24, (n,), generator=g)]
    seeds = list(range(1000 * k + 1, 1000 * k + 1 + n))
    res = cuda.generate_sampled(prompts, 40, seeds, stop_ids=stop_ids, keep_logits=True, **cfg)
    dev_rows = res.logits.cpu()  # raw logits of every decode step, [n, 40, vocab]
    # the sampler decides on the device's own logits (boundary margin 1e-4); those logits must be
    # within the step's 2e-4 of the oracle's
    summary = verify_sampled(BatchScorer(orc), prompts, res.sampled, seeds, 40,
                             stop_token=set(stop_ids) if stop_ids else None, device_logits=dev_rows,
                             margin_tol=MARGIN, logit_tol=2e-4, **cfg)
    assert summary["failures"] == [], summary
    assert summary["exact"] >= summary["picks"] - max(1, summary["picks"] // 100), summary


def test_sampling_argument_errors(tiny):
    cuda, _ = tiny
    with pytest.raises(ValueError):
        generate(cuda, [5, 6], 4, cuda.device, repetition_penalty=0.0)
    with pytest.raises(ValueError):
        generate(cuda, [5, 6], 4, cuda.device, no_repeat_ngram_size=-1)
