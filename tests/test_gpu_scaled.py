"""GPU: the scaled 1.1B-shape config as configured (dim 2048, 22 layers, 32
heads / 4 kv heads, hidden 5632, vocab 32000, context 256), weights
N(0, 0.02) from a seed, Q6W-quantized by the device writer, against the
oracle.

A 128-token random prompt plus 8 greedy tokens at B=1 (streaming GEMVs)
and at B=64 (general tensor-core linears).  The streams are verified by
teacher forcing through the oracle: every pick is the oracle's argmax or an
FP32 near-tie within 1e-4 of its maximum.  The logits of the first decode
step at B=1 are compared with the oracle's B=1 step.  B=64 checks four of
the 64 sequences (the oracle costs ~0.1 s per position per sequence group
on the host).
"""

import pytest
import torch

from oracle.model import BatchScorer, OracleModel
from q6w_b200 import format as fmt
from q6w_b200.model import Q6WCudaTransformer

pytestmark = [pytest.mark.gpu, pytest.mark.slow]
PROMPT, NEW = 128, 8
# Logit tolerance of the 22-layer model (the tiny model's is 2e-4): both
# sides sum in FP32 in different orders and the error grows with depth and
# width; measured ~2e-5 on the B200.
LOGIT_TOL_22 = 2e-4


@pytest.fixture(scope="module")
def scaled(tmp_path_factory):
    d = tmp_path_factory.mktemp("scaled22")
    b, m = d / "scaled.bin", d / "scaled.json"
    fmt.write_synthetic(dict(fmt.SCALED_ARGS), 2026, b, m, device="cuda")
    cuda = Q6WCudaTransformer.from_q6w(b, m)
    orc = OracleModel.from_q6w(b, m)
    return cuda, orc


def _prompts(n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(3, fmt.SCALED_ARGS["vocab_size"], (n, PROMPT), generator=g).tolist()


def test_scaled_22_layers_b1(scaled):
    cuda, orc = scaled
    prompt = _prompts(1, 31)[0]
    res = cuda.generate_greedy([prompt], NEW, keep_logits=True)
    assert len(res.sampled[0]) == NEW
    summary = BatchScorer(orc).verify_greedy([prompt], res.sampled, NEW)
    assert summary["failures"] == [], summary
    # first decode step's logits against the oracle's own B=1 step over the prompt
    k, v = orc.new_cache()
    with torch.inference_mode():
        for pos, tok in enumerate(prompt):
            logits = orc.step(tok, pos, k, v)
    err = float((res.logits[0, 0].cpu() - logits).abs().max())
    assert err <= LOGIT_TOL_22, err


def test_scaled_22_layers_b64(scaled):
    cuda, orc = scaled
    prompts = _prompts(64, 32)
    res = cuda.generate_greedy(prompts, NEW)
    assert all(len(s) == NEW for s in res.sampled)
    pick = [0, 21, 42, 63]
    summary = BatchScorer(orc).verify_greedy([prompts[i] for i in pick], [res.sampled[i] for i in pick], NEW)
    assert summary["failures"] == [], summary
    assert summary["picks"] == len(pick) * NEW
