"""GPU: the non-cached forward with targets (q6w_forward_all), the
Transformer.forward(tokens, targets) of training/model.py:249-269, against the
reference's own recorded forward and the oracle.

Tolerances: logits within 2e-4 of the reference (the cached-step tolerance;
here the reference attends with scaled_dot_product_attention, the device
with the decode kernels over the filled caches); the mean cross entropy
within 1e-5 relative (FP64 mean of FP32 per-row values here, FP32 torch
there).
"""

import json

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import GOLDEN
from oracle.model import OracleModel, forward_all
from q6w_b200.model import Q6WCudaTransformer

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny(tiny_files):
    return Q6WCudaTransformer.from_q6w(*tiny_files), OracleModel.from_q6w(*tiny_files)


def test_forward_matches_reference_training_forward(tiny):
    cuda, _ = tiny
    doc = json.loads((GOLDEN / "forward_all.json").read_text())
    rows = np.load(GOLDEN / "forward_all_logits.npz")["rows"]
    logits = cuda.forward(torch.tensor(doc["tokens"]), torch.tensor(doc["targets"]))
    assert tuple(logits.shape) == (2, 40, 4096)
    got = logits[:, :: doc["rows_every"]].cpu().numpy()
    assert np.abs(got - rows).max() <= 2e-4
    assert float(cuda.last_loss) == pytest.approx(doc["loss"], rel=1e-5)
    last = cuda.forward(torch.tensor(doc["tokens"]))  # inference branch: last position only
    assert tuple(last.shape) == (2, 1, 4096)
    assert float((last[:, 0].cpu() - logits[:, -1].cpu()).abs().max()) <= 2e-4


@pytest.mark.parametrize("n", [3, 70])
def test_forward_all_ragged_against_oracle(tiny, n):
    """Ragged prompts (SIMT rows below 64 token rows, tensor cores above),
    targets with ignored positions."""
    cuda, orc = tiny
    g = torch.Generator().manual_seed(n)
    prompts = [torch.randint(3, 4096, (int(L),), generator=g).tolist() for L in torch.randint(1, 25, (n,), generator=g)]
    targets = [[(t if (i + j) % 5 else -1) for j, t in enumerate(p[1:] + [7])] for i, p in enumerate(prompts)]
    lg, loss = cuda.forward_all(prompts, targets)
    want, want_loss = forward_all(orc, prompts, targets)
    for a, b in zip(lg, want):
        assert float((a.cpu() - b).abs().max()) <= 2e-4
    assert float(loss) == pytest.approx(want_loss, rel=1e-5)
    flat = torch.cat([x.cpu() for x in lg])
    tg = torch.tensor([t for row in targets for t in row])
    assert float(loss) == pytest.approx(float(F.cross_entropy(flat, tg, ignore_index=-1)), rel=1e-5)


def test_forward_all_every_target_ignored_gives_nan(tiny):
    cuda, _ = tiny
    _, loss = cuda.forward_all([[5, 6, 7]], [[-1, -1, -1]])
    assert torch.isnan(loss)
