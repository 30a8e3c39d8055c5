"""GPU: FP16 KV storage (q6w_model_set_kv_dtype), the reference's FP16-KV
wrapper (quantization/compare_kv_cache.py:15-72: K/V rows rounded to FP16 by
copy_, attention in FP32 on the widened rows), against its recorded output
and the oracle restatement (OracleModel(kv_dtype=float16)).

Tolerances as for the FP32 cache: logits within 2e-4 of the reference, greedy
tokens exact on the golden request, batched streams verified by teacher
forcing.  Cache rows: the device rounds its own FP32 K/V (within ~1e-7 of the
oracle's) to FP16, so a stored value may differ from the oracle's by one
FP16 step (relative 2^-10) where that FP32 value sat at a rounding boundary.
"""

import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN, small_model_files
from oracle.model import BatchScorer, OracleModel, greedy_request
from q6w_b200 import format as fmt
from q6w_b200 import generate
from q6w_b200.model import Q6WCudaTransformer

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-4


@pytest.fixture(scope="module")
def tiny16(tiny_files):
    return (Q6WCudaTransformer.from_q6w(*tiny_files, kv_dtype=torch.float16),
            OracleModel.from_q6w(*tiny_files, kv_dtype=torch.float16))


def test_fp16_kv_step_matches_reference_wrapper(tiny16):
    cuda, orc = tiny16
    doc = json.loads((GOLDEN / "fp16_kv.json").read_text())
    rows = np.load(GOLDEN / "fp16_kv_logits.npz")["rows"]
    k, v = cuda.new_cache()
    assert k.dtype == torch.float16
    ko, vo = orc.new_cache()
    got = []
    seq = doc["prompt"] + doc["generated"][:4]
    for pos, tok in enumerate(seq):
        lg = cuda.step(tok, pos, k, v)
        with torch.inference_mode():
            orc.step(tok, pos, ko, vo)
        if pos >= len(doc["prompt"]) - 1:
            got.append(lg.cpu().numpy())
    assert np.abs(np.stack(got) - rows).max() <= LOGIT_TOL
    P = len(seq)
    for dev, ref in ((k, ko), (v, vo)):
        d = dev[:, :P].float().cpu()
        r = ref[:, :P].float()
        # layer 0: both sides round FP32 rows that differ only by FP32 summation order -> at
        # most one FP16 step apart; deeper layers also carry earlier layers' FP16 roundings
        bad0 = (d[0] - r[0]).abs() > r[0].abs() * 2.0 ** -10 + 2.0 ** -24
        assert not bad0.any(), int(bad0.sum())
        # within 4 FP16 steps of the head row's largest value (a small value from cancellation
        # carries the error of the terms that cancelled)
        scale = r.abs().amax(-1, keepdim=True)
        assert ((d - r).abs() <= scale * 2.0 ** -8 + 2.0 ** -20).all()
        assert float((d == r).float().mean()) > 0.97  # measured 0.987 over all five layers


def test_fp16_kv_generate_token_exact(tiny16):
    cuda, _ = tiny16
    doc = json.loads((GOLDEN / "fp16_kv.json").read_text())
    gen, *_ = generate(cuda, doc["prompt"], 128, cuda.device)
    assert gen == doc["generated"]


@pytest.mark.parametrize("n", [40, 300])
def test_fp16_kv_batched_teacher_forced(tiny16, n):
    """The batched step (SIMT below 64 sequences, tensor cores above) with
    FP16 caches, every stream teacher-forced through the FP16 oracle."""
    cuda, orc = tiny16
    g = torch.Generator().manual_seed(n)
    prompts = [torch.randint(3, 4096, (int(L),), generator=g).tolist() for L in torch.randint(2, 30, (n,), generator=g)]
    res = cuda.generate_greedy(prompts, 24)
    summary = BatchScorer(orc).verify_greedy(prompts, res.sampled, 24)
    assert summary["failures"] == [], summary


def test_fp16_kv_prefill(tiny16):
    cuda, orc = tiny16
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(3, 4096, (int(L),), generator=g).tolist() for L in (5, 17, 64, 1)]
    logits, (k, v) = cuda.prefill_batch(prompts)
    for i, p in enumerate(prompts):
        ko, vo = orc.new_cache()
        with torch.inference_mode():
            for pos, tok in enumerate(p):
                want = orc.step(tok, pos, ko, vo)
        assert float((logits[i].cpu() - want).abs().max()) <= LOGIT_TOL
        assert k.dtype == torch.float16


def test_fp16_kv_scaled_head_dim_64(tmp_path_factory):
    """Head dim 64 (the 1.1B shape's heads, one layer): per-head kernel at
    few sequences, group kernel at many, general tensor-core linears."""
    args = dict(fmt.SCALED_ARGS, n_layers=1, max_seq_len=32)
    b, m = small_model_files(tmp_path_factory, args, 5, "scaled16")
    cuda = Q6WCudaTransformer.from_q6w(b, m, kv_dtype=torch.float16)
    orc = OracleModel.from_q6w(b, m, kv_dtype=torch.float16)
    prompt = [17, 2500, 31999, 4, 1234]
    k, v = cuda.new_cache()
    ko, vo = orc.new_cache()
    for p, t in enumerate(prompt):
        a = cuda.step(t, p, k, v).cpu()
        with torch.inference_mode():
            want = orc.step(t, p, ko, vo)
        assert float((a - want).abs().max()) <= LOGIT_TOL
    for n in (4, 40):
        kb, vb = cuda.new_batch_cache(n)
        for p, t in enumerate(prompt):
            lg, _ = cuda.forward_batch(torch.full((n,), t, dtype=torch.int32).cuda(),
                                       torch.full((n,), p, dtype=torch.int32).cuda(), kb, vb)
        assert float((lg.cpu() - want).abs().max()) <= LOGIT_TOL


def test_fp16_kv_rejects_fp32_cache(tiny16):
    cuda, _ = tiny16
    k = torch.empty(5, 256, 4, 16, device="cuda")
    with pytest.raises(ValueError):
        cuda.step(3, 0, k, k)
