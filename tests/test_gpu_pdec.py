"""GPU: the persistent B=1 step (pdec.cuh, opt-in with Q6W_PDEC=1 at model
creation) -- one cooperative launch per model step for models with
streaming-GEMV widths (the 1.1B shape) -- against the per-kernel step and the
oracle.

The persistent kernel keeps the per-kernel step's arithmetic and summation
orders (the streaming GEMV's unit decode, eight-row reductions and per-group
sums; the per-head attention kernel's reductions), so logits and caches are
compared bit for bit.  The profiler confirms the persistent kernel is the
one that ran.
"""

import os

import pytest
import torch
from torch.profiler import ProfilerActivity, profile

from conftest import small_model_files
from oracle.model import BatchScorer, OracleModel
from q6w_b200 import format as fmt
from q6w_b200.model import Q6WCudaTransformer

pytestmark = pytest.mark.gpu


def _persistent(b, m, **kw):
    os.environ["Q6W_PDEC"] = "1"
    try:
        return Q6WCudaTransformer.from_q6w(b, m, **kw)
    finally:
        del os.environ["Q6W_PDEC"]


def _kernels(fn):
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return {e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA}


@pytest.fixture(scope="module")
def pair(tmp_path_factory):
    args = dict(fmt.SCALED_ARGS, n_layers=2, max_seq_len=64)
    b, m = small_model_files(tmp_path_factory, args, 9, "pdec2")
    return _persistent(b, m), Q6WCudaTransformer.from_q6w(b, m), (b, m)


def test_persistent_step_bit_identical(pair):
    fast, ref, _ = pair
    g = torch.Generator().manual_seed(2)
    toks = torch.randint(3, 32000, (20,), generator=g).tolist()
    kf, vf = fast.new_cache()
    kr, vr = ref.new_cache()
    names = _kernels(lambda: fast.step(toks[0], 0, kf, vf))
    assert any("pdec_kernel" in n for n in names), names
    assert not any("pdec_kernel" in n for n in _kernels(lambda: ref.step(toks[0], 0, kr, vr)))
    for pos, t in enumerate(toks[1:], start=1):
        a = fast.step(t, pos, kf, vf)
        b = ref.step(t, pos, kr, vr)
        assert torch.equal(a, b), (pos, float((a - b).abs().max()))
    P = len(toks)
    assert torch.equal(kf[:, :P], kr[:, :P]) and torch.equal(vf[:, :P], vr[:, :P])


def test_persistent_generation_matches_and_oracle(pair):
    fast, ref, (b, m) = pair
    g = torch.Generator().manual_seed(3)
    prompt = torch.randint(3, 32000, (9,), generator=g).tolist()
    rf = fast.generate_greedy([prompt], 30)
    rr = ref.generate_greedy([prompt], 30)
    assert rf.sampled == rr.sampled
    orc = OracleModel.from_q6w(b, m)
    summary = BatchScorer(orc).verify_greedy([prompt], rf.sampled, 30)
    assert summary["failures"] == [], summary


def test_persistent_step_fp16_kv(tmp_path_factory):
    args = dict(fmt.SCALED_ARGS, n_layers=1, max_seq_len=32)
    b, m = small_model_files(tmp_path_factory, args, 10, "pdec16")
    fast = _persistent(b, m, kv_dtype=torch.float16)
    ref = Q6WCudaTransformer.from_q6w(b, m, kv_dtype=torch.float16)
    kf, vf = fast.new_cache()
    kr, vr = ref.new_cache()
    for pos, t in enumerate([5, 900, 31000, 17, 4242, 8]):
        a = fast.step(t, pos, kf, vf)
        b2 = ref.step(t, pos, kr, vr)
        assert torch.equal(a, b2), pos
    assert torch.equal(kf[:, :6], kr[:, :6])
