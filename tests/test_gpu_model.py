"""GPU: the cached step, the batched step and the device greedy loop against
the oracle (and through it, the reference's golden requests).

Tolerances: logits within 2e-4 absolute of the oracle (the reference's own
cached-vs-uncached check, benchmarks/torch_benchmark.py:316); greedy token
ids and per-step argmaxes exactly equal on the golden requests; batched
device streams verified by teacher forcing (every pick is the oracle's
argmax, or an FP32 near-tie within 1e-4 of the oracle's maximum, and the
stop/length contract holds).
"""

import numpy as np
import pytest
import torch

from conftest import GOLDEN, small_model_files
from oracle.model import BatchScorer, OracleModel, greedy_request
from q6w_b200 import format as fmt
from q6w_b200 import generate, ops
from q6w_b200.model import Q6WCudaTransformer

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-4


@pytest.fixture(scope="module")
def tiny(tiny_files):
    return Q6WCudaTransformer.from_q6w(*tiny_files), OracleModel.from_q6w(*tiny_files)


def test_step_logits_match_oracle(tiny, golden_tiny):
    cuda, orc = tiny
    k, v = cuda.new_cache()
    ko, vo = orc.new_cache()
    worst = 0.0
    with torch.inference_mode():
        for pos, tok in enumerate(golden_tiny["prompt"]):
            a = cuda.step(tok, pos, k, v).cpu()
            b = orc.step(tok, pos, ko, vo)
            worst = max(worst, float((a - b).abs().max()))
    assert worst <= LOGIT_TOL
    ref = np.load(GOLDEN / "tiny_logits.npz")["prompt_last"]
    assert np.abs(a.numpy() - ref).max() <= LOGIT_TOL
    # cache contents: rotated keys and raw values of every prompt position
    P = len(golden_tiny["prompt"])
    assert (k[:, :P].cpu() - ko[:, :P]).abs().max() <= 1e-4
    assert (v[:, :P].cpu() - vo[:, :P]).abs().max() <= 1e-4


def test_drop_in_host_loop_is_token_exact(tiny, golden_tiny):
    """The oracle's own greedy loop driving Q6WCudaTransformer.step."""
    cuda, _ = tiny
    out = greedy_request(cuda, golden_tiny["prompt"], golden_tiny["new_tokens"])
    assert out["generated"] == golden_tiny["generated"]


def test_generate_device_loop_is_token_exact(tiny, golden_tiny):
    cuda, _ = tiny
    gen, pre_s, dec_s, stopped, reason = generate(cuda, golden_tiny["prompt"], golden_tiny["new_tokens"], cuda.device)
    assert gen == golden_tiny["generated"] and not stopped and reason is None
    assert pre_s > 0 and dec_s > 0


def test_generate_stop_contract(tiny, golden_tiny):
    cuda, _ = tiny
    case = golden_tiny["stop_case"]
    res = cuda.generate_greedy([golden_tiny["prompt"]], golden_tiny["new_tokens"], case["stop_ids"],
                               case["min_new_tokens"], keep_logits=True)
    assert res.sampled[0] == case["sampled"]
    assert res.generated[0] == case["generated"]
    assert res.stop_reason[0] == case["stopped_on"]
    first = np.load(GOLDEN / "tiny_logits.npz")["stop_run_first"]
    assert np.abs(res.logits[0, 0].cpu().numpy() - first).max() <= LOGIT_TOL


def test_generate_matches_reference_signature_errors(tiny):
    cuda, _ = tiny
    with pytest.raises(ValueError):
        generate(cuda, [5, 6], 4, cuda.device, min_new_tokens=5)
    with pytest.raises(ValueError):
        generate(cuda, [5, 6], 4, cuda.device, temperature=0.7, repetition_penalty=-1.0)
    with pytest.raises(ValueError):
        cuda.generate_greedy([[1] * 250], 10)  # exceeds the 256-position context


def test_step_range_errors(tiny):
    cuda, _ = tiny
    k, v = cuda.new_cache()
    with pytest.raises(IndexError):
        cuda.step(1, cuda.args.max_seq_len, k, v)
    with pytest.raises(IndexError):
        cuda.step(cuda.args.vocab_size, 0, k, v)


def test_forward_batch_bad_token_flagged(tiny):
    cuda, _ = tiny
    k, v = cuda.new_batch_cache(3)
    toks = torch.tensor([5, 99999, 7], dtype=torch.int32, device="cuda")
    pos = torch.zeros(3, dtype=torch.int32, device="cuda")
    lg, _ = cuda.forward_batch(toks, pos, k, v)
    ws, _ = cuda.workspace(3)
    from q6w_b200 import Q6WError

    with pytest.raises(Q6WError):
        cuda.check_device_status(ws)
    cuda.check_device_status(ws)  # cleared


@pytest.mark.parametrize("n", [1, 3, 8, 37, 200])
def test_forward_batch_matches_oracle(tiny, n):
    cuda, orc = tiny
    g = torch.Generator().manual_seed(n)
    T = 6
    toks = torch.randint(0, 4096, (T, n), generator=g)
    k, v = cuda.new_batch_cache(n)
    for t in range(T):
        lg, am = cuda.forward_batch(toks[t].int().cuda(), torch.full((n,), t, dtype=torch.int32).cuda(), k, v,
                                    argmax=True)
    # ragged positions: re-run some sequences at an earlier position
    pos = torch.tensor([T if i % 3 else T - 3 for i in range(n)], dtype=torch.int32)
    last = torch.randint(0, 4096, (n,), generator=g)
    lg, am = cuda.forward_batch(last.int().cuda(), pos.cuda(), k, v, argmax=True)
    lg = lg.cpu()
    assert torch.equal(am.cpu().long(), lg.argmax(dim=1))
    for i in range(0, n, max(1, n // 12)):
        ko, vo = orc.new_cache()
        with torch.inference_mode():
            for t in range(T):
                orc.step(int(toks[t, i]), t, ko, vo)
            want = orc.step(int(last[i]), int(pos[i]), ko, vo)
        assert float((lg[i] - want).abs().max()) <= LOGIT_TOL, i


def _ragged_prompts(n, seed, lo=1, hi=40):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(lo, hi + 1, (n,), generator=g).tolist()
    return [torch.randint(3, 4096, (L,), generator=g).tolist() for L in lens]


@pytest.mark.parametrize("n,new", [(64, 24), (600, 12)])
def test_generate_batch_teacher_forced(tiny, n, new):
    cuda, orc = tiny
    prompts = _ragged_prompts(n, n)
    res = cuda.generate_greedy(prompts, new)
    idx = list(range(0, n, max(1, n // 64)))
    summary = BatchScorer(orc).verify_greedy([prompts[i] for i in idx], [res.sampled[i] for i in idx], new)
    assert summary["failures"] == [], summary["failures"][:5]
    assert summary["exact"] >= 0.99 * summary["picks"]
    assert all(len(s) == new for s in res.sampled)


def test_generate_batch_with_stops(tiny, golden_tiny):
    cuda, orc = tiny
    case = golden_tiny["stop_case"]
    prompts = _ragged_prompts(16, 3) + [golden_tiny["prompt"]]
    res = cuda.generate_greedy(prompts, 60, case["stop_ids"], case["min_new_tokens"])
    assert res.sampled[-1] == case["sampled"][:60] or res.sampled[-1] == case["sampled"]
    summary = BatchScorer(orc).verify_greedy(prompts, res.sampled, 60, case["stop_ids"], case["min_new_tokens"])
    assert summary["failures"] == []


@pytest.fixture(scope="module")
def shipped_shape(tmp_path_factory):
    """Synthetic model with the shipped artifact's shapes: 4 q heads, 2 kv heads,
    head_dim 32, hidden 352 (from the multiple_of rule), context 512."""
    args = {"dim": 128, "n_layers": 5, "n_heads": 4, "n_kv_heads": 2, "vocab_size": 4096, "multiple_of": 32,
            "max_seq_len": 512, "dropout": 0.0}
    b, m = small_model_files(tmp_path_factory, args, 77, "shipshape")
    return Q6WCudaTransformer.from_q6w(b, m), OracleModel.from_q6w(b, m)


def test_shipped_shapes_parity(shipped_shape):
    cuda, orc = shipped_shape
    assert cuda.hidden_dim == 352
    prompt = _ragged_prompts(1, 11, 20, 20)[0]
    want = greedy_request(orc, prompt, 48)
    res = cuda.generate_greedy([prompt], 48)
    assert res.generated[0] == want["generated"]
    k, v = cuda.new_cache()
    ko, vo = orc.new_cache()
    for p, t in enumerate(prompt[:5]):
        a = cuda.step(t, p, k, v).cpu()
        b = orc.step(t, p, ko, vo)
    assert float((a - b).abs().max()) <= LOGIT_TOL


def test_scaled_shapes_parity(tmp_path_factory):
    """The 1.1B-shape config's matrices (dim 2048, 32 heads, 4 kv heads,
    hidden 5632, vocab 32000) with one layer, against the oracle."""
    args = dict(fmt.SCALED_ARGS, n_layers=1, max_seq_len=32)
    b, m = small_model_files(tmp_path_factory, args, 5, "scaled1")
    cuda, orc = Q6WCudaTransformer.from_q6w(b, m), OracleModel.from_q6w(b, m)
    k, v = cuda.new_cache()
    ko, vo = orc.new_cache()
    prompt = [17, 2500, 31999, 4, 1234]
    for p, t in enumerate(prompt):
        a = cuda.step(t, p, k, v).cpu()
        with torch.inference_mode():
            bb = orc.step(t, p, ko, vo)
        assert float((a - bb).abs().max()) <= LOGIT_TOL
    # batched path on the same model (gemv n<=8 and tiled n>8 kernels)
    for n in (4, 20):
        kb, vb = cuda.new_batch_cache(n)
        for p, t in enumerate(prompt):
            lg, _ = cuda.forward_batch(torch.full((n,), t, dtype=torch.int32).cuda(),
                                       torch.full((n,), p, dtype=torch.int32).cuda(), kb, vb)
        assert float((lg.cpu() - bb).abs().max()) <= LOGIT_TOL
    # single-request device loop (streaming GEMVs in a captured graph), teacher-forced
    res = cuda.generate_greedy([prompt], 12)
    summary = BatchScorer(orc).verify_greedy([prompt], res.sampled, 12)
    assert summary["failures"] == []


def test_shipped_artifact_request(shipped_files_env, golden_shipped):
    cuda = Q6WCudaTransformer.from_q6w(*shipped_files_env)
    g = golden_shipped
    res = cuda.generate_greedy([g["prompt"]], g["new_tokens"], g["stop_ids"], g["min_new_tokens"])
    assert res.sampled[0] == g["sampled"]
    assert res.generated[0] == g["generated"]


@pytest.mark.parametrize("n,L,KV,rep,hd", [(5, 40, 4, 2, 16), (3, 300, 4, 8, 64), (2, 70, 2, 2, 128), (1, 256, 4, 8, 64)])
def test_gqa_attention_op(tiny, n, L, KV, rep, hd):
    """The public attention op against torch's softmax attention (head dims
    16 / 32 take the warp-per-sequence kernel, 64 / 128 the per-head kernel;
    300 positions exceed one pass of its 256 threads)."""
    torch.manual_seed(3 + hd)
    q = torch.randn(n, KV * rep, hd)
    kk = torch.randn(n, L, KV, hd)
    vv = torch.randn(n, L, KV, hd)
    lens = torch.tensor([1, 7, 40, 33, 12, L, L - 1][:n], dtype=torch.int32).clamp(max=L)
    if n <= 3:
        lens[-1] = L
    out = ops.gqa_attention(q.cuda(), kk.cuda(), vv.cuda(), lens.cuda(), rep).cpu()
    for i in range(n):
        T = int(lens[i])
        ks = kk[i, :T].permute(1, 0, 2).repeat_interleave(rep, 0)
        vs = vv[i, :T].permute(1, 0, 2).repeat_interleave(rep, 0)
        w = torch.softmax((q[i].unsqueeze(1) @ ks.transpose(1, 2)) / hd ** 0.5, -1)
        want = (w @ vs).squeeze(1)
        assert (out[i] - want).abs().max() <= 1e-5


@pytest.mark.parametrize("n,L,KV,rep,hd", [(40, 300, 4, 8, 64), (70, 70, 2, 4, 128), (64, 256, 4, 8, 64)])
def test_gqa_group_kernel_matches_per_head(tiny, n, L, KV, rep, hd):
    """With many (sequence, kv head) pairs the op runs one CTA per kv head for
    all of its query heads; that output is bit-identical to the per-head
    kernel's (the same sequences one at a time) and within 1e-5 of torch."""
    g = torch.Generator().manual_seed(11 + hd + n)
    q = torch.randn(n, KV * rep, hd, generator=g)
    kk = torch.randn(n, L, KV, hd, generator=g)
    vv = torch.randn(n, L, KV, hd, generator=g)
    lens = torch.randint(1, L + 1, (n,), generator=g, dtype=torch.int32)
    lens[0], lens[1] = L, 1
    out = ops.gqa_attention(q.cuda(), kk.cuda(), vv.cuda(), lens.cuda(), rep).cpu()
    for i in range(n):
        one = ops.gqa_attention(q[i : i + 1].cuda(), kk[i : i + 1].cuda(), vv[i : i + 1].cuda(),
                                lens[i : i + 1].cuda(), rep).cpu()
        assert torch.equal(out[i], one[0]), i
    for i in (0, 1, n // 2, n - 1):
        T = int(lens[i])
        ks = kk[i, :T].permute(1, 0, 2).repeat_interleave(rep, 0)
        vs = vv[i, :T].permute(1, 0, 2).repeat_interleave(rep, 0)
        w = torch.softmax((q[i].unsqueeze(1) @ ks.transpose(1, 2)) / hd ** 0.5, -1)
        assert (out[i] - (w @ vs).squeeze(1)).abs().max() <= 1e-5


@pytest.mark.parametrize("n", [64, 130, 513, 9600])
def test_tensor_core_step_matches_simt_step(tiny_files, monkeypatch, n):
    """The tcgen05 batched step (n >= 64) against the FP32 SIMT step on the
    same inputs, and both against the oracle on a sample of sequences.  Up to
    74 tiles of 128 sequences the residual + RMSNorm GEMM runs as 2-CTA
    clusters of column halves; 9600 sequences (75 tiles) take the one-CTA
    form on a 148-SM B200."""
    tc_model = Q6WCudaTransformer.from_q6w(*tiny_files)
    monkeypatch.setenv("Q6W_DISABLE_TC", "1")
    simt_model = Q6WCudaTransformer.from_q6w(*tiny_files)
    g = torch.Generator().manual_seed(100 + n)
    T = 5
    toks = torch.randint(0, 4096, (T, n), generator=g).int()
    outs = []
    for mdl in (tc_model, simt_model):
        k, v = mdl.new_batch_cache(n)
        for t in range(T):
            lg, am = mdl.forward_batch(toks[t].cuda(), torch.full((n,), t, dtype=torch.int32).cuda(), k, v,
                                       argmax=True)
        outs.append((lg.cpu(), am.cpu(), k[:, :, :T].cpu(), v[:, :, :T].cpu()))
    (a_lg, a_am, a_k, a_v), (b_lg, b_am, b_k, b_v) = outs
    assert float((a_lg - b_lg).abs().max()) <= LOGIT_TOL
    assert float((a_k - b_k).abs().max()) <= 1e-4 and float((a_v - b_v).abs().max()) <= 1e-4
    assert torch.equal(a_am.long(), a_lg.argmax(1))
    orc = OracleModel.from_q6w(*tiny_files)
    for i in (0, n // 2, n - 1):
        ko, vo = orc.new_cache()
        with torch.inference_mode():
            for t in range(T):
                want = orc.step(int(toks[t, i]), t, ko, vo)
        assert float((a_lg[i] - want).abs().max()) <= LOGIT_TOL


def test_b1_cluster_kernel_matches_graph_path(tiny_files, monkeypatch):
    """Single requests run as one cluster kernel; compare with the per-step
    CUDA-graph path on the same prompts (logits and KV caches) and verify the
    tokens against the oracle by teacher forcing."""
    fast = Q6WCudaTransformer.from_q6w(*tiny_files)
    monkeypatch.setenv("Q6W_DISABLE_B1", "1")
    graph = Q6WCudaTransformer.from_q6w(*tiny_files)
    orc = OracleModel.from_q6w(*tiny_files)
    prompts = _ragged_prompts(4, 21, 1, 60)
    new = 40
    picks = []
    for p in prompts:
        a = fast.generate_greedy([p], new, keep_logits=True)
        b = graph.generate_greedy([p], new, keep_logits=True)
        n = min(len(a.sampled[0]), len(b.sampled[0]))
        assert float((a.logits[0, :n] - b.logits[0, :n]).abs().max()) <= LOGIT_TOL
        T = len(p) + new - 1
        ka, va = a.caches
        kb, vb = b.caches
        assert float((ka[0, :, :T] - kb[0, :, :T]).abs().max()) <= 1e-4
        assert float((va[0, :, :T] - vb[0, :, :T]).abs().max()) <= 1e-4
        picks.append(a.sampled[0])
    summary = BatchScorer(orc).verify_greedy(prompts, picks, new)
    assert summary["failures"] == []


def test_b1_cluster_kernel_long_context(tmp_path_factory, monkeypatch):
    """A single request past 256 positions (shipped shapes, 512-position
    context): each thread of the cluster kernel's attention then holds two
    positions."""
    args = {"dim": 128, "n_layers": 5, "n_heads": 4, "n_kv_heads": 2, "vocab_size": 4096, "multiple_of": 32,
            "max_seq_len": 512, "dropout": 0.0}
    files = small_model_files(tmp_path_factory, args, 78, "longctx")
    fast = Q6WCudaTransformer.from_q6w(*files)
    monkeypatch.setenv("Q6W_DISABLE_B1", "1")
    graph = Q6WCudaTransformer.from_q6w(*files)
    orc = OracleModel.from_q6w(*files)
    p = _ragged_prompts(1, 77, 200, 200)[0]
    new = 300
    a = fast.generate_greedy([p], new, keep_logits=True)
    b = graph.generate_greedy([p], new, keep_logits=True)
    n = min(len(a.sampled[0]), len(b.sampled[0]))
    assert float((a.logits[0, :n] - b.logits[0, :n]).abs().max()) <= LOGIT_TOL
    summary = BatchScorer(orc).verify_greedy([p], [a.sampled[0]], new)
    assert summary["failures"] == []


@pytest.mark.parametrize("n", [16, 64, 100])
def test_general_tensor_core_step(tmp_path_factory, monkeypatch, n):
    """The general tcgen05 linears (weights as the MMA's M operand, the three
    bf16 activation parts stacked as N) on a 1.1B-shape layer: against the SIMT
    step on the same inputs and the oracle on a sample."""
    args = dict(fmt.SCALED_ARGS, n_layers=1, max_seq_len=16)
    b, m = small_model_files(tmp_path_factory, args, 5, f"tcg{n}")
    tc_model = Q6WCudaTransformer.from_q6w(b, m)
    monkeypatch.setenv("Q6W_DISABLE_TCG", "1")
    simt_model = Q6WCudaTransformer.from_q6w(b, m)
    orc = OracleModel.from_q6w(b, m)
    g = torch.Generator().manual_seed(200 + n)
    T = 4
    toks = torch.randint(0, args["vocab_size"], (T, n), generator=g).int()
    outs = []
    for mdl in (tc_model, simt_model):
        k, v = mdl.new_batch_cache(n)
        for t in range(T):
            lg, am = mdl.forward_batch(toks[t].cuda(), torch.full((n,), t, dtype=torch.int32).cuda(), k, v,
                                       argmax=True)
        outs.append((lg.cpu(), am.cpu(), k[:, :, :T].cpu(), v[:, :, :T].cpu()))
    (a_lg, a_am, a_k, a_v), (b_lg, b_am, b_k, b_v) = outs
    assert float((a_lg - b_lg).abs().max()) <= LOGIT_TOL
    assert float((a_k - b_k).abs().max()) <= 1e-4 and float((a_v - b_v).abs().max()) <= 1e-4
    assert torch.equal(a_am.long(), a_lg.argmax(1))
    for i in range(0, n, max(1, n // 4)):
        ko, vo = orc.new_cache()
        with torch.inference_mode():
            for t in range(T):
                want = orc.step(int(toks[t, i]), t, ko, vo)
        assert float((a_lg[i] - want).abs().max()) <= LOGIT_TOL, i


def test_dim128_wide_hidden_leaves_tensor_core_step(tmp_path_factory):
    """dim 128 with hidden 512 (multiple_of 256): the packed w2 rows of a
    128-row residual tile would not fit the tensor-core step's staging area,
    so the model takes the FP32 SIMT step, token-exact against the oracle."""
    from torch.profiler import ProfilerActivity, profile

    args = {"dim": 128, "n_layers": 2, "n_heads": 8, "n_kv_heads": 4, "vocab_size": 4096, "multiple_of": 256,
            "max_seq_len": 64, "dropout": 0.0}
    b, m = small_model_files(tmp_path_factory, args, 31, "wide_hidden")
    cuda, orc = Q6WCudaTransformer.from_q6w(b, m), OracleModel.from_q6w(b, m)
    assert cuda.hidden_dim == 512
    prompts = _ragged_prompts(96, 31, 4, 20)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        res = cuda.generate_greedy(prompts, 8)
        torch.cuda.synchronize()
    names = {e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA}
    assert not any("tc_gemm_kernel" in s for s in names), sorted(names)
    idx = list(range(0, 96, 8))
    summary = BatchScorer(orc).verify_greedy([prompts[i] for i in idx], [res.sampled[i] for i in idx], 8)
    assert summary["failures"] == [], summary["failures"][:5]
