"""GPU: batched ragged prefill (q6w_prefill) against the oracle's own prompt
loop (CachedTransformer.step over every prompt position in order,
torch_benchmark.py:263-264).

Tolerances as the step tests: last-position logits within 2e-4 absolute of
the oracle, K/V cache rows within 1e-4, argmax the first maximum of the
device logits.
"""

import numpy as np
import pytest
import torch

from conftest import small_model_files
from oracle.model import OracleModel
from q6w_b200 import Q6WError
from q6w_b200 import format as fmt
from q6w_b200.model import Q6WCudaTransformer

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-4


def ragged(n, seed, lo, hi, vocab):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(lo, hi + 1, (n,), generator=g).tolist()
    return [torch.randint(3, vocab, (L,), generator=g).tolist() for L in lens]


def check_against_oracle(cuda, orc, prompts, sample):
    lg, (k, v) = cuda.prefill_batch(prompts)
    lg = lg.cpu()
    for i in sample:
        p = prompts[i]
        ko, vo = orc.new_cache()
        with torch.inference_mode():
            for pos, t in enumerate(p):
                want = orc.step(t, pos, ko, vo)
        assert float((lg[i] - want).abs().max()) <= LOGIT_TOL, i
        L = len(p)
        assert float((k[i, :, :L].cpu() - ko[:, :L]).abs().max()) <= 1e-4, i
        assert float((v[i, :, :L].cpu() - vo[:, :L]).abs().max()) <= 1e-4, i
    return lg


@pytest.fixture(scope="module")
def tiny_pair(tiny_files):
    return Q6WCudaTransformer.from_q6w(*tiny_files), OracleModel.from_q6w(*tiny_files)


def test_prefill_tensor_core_rows(tiny_pair):
    """~1100 token rows: the tensor-core step (tiny model) with the row ->
    prompt map in its QKV epilogue and attention."""
    cuda, orc = tiny_pair
    prompts = ragged(37, 5, 1, 60, 4096)
    check_against_oracle(cuda, orc, prompts, range(0, 37, 4))


def test_prefill_few_rows_and_argmax(tiny_pair):
    """15 token rows (SIMT linears), single-token prompts included; argmax of
    the last positions."""
    cuda, orc = tiny_pair
    prompts = [[7], [3, 9, 4000, 12, 5], [100 + i for i in range(9)]]
    lg = check_against_oracle(cuda, orc, prompts, range(3))
    pr = torch.zeros((3, 9), dtype=torch.int32)
    for i, p in enumerate(prompts):
        pr[i, : len(p)] = torch.tensor(p)
    ln = torch.tensor([len(p) for p in prompts], dtype=torch.int32)
    _, am, _, ws = cuda.prefill_batch_device(pr.cuda(), ln.cuda(), 9, 15)
    cuda.check_device_status(ws)
    assert torch.equal(am.cpu().long(), lg.argmax(1))


def test_prefill_simt_path(tiny_files, monkeypatch):
    monkeypatch.setenv("Q6W_DISABLE_TC", "1")
    cuda, orc = Q6WCudaTransformer.from_q6w(*tiny_files), OracleModel.from_q6w(*tiny_files)
    prompts = ragged(20, 6, 8, 50, 4096)
    check_against_oracle(cuda, orc, prompts, range(0, 20, 5))


@pytest.mark.parametrize("tag,args", [
    ("pf_ship", {"dim": 128, "n_layers": 2, "n_heads": 4, "n_kv_heads": 2, "vocab_size": 4096, "multiple_of": 32,
                 "max_seq_len": 512, "dropout": 0.0}),
    ("pf_scaled", dict(fmt.SCALED_ARGS, n_layers=1, max_seq_len=64)),
])
def test_prefill_other_head_layouts(tmp_path_factory, tag, args):
    """head_dim 32 (shipped shapes, 300-token prompt) and head_dim 64 (the
    1.1B-shape layer: per-head attention kernel with the row map)."""
    b, m = small_model_files(tmp_path_factory, args, 21, tag)
    cuda, orc = Q6WCudaTransformer.from_q6w(b, m), OracleModel.from_q6w(b, m)
    vocab = args["vocab_size"]
    if tag == "pf_ship":
        prompts = ragged(5, 8, 1, 40, vocab) + ragged(1, 9, 300, 300, vocab)
    else:
        prompts = ragged(6, 8, 1, 40, vocab)
    check_against_oracle(cuda, orc, prompts, range(len(prompts)))


def test_prefill_flags_bad_input(tiny_pair):
    """A total that does not match the lengths, and a token outside the
    vocabulary, are reported by the device status check."""
    cuda, _ = tiny_pair
    pr = torch.tensor([[5, 6, 7], [8, 9, 0]], dtype=torch.int32).cuda()
    ln = torch.tensor([3, 2], dtype=torch.int32).cuda()
    _, _, _, ws = cuda.prefill_batch_device(pr, ln, 3, 6)  # lengths sum to 5
    with pytest.raises(Q6WError):
        cuda.check_device_status(ws)
    pr2 = torch.tensor([[5, 99999, 7]], dtype=torch.int32).cuda()
    _, _, _, ws = cuda.prefill_batch_device(pr2, torch.tensor([3], dtype=torch.int32).cuda(), 3, 3)
    with pytest.raises(Q6WError):
        cuda.check_device_status(ws)
    cuda.check_device_status(ws)  # cleared
