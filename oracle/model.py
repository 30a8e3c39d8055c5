"""Oracle restatement of the cached Q6 transformer (test infrastructure only).

``OracleModel.step`` restates ``CachedTransformer.step``
(benchmarks/torch_benchmark.py:96-125) with torch CPU FP32 operators applied
in the same order and on the same tensor shapes as the reference, so that on
one machine it reproduces the reference's logits bit for bit.  The steps of
the algorithm (RMSNorm, per-pair RoPE, GQA attention over the cache, SwiGLU,
tied vocab head) necessarily match the reference; the code is organised as
plain functions over a weight dict.

``greedy_request`` restates the greedy contract shared by
``generate`` (torch_benchmark.py:233-296, temperature 0 branch of
``sample_token`` at :148-150) and the golden-request builder
(scripts/prepare_e2e.py:121-143): stop ids are masked to -inf before
``min_new_tokens`` tokens exist, argmax takes the first maximum, and a stop id
picked afterwards ends the request without being appended.

``BatchScorer`` runs the same model over many sequences at once (batched
matmuls: a different FP32 summation order, so agreement with the B=1 path is
within tolerance rather than bitwise) and verifies a device-produced token
stream by teacher forcing.
"""

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .codec import load_state


@dataclass
class OracleArgs:
    """Model arguments; defaults follow torch_benchmark.py:447-455."""

    dim: int
    n_layers: int
    n_heads: int
    vocab_size: int
    n_kv_heads: int = None
    hidden_dim: int = None
    multiple_of: int = 256
    norm_eps: float = 1e-5
    max_seq_len: int = 2048

    @classmethod
    def from_model_args(cls, model_args, max_seq_len=None):
        keys = cls.__dataclass_fields__
        args = cls(**{k: v for k, v in model_args.items() if k in keys})
        if max_seq_len is not None:
            args.max_seq_len = int(max_seq_len)
        return args

    @property
    def kv_heads(self):
        return self.n_heads if self.n_kv_heads is None else self.n_kv_heads

    @property
    def head_dim(self):
        return self.dim // self.n_heads

    @property
    def ffn_dim(self):
        """Hidden width rule of torch_benchmark.py:61-64."""
        if self.hidden_dim is not None:
            return self.hidden_dim
        h = int(2 * (4 * self.dim) / 3)
        return self.multiple_of * ((h + self.multiple_of - 1) // self.multiple_of)


def rope_tables(args):
    """cos/sin tables of torch_benchmark.py:72-77, [max_seq_len, head_dim/2] f32."""
    hd = args.head_dim
    inv_freq = 1.0 / (10000.0 ** (torch.arange(0, hd, 2).float() / hd))
    ang = torch.outer(torch.arange(args.max_seq_len).float(), inv_freq)
    return torch.cos(ang), torch.sin(ang)


def _rms(x, weight, eps):
    # torch_benchmark.py:22-24
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).type_as(x) * weight


def _rotate_pairs(x, cos, sin):
    # torch_benchmark.py:79-85: rotate adjacent (2j, 2j+1) pairs
    re, im = x.float().reshape(*x.shape[:-1], -1, 2).unbind(-1)
    c = cos.view(1, 1, 1, -1)
    s = sin.view(1, 1, 1, -1)
    return torch.stack((re * c - im * s, re * s + im * c), dim=-1).flatten(-2).type_as(x)


class OracleModel:
    """B=1 cached transformer over dequantized Q6 weights (CPU, FP32).

    ``kv_dtype=torch.float16`` restates the reference's FP16-KV wrapper
    (quantization/compare_kv_cache.py:15-72): the cache holds FP16 (the new
    rows rounded by ``copy_``) and is read back with ``.float()``.
    """

    def __init__(self, args, state, kv_dtype=torch.float32):
        self.args = args
        self.w = {k: v.float().contiguous() for k, v in state.items()}
        self.freqs_cos, self.freqs_sin = rope_tables(args)
        self.hidden_dim = args.ffn_dim
        self.kv_dtype = kv_dtype

    @classmethod
    def from_q6w(cls, binary_path, manifest_path, max_seq_len=None, kv_dtype=torch.float32):
        state, manifest = load_state(binary_path, manifest_path)
        return cls(OracleArgs.from_model_args(manifest["model_args"], max_seq_len), state, kv_dtype)

    def new_cache(self, device="cpu"):
        """torch_benchmark.py:87-94 (zero-filled here; unread slots never matter)."""
        a = self.args
        shape = (a.n_layers, a.max_seq_len, a.kv_heads, a.head_dim)
        return torch.zeros(shape, dtype=self.kv_dtype), torch.zeros(shape, dtype=self.kv_dtype)

    def step(self, token_id, position, key_cache, value_cache):
        """One cached decode step; returns logits [vocab] (torch_benchmark.py:96-125)."""
        a, w = self.args, self.w
        H, KV, hd = a.n_heads, a.kv_heads, a.head_dim
        rep = H // KV
        x = F.embedding(torch.tensor([[token_id]], dtype=torch.long), w["tok_embeddings.weight"])
        cos, sin = self.freqs_cos[position], self.freqs_sin[position]
        denom = (a.dim // a.n_heads) ** 0.5
        for l in range(a.n_layers):
            p = f"layers.{l}."
            u = _rms(x, w[p + "attention_norm.weight"], a.norm_eps)
            q = F.linear(u, w[p + "attention.wq.weight"]).view(1, 1, H, hd)
            k = F.linear(u, w[p + "attention.wk.weight"]).view(1, 1, KV, hd)
            v = F.linear(u, w[p + "attention.wv.weight"]).view(1, 1, KV, hd)
            q = _rotate_pairs(q, cos, sin).transpose(1, 2)
            k = _rotate_pairs(k, cos, sin)
            key_cache[l, position].copy_(k[0, 0])
            value_cache[l, position].copy_(v[0, 0])
            ks = key_cache[l, : position + 1].float().permute(1, 0, 2).repeat_interleave(rep, dim=0).unsqueeze(0)
            vs = value_cache[l, : position + 1].float().permute(1, 0, 2).repeat_interleave(rep, dim=0).unsqueeze(0)
            att = torch.softmax((torch.matmul(q, ks.transpose(-2, -1)) / denom).float(), dim=-1).type_as(q)
            o = torch.matmul(att, vs).transpose(1, 2).contiguous().view(1, 1, -1)
            x = x + F.linear(o, w[p + "attention.wo.weight"])
            u = _rms(x, w[p + "ffn_norm.weight"], a.norm_eps)
            g = F.silu(F.linear(u, w[p + "feed_forward.w1.weight"])) * F.linear(u, w[p + "feed_forward.w3.weight"])
            x = x + F.linear(g, w[p + "feed_forward.w2.weight"])
        return F.linear(_rms(x, w["norm.weight"], a.norm_eps), w["output.weight"])[0, 0]


def masked_argmax(logits, index, stop_ids, min_new_tokens):
    """Greedy pick with early stop masking (prepare_e2e.py:132-136).

    ``torch.argmax`` returns the first index of the maximum.
    """
    scores = logits
    if stop_ids and index < min_new_tokens:
        scores = logits.clone()
        for t in stop_ids:
            scores[t] = -float("inf")
    return int(torch.argmax(scores).item())


def greedy_request(model, prompt_ids, new_tokens, stop_ids=(), min_new_tokens=0, keep_logits=False):
    """Prefill + greedy decode of one request (prepare_e2e.py:121-143).

    Returns a dict with ``sampled`` (every argmax, including a final stop id),
    ``generated`` (tokens appended, as returned by torch_benchmark.generate),
    ``stopped_on``, ``margins`` (top-1 minus top-2 of each sampled step's
    masked logits) and optionally ``logits`` (one row per sampled step).
    """
    stop_ids = sorted(set(int(t) for t in stop_ids))
    k, v = model.new_cache()
    with torch.inference_mode():
        logits = None
        for pos, tok in enumerate(prompt_ids):
            logits = model.step(int(tok), pos, k, v)
        sampled, generated, margins, rows = [], [], [], []
        stopped_on = None
        for index in range(new_tokens):
            if keep_logits:
                rows.append(logits.clone())
            t = masked_argmax(logits, index, stop_ids, min_new_tokens)
            scores = logits.clone()
            if stop_ids and index < min_new_tokens:
                scores[stop_ids] = -float("inf")
            top2 = torch.topk(scores, 2).values
            margins.append(float(top2[0] - top2[1]))
            sampled.append(t)
            if index >= min_new_tokens and t in stop_ids:
                stopped_on = t
                break
            generated.append(t)
            if index + 1 < new_tokens:
                logits = model.step(t, len(prompt_ids) + index, k, v)
    out = {"sampled": sampled, "generated": generated, "stopped_on": stopped_on, "margins": margins}
    if keep_logits:
        out["logits"] = torch.stack(rows) if rows else torch.empty(0)
    return out


def forward_all(model, token_rows, target_rows=None):
    """Logits of every position of each token row, and with targets the mean
    cross entropy over positions whose target is not -1: the non-cached
    ``Transformer.forward(tokens, targets)`` of training/model.py:249-269
    (F.cross_entropy(..., ignore_index=-1)), computed here with the cached
    step over each row (the same arithmetic up to summation order).
    Returns (list of [len, vocab] logits, loss or None)."""
    out = []
    with torch.inference_mode():
        for row in token_rows:
            k, v = model.new_cache()
            out.append(torch.stack([model.step(int(t), p, k, v) for p, t in enumerate(row)]))
        loss = None
        if target_rows is not None:
            tg = torch.cat([torch.as_tensor(t, dtype=torch.long) for t in target_rows])
            loss = float(F.cross_entropy(torch.cat(out), tg, ignore_index=-1))
    return out, loss


class BatchScorer:
    """Many-sequence FP32 CPU forward used to verify device token streams.

    Each sequence keeps a private cache laid out like ``new_cache``.  The
    linears run as batched ``F.linear`` calls and attention as padded,
    masked batched matmuls -- the same arithmetic as ``OracleModel.step``
    summed in a different order.
    """

    def __init__(self, model):
        self.m = model
        self.args = model.args

    def _step(self, tokens, positions, kc, vc, rows):
        a, w = self.args, self.m.w
        B = tokens.shape[0]
        H, KV, hd = a.n_heads, a.kv_heads, a.head_dim
        rep = H // KV
        denom = (a.dim // a.n_heads) ** 0.5
        x = F.embedding(tokens.view(B, 1), w["tok_embeddings.weight"])  # [B,1,dim]
        cos = self.m.freqs_cos[positions].view(B, 1, 1, -1)
        sin = self.m.freqs_sin[positions].view(B, 1, 1, -1)
        T = int(positions.max()) + 1
        mask = torch.arange(T).view(1, 1, 1, T) > positions.view(B, 1, 1, 1)

        def rot(t):
            re, im = t.reshape(*t.shape[:-1], -1, 2).unbind(-1)
            return torch.stack((re * cos - im * sin, re * sin + im * cos), dim=-1).flatten(-2)

        for l in range(a.n_layers):
            p = f"layers.{l}."
            u = _rms(x, w[p + "attention_norm.weight"], a.norm_eps)
            q = rot(F.linear(u, w[p + "attention.wq.weight"]).view(B, 1, H, hd)).transpose(1, 2)
            k = rot(F.linear(u, w[p + "attention.wk.weight"]).view(B, 1, KV, hd))
            v = F.linear(u, w[p + "attention.wv.weight"]).view(B, KV, hd)
            kc[rows, l, positions] = k[:, 0].to(kc.dtype)  # an FP16 cache rounds as copy_ does
            vc[rows, l, positions] = v.to(vc.dtype)
            ks = kc[rows, l, :T].float().permute(0, 2, 1, 3).repeat_interleave(rep, dim=1)  # [B,H,T,hd]
            vs = vc[rows, l, :T].float().permute(0, 2, 1, 3).repeat_interleave(rep, dim=1)
            sc = torch.matmul(q, ks.transpose(-2, -1)) / denom  # [B,H,1,T]
            sc = sc.masked_fill(mask, -float("inf"))
            o = torch.matmul(torch.softmax(sc, dim=-1), vs).transpose(1, 2).reshape(B, 1, -1)
            x = x + F.linear(o, w[p + "attention.wo.weight"])
            u = _rms(x, w[p + "ffn_norm.weight"], a.norm_eps)
            g = F.silu(F.linear(u, w[p + "feed_forward.w1.weight"])) * F.linear(u, w[p + "feed_forward.w3.weight"])
            x = x + F.linear(g, w[p + "feed_forward.w2.weight"])
        return F.linear(_rms(x, w["norm.weight"], a.norm_eps), w["output.weight"])[:, 0]

    def verify_greedy(self, prompts, sampled, new_tokens, stop_ids=(), min_new_tokens=0, tie_tol=1e-4, chunk=256):
        """Teacher-forced check of device greedy output.

        ``prompts``: list of prompt id lists.  ``sampled``: list of the
        device's argmax picks per sequence (as ``greedy_request['sampled']``).
        Every pick must be the oracle's masked argmax, or within ``tie_tol``
        of the oracle's maximum (an FP32 near-tie), and the stream must stop
        exactly where the greedy contract says.  Returns a summary dict;
        ``failures`` lists the violating (sequence, index) pairs.
        """
        a = self.args
        stop_ids = sorted(set(int(t) for t in stop_ids))
        summary = {"sequences": len(prompts), "picks": 0, "exact": 0, "near_ties": 0, "failures": [],
                   "min_margin": math.inf}
        for c0 in range(0, len(prompts), chunk):
            idx = list(range(c0, min(len(prompts), c0 + chunk)))
            feeds = []
            for i in idx:
                s = list(sampled[i])
                gen = s[:-1] if (stop_ids and s and s[-1] in stop_ids and len(s) - 1 >= min_new_tokens) else s
                feeds.append(list(prompts[i]) + gen[: new_tokens - 1])
            B = len(idx)
            steps = max(len(f) for f in feeds)
            shape = (B, a.n_layers, a.max_seq_len, a.kv_heads, a.head_dim)
            kc, vc = torch.zeros(shape, dtype=self.m.kv_dtype), torch.zeros(shape, dtype=self.m.kv_dtype)
            with torch.inference_mode():
                for t in range(steps):
                    live = [j for j in range(B) if t < len(feeds[j])]
                    if not live:
                        break
                    lv = torch.tensor(live)
                    toks = torch.tensor([feeds[j][t] for j in live])
                    pos = torch.full((len(live),), t, dtype=torch.long)
                    logits = self._step(toks, pos, kc, vc, lv)
                    for r, j in enumerate(live):
                        i = idx[j]
                        index = t - (len(prompts[i]) - 1)
                        if index < 0 or index >= len(sampled[i]):
                            continue
                        row = logits[r].clone()
                        if stop_ids and index < min_new_tokens:
                            row[stop_ids] = -float("inf")
                        pick = int(sampled[i][index])
                        best = int(torch.argmax(row))
                        top2 = torch.topk(row, 2).values
                        summary["picks"] += 1
                        summary["min_margin"] = min(summary["min_margin"], float(top2[0] - top2[1]))
                        if pick == best:
                            summary["exact"] += 1
                        elif float(row[best] - row[pick]) <= tie_tol:
                            summary["near_ties"] += 1
                        else:
                            summary["failures"].append((i, index, pick, best, float(row[best] - row[pick])))
            for j, i in enumerate(idx):
                s = list(sampled[i])
                stopped = bool(stop_ids) and s and s[-1] in stop_ids and len(s) - 1 >= min_new_tokens
                early_stop = [n for n, t in enumerate(s[:-1]) if t in stop_ids and n >= min_new_tokens]
                if early_stop or (not stopped and len(s) != new_tokens) or len(s) > new_tokens:
                    summary["failures"].append((i, -1, "length/stop contract", len(s), None))
        return summary
