"""Oracle restatement of the reference's sampler and sampled generation loop
(test infrastructure only).

Follows benchmarks/torch_benchmark.py:
* ``XorShift64``            -- :133-144 (64-bit xorshift, multiply, top 24 bits)
* ``sample_token``          -- :147-185 (temperature softmax; plain scan, or
                               nucleus over the probabilities sorted in
                               descending order above the cutoff)
* ``penalize_repeated``     -- :188-198
* ``bias_stop_tokens``      -- :201-208
* ``block_repeated_ngrams`` -- :211-230
* ``sampled_request``       -- the decode loop of ``generate`` :233-296
with the same torch CPU FP32 operations, so that on one machine it returns
the reference's tokens.  ``decision`` additionally reports how close each
sampling decision came to a boundary, which the device tests use to tell a
rounding-level difference in the probabilities from a real mismatch.
"""

import math

import torch
import torch.nn.functional as F

MASK64 = (1 << 64) - 1


class XorShift64:
    def __init__(self, seed):
        self.state = int(seed) & MASK64

    def random_f32(self):
        s = self.state
        s ^= s >> 12
        s ^= (s << 25) & MASK64
        s ^= s >> 27
        self.state = s
        value = (s * 0x2545F4914F6CDD1D) & MASK64
        return ((value >> 32) >> 8) / 16777216.0


def sample_token(logits, temperature, top_p, rng):
    """torch_benchmark.py:147-185; returns the token id."""
    return decision(logits, temperature, top_p, rng)["token"]


def decision(logits, temperature, top_p, rng):
    """The reference's sampling decision plus its distance to a boundary.

    ``margin``: the smallest gap, relative to the probability mass involved,
    between the sampled quantity (coin, or coin * nucleus mass) and the
    cumulative sum it was compared with, and between the nucleus sum and
    top_p; ``tie``: the pick sat in a group of equal probabilities (the
    reference's unstable sort orders such a group arbitrarily).
    """
    if temperature == 0:
        return {"token": int(torch.argmax(logits).item()), "margin": math.inf, "tie": False}
    probabilities = F.softmax(logits.float() / temperature, dim=-1)
    coin = rng.random_f32()
    probs = probabilities.tolist()
    if top_p <= 0 or top_p >= 1:
        cumulative = 0.0
        for token_id, p in enumerate(probs):
            prev = cumulative
            cumulative += p
            if coin < cumulative:
                m = min(coin - prev, cumulative - coin)
                return {"token": token_id, "margin": m, "tie": False}
        return {"token": len(probs) - 1, "margin": coin - cumulative, "tie": False}
    sorted_probabilities, sorted_ids = torch.sort(probabilities, descending=True)
    cutoff = (1.0 - top_p) / (probabilities.numel() - 1)
    keep = sorted_probabilities >= cutoff
    cand_p = sorted_probabilities[keep].tolist()
    cand_i = sorted_ids[keep].tolist()
    cumulative_probability = 0.0
    last_index = len(cand_p) - 1
    margin = math.inf
    for index, p in enumerate(cand_p):
        cumulative_probability += p
        if cumulative_probability > top_p:
            last_index = index
            margin = min(margin, cumulative_probability - top_p, top_p - (cumulative_probability - p))
            break
    target = coin * cumulative_probability
    cumulative = 0.0
    for index in range(last_index + 1):
        prev = cumulative
        cumulative += cand_p[index]
        if target < cumulative:
            margin = min(margin, target - prev, cumulative - target)
            tie = cand_p.count(cand_p[index]) > 1
            return {"token": cand_i[index], "margin": margin, "tie": tie}
    return {"token": cand_i[last_index], "margin": margin, "tie": False}


def penalize_repeated(logits, generated, repetition_penalty):
    """torch_benchmark.py:188-198."""
    if repetition_penalty == 1.0 or not generated:
        return logits
    adjusted = logits.clone()
    ids = torch.tensor(sorted(set(generated)), dtype=torch.long)
    rep = adjusted[ids]
    adjusted[ids] = torch.where(rep < 0, rep * repetition_penalty, rep / repetition_penalty)
    return adjusted


def bias_stop_tokens(logits, stop_tokens, stop_token_bias):
    """torch_benchmark.py:201-208 (stop_tokens a collection)."""
    if stop_tokens is None or stop_token_bias == 0:
        return logits
    adjusted = logits.clone()
    for t in stop_tokens:
        adjusted[t] += stop_token_bias
    return adjusted


def block_repeated_ngrams(logits, generated, ngram_size):
    """torch_benchmark.py:211-230."""
    if ngram_size == 0 or not generated:
        return logits
    if ngram_size == 1:
        banned = set(generated)
    elif len(generated) < ngram_size - 1:
        return logits
    else:
        prefix = generated[-(ngram_size - 1):]
        banned = {generated[i + ngram_size - 1] for i in range(len(generated) - ngram_size + 1)
                  if generated[i: i + ngram_size - 1] == prefix}
    if not banned:
        return logits
    adjusted = logits.clone()
    adjusted[torch.tensor(sorted(banned), dtype=torch.long)] = -torch.inf
    if not torch.isfinite(adjusted).any():
        return logits
    return adjusted


def process_logits(logits, generated, index, stop_tokens, min_new_tokens, bias_after, stop_token_bias,
                   repetition_penalty, no_repeat_ngram_size):
    """The logit shaping of one decode index, in the order of torch_benchmark.py:272-283."""
    out = penalize_repeated(logits, generated, repetition_penalty)
    out = block_repeated_ngrams(out, generated, no_repeat_ngram_size)
    if stop_tokens is not None:
        if index < min_new_tokens:
            out = out.clone()
            for t in stop_tokens:
                out[t] = -torch.inf
        elif index >= bias_after:
            out = bias_stop_tokens(out, stop_tokens, stop_token_bias)
    return out


def verify_sampled(scorer, prompts, streams, seeds, new_tokens, stop_token=None, temperature=0.0, top_p=0.9,
                   repetition_penalty=1.0, min_new_tokens=0, stop_token_bias=0.0, stop_token_bias_after=None,
                   no_repeat_ngram_size=0, margin_tol=1e-5, device_logits=None, logit_tol=2e-4):
    """Teacher-forced check of device sampled streams.

    ``scorer``: an ``oracle.model.BatchScorer``; ``streams[i]``: the device's
    picks for prompt i (a final stop id included).  At every step the oracle
    shapes the logits with the device stream's history, draws from its own
    XorShift64(seeds[i]) and makes the reference's decision; the device pick
    must equal it, or the decision must have been within ``margin_tol`` of a
    boundary (or inside an equal-probability group), where rounding-level
    differences in the probabilities may flip it.  Every stream must stop
    exactly where generate stops.

    With ``device_logits`` (per sequence, the raw logits row of every
    decode step, as the device computed it), the decision is made on those
    rows -- the sampler's own parity -- and each row must also be within
    ``logit_tol`` of the oracle's logits for that step.  Without it the
    oracle's logits are used, and ``margin_tol`` must cover the logit error
    as well.  Returns a summary dict.
    """
    a = scorer.args
    bias_after = min_new_tokens if stop_token_bias_after is None else stop_token_bias_after
    stops = None
    if stop_token is not None:
        stops = tuple(stop_token) if isinstance(stop_token, (set, tuple, list)) else (stop_token,)
    B = len(prompts)
    rngs = [XorShift64(s) for s in seeds]
    summary = {"picks": 0, "exact": 0, "boundary": 0, "failures": [], "min_margin": math.inf}
    feeds = []
    for i in range(B):
        s = list(streams[i])
        gen = s[:-1] if (stops and s and s[-1] in stops) else s
        feeds.append(list(prompts[i]) + gen[: new_tokens - 1])
    steps = max(len(f) for f in feeds)
    shape = (B, a.n_layers, a.max_seq_len, a.kv_heads, a.head_dim)
    kc, vc = torch.zeros(shape, dtype=scorer.m.kv_dtype), torch.zeros(shape, dtype=scorer.m.kv_dtype)
    with torch.inference_mode():
        for t in range(steps):
            live = [j for j in range(B) if t < len(feeds[j])]
            if not live:
                break
            logits = scorer._step(torch.tensor([feeds[j][t] for j in live]), torch.full((len(live),), t),
                                  kc, vc, torch.tensor(live))
            for r, j in enumerate(live):
                index = t - (len(prompts[j]) - 1)
                if index < 0 or index >= len(streams[j]):
                    continue
                history = list(streams[j][:index])
                row = logits[r]
                if device_logits is not None:
                    dev_row = torch.as_tensor(device_logits[j][index]).float()
                    err = float((dev_row - row).abs().max())
                    summary["max_logit_diff"] = max(summary.get("max_logit_diff", 0.0), err)
                    if err > logit_tol:
                        summary["failures"].append((j, index, "logits", err, None))
                    row = dev_row
                shaped = process_logits(row, history, index, stops, min_new_tokens, bias_after,
                                        stop_token_bias, repetition_penalty, no_repeat_ngram_size)
                d = decision(shaped, temperature, top_p, rngs[j])
                pick = int(streams[j][index])
                summary["picks"] += 1
                summary["min_margin"] = min(summary["min_margin"], d["margin"])
                if pick == d["token"]:
                    summary["exact"] += 1
                elif d["margin"] <= margin_tol or d["tie"]:
                    summary["boundary"] += 1
                else:
                    summary["failures"].append((j, index, pick, d["token"], d["margin"]))
    for j in range(B):
        s = list(streams[j])
        early = [n for n, tk in enumerate(s[:-1]) if stops and tk in stops]
        stopped = bool(stops) and bool(s) and s[-1] in stops
        if early or (not stopped and len(s) != new_tokens) or len(s) > new_tokens:
            summary["failures"].append((j, -1, "length/stop contract", len(s), None))
    return summary


def sampled_request(model, prompt_ids, new_tokens, stop_token=None, temperature=0.0, top_p=0.9, seed=1,
                    repetition_penalty=1.0, min_new_tokens=0, stop_token_bias=0.0, stop_token_bias_after=None,
                    no_repeat_ngram_size=0, keep_logits=False):
    """The prefill + decode loop of torch_benchmark.generate (:233-296) on an
    oracle model.  Returns dict(generated, stopped, stop_reason, decisions,
    logits) -- ``logits`` the raw rows each decision saw (when kept)."""
    bias_after = min_new_tokens if stop_token_bias_after is None else stop_token_bias_after
    stops = None
    if stop_token is not None:
        stops = tuple(stop_token) if isinstance(stop_token, (set, tuple, list)) else (stop_token,)
    k, v = model.new_cache()
    rng = XorShift64(seed)
    rows, decisions, generated = [], [], []
    stopped, reason = False, None
    with torch.inference_mode():
        logits = None
        for pos, tok in enumerate(prompt_ids):
            logits = model.step(int(tok), pos, k, v)
        for index in range(new_tokens):
            if keep_logits:
                rows.append(logits.clone())
            shaped = process_logits(logits, generated, index, stops, min_new_tokens, bias_after, stop_token_bias,
                                    repetition_penalty, no_repeat_ngram_size)
            d = decision(shaped, temperature, top_p, rng)
            decisions.append(d)
            t = d["token"]
            if stops is not None and t in stops:
                stopped, reason = True, t
                break
            generated.append(t)
            if index + 1 < new_tokens:
                logits = model.step(t, len(prompt_ids) + index, k, v)
    out = {"generated": generated, "stopped": stopped, "stop_reason": reason, "decisions": decisions}
    if keep_logits:
        out["logits"] = torch.stack(rows) if rows else torch.empty(0)
    return out
