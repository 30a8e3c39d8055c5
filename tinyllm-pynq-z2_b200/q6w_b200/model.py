"""Drop-in CUDA replacement for the reference's cached Q6 transformer.

``Q6WCudaTransformer`` offers the interface that ``generate`` / ``benchmark``
(benchmarks/torch_benchmark.py:233-395), ``compare_logits``
(quantization/evaluate_q6w.py:48-65) and the golden-request builder
(scripts/prepare_e2e.py:120-143) use on ``CachedTransformer``
(torch_benchmark.py:57-125): ``args``, ``hidden_dim``, ``eval()``, ``to()``,
``new_cache(device)`` and ``step(token_id, position, key_cache,
value_cache) -> logits``.  The weights stay packed on the GPU (the Q6W
file's bytes, unchanged); every op runs in the sm_100a kernels behind the C
ABI.  Batched entry points (``forward_batch``, ``generate_greedy``) serve
many independent sequences per call with the whole greedy loop on the
device.

There is no CPU path: constructing the model without a CUDA device or
without the compiled library raises.
"""

import tempfile
import time
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

from . import _lib
from . import format as fmt
from .format import Q6WImage, ffn_dim
from .ops import DeviceImage

MODEL_DEFAULTS = {"hidden_dim": None, "multiple_of": 256, "norm_eps": 1e-5, "n_kv_heads": None,
                  "max_seq_len": 2048, "dropout": 0.0}


def runtime_args(model_args, max_seq_len=None):
    """``model_args`` merged over the reference's defaults (torch_benchmark.py:447-455)."""
    args = SimpleNamespace(**{**MODEL_DEFAULTS, **model_args})
    if max_seq_len is not None:
        args.max_seq_len = int(max_seq_len)
    return args


def rope_tables(head_dim, max_seq_len):
    """RoPE cos/sin tables, built on the host with torch CPU exactly as the
    reference builds them (torch_benchmark.py:72-77), so the device reads the
    same FP32 values the reference uses.  [max_seq_len, head_dim // 2] each.
    """
    inv = 1.0 / (10000.0 ** (torch.arange(0, head_dim, 2).float() / head_dim))
    ang = torch.outer(torch.arange(max_seq_len).float(), inv)
    return torch.cos(ang), torch.sin(ang)


class GreedyResult(SimpleNamespace):
    """Per-sequence greedy output (host lists) plus optional device logits.

    ``sampled[i]``: every argmax pick of sequence i, including a final stop
    id (prepare_e2e.py ``reference_sampled_ids``); ``generated[i]``: the
    appended tokens (torch_benchmark.generate's list); ``stop_reason[i]``:
    the stop id or None.
    """


class Q6WCudaTransformer:
    """``kv_dtype``: torch.float32 (the reference's ``CachedTransformer``) or
    torch.float16 (its FP16-KV wrapper, quantization/compare_kv_cache.py:15-72:
    K/V rows stored as FP16, attention in FP32); the caches ``new_cache`` and
    ``new_batch_cache`` return have that dtype."""

    def __init__(self, image, device="cuda", max_seq_len=None, kv_dtype=torch.float32):
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("Q6WCudaTransformer runs on a CUDA device")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self._lib = _lib.load()
        self.device = device
        if kv_dtype not in (torch.float32, torch.float16):
            raise ValueError("kv_dtype must be torch.float32 or torch.float16")
        self._max_seq_len = max_seq_len
        self._ws = {}
        self._attach(image, kv_dtype)

    def _attach(self, image, kv_dtype):
        """Upload ``image`` and create the device model (replacing any earlier one)."""
        old = getattr(self, "_handle", None)
        self.image = image
        self.args = runtime_args(image.model_args, self._max_seq_len)
        a = self.args
        self.n_kv_heads = a.n_kv_heads or a.n_heads
        self.head_dim = a.dim // a.n_heads
        self.hidden_dim = ffn_dim(vars(a))
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            if old is not None and old.value:
                self._lib.q6w_model_destroy(old)
                self._handle = None
            self.dimg = DeviceImage(image, self.device)
            cos, sin = rope_tables(self.head_dim, a.max_seq_len)
            self.freqs_cos = cos.to(self.device)
            self.freqs_sin = sin.to(self.device)
            self._build_desc()
            handle = ctypes_void()
            _lib.check(self._lib.q6w_model_create(self._desc, handle), "q6w_model_create")
            self._handle = handle
        _lib.check(self._lib.q6w_model_set_kv_dtype(self._handle, 1 if kv_dtype == torch.float16 else 0),
                   "q6w_model_set_kv_dtype")
        self.kv_dtype = kv_dtype

    # -- construction ----------------------------------------------------------
    @classmethod
    def from_q6w(cls, binary_path, manifest_path, device="cuda", max_seq_len=None, kv_dtype=torch.float32):
        """Load a Q6W binary + manifest (SHA and header checked) onto ``device``."""
        return cls(Q6WImage(binary_path, manifest_path), device, max_seq_len, kv_dtype)

    def _qmat(self, name):
        packed, scales, rows, cols = self.dimg.qmat(name)
        return _lib.QMat(packed.data_ptr(), scales.data_ptr(), rows, cols)

    def _build_desc(self):
        a = self.args
        layers = (_lib.LayerWeights * a.n_layers)()
        for l in range(a.n_layers):
            p = f"layers.{l}."
            L = layers[l]
            for short, key in (("wq", "attention.wq"), ("wk", "attention.wk"), ("wv", "attention.wv"),
                               ("wo", "attention.wo"), ("w1", "feed_forward.w1"), ("w2", "feed_forward.w2"),
                               ("w3", "feed_forward.w3")):
                setattr(L, short, self._qmat(p + key + ".weight"))
            L.attention_norm = self.dimg.fp32(p + "attention_norm.weight").data_ptr()
            L.ffn_norm = self.dimg.fp32(p + "ffn_norm.weight").data_ptr()
        self._layers = layers
        d = _lib.ModelDesc()
        d.dim, d.n_layers, d.n_heads = a.dim, a.n_layers, a.n_heads
        d.n_kv_heads, d.vocab_size = self.n_kv_heads, a.vocab_size
        d.hidden_dim, d.max_seq_len, d.norm_eps = self.hidden_dim, a.max_seq_len, a.norm_eps
        d.tok_embeddings = self._qmat("tok_embeddings.weight")
        d.norm = self.dimg.fp32("norm.weight").data_ptr()
        d.rope_cos, d.rope_sin = self.freqs_cos.data_ptr(), self.freqs_sin.data_ptr()
        d.layers = layers
        self._desc = d

    def __del__(self):
        h = getattr(self, "_handle", None)
        if h is not None and h.value:
            try:
                self._lib.q6w_model_destroy(h)
            except Exception:
                pass

    # -- nn.Module-style no-ops kept for drop-in use ----------------------------
    def eval(self):
        return self

    def load_state_dict(self, state_dict, strict=True):
        """Take FP32 weights by name, as ``CachedTransformer.load_state_dict``
        does (evaluate_q6w.py:158-163): every quantized tensor is quantized and
        packed on this GPU with the reference's row rule (q6w_format.py:84-98),
        so the model equals what ``export_q6w`` + ``from_q6w`` give for the same
        weights; norm weights are used as given.  A state that holds a Q6W
        file's dequantized weights round-trips to the same codes, with scales
        within one rounding of the file's.

        The model needs every quantized and norm tensor, so missing keys raise
        whatever ``strict`` says; with ``strict``, keys the model does not have
        raise too (``output.weight``, tied to the embedding, is accepted when
        it equals ``tok_embeddings.weight``).  Returns (missing, unexpected)
        key lists, as torch does."""
        args = dict(self.image.model_args)
        n_layers = int(args["n_layers"])
        want = fmt.quant_keys(n_layers) + fmt.norm_keys(n_layers)
        missing = [k for k in want if k not in state_dict]
        unexpected = [k for k in state_dict if k not in want and k != "output.weight"]
        if "output.weight" in state_dict and "tok_embeddings.weight" in state_dict and not torch.equal(
                state_dict["output.weight"].detach().cpu(), state_dict["tok_embeddings.weight"].detach().cpu()):
            raise ValueError("output.weight must equal tok_embeddings.weight (the head is tied)")
        if missing:
            raise RuntimeError(f"state_dict lacks tensors the model needs: {missing[:4]}")
        if strict and unexpected:
            raise RuntimeError(f"unexpected keys in state_dict: {unexpected[:4]}")
        state = {k: state_dict[k].detach().float().contiguous() for k in want}
        with tempfile.TemporaryDirectory() as d:
            b, m = Path(d) / "state.bin", Path(d) / "state.json"
            fmt.write_q6w(state, args, b, m, {"load_state_dict": True}, device=self.device)
            image = Q6WImage(b, m)
        self._attach(image, self.kv_dtype)
        return SimpleNamespace(missing_keys=[], unexpected_keys=unexpected)

    def to(self, device):
        if torch.device(device) != self.device and not (torch.device(device).type == "cuda" and torch.device(device).index is None):
            raise ValueError("Q6WCudaTransformer is bound to the device it was loaded on")
        return self

    def __call__(self, *a, **k):
        return self.step(*a, **k)

    # -- workspace -------------------------------------------------------------
    def workspace(self, n_seqs):
        """Zeroed device scratch for up to n_seqs sequences (cached by size)."""
        need = int(self._lib.q6w_workspace_bytes(self._handle, int(n_seqs)))
        for cap, buf in self._ws.items():
            if cap >= n_seqs:
                return buf, buf.numel()
        buf = torch.zeros(need + 256, dtype=torch.uint8, device=self.device)
        off = (-buf.data_ptr()) % 256
        buf = buf[off: off + need]
        self._ws = {n_seqs: buf}
        return buf, need

    def check_device_status(self, ws):
        """Raise if a kernel flagged an out-of-range token/position (synchronises)."""
        _lib.check(self._lib.q6w_workspace_status(ws.data_ptr(), _lib.stream_handle()), "device status")

    # -- reference API -----------------------------------------------------------
    def new_cache(self, device=None):
        """(K, V), each [n_layers, max_seq_len, n_kv_heads, head_dim] FP32 (torch_benchmark.py:87-94)."""
        a = self.args
        shape = (a.n_layers, a.max_seq_len, self.n_kv_heads, self.head_dim)
        dev = self.device if device is None else torch.device(device)
        if dev.type != "cuda":
            raise ValueError("the KV cache must live on the model's CUDA device")
        return (torch.empty(shape, device=self.device, dtype=self.kv_dtype),
                torch.empty(shape, device=self.device, dtype=self.kv_dtype))

    def _check_cache(self, k, v, n=None):
        a = self.args
        shape = (a.n_layers, a.max_seq_len, self.n_kv_heads, self.head_dim)
        for c in (k, v):
            if c.dtype != self.kv_dtype or c.device != self.device or not c.is_contiguous():
                raise ValueError(f"KV cache must be contiguous {self.kv_dtype} on the model's device")
            if tuple(c.shape[-4:]) != shape or (n is not None and (c.dim() != 5 or c.shape[0] < n)):
                raise ValueError(f"KV cache shape {tuple(c.shape)} does not match {shape}")

    def step(self, token_id, position, key_cache, value_cache):
        """One cached step; returns logits [vocab] on the device (torch_benchmark.py:96-125)."""
        token_id, position = int(token_id), int(position)
        if not 0 <= position < self.args.max_seq_len:
            raise IndexError(f"position {position} is out of range for max_seq_len {self.args.max_seq_len}")
        if not 0 <= token_id < self.args.vocab_size:
            raise IndexError(f"token id {token_id} is out of range for vocab_size {self.args.vocab_size}")
        self._check_cache(key_cache, value_cache)
        logits = torch.empty(self.args.vocab_size, dtype=torch.float32, device=self.device)
        ws, nbytes = self.workspace(1)
        with torch.cuda.device(self.device):
            _lib.check(self._lib.q6w_step(self._handle, token_id, position, key_cache.data_ptr(),
                                          value_cache.data_ptr(), logits.data_ptr(), ws.data_ptr(), nbytes,
                                          _lib.stream_handle()), "q6w_step")
        return logits

    # -- batched API -------------------------------------------------------------
    def new_batch_cache(self, n_seqs):
        """(K, V), each [n_seqs, n_layers, max_seq_len, n_kv_heads, head_dim]; sequence i's
        slice is a ``new_cache`` cache."""
        a = self.args
        shape = (n_seqs, a.n_layers, a.max_seq_len, self.n_kv_heads, self.head_dim)
        return (torch.empty(shape, device=self.device, dtype=self.kv_dtype),
                torch.empty(shape, device=self.device, dtype=self.kv_dtype))

    def forward_batch(self, tokens, positions, key_cache, value_cache, logits=True, argmax=False):
        """One cached step of n independent sequences (device int32 tokens/positions).

        Returns (logits [n, vocab] or None, argmax [n] int32 or None).
        """
        n = int(tokens.numel())
        self._check_cache(key_cache, value_cache, n)
        tok = tokens.to(self.device, torch.int32).contiguous()
        pos = positions.to(self.device, torch.int32).contiguous()
        lg = torch.empty((n, self.args.vocab_size), dtype=torch.float32, device=self.device) if logits else None
        am = torch.empty(n, dtype=torch.int32, device=self.device) if argmax else None
        ws, nbytes = self.workspace(n)
        stride = key_cache[0].numel() if n > 0 else 0
        with torch.cuda.device(self.device):
            _lib.check(self._lib.q6w_forward_batch(
                self._handle, n, tok.data_ptr(), pos.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
                stride, lg.data_ptr() if lg is not None else None, am.data_ptr() if am is not None else None,
                ws.data_ptr(), nbytes, _lib.stream_handle()), "q6w_forward_batch")
        return lg, am

    def _prefill_workspace(self, n_prompts, total_tokens):
        need = int(self._lib.q6w_prefill_workspace_bytes(self._handle, int(n_prompts), int(total_tokens)))
        if need == 0:
            raise ValueError(f"{total_tokens} prompt tokens exceed the per-call prefill limit")
        buf = getattr(self, "_pws", None)
        if buf is None or buf.numel() < need:
            raw = torch.zeros(need + 256, dtype=torch.uint8, device=self.device)
            off = (-raw.data_ptr()) % 256
            buf = raw[off: off + need]
            self._pws = buf
        return buf, need

    def prefill_batch_device(self, prompts, prompt_lens, max_prompt_len, total_tokens, caches=None, logits=True,
                             argmax=True):
        """Batched prefill on device arrays (no host sync inside).

        ``prompts``: device int32 [n, stride]; ``prompt_lens``: device int32 [n];
        ``total_tokens``: the sum of the lengths.  Returns (last_logits
        [n, vocab] or None, last_argmax [n] or None, caches, workspace).
        """
        n = int(prompts.shape[0])
        if caches is None:
            caches = self.new_batch_cache(n)
        k, v = caches
        self._check_cache(k, v, n)
        lg = torch.empty((n, self.args.vocab_size), dtype=torch.float32, device=self.device) if logits else None
        am = torch.empty(n, dtype=torch.int32, device=self.device) if argmax else None
        ws, nbytes = self._prefill_workspace(n, total_tokens)
        with torch.cuda.device(self.device):
            _lib.check(self._lib.q6w_prefill(
                self._handle, n, prompts.data_ptr(), prompt_lens.data_ptr(), int(prompts.shape[1]),
                int(max_prompt_len), int(total_tokens), k.data_ptr(), v.data_ptr(), k[0].numel(),
                lg.data_ptr() if lg is not None else None, am.data_ptr() if am is not None else None,
                ws.data_ptr(), nbytes, _lib.stream_handle()), "q6w_prefill")
        return lg, am, caches, ws

    def prefill_batch(self, prompts):
        """Prefill a list of prompt id lists at once: (last_logits [B, vocab],
        (K, V) caches [B, n_layers, max_seq_len, n_kv_heads, head_dim]).

        The logits of prompt i equal those ``step`` returns at its last
        position after stepping through the prompt in order
        (torch_benchmark.py:263-264), and cache slice i equals that run's cache.
        """
        n = len(prompts)
        lens = [len(p) for p in prompts]
        if n == 0:
            raise ValueError("no prompts")
        if min(lens) < 1:
            raise ValueError("every prompt needs at least one token")
        if max(lens) > self.args.max_seq_len:
            raise ValueError("Prompt exceeds the model context")
        L = max(lens)
        host = np.zeros((n, L), dtype=np.int32)
        for i, p in enumerate(prompts):
            host[i, : len(p)] = p
        pr = torch.from_numpy(host).to(self.device)
        ln = torch.tensor(lens, dtype=torch.int32, device=self.device)
        lg, _, caches, ws = self.prefill_batch_device(pr, ln, L, sum(lens), argmax=False)
        self.check_device_status(ws)
        return lg, caches

    def forward_all(self, prompts, targets=None):
        """Logits of every position of each prompt (a list of [len, vocab]
        device tensors, views of one [sum(len), vocab] buffer) and, with
        ``targets`` (a list of id lists of the same lengths, -1 = ignored),
        the mean cross entropy as a device scalar -- the non-cached
        ``Transformer.forward(tokens, targets)`` of training/model.py:249-269
        on ragged prompts.  Returns (logits list, loss or None)."""
        n = len(prompts)
        lens = [len(p) for p in prompts]
        if n == 0 or min(lens) < 1:
            raise ValueError("every prompt needs at least one token")
        if max(lens) > self.args.max_seq_len:
            raise ValueError("Prompt exceeds the model context")
        if targets is not None and [len(t) for t in targets] != lens:
            raise ValueError("targets must have the prompts' lengths")
        L, total = max(lens), sum(lens)
        host = np.zeros((n, L), dtype=np.int32)
        th = np.full((n, L), -1, dtype=np.int32)
        for i, p in enumerate(prompts):
            host[i, : len(p)] = p
            if targets is not None:
                th[i, : len(p)] = targets[i]
        pr = torch.from_numpy(host).to(self.device)
        ln = torch.tensor(lens, dtype=torch.int32, device=self.device)
        tg = torch.from_numpy(th).to(self.device) if targets is not None else None
        k, v = self.new_batch_cache(n)
        logits = torch.empty((total, self.args.vocab_size), dtype=torch.float32, device=self.device)
        loss = torch.empty(1, dtype=torch.float32, device=self.device) if targets is not None else None
        ws, nbytes = self._prefill_workspace(n, total)
        with torch.cuda.device(self.device):
            _lib.check(self._lib.q6w_forward_all(
                self._handle, n, pr.data_ptr(), ln.data_ptr(), L, L, total, k.data_ptr(), v.data_ptr(),
                k[0].numel(), logits.data_ptr(), tg.data_ptr() if tg is not None else None,
                loss.data_ptr() if loss is not None else None, ws.data_ptr(), nbytes, _lib.stream_handle()),
                "q6w_forward_all")
        self.check_device_status(ws)
        return list(torch.split(logits, lens)), (loss[0] if loss is not None else None)

    def forward(self, tokens, targets=None):
        """``Transformer.forward`` of training/model.py:249-269 on a [B, T]
        token batch: with ``targets`` ([B, T], -1 ignored) the logits of every
        position [B, T, vocab] and ``self.last_loss`` = the mean cross
        entropy; without, the last position's logits [B, 1, vocab] and
        ``last_loss`` None."""
        tok = torch.as_tensor(tokens)
        if tok.dim() != 2:
            raise ValueError("tokens must be [batch, seq_len]")
        rows = tok.tolist()
        if targets is None:
            lg, _ = self.prefill_batch(rows)
            self.last_loss = None
            return lg[:, None, :]
        lg, loss = self.forward_all(rows, torch.as_tensor(targets).tolist())
        self.last_loss = loss
        return torch.stack(lg)

    def generate_greedy_device(self, prompts, prompt_lens, max_prompt_len, new_tokens, stop_ids=(),
                               min_new_tokens=0, caches=None, keep_logits=False, prefill_event=None, sampling=None):
        """Device-resident generation (no host sync inside).

        ``prompts``: device int32 [n, stride]; ``prompt_lens``: device int32 [n].
        ``sampling``: None (greedy) or a ``sampling_args(...)`` dict (the
        reference's temperature / top-p sampler and logit processors, one
        seed per sequence).  Returns device tensors (sampled [n, new_tokens],
        n_sampled [n], stop_reason [n], step_logits or None, caches, workspace).
        Does not synchronise.
        """
        n = int(prompts.shape[0])
        if caches is None:
            caches = self.new_batch_cache(n)
        k, v = caches
        self._check_cache(k, v, n)
        dev = self.device
        sampled = torch.empty((n, new_tokens), dtype=torch.int32, device=dev)
        n_sampled = torch.empty(n, dtype=torch.int32, device=dev)
        stop_reason = torch.empty(n, dtype=torch.int32, device=dev)
        step_logits = (torch.empty((n, new_tokens, self.args.vocab_size), dtype=torch.float32, device=dev)
                       if keep_logits else None)
        ws, nbytes = self.workspace(n)
        stop = sorted(set(int(t) for t in stop_ids))
        arr = (_lib.c_int32 * max(1, len(stop)))(*stop) if stop else None
        ga = _lib.GreedyArgs()
        ga.n_seqs = n
        ga.prompts, ga.prompt_lens = prompts.data_ptr(), prompt_lens.data_ptr()
        ga.prompt_stride, ga.max_prompt_len, ga.new_tokens = int(prompts.shape[1]), int(max_prompt_len), int(new_tokens)
        ga.stop_ids = arr
        ga.n_stop, ga.min_new_tokens = len(stop), int(min_new_tokens)
        ga.sampled, ga.n_sampled, ga.stop_reason = sampled.data_ptr(), n_sampled.data_ptr(), stop_reason.data_ptr()
        ga.k_cache, ga.v_cache = k.data_ptr(), v.data_ptr()
        ga.cache_seq_stride = k[0].numel()
        ga.step_logits = step_logits.data_ptr() if step_logits is not None else None
        if prefill_event is not None and not prefill_event.cuda_event:
            with torch.cuda.device(dev):
                prefill_event.record()  # torch creates the CUDA event on its first record
        ga.prefill_event = prefill_event.cuda_event if prefill_event is not None else None
        sa = None
        if sampling is not None:
            seeds = sampling["seeds"]
            if seeds.numel() != n:
                raise ValueError("one seed per sequence")
            seeds = seeds.to(dev, torch.int64).contiguous()
            sa = _lib.SampleArgs(float(sampling["temperature"]), float(sampling["top_p"]),
                                 float(sampling["repetition_penalty"]), int(sampling["no_repeat_ngram_size"]),
                                 float(sampling["stop_token_bias"]), int(sampling["stop_token_bias_after"]),
                                 seeds.data_ptr())
            self._seeds = seeds  # alive until the init kernel has read it
        with torch.cuda.device(dev):
            if sa is None:
                _lib.check(self._lib.q6w_generate_greedy(self._handle, ga, ws.data_ptr(), nbytes,
                                                         _lib.stream_handle()), "q6w_generate_greedy")
            else:
                _lib.check(self._lib.q6w_generate(self._handle, ga, sa, ws.data_ptr(), nbytes, _lib.stream_handle()),
                           "q6w_generate")
        return sampled, n_sampled, stop_reason, step_logits, caches, ws

    def generate_sampled(self, prompts, new_tokens, seeds, stop_ids=(), min_new_tokens=0, temperature=0.0,
                         top_p=0.9, repetition_penalty=1.0, stop_token_bias=0.0, stop_token_bias_after=None,
                         no_repeat_ngram_size=0, keep_logits=False):
        """Generation with the reference's sampler for a list of prompts, one
        XorShift64 seed per prompt: each sequence follows
        torch_benchmark.generate (:233-296) with those arguments.  Host results
        as ``generate_greedy``."""
        bias_after = min_new_tokens if stop_token_bias_after is None else stop_token_bias_after
        if (repetition_penalty <= 0 or not np.isfinite(stop_token_bias) or min_new_tokens < 0
                or min_new_tokens > new_tokens or bias_after < 0 or no_repeat_ngram_size < 0):
            raise ValueError("repetition_penalty must be positive, stop_token_bias finite, min_new_tokens within the "
                             "limit, and bias/ngram settings nonnegative")
        seeds = [int(s) & ((1 << 64) - 1) for s in seeds]
        if len(seeds) != len(prompts):
            raise ValueError("one seed per prompt")
        signed = [s - (1 << 64) if s >= (1 << 63) else s for s in seeds]  # int64 storage of the u64 seeds
        sampling = sampling_args(temperature, top_p, repetition_penalty, no_repeat_ngram_size,
                                 stop_token_bias if stop_ids else 0.0, bias_after,
                                 torch.tensor(signed, dtype=torch.int64, device=self.device))
        return self.generate_greedy(prompts, new_tokens, stop_ids, min_new_tokens, keep_logits, sampling=sampling)

    def decode_greedy_batch(self, prompts, new_tokens, stop_ids=None, min_new_tokens=0):
        """Batched greedy decode of a list of prompt id lists: (ids,
        per_step_argmax).  ids[b] is what ``torch_benchmark.generate`` returns
        for request b at temperature 0 (at most ``new_tokens`` ids, a stop id
        not appended); per_step_argmax[b] is the argmax of every decode step
        (the stop id, when one ended the request, last)."""
        r = self.generate_greedy(prompts, new_tokens, tuple(stop_ids or ()), min_new_tokens)
        return r.generated, r.sampled

    def generate_greedy(self, prompts, new_tokens, stop_ids=(), min_new_tokens=0, keep_logits=False, sampling=None):
        """Greedy generation for a list of prompt id lists; host results.

        Contract of prepare_e2e.py:121-143 / torch_benchmark.generate at
        temperature 0, per sequence (``sampling``: see ``generate_sampled``).
        """
        n = len(prompts)
        if n == 0:
            return GreedyResult(sampled=[], generated=[], stop_reason=[], logits=None)
        lens = [len(p) for p in prompts]
        if min(lens) < 1:
            raise ValueError("every prompt needs at least one token")
        if max(lens) + new_tokens - 1 > self.args.max_seq_len:
            raise ValueError("Prompt plus requested generation exceeds the model context")
        if not 0 <= min_new_tokens <= new_tokens:
            raise ValueError("min_new_tokens must be within the token limit")
        L = max(lens)
        host = np.zeros((n, L), dtype=np.int32)
        for i, p in enumerate(prompts):
            host[i, : len(p)] = p
        pr = torch.from_numpy(host).to(self.device)
        ln = torch.tensor(lens, dtype=torch.int32, device=self.device)
        sampled, n_sampled, stop_reason, logits, caches, ws = self.generate_greedy_device(
            pr, ln, L, new_tokens, stop_ids, min_new_tokens, keep_logits=keep_logits, sampling=sampling)
        self.check_device_status(ws)
        s = sampled.cpu().numpy()
        ns = n_sampled.cpu().numpy()
        sr = stop_reason.cpu().numpy()
        out_s, out_g, out_r = [], [], []
        for i in range(n):
            picks = s[i, : ns[i]].tolist()
            out_s.append(picks)
            stopped = int(sr[i]) >= 0
            out_g.append(picks[:-1] if stopped else picks)
            out_r.append(int(sr[i]) if stopped else None)
        return GreedyResult(sampled=out_s, generated=out_g, stop_reason=out_r, logits=logits, caches=caches,
                            n_sampled=ns)


def ctypes_void():
    import ctypes

    return ctypes.c_void_p()


def sampling_args(temperature, top_p, repetition_penalty, no_repeat_ngram_size, stop_token_bias,
                  stop_token_bias_after, seeds):
    """The sampler settings of one generation call (q6w_sample_args); ``seeds``
    a device int64 tensor holding each sequence's 64-bit XorShift64 seed."""
    return {"temperature": temperature, "top_p": top_p, "repetition_penalty": repetition_penalty,
            "no_repeat_ngram_size": no_repeat_ngram_size, "stop_token_bias": stop_token_bias,
            "stop_token_bias_after": stop_token_bias_after, "seeds": seeds}


def generate(model, prompt_ids, new_tokens, device=None, stop_token=None, temperature=0.0, top_p=0.9, seed=1,
             repetition_penalty=1.0, min_new_tokens=0, stop_token_bias=0.0, stop_token_bias_after=None,
             no_repeat_ngram_size=0):
    """``torch_benchmark.generate`` (benchmarks/torch_benchmark.py:233-296) on the device.

    Same signature, argument checks and return value ``(generated,
    prefill_seconds, decode_seconds, stopped, stop_reason)``.  The whole
    request runs as one device-resident loop: greedy decoding, or the
    reference's sampler (XorShift64 seeded with ``seed``, temperature and
    top-p, repetition penalty, n-gram blocking, stop-id masking and bias) in
    the step graph.  Prefill and decode times come from CUDA events.
    """
    import math

    bias_after = min_new_tokens if stop_token_bias_after is None else stop_token_bias_after
    if (repetition_penalty <= 0 or not math.isfinite(stop_token_bias) or min_new_tokens < 0
            or min_new_tokens > new_tokens or bias_after < 0 or no_repeat_ngram_size < 0):
        raise ValueError("repetition_penalty must be positive, stop_token_bias finite, min_new_tokens within the "
                         "limit, and bias/ngram settings nonnegative")
    if new_tokens < 1:
        return [], 0.0, 0.0, False, None
    stops = () if stop_token is None else (tuple(stop_token) if isinstance(stop_token, (set, tuple, list))
                                          else (stop_token,))
    P = len(prompt_ids)
    dev = model.device
    sampling = None
    if temperature != 0 or repetition_penalty != 1.0 or no_repeat_ngram_size != 0 or (stops and stop_token_bias != 0):
        s = int(seed) & ((1 << 64) - 1)
        sampling = sampling_args(temperature, top_p, repetition_penalty, no_repeat_ngram_size,
                                 stop_token_bias if stops else 0.0, bias_after,
                                 torch.tensor([s - (1 << 64) if s >= (1 << 63) else s], dtype=torch.int64, device=dev))
    pr = torch.tensor([list(prompt_ids)], dtype=torch.int32, device=dev)
    ln = torch.tensor([P], dtype=torch.int32, device=dev)
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    torch.cuda.synchronize(dev)
    e0.record()
    e1.record()  # creates the event; the device loop re-records it after the prefill steps
    sampled, n_sampled, stop_reason, _, _, ws = model.generate_greedy_device(
        pr, ln, P, new_tokens, stops, min_new_tokens, prefill_event=e1, sampling=sampling)
    e2.record()
    model.check_device_status(ws)
    picks = sampled[0, : int(n_sampled[0])].tolist()
    reason = int(stop_reason[0])
    stopped = reason >= 0
    generated = picks[:-1] if stopped else picks
    return generated, e0.elapsed_time(e1) / 1e3, e1.elapsed_time(e2) / 1e3, stopped, (reason if stopped else None)
