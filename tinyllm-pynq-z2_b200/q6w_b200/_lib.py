"""ctypes binding of libq6w_b200.so (the C ABI declared in include/q6w_b200.h).

The library is loaded from this package directory.  There is no fallback:
if the shared object is missing or cannot be loaded, every entry point
raises ``Q6WLibraryError``.
"""

import ctypes
import os
from ctypes import POINTER, c_float, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path

LIB_NAME = "libq6w_b200.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

Q6W_OK = 0
Q6W_ERR_ARG = -1
Q6W_ERR_ALIGN = -2
Q6W_ERR_RANGE = -3
Q6W_ERR_CUDA = -4
Q6W_ERR_DEVICE = -5

# Every symbol include/q6w_b200.h declares.
EXPORTS = (
    "q6w_last_error", "q6w_abi_version", "q6w_unpack", "q6w_dequant", "q6w_linear",
    "q6w_model_create", "q6w_model_destroy", "q6w_workspace_bytes", "q6w_step",
    "q6w_forward_batch", "q6w_generate_greedy", "q6w_workspace_status", "q6w_linear_argmax",
    "q6w_rmsnorm", "q6w_gqa_attention", "q6w_linear_argmax_noalloc", "q6w_prefill_workspace_bytes",
    "q6w_prefill", "q6w_quantize_rows", "q6w_linear_workspace_bytes", "q6w_linear_ex", "q6w_generate",
    "q6w_sample", "q6w_model_set_kv_dtype", "q6w_forward_all", "q6w_selftest_wait_timeout",
)


class Q6WLibraryError(RuntimeError):
    pass


class Q6WError(RuntimeError):
    """A negative status from the library; ``.code`` holds it."""

    def __init__(self, code, message):
        super().__init__(f"{message} (status {code})")
        self.code = code


class QMat(ctypes.Structure):
    _fields_ = [("packed", c_void_p), ("scales", c_void_p), ("rows", c_int32), ("cols", c_int32)]


class LayerWeights(ctypes.Structure):
    _fields_ = [(n, QMat) for n in ("wq", "wk", "wv", "wo", "w1", "w2", "w3")] + [
        ("attention_norm", c_void_p), ("ffn_norm", c_void_p)]


class ModelDesc(ctypes.Structure):
    _fields_ = [("dim", c_int32), ("n_layers", c_int32), ("n_heads", c_int32), ("n_kv_heads", c_int32),
                ("vocab_size", c_int32), ("hidden_dim", c_int32), ("max_seq_len", c_int32),
                ("norm_eps", c_float), ("tok_embeddings", QMat), ("norm", c_void_p),
                ("rope_cos", c_void_p), ("rope_sin", c_void_p), ("layers", POINTER(LayerWeights))]


class SampleArgs(ctypes.Structure):
    _fields_ = [("temperature", c_float), ("top_p", ctypes.c_double), ("repetition_penalty", c_float),
                ("no_repeat_ngram_size", c_int32), ("stop_token_bias", c_float), ("stop_token_bias_after", c_int32),
                ("seeds", c_void_p)]


class GreedyArgs(ctypes.Structure):
    _fields_ = [("n_seqs", c_int32), ("prompts", c_void_p), ("prompt_lens", c_void_p),
                ("prompt_stride", c_int32), ("max_prompt_len", c_int32), ("new_tokens", c_int32),
                ("stop_ids", POINTER(c_int32)), ("n_stop", c_int32), ("min_new_tokens", c_int32),
                ("sampled", c_void_p), ("n_sampled", c_void_p), ("stop_reason", c_void_p),
                ("k_cache", c_void_p), ("v_cache", c_void_p), ("cache_seq_stride", c_int64),
                ("step_logits", c_void_p), ("prefill_event", c_void_p)]


_lib = None
_load_error = None


def _declare(lib):
    S = c_void_p  # stream
    sig = {
        "q6w_last_error": (ctypes.c_char_p, []),
        "q6w_abi_version": (c_int32, []),
        "q6w_unpack": (c_int32, [c_void_p, c_void_p, c_int64, c_int64, S]),
        "q6w_dequant": (c_int32, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, S]),
        "q6w_quantize_rows": (c_int32, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, S]),
        "q6w_linear_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64]),
        "q6w_linear_ex": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p,
                                    c_size_t, S]),
        "q6w_linear": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, S]),
        "q6w_model_create": (c_int32, [POINTER(ModelDesc), POINTER(c_void_p)]),
        "q6w_model_destroy": (None, [c_void_p]),
        "q6w_model_set_kv_dtype": (c_int32, [c_void_p, c_int32]),
        "q6w_workspace_bytes": (c_size_t, [c_void_p, c_int32]),
        "q6w_step": (c_int32, [c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, S]),
        "q6w_forward_batch": (c_int32, [c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                                        c_void_p, c_void_p, c_void_p, c_size_t, S]),
        "q6w_generate_greedy": (c_int32, [c_void_p, POINTER(GreedyArgs), c_void_p, c_size_t, S]),
        "q6w_generate": (c_int32, [c_void_p, POINTER(GreedyArgs), POINTER(SampleArgs), c_void_p, c_size_t, S]),
        "q6w_sample": (c_int32, [c_void_p, c_int64, c_int32, c_int32, c_void_p, c_int64, c_void_p, c_void_p,
                                 POINTER(SampleArgs), POINTER(c_int32), c_int32, c_int32, c_void_p, S]),
        "q6w_workspace_status": (c_int32, [c_void_p, S]),
        "q6w_selftest_wait_timeout": (c_int32, [c_void_p, c_int64, S]),
        "q6w_linear_argmax": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
                                        c_int64, c_int64, c_int64, S]),
        "q6w_linear_argmax_noalloc": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                                                c_int64, c_int64, S]),
        "q6w_rmsnorm": (c_int32, [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_float, S]),
        "q6w_prefill_workspace_bytes": (c_size_t, [c_void_p, c_int32, c_int64]),
        "q6w_forward_all": (c_int32, [c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_int32, c_int64, c_void_p,
                                      c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, S]),
        "q6w_prefill": (c_int32, [c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_int32, c_int64, c_void_p,
                                  c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_size_t, S]),
        "q6w_gqa_attention": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32,
                                        c_int32, c_int32, c_int32, c_int64, S]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def load(path=None):
    """Load (once) and return the ctypes library handle."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    p = Path(path or os.environ.get("Q6W_B200_LIB", LIB_PATH))
    if not p.exists():
        raise Q6WLibraryError(f"{p} not found: build it with `python tinyllm-pynq-z2_b200/build.py`")
    try:
        lib = ctypes.CDLL(str(p))
        _declare(lib)
    except OSError as e:  # pragma: no cover - depends on the host
        _load_error = e
        raise Q6WLibraryError(f"cannot load {p}: {e}") from e
    _lib = lib
    return lib


def check(status, what=""):
    if status != Q6W_OK:
        msg = load().q6w_last_error().decode(errors="replace")
        raise Q6WError(status, f"{what}: {msg}" if what else msg)
    return status


def stream_handle(stream=None):
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return c_void_p(s.cuda_stream)
