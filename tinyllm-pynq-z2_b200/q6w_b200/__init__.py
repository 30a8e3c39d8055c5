"""q6w_b200 -- the Q6W inference hot path on NVIDIA B200 (sm_100a).

Host side of the library: the Q6W file format (``format``), device codec and
linear ops (``ops``), and the drop-in cached transformer plus the
device-resident greedy loop (``model``), all calling the compiled kernels in
``libq6w_b200.so`` through the C ABI of include/q6w_b200.h.
"""

from . import format
from ._lib import EXPORTS, Q6WError, Q6WLibraryError, load as load_library
from .format import (QUANT_KEYS, NORM_KEYS, SCALED_ARGS, TINY_ARGS, Q6WImage, export_q6w, pack_signed_int6,
                     quant_keys, norm_keys, quantize_rows, synthetic_state, write_q6w, write_synthetic)

__all__ = [
    "format", "EXPORTS", "Q6WError", "Q6WLibraryError", "load_library", "QUANT_KEYS", "NORM_KEYS", "SCALED_ARGS",
    "TINY_ARGS", "Q6WImage", "export_q6w", "pack_signed_int6", "quant_keys", "norm_keys", "quantize_rows",
    "synthetic_state", "write_q6w", "write_synthetic", "Q6WCudaTransformer", "generate", "unpack_signed_int6",
    "dequantize_rows", "q6w_linear", "load_dequantized_state",
]


def __getattr__(name):
    # torch-dependent device modules are imported on first use
    if name in ("Q6WCudaTransformer", "generate", "runtime_args", "rope_tables"):
        from . import model

        return getattr(model, name)
    if name in ("unpack_signed_int6", "dequantize_rows", "q6w_linear", "load_dequantized_state", "DeviceImage",
                "linear_argmax", "rmsnorm", "gqa_attention"):
        from . import ops

        return getattr(ops, name)
    raise AttributeError(name)
