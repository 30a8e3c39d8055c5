"""CPU: the C-ABI library loads and exports every symbol include/q6w_b200.h
declares; host-side argument checks answer without touching a GPU."""

import ctypes
import re

import pytest

from conftest import REPO
from q6w_b200 import _lib

HEADER = REPO / "include" / "q6w_b200.h"


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"Q6W_API\s+[\w\s\*]+?\b(q6w_\w+)\s*\(", text)))


def test_header_declares_exports():
    assert declared() == sorted(_lib.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared():
        assert hasattr(lib, name), name
    assert lib.q6w_abi_version() == 1


def test_host_side_argument_errors_need_no_gpu():
    lib = _lib.load()
    S = ctypes.c_void_p(0)
    assert lib.q6w_unpack(None, None, 2, 6, S) == _lib.Q6W_ERR_ARG
    assert b"divisible by four" in lib.q6w_last_error()
    assert lib.q6w_unpack(None, None, -1, 4, S) == _lib.Q6W_ERR_ARG
    assert lib.q6w_unpack(None, None, 0, 4, S) == _lib.Q6W_OK  # empty is a no-op
    assert lib.q6w_dequant(None, None, None, 3, 7, S) == _lib.Q6W_ERR_ARG
    assert lib.q6w_linear(None, None, None, None, 4, 8, 1, S) == _lib.Q6W_ERR_ARG
    assert lib.q6w_linear(None, None, None, None, 4, 8, 0, S) == _lib.Q6W_OK
    assert lib.q6w_model_create(None, None) == _lib.Q6W_ERR_ARG
    assert lib.q6w_workspace_bytes(None, 4) == 0


def test_model_create_rejects_bad_shapes_without_gpu():
    lib = _lib.load()
    d = _lib.ModelDesc()
    d.dim, d.n_layers, d.n_heads, d.n_kv_heads = 128, 1, 3, 1
    d.vocab_size, d.hidden_dim, d.max_seq_len, d.norm_eps = 64, 384, 16, 1e-5
    h = ctypes.c_void_p()
    assert lib.q6w_model_create(ctypes.byref(d), ctypes.byref(h)) == _lib.Q6W_ERR_ARG
    d.n_heads = 8
    d.dim = 8 * 24  # head_dim 24 unsupported
    assert lib.q6w_model_create(ctypes.byref(d), ctypes.byref(h)) == _lib.Q6W_ERR_ARG
    assert b"head_dim" in lib.q6w_last_error()
