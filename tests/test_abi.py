"""The C ABI: libllamacuda.so loads and exports every entry point declared in
include/llamacuda.h.  CPU only (no kernel is launched)."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "llamacuda.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lc_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from llamahat import _lib
    return _lib.load()


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for must in ("lc_gemv_f16", "lc_rmsnorm", "lc_rope", "lc_silu", "lc_softmax", "lc_softmax_row",
                 "lc_attn_scores", "lc_attn_values", "lc_forward", "lc_generate", "lc_argmax"):
        assert must in syms


def test_every_declared_symbol_is_exported(lib):
    so = lib._name
    out = subprocess.run(["nm", "-D", "--defined-only", so], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (lc_\w+)", out))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing


def test_binding_covers_header():
    from llamahat._lib import SIGNATURES
    assert sorted(SIGNATURES) == declared_symbols()


def test_abi_version(lib):
    assert lib.lc_abi_version() == 1


def test_errors_without_device(lib):
    from llamahat import _lib
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    n = ctypes.c_int(-1)
    rc = lib.lc_device_count(ctypes.byref(n))
    assert rc == _lib.LC_ERR_CUDA or n.value == 0
    h = ctypes.c_void_p()
    rc = lib.lc_context_create(0, ctypes.byref(h))
    assert rc != 0
    assert len(_lib.last_error()) > 0
    with pytest.raises(_lib.LlamaCudaError):
        _lib.check(rc)


def test_null_arguments_rejected(lib):
    from llamahat import _lib
    assert lib.lc_gemv_f16(None, None, None, None, 1, 1) == _lib.LC_ERR_INVALID_ARG
    assert lib.lc_forward(None, 0, 0, None, None) == _lib.LC_ERR_INVALID_ARG
    assert lib.lc_model_upload_tensor(None, b"x", None, 0, 0) == _lib.LC_ERR_INVALID_ARG


def test_config_constants(lib):
    from llamahat._lib import LcConfig
    from llamahat.config import LLAMA_3_2_1B
    c = LcConfig()
    lib.lc_config_llama32_1b(ctypes.byref(c))
    ref = LLAMA_3_2_1B.to_lc()
    for name, _ in LcConfig._fields_[:-1]:
        assert getattr(c, name) == getattr(ref, name), name
    assert LLAMA_3_2_1B.weight_bytes() == 2_471_493_632
