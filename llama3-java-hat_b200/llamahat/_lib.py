"""ctypes binding of libllamacuda.so (include/llamacuda.h).

Loading fails loudly when the library is missing: there is no CPU fallback
anywhere in this package.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_uint16, c_void_p

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG, "_build", "libllamacuda.so")

LC_OK = 0
LC_ERR_INVALID_ARG = -1
LC_ERR_CUDA = -2
LC_ERR_OUT_OF_MEMORY = -3
LC_ERR_NOT_FOUND = -4
LC_ERR_SHAPE = -5
LC_ERR_IO = -6
LC_ERR_TIMEOUT = -7
LC_ERR_STATE = -8
LC_ERR_UNSUPPORTED = -9


class LlamaCudaError(RuntimeError):
    """Base error; `code` is the LC_ERR_* status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code


class IllegalArgumentError(LlamaCudaError, ValueError):
    """IllegalArgumentException of the reference (bad argument / architecture)."""


class ModelIOError(LlamaCudaError, IOError):
    """IOException of the reference (tensor not found, shape mismatch, bad GGUF)."""


class IllegalStateError(LlamaCudaError):
    """IllegalStateException of the reference."""


class DeviceTimeoutError(LlamaCudaError):
    """A bounded device-side wait expired (the context stays usable)."""


_CODE_CLASS = {
    LC_ERR_INVALID_ARG: IllegalArgumentError,
    LC_ERR_NOT_FOUND: ModelIOError,
    LC_ERR_SHAPE: ModelIOError,
    LC_ERR_IO: ModelIOError,
    LC_ERR_STATE: IllegalStateError,
    LC_ERR_TIMEOUT: DeviceTimeoutError,
}


class LcConfig(ctypes.Structure):
    _fields_ = [
        ("dim", c_int32), ("hidden", c_int32), ("n_layers", c_int32), ("n_heads", c_int32),
        ("n_kv_heads", c_int32), ("head_dim", c_int32), ("vocab", c_int32), ("max_seq", c_int32),
        ("rope_theta", c_float), ("rms_eps", c_float), ("weight_mode", c_int32), ("reserved", c_int32 * 5),
    ]


# lc_token_callback: void (*)(int32_t token, int32_t index, void* user)
TOKEN_CALLBACK = ctypes.CFUNCTYPE(None, c_int32, c_int32, c_void_p)

# name -> (restype, argtypes).  Every symbol of include/llamacuda.h.
SIGNATURES = {
    "lc_last_error": (c_int, [c_char_p, c_size_t]),
    "lc_abi_version": (c_int, []),
    "lc_device_count": (c_int, [POINTER(c_int)]),
    "lc_context_create": (c_int, [c_int, POINTER(c_void_p)]),
    "lc_context_destroy": (c_int, [c_void_p]),
    "lc_context_synchronize": (c_int, [c_void_p]),
    "lc_context_stream": (c_void_p, [c_void_p]),
    "lc_context_sm_count": (c_int, [c_void_p]),
    "lc_gemv_f16": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int]),
    "lc_gemv_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int]),
    "lc_gemv_f16_batched": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int]),
    "lc_weights_tile": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int]),
    "lc_gemm_f16_tiled_argmax": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int32,
                                         c_void_p]),
    "lc_batch_create": (c_int, [c_void_p, c_int32, POINTER(c_void_p)]),
    "lc_batch_destroy": (c_int, [c_void_p]),
    "lc_batch_generate": (c_int, [c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_void_p, c_int32, c_void_p]),
    "lc_batch_last_ms": (c_int, [c_void_p, POINTER(c_float), POINTER(c_float), POINTER(c_int32)]),
    "lc_batch_logits": (c_int, [c_void_p, c_int32, c_void_p]),
    "lc_gemm_f16_tiled": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int]),
    "lc_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_int]),
    "lc_rmsnorm_rows": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_float]),
    "lc_rope": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_float]),
    "lc_rope_rows": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_float]),
    "lc_silu": (c_int, [c_void_p, c_void_p, c_int]),
    "lc_swiglu": (c_int, [c_void_p, c_void_p, c_void_p, c_int]),
    "lc_softmax": (c_int, [c_void_p, c_void_p, c_int]),
    "lc_softmax_row": (c_int, [c_void_p, c_void_p, c_int, c_int]),
    "lc_softmax_rows": (c_int, [c_void_p, c_void_p, c_int, c_int]),
    "lc_attn_scores": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int]),
    "lc_attn_values": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int]),
    "lc_attention_decode": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                    c_int, c_int, c_int64, c_int64, c_int64]),
    "lc_attention_decode_maxlen": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                           c_int, c_int, c_int, c_int64, c_int64, c_int64, c_int]),
    "lc_attention_decode_static": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                           c_int, c_int, c_int, c_int64, c_int64, c_int64]),
    "lc_argmax": (c_int, [c_void_p, c_void_p, c_int, c_void_p]),
    "lc_config_llama32_1b": (None, [POINTER(LcConfig)]),
    "lc_model_create": (c_int, [c_void_p, POINTER(LcConfig), POINTER(c_void_p)]),
    "lc_model_upload_tensor": (c_int, [c_void_p, c_char_p, c_void_p, c_int64, c_int32]),
    "lc_model_finalize": (c_int, [c_void_p]),
    "lc_model_load_gguf": (c_int, [c_void_p, c_char_p, c_int32, POINTER(c_void_p)]),
    "lc_model_load_gguf_mode": (c_int, [c_void_p, c_char_p, c_int32, c_int32, POINTER(c_void_p)]),
    "lc_model_get_config": (c_int, [c_void_p, POINTER(LcConfig)]),
    "lc_model_destroy": (c_int, [c_void_p]),
    "lc_session_create": (c_int, [c_void_p, POINTER(c_void_p)]),
    "lc_session_destroy": (c_int, [c_void_p]),
    "lc_forward": (c_int, [c_void_p, c_int32, c_int32, c_void_p, c_void_p]),
    "lc_generate": (c_int, [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_int32, c_void_p, c_void_p]),
    "lc_generate_stream": (c_int, [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_int32, TOKEN_CALLBACK, c_void_p,
                                   c_void_p, c_void_p]),
    "lc_decode": (c_int, [c_void_p, c_int32, c_int32, c_int32, c_void_p]),
    "lc_session_enable_trace": (c_int, [c_void_p, c_int32]),
    "lc_session_read_trace": (c_int, [c_void_p, c_void_p, c_int64, POINTER(c_int32), POINTER(c_int32)]),
    "lc_session_last_ms": (c_int, [c_void_p, POINTER(c_float)]),
    "lc_keyx_create": (c_int, [c_void_p, c_int32, c_int32, c_int32, POINTER(c_void_p), c_void_p]),
    "lc_keyx_open": (c_int, [c_void_p, c_void_p]),
    "lc_keyx_allreduce": (c_int, [c_void_p, c_void_p, c_int32]),
    "lc_keyx_destroy": (c_int, [c_void_p]),
}

_lib = None


def load(path: str | None = None) -> ctypes.CDLL:
    """Loads libllamacuda.so (built in-tree by build.py) once."""
    global _lib
    if _lib is not None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise ImportError(
            f"libllamacuda.so not found at {p}; run `python llama3-java-hat_b200/build.py` "
            "(or __graft_entry__.build()) first")
    lib = ctypes.CDLL(p)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error() -> str:
    lib = load()
    buf = ctypes.create_string_buffer(1024)
    lib.lc_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    """Raises the exception class matching an LC_ERR_* status."""
    if rc == LC_OK:
        return
    cls = _CODE_CLASS.get(rc, LlamaCudaError)
    raise cls(rc, last_error())
