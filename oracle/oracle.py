"""ctypes binding of the CPU oracle (oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference arm, never by the product path.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, c_float, c_int, c_uint16, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "liboracle.so")
MAX_LAYERS = 64


def build() -> str:
    """Compiles liboracle.so with the committed Makefile recipe."""
    r = subprocess.run(["make", "-C", HERE], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}{r.stderr}")
    return LIB


class _Model(ctypes.Structure):
    _fields_ = [
        ("dim", c_int), ("hidden", c_int), ("n_layers", c_int), ("n_heads", c_int), ("n_kv_heads", c_int),
        ("head_dim", c_int), ("vocab", c_int), ("max_seq", c_int), ("rope_theta", c_float), ("rms_eps", c_float),
        ("tok_emb", c_void_p), ("out_norm", c_void_p), ("out_w", c_void_p),
        ("attn_norm", c_void_p * MAX_LAYERS), ("wq", c_void_p * MAX_LAYERS), ("wk", c_void_p * MAX_LAYERS),
        ("wv", c_void_p * MAX_LAYERS), ("wo", c_void_p * MAX_LAYERS), ("ffn_norm", c_void_p * MAX_LAYERS),
        ("wgate", c_void_p * MAX_LAYERS), ("wup", c_void_p * MAX_LAYERS), ("wdown", c_void_p * MAX_LAYERS),
        ("f32", c_int),
    ]


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        vp = c_void_p
        sigs = {
            "or_f16_to_f32": (c_float, [c_uint16]),
            "or_set_threads": (None, [c_int]),
            "or_max_threads": (c_int, []),
            "or_gemv_f32": (None, [vp, vp, vp, c_int, c_int]),
            "or_gemv_f16": (None, [vp, vp, vp, c_int, c_int]),
            "or_rmsnorm": (None, [vp, vp, c_int]),
            "or_rmsnorm_eps": (None, [vp, vp, c_int, c_float]),
            "or_rope": (None, [vp, c_int, c_int, c_int, c_float]),
            "or_silu": (None, [vp, c_int]),
            "or_swiglu": (None, [vp, vp, c_int]),
            "or_softmax": (None, [vp, c_int]),
            "or_softmax_row": (None, [vp, c_int, c_int]),
            "or_attn_scores": (None, [vp, vp, vp, c_int, c_int]),
            "or_attn_values": (None, [vp, vp, vp, c_int, c_int]),
            "or_gqa_attention": (None, [vp, vp, vp, vp, c_int, c_int, c_int, c_int, vp]),
            "or_argmax": (c_int, [vp, c_int]),
            "or_state_create": (vp, [POINTER(_Model)]),
            "or_state_destroy": (None, [vp]),
            "or_state_x": (POINTER(c_float), [vp]),
            "or_state_logits": (POINTER(c_float), [vp]),
            "or_state_kcache": (POINTER(c_float), [vp]),
            "or_state_vcache": (POINTER(c_float), [vp]),
            "or_block_forward": (None, [POINTER(_Model), c_int, vp, c_int]),
            "or_forward": (None, [POINTER(_Model), vp, c_int, c_int, vp]),
            "or_generate": (c_int, [POINTER(_Model), vp, vp, c_int, c_int, vp, c_int, vp]),
        }
        for n, (r, a) in sigs.items():
            f = getattr(L, n)
            f.restype = r
            f.argtypes = a
        _lib = L
    return _lib


def _p(a: np.ndarray, dtype) -> int:
    if a.dtype != dtype or not a.flags.c_contiguous:
        raise TypeError(f"expected contiguous {dtype}, got {a.dtype}")
    return a.ctypes.data


def f16_bits(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a)
    return a.view(np.uint16) if a.dtype == np.float16 else a


def set_threads(n: int) -> None:
    lib().or_set_threads(n)


def max_threads() -> int:
    return lib().or_max_threads()


# --------------------------------------------------------------- kernels
# Each returns a new array (inputs are copied) unless noted.

def gemv_f16(W: np.ndarray, x: np.ndarray) -> np.ndarray:
    Wb = f16_bits(W)
    rows, cols = Wb.shape
    y = np.empty(rows, np.float32)
    lib().or_gemv_f16(_p(Wb, np.uint16), _p(np.ascontiguousarray(x, np.float32), np.float32), y.ctypes.data, rows, cols)
    return y


def gemv_f32(W: np.ndarray, x: np.ndarray) -> np.ndarray:
    W = np.ascontiguousarray(W, np.float32)
    rows, cols = W.shape
    y = np.empty(rows, np.float32)
    lib().or_gemv_f32(W.ctypes.data, _p(np.ascontiguousarray(x, np.float32), np.float32), y.ctypes.data, rows, cols)
    return y


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float | None = None) -> np.ndarray:
    x = np.array(x, np.float32, copy=True)
    w = np.ascontiguousarray(w, np.float32)
    if eps is None:
        lib().or_rmsnorm(x.ctypes.data, w.ctypes.data, x.size)
    else:
        lib().or_rmsnorm_eps(x.ctypes.data, w.ctypes.data, x.size, eps)
    return x


def rope(v: np.ndarray, pos: int, n_heads: int, head_dim: int, theta: float) -> np.ndarray:
    v = np.array(v, np.float32, copy=True)
    lib().or_rope(v.ctypes.data, pos, n_heads, head_dim, theta)
    return v


def silu(x: np.ndarray) -> np.ndarray:
    x = np.array(x, np.float32, copy=True)
    lib().or_silu(x.ctypes.data, x.size)
    return x


def swiglu(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.array(g, np.float32, copy=True)
    lib().or_swiglu(g.ctypes.data, _p(np.ascontiguousarray(u, np.float32), np.float32), g.size)
    return g


def softmax(x: np.ndarray) -> np.ndarray:
    x = np.array(x, np.float32, copy=True)
    lib().or_softmax(x.ctypes.data, x.size)
    return x


def softmax_row(x: np.ndarray, off: int, n: int) -> np.ndarray:
    x = np.array(x, np.float32, copy=True)
    lib().or_softmax_row(x.ctypes.data, off, n)
    return x


def attn_scores(q: np.ndarray, K: np.ndarray, seq_len: int, head_dim: int) -> np.ndarray:
    s = np.empty(seq_len, np.float32)
    lib().or_attn_scores(_p(np.ascontiguousarray(q, np.float32), np.float32),
                         _p(np.ascontiguousarray(K, np.float32), np.float32), s.ctypes.data, seq_len, head_dim)
    return s


def attn_values(p: np.ndarray, V: np.ndarray, seq_len: int, head_dim: int) -> np.ndarray:
    o = np.empty(head_dim, np.float32)
    lib().or_attn_values(_p(np.ascontiguousarray(p, np.float32), np.float32),
                         _p(np.ascontiguousarray(V, np.float32), np.float32), o.ctypes.data, seq_len, head_dim)
    return o


def gqa_attention(q: np.ndarray, kcache: np.ndarray, vcache: np.ndarray, seq_len: int, n_heads: int,
                  n_kv_heads: int, head_dim: int) -> np.ndarray:
    """q [n_heads*head_dim]; caches position-major [>=seq_len][n_kv][head_dim]."""
    out = np.empty(n_heads * head_dim, np.float32)
    scratch = np.empty(n_heads * seq_len, np.float32)
    lib().or_gqa_attention(_p(np.ascontiguousarray(q, np.float32), np.float32),
                           _p(np.ascontiguousarray(kcache, np.float32), np.float32),
                           _p(np.ascontiguousarray(vcache, np.float32), np.float32), out.ctypes.data, seq_len,
                           n_heads, n_kv_heads, head_dim, scratch.ctypes.data)
    return out


def argmax(v: np.ndarray) -> int:
    v = np.ascontiguousarray(v, np.float32)
    return int(lib().or_argmax(v.ctypes.data, v.size))


def f16_to_f32(bits: int) -> float:
    return float(lib().or_f16_to_f32(bits))


# ----------------------------------------------------------------- model

class OracleModel:
    """LlamaInference with PlainJavaKernelFactory, restated in C (host memory).

    f32=True is WeightStorageMode.F32 (H/LlamaInference.java:102-108): the
    embedding and the projections are fp32 (F16 tensors widened exactly, F32
    tensors as given) and go through GEMV.apply(F32Array, ...)."""

    def __init__(self, cfg, weights: dict[str, np.ndarray], f32: bool = False):
        if cfg.n_layers > MAX_LAYERS:
            raise ValueError("too many layers")
        self.cfg = cfg
        self._keep = {}

        def ptr(name, dtype):
            a = weights[name]
            if dtype == np.uint16 and f32:
                a = np.ascontiguousarray(a.astype(np.float32) if a.dtype == np.float16 else a, np.float32)
            elif dtype == np.uint16:
                a = f16_bits(a)
            else:
                a = np.ascontiguousarray(a, np.float32)
            self._keep[name] = a
            return a.ctypes.data

        m = _Model()
        m.dim, m.hidden, m.n_layers, m.n_heads = cfg.dim, cfg.hidden, cfg.n_layers, cfg.n_heads
        m.n_kv_heads, m.head_dim, m.vocab, m.max_seq = cfg.n_kv_heads, cfg.head_dim, cfg.vocab, cfg.max_seq
        m.rope_theta, m.rms_eps = cfg.rope_theta, cfg.rms_eps
        m.tok_emb = ptr("token_embd.weight", np.uint16)
        m.out_norm = ptr("output_norm.weight", np.float32)
        m.out_w = ptr("output.weight", np.uint16) if "output.weight" in weights else m.tok_emb
        for l in range(cfg.n_layers):
            p = f"blk.{l}."
            m.attn_norm[l] = ptr(p + "attn_norm.weight", np.float32)
            m.wq[l] = ptr(p + "attn_q.weight", np.uint16)
            m.wk[l] = ptr(p + "attn_k.weight", np.uint16)
            m.wv[l] = ptr(p + "attn_v.weight", np.uint16)
            m.wo[l] = ptr(p + "attn_output.weight", np.uint16)
            m.ffn_norm[l] = ptr(p + "ffn_norm.weight", np.float32)
            m.wgate[l] = ptr(p + "ffn_gate.weight", np.uint16)
            m.wup[l] = ptr(p + "ffn_up.weight", np.uint16)
            m.wdown[l] = ptr(p + "ffn_down.weight", np.uint16)
        m.f32 = 1 if f32 else 0
        self.m = m
        self.state = lib().or_state_create(ctypes.byref(m))
        if not self.state:
            raise MemoryError("oracle state")

    def __del__(self):
        st = getattr(self, "state", None)
        if st:
            lib().or_state_destroy(st)
            self.state = None

    def forward(self, token: int, pos: int) -> np.ndarray:
        out = np.empty(self.cfg.vocab, np.float32)
        lib().or_forward(ctypes.byref(self.m), self.state, int(token), int(pos), out.ctypes.data)
        return out

    def generate(self, prompt, max_new: int, stop=(128001,)) -> np.ndarray:
        p = np.ascontiguousarray(np.asarray(prompt, np.int32))
        st = np.ascontiguousarray(np.asarray(list(stop), np.int32))
        out = np.zeros(max(max_new, 1), np.int32)
        n = lib().or_generate(ctypes.byref(self.m), self.state, p.ctypes.data, p.size, int(max_new),
                              st.ctypes.data if st.size else None, st.size, out.ctypes.data)
        return out[:n].copy()

    def kcache(self) -> np.ndarray:
        c = self.cfg
        n = c.n_layers * c.max_seq * c.kv_dim
        return np.ctypeslib.as_array(lib().or_state_kcache(self.state), shape=(n,)).reshape(
            c.n_layers, c.max_seq, c.n_kv_heads, c.head_dim)

    def block_forward(self, layer: int, x: np.ndarray, pos: int) -> np.ndarray:
        """TransformerBlock.forward on a given hidden state (KV cache of this
        model's state)."""
        xs = np.ctypeslib.as_array(lib().or_state_x(self.state), shape=(self.cfg.dim,))
        xs[:] = np.asarray(x, np.float32)
        lib().or_block_forward(ctypes.byref(self.m), int(layer), self.state, int(pos))
        return xs.copy()
