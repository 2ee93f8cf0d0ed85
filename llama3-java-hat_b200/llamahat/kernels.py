"""Host-side mirror of the reference's kernel strategy API.

Reference: src/main/java/com/arturskowronski/llama3babylon/hat/kernels/
  IKernelFactory.java:9-40, IGEMV.java:11-69, IRMSNorm.java:8-18, IRoPE.java:8-20,
  ISiLU.java:8-17, ISoftmax.java:8-27, IAttention.java:8-31.

`CudaKernelFactory` sits where `PlainJavaKernelFactory` / `HybridKernelFactory`
sit: same method names, same argument meaning, same in-place behaviour.  Each
kernel object forwards to the C ABI of libllamacuda.so; buffers may be numpy
arrays (host memory, staged by the library) or torch tensors (host or CUDA).
`Accelerator` stands in for hat.Accelerator: it owns the CUDA context of one
device.
"""
from __future__ import annotations

import ctypes
import weakref
from abc import ABC, abstractmethod

import numpy as np

from . import _lib


def _addr(buf, kind: str, min_len: int, writable: bool = False) -> int:
    """Address of a contiguous buffer of the expected element type.

    kind: "f32", "f16" (IEEE half bits; numpy float16 or uint16), "i32".
    """
    want = {"f32": (np.float32,), "f16": (np.float16, np.uint16), "i32": (np.int32,)}[kind]
    if isinstance(buf, np.ndarray):
        if buf.dtype.type not in want:
            raise TypeError(f"expected {kind} buffer, got numpy {buf.dtype}")
        if not buf.flags.c_contiguous:
            raise ValueError("buffer must be C-contiguous")
        if writable and not buf.flags.writeable:
            raise ValueError("buffer is read-only")
        if buf.size < min_len:
            raise ValueError(f"buffer holds {buf.size} elements, need {min_len}")
        return buf.ctypes.data
    try:
        import torch
    except ImportError:  # pragma: no cover
        torch = None
    if torch is not None and isinstance(buf, torch.Tensor):
        tw = {"f32": (torch.float32,), "f16": (torch.float16, torch.int16), "i32": (torch.int32,)}[kind]
        if buf.dtype not in tw:
            raise TypeError(f"expected {kind} tensor, got {buf.dtype}")
        if not buf.is_contiguous():
            raise ValueError("tensor must be contiguous")
        if buf.numel() < min_len:
            raise ValueError(f"tensor holds {buf.numel()} elements, need {min_len}")
        return buf.data_ptr()
    raise TypeError(f"unsupported buffer type {type(buf)!r}")


class Accelerator:
    """Device handle (hat.Accelerator's role): one lc_context per instance."""

    def __init__(self, device: int = 0):
        lib = _lib.load()
        h = ctypes.c_void_p()
        _lib.check(lib.lc_context_create(device, ctypes.byref(h)))
        self.device = device
        self.handle = h
        self._fin = weakref.finalize(self, lib.lc_context_destroy, h)

    def synchronize(self) -> None:
        _lib.check(_lib.load().lc_context_synchronize(self.handle))

    @property
    def stream(self) -> int:
        return _lib.load().lc_context_stream(self.handle) or 0

    @property
    def sm_count(self) -> int:
        return _lib.load().lc_context_sm_count(self.handle)

    def close(self) -> None:
        self._fin()


_default_acc: Accelerator | None = None


def default_accelerator() -> Accelerator:
    global _default_acc
    if _default_acc is None:
        _default_acc = Accelerator(0)
    return _default_acc


# ---------------------------------------------------------------- interfaces

class IGEMV(ABC):
    """IGEMV.java:11-69: y = A x, A row-major [rows][cols]."""

    @abstractmethod
    def apply(self, matrix, vector, result, rows: int, cols: int) -> None: ...


class IRMSNorm(ABC):
    """IRMSNorm.java:8-18: in-place RMSNorm."""

    @abstractmethod
    def apply(self, input, weight, size: int) -> None: ...


class IRoPE(ABC):
    """IRoPE.java:8-20: in-place interleaved rotary embedding."""

    @abstractmethod
    def apply(self, vec, pos: int, numHeads: int, headDim: int, theta: float) -> None: ...


class ISiLU(ABC):
    """ISiLU.java:8-17: in-place SiLU."""

    @abstractmethod
    def apply(self, input, size: int) -> None: ...


class ISoftmax(ABC):
    """ISoftmax.java:8-27: in-place softmax of a vector / of one row."""

    @abstractmethod
    def apply(self, input, size: int) -> None: ...

    @abstractmethod
    def applyRow(self, input, rowOffset: int, rowSize: int) -> None: ...


class IAttention(ABC):
    """IAttention.java:8-31: scores and weighted values of one query head."""

    @abstractmethod
    def computeScores(self, query, keys, scores, seqLen: int, headDim: int) -> None: ...

    @abstractmethod
    def computeValues(self, scores, values, output, seqLen: int, headDim: int) -> None: ...


class IKernelFactory(ABC):
    """IKernelFactory.java:9-40."""

    @abstractmethod
    def createGEMV(self, acc: Accelerator | None = None) -> IGEMV: ...

    @abstractmethod
    def createRMSNorm(self, acc: Accelerator | None = None) -> IRMSNorm: ...

    @abstractmethod
    def createRoPE(self, acc: Accelerator | None = None) -> IRoPE: ...

    @abstractmethod
    def createSiLU(self, acc: Accelerator | None = None) -> ISiLU: ...

    @abstractmethod
    def createSoftmax(self, acc: Accelerator | None = None) -> ISoftmax: ...

    @abstractmethod
    def createAttention(self, acc: Accelerator | None = None) -> IAttention: ...


# ----------------------------------------------------------- CUDA kernels

class _CudaKernel:
    def __init__(self, acc: Accelerator | None):
        self.acc = acc or default_accelerator()
        self.lib = _lib.load()

    @property
    def ctx(self):
        return self.acc.handle


class CudaGEMV(_CudaKernel, IGEMV):
    """GEMV on the GPU.  F16 matrices (numpy float16/uint16, the F16Array /
    F16Weights overloads, IGEMV.java:34,50) use the streaming F16 kernel;
    F32 matrices (IGEMV.java:22) the fp32 kernel."""

    def apply(self, matrix, vector, result, rows: int, cols: int) -> None:
        n = rows * cols
        is_f16 = (isinstance(matrix, np.ndarray) and matrix.dtype.type in (np.float16, np.uint16)) or (
            not isinstance(matrix, np.ndarray) and str(getattr(matrix, "dtype", "")) in ("torch.float16", "torch.int16"))
        x = _addr(vector, "f32", cols)
        y = _addr(result, "f32", rows, writable=True)
        if is_f16:
            _lib.check(self.lib.lc_gemv_f16(self.ctx, _addr(matrix, "f16", n), x, y, rows, cols))
        else:
            _lib.check(self.lib.lc_gemv_f32(self.ctx, _addr(matrix, "f32", n), x, y, rows, cols))

    def apply_batched(self, matrix, X, Y, rows: int, cols: int, batch: int) -> None:
        """Y[b] = matrix @ X[b] for b < batch (no reference counterpart)."""
        _lib.check(self.lib.lc_gemv_f16_batched(self.ctx, _addr(matrix, "f16", rows * cols),
                                                _addr(X, "f32", batch * cols),
                                                _addr(Y, "f32", batch * rows, writable=True), rows, cols, batch))

    def tile(self, matrix, tiled, rows: int, cols: int) -> None:
        """Row-major F16 matrix -> the tiled layout of the tensor-core product
        (`tiled`: device memory, rows * cols halves)."""
        n = rows * cols
        _lib.check(self.lib.lc_weights_tile(self.ctx, _addr(matrix, "f16", n), _addr(tiled, "f16", n, writable=True),
                                            rows, cols))

    def apply_batched_tiled_argmax(self, tiled, X, Y, rows: int, cols: int, batch: int, index_offset: int,
                                   keys) -> None:
        """apply_batched_tiled plus packed argmax keys per row (keys: uint64 /
        int64 buffer of `batch`; Y may be None)."""
        y = None if Y is None else _addr(Y, "f32", batch * rows, writable=True)
        if isinstance(keys, np.ndarray):
            if keys.dtype not in (np.uint64, np.int64) or keys.size < batch:
                raise TypeError("keys must be a uint64/int64 array of `batch` entries")
            k = keys.ctypes.data
        else:
            if str(keys.dtype) not in ("torch.int64", "torch.uint64") or keys.numel() < batch:
                raise TypeError("keys must be an int64 tensor of `batch` entries")
            k = keys.data_ptr()
        _lib.check(self.lib.lc_gemm_f16_tiled_argmax(self.ctx, _addr(tiled, "f16", rows * cols),
                                                     _addr(X, "f32", batch * cols), y, rows, cols, batch,
                                                     int(index_offset), k))

    def apply_batched_tiled(self, tiled, X, Y, rows: int, cols: int, batch: int) -> None:
        """Y[b] = W @ X[b] for b < batch <= 64 on the tcgen05 tensor cores; W
        given in the tiled layout (`tile`)."""
        _lib.check(self.lib.lc_gemm_f16_tiled(self.ctx, _addr(tiled, "f16", rows * cols),
                                              _addr(X, "f32", batch * cols),
                                              _addr(Y, "f32", batch * rows, writable=True), rows, cols, batch))


class CudaRMSNorm(_CudaKernel, IRMSNorm):
    """RMSNorm.java:35-50 on the GPU: one fused reduce + normalise kernel."""

    def apply(self, input, weight, size: int) -> None:
        _lib.check(self.lib.lc_rmsnorm(self.ctx, _addr(input, "f32", size, True), _addr(weight, "f32", size), size))

    def apply_rows(self, input, weight, rows: int, width: int, eps: float = 1e-5) -> None:
        _lib.check(self.lib.lc_rmsnorm_rows(self.ctx, _addr(input, "f32", rows * width, True),
                                            _addr(weight, "f32", width), rows, width, eps))


class CudaRoPE(_CudaKernel, IRoPE):
    """RoPE.java:36-52 on the GPU."""

    def apply(self, vec, pos: int, numHeads: int, headDim: int, theta: float) -> None:
        _lib.check(self.lib.lc_rope(self.ctx, _addr(vec, "f32", numHeads * headDim, True), pos, numHeads, headDim,
                                    theta))

    def apply_rows(self, vec, positions, rows: int, numHeads: int, headDim: int, theta: float) -> None:
        _lib.check(self.lib.lc_rope_rows(self.ctx, _addr(vec, "f32", rows * numHeads * headDim, True),
                                         _addr(positions, "i32", rows), rows, numHeads, headDim, theta))


class CudaSiLU(_CudaKernel, ISiLU):
    """SiLU.java:32-40 on the GPU."""

    def apply(self, input, size: int) -> None:
        _lib.check(self.lib.lc_silu(self.ctx, _addr(input, "f32", size, True), size))

    def swiglu(self, gate, up, n: int) -> None:
        """gate = silu(gate) * up (TransformerBlock.java:209-210)."""
        _lib.check(self.lib.lc_swiglu(self.ctx, _addr(gate, "f32", n, True), _addr(up, "f32", n), n))


class CudaSoftmax(_CudaKernel, ISoftmax):
    """Softmax.java:28-84 on the GPU (online-statistics single kernel)."""

    def apply(self, input, size: int) -> None:
        _lib.check(self.lib.lc_softmax(self.ctx, _addr(input, "f32", size, True), size))

    def applyRow(self, input, rowOffset: int, rowSize: int) -> None:
        _lib.check(self.lib.lc_softmax_row(self.ctx, _addr(input, "f32", rowOffset + rowSize, True), rowOffset,
                                           rowSize))

    def apply_rows(self, input, rows: int, width: int) -> None:
        _lib.check(self.lib.lc_softmax_rows(self.ctx, _addr(input, "f32", rows * width, True), rows, width))


class CudaAttention(_CudaKernel, IAttention):
    """Attention.java:32-61 on the GPU, plus the fused GQA decode kernel."""

    def computeScores(self, query, keys, scores, seqLen: int, headDim: int) -> None:
        _lib.check(self.lib.lc_attn_scores(self.ctx, _addr(query, "f32", headDim), _addr(keys, "f32", seqLen * headDim),
                                           _addr(scores, "f32", seqLen, True), seqLen, headDim))

    def computeValues(self, scores, values, output, seqLen: int, headDim: int) -> None:
        _lib.check(self.lib.lc_attn_values(self.ctx, _addr(scores, "f32", seqLen), _addr(values, "f32", seqLen * headDim),
                                           _addr(output, "f32", headDim, True), seqLen, headDim))

    def decode(self, q, k, v, out, seq_len, batch: int, n_heads: int, n_kv_heads: int, head_dim: int,
               seq_stride: int, head_stride: int, pos_stride: int) -> None:
        """Fused GQA attention for one query token per sequence (see lc_attention_decode)."""
        _lib.check(self.lib.lc_attention_decode(
            self.ctx, _addr(q, "f32", batch * n_heads * head_dim), _addr(k, "f32", 1), _addr(v, "f32", 1),
            _addr(out, "f32", batch * n_heads * head_dim, True), _addr(seq_len, "i32", batch), batch, n_heads,
            n_kv_heads, head_dim, seq_stride, head_stride, pos_stride))

    def decode_maxlen(self, q, k, v, out, seq_len, batch: int, n_heads: int, n_kv_heads: int, head_dim: int,
                      seq_stride: int, head_stride: int, pos_stride: int, max_len: int) -> None:
        """decode with the split plan sized for max_len >= every seq_len (see
        lc_attention_decode_maxlen): enqueue-only with device buffers."""
        _lib.check(self.lib.lc_attention_decode_maxlen(
            self.ctx, _addr(q, "f32", batch * n_heads * head_dim), _addr(k, "f32", 1), _addr(v, "f32", 1),
            _addr(out, "f32", batch * n_heads * head_dim, True), _addr(seq_len, "i32", batch), batch, n_heads,
            n_kv_heads, head_dim, seq_stride, head_stride, pos_stride, max_len))


class CudaKernelFactory(IKernelFactory):
    """The B200 sibling of PlainJavaKernelFactory (PlainJavaKernelFactory.java:9-40)."""

    def createGEMV(self, acc=None) -> CudaGEMV:
        return CudaGEMV(acc)

    def createRMSNorm(self, acc=None) -> CudaRMSNorm:
        return CudaRMSNorm(acc)

    def createRoPE(self, acc=None) -> CudaRoPE:
        return CudaRoPE(acc)

    def createSiLU(self, acc=None) -> CudaSiLU:
        return CudaSiLU(acc)

    def createSoftmax(self, acc=None) -> CudaSoftmax:
        return CudaSoftmax(acc)

    def createAttention(self, acc=None) -> CudaAttention:
        return CudaAttention(acc)


def argmax(values, acc: Accelerator | None = None) -> int:
    """LlamaInference.argmax (LlamaInference.java:252-262) on the GPU."""
    acc = acc or default_accelerator()
    out = np.zeros(1, np.int32)
    _lib.check(_lib.load().lc_argmax(acc.handle, _addr(values, "f32", 1), int(np.asarray(values).size if isinstance(values, np.ndarray) else values.numel()), out.ctypes.data))
    return int(out[0])
