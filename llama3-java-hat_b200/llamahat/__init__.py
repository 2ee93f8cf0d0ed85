"""llamahat -- B200 (sm_100a) CUDA implementation of the llama3-java-hat decode path.

Python host mirror of the reference's kernel strategy API (`CudaKernelFactory`)
and inference driver (`LlamaInference`) over the C ABI of libllamacuda.so.
"""
from ._lib import (DeviceTimeoutError, IllegalArgumentError, IllegalStateError, LlamaCudaError, ModelIOError,
                   load as load_library)
from .config import LLAMA_3_2_1B, TINY, LlamaConfig, WeightStorageMode
from .kernels import (Accelerator, CudaAttention, CudaGEMV, CudaKernelFactory, CudaRMSNorm, CudaRoPE, CudaSiLU,
                      CudaSoftmax, IAttention, IGEMV, IKernelFactory, IRMSNorm, IRoPE, ISiLU, ISoftmax,
                      default_accelerator)
from .inference import EOS_TOKEN, Batch, CudaModel, LlamaInference, Session
from .tokenizer import ChatFormat, Message, Role, StreamDecoder, Tokenizer

__all__ = [
    "WeightStorageMode",
    "Accelerator", "Batch", "ChatFormat", "CudaAttention", "CudaGEMV", "CudaKernelFactory", "CudaModel",
    "CudaRMSNorm", "CudaRoPE", "CudaSiLU", "CudaSoftmax", "DeviceTimeoutError", "EOS_TOKEN", "IAttention", "IGEMV", "IKernelFactory",
    "IRMSNorm", "IRoPE", "ISiLU", "ISoftmax", "IllegalArgumentError", "IllegalStateError", "LLAMA_3_2_1B",
    "LlamaConfig", "LlamaCudaError", "LlamaInference", "Message", "ModelIOError", "Role", "Session",
    "StreamDecoder", "TINY", "Tokenizer", "default_accelerator", "load_library",
]
