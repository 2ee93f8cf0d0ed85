"""Model configuration.

LLAMA_3_2_1B holds the constants the reference hard-codes
(src/main/java/com/arturskowronski/llama3babylon/hat/LlamaModel.java:30-37,
rope theta TransformerBlock.java:136, eps kernels/RMSNorm.java:22).
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, replace

from ._lib import LcConfig


@dataclass(frozen=True)
class LlamaConfig:
    dim: int = 2048
    hidden: int = 8192
    n_layers: int = 16
    n_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 64
    vocab: int = 128256
    max_seq: int = 2048
    rope_theta: float = 500000.0
    rms_eps: float = 1e-5

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    def with_(self, **kw) -> "LlamaConfig":
        return replace(self, **kw)

    def to_lc(self) -> LcConfig:
        c = LcConfig()
        c.dim, c.hidden, c.n_layers, c.n_heads = self.dim, self.hidden, self.n_layers, self.n_heads
        c.n_kv_heads, c.head_dim, c.vocab, c.max_seq = self.n_kv_heads, self.head_dim, self.vocab, self.max_seq
        c.rope_theta, c.rms_eps = self.rope_theta, self.rms_eps
        return c

    @staticmethod
    def from_lc(c: LcConfig) -> "LlamaConfig":
        return LlamaConfig(c.dim, c.hidden, c.n_layers, c.n_heads, c.n_kv_heads, c.head_dim, c.vocab, c.max_seq,
                           float(c.rope_theta), float(c.rms_eps))

    def weight_bytes(self) -> int:
        """F16 projection + embedding bytes streamed by one batch-1 decode step."""
        per_layer = 2 * (self.dim * (self.q_dim + 2 * self.kv_dim) + self.dim * self.q_dim + 3 * self.dim * self.hidden)
        return self.n_layers * per_layer + 2 * self.vocab * self.dim


LLAMA_3_2_1B = LlamaConfig()

# Small configuration with the same structure (GQA 4:1, head_dim 64) for fast tests.
TINY = LlamaConfig(dim=512, hidden=1024, n_layers=2, n_heads=8, n_kv_heads=2, head_dim=64, vocab=1000, max_seq=256)


class WeightStorageMode(enum.Enum):
    """How the projection weights are stored (H/WeightStorageMode.java).

    F16 and F16_FAST differ only in the Java host's storage; on the GPU both
    keep the F16 weights (tiled for the fused decode kernel).  F32 keeps the
    projections and the embedding in fp32 (twice the memory) and decodes with
    fp32-weight GEMVs.  The value is the C ABI's weight_mode."""
    F32 = 1
    F16 = 0
    F16_FAST = 2

    @property
    def device_mode(self) -> int:
        return 1 if self is WeightStorageMode.F32 else 0

    @staticmethod
    def fromString(s: str) -> "WeightStorageMode":
        """WeightStorageMode.fromString (H/WeightStorageMode.java:63-70)."""
        key = s.strip().upper()
        if key == "F32":
            return WeightStorageMode.F32
        if key == "F16":
            return WeightStorageMode.F16
        if key in ("F16_FAST", "F16FAST", "FAST"):
            return WeightStorageMode.F16_FAST
        raise ValueError(f"Unknown weight storage mode: '{s}'. Valid: F16, F16_FAST, F32")
