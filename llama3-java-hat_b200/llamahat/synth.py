"""Seeded synthetic model weights and prompts (no checkpoint or dataset exists here).

Generator: numpy PCG64, one independent stream per tensor,
SeedSequence([seed, tensor_index]).  Projection and embedding weights are
N(0, 0.02) rounded to IEEE half (round-to-nearest-even); norm weights are
1 + N(0, 0.01) in float32.  Prompts are ids uniform in [0, 128000).
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from .config import LlamaConfig

PER_LAYER = ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "ffn_norm", "ffn_gate", "ffn_up", "ffn_down")


def tensor_specs(cfg: LlamaConfig) -> list[tuple[str, tuple[int, ...], str]]:
    """(GGUF name, shape (rows=out, cols=in) or (n,), kind) in generation order."""
    specs = [("token_embd.weight", (cfg.vocab, cfg.dim), "proj"), ("output_norm.weight", (cfg.dim,), "norm")]
    for l in range(cfg.n_layers):
        p = f"blk.{l}."
        specs += [
            (p + "attn_norm.weight", (cfg.dim,), "norm"),
            (p + "attn_q.weight", (cfg.q_dim, cfg.dim), "proj"),
            (p + "attn_k.weight", (cfg.kv_dim, cfg.dim), "proj"),
            (p + "attn_v.weight", (cfg.kv_dim, cfg.dim), "proj"),
            (p + "attn_output.weight", (cfg.dim, cfg.q_dim), "proj"),
            (p + "ffn_norm.weight", (cfg.dim,), "norm"),
            (p + "ffn_gate.weight", (cfg.hidden, cfg.dim), "proj"),
            (p + "ffn_up.weight", (cfg.hidden, cfg.dim), "proj"),
            (p + "ffn_down.weight", (cfg.dim, cfg.hidden), "proj"),
        ]
    return specs


def _make(seed: int, idx: int, shape, kind: str, std: float, norm_std: float) -> np.ndarray:
    g = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, idx])))
    a = g.standard_normal(int(np.prod(shape)), dtype=np.float32)
    if kind == "proj":
        a *= np.float32(std)
        return a.astype(np.float16).reshape(shape)
    a *= np.float32(norm_std)
    a += np.float32(1.0)
    return a.reshape(shape)


def synth_weights(cfg: LlamaConfig, seed: int = 1234, std: float = 0.02, norm_std: float = 0.01,
                  threads: int | None = None) -> dict[str, np.ndarray]:
    """All tensors of the model; F16 tensors as numpy float16."""
    specs = tensor_specs(cfg)
    threads = threads or min(16, os.cpu_count() or 1)
    with ThreadPoolExecutor(threads) as ex:
        arrs = list(ex.map(lambda t: _make(seed, t[0], t[1][1], t[1][2], std, norm_std), enumerate(specs)))
    return {name: a for (name, _, _), a in zip(specs, arrs)}


def synth_prompt(n: int, seed: int = 1234, high: int = 128000) -> np.ndarray:
    g = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, 0x50524F4D])))
    return g.integers(0, high, size=n, dtype=np.int64).astype(np.int32)
