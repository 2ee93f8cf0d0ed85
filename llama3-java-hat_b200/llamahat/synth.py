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


# A few sentences to learn byte-pair merges from, so that the synthetic
# vocabulary tokenises ordinary text into multi-byte tokens the way a real
# Llama 3 vocabulary does (the real one is not available here).  The first
# four lines are the strings the reference's own tests and benchmark feed
# the chat path.
_BPE_CORPUS = """You are a helpful assistant.
Tell a joke about programming
Say hi
Hello, world!
The decoder reads every weight of the model once for each new token, so the
speed of a single stream is set by how fast the memory can deliver bytes.
Sixteen layers follow one another: a norm, the attention over the cached keys
and values, a second norm and the feed forward block with its gate and up
projections.  The last norm feeds the output head, and the largest logit names
the next token.  A prompt is read first; then the model writes its answer one
token at a time until it emits a stop token or reaches the limit.
Numbers such as 2048, 8192 and 128256 appear in the shapes of the weights.
It's easy to say hi; they'll answer when they're ready, and we've seen it.
"""


def train_bpe(text: str, n_merges: int) -> list[tuple[str, str]]:
    """Byte-level BPE training: pre-tokenise with the Llama 3 pattern, start
    from one symbol per byte (GPT-2 byte map) and repeatedly merge the most
    frequent adjacent pair (ties: the smallest pair of strings); stops early
    when no pair occurs twice.  Deterministic."""
    from collections import Counter

    from .tokenizer import _PATTERN, BYTE_ENCODER
    words = Counter(tuple(chr(BYTE_ENCODER[b]) for b in m.group().encode("utf-8")) for m in _PATTERN.finditer(text))
    merges: list[tuple[str, str]] = []
    for _ in range(n_merges):
        pairs: Counter = Counter()
        for w, c in words.items():
            for p in zip(w, w[1:]):
                pairs[p] += c
        if not pairs:
            break
        top = max(pairs.values())
        if top < 2:
            break
        best = min(p for p, c in pairs.items() if c == top)
        merges.append(best)
        nxt: Counter = Counter()
        for w, c in words.items():
            out, i = [], 0
            while i < len(w):
                if i + 1 < len(w) and (w[i], w[i + 1]) == best:
                    out.append(w[i] + w[i + 1])
                    i += 2
                else:
                    out.append(w[i])
                    i += 1
            nxt[tuple(out)] += c
        words = nxt
    return merges


def synth_tokenizer(vocab: int, n_merges: int = 400) -> tuple[list[str], list[str]]:
    """(token strings, merge rules) of a synthetic GGUF tokenizer: ids 0..255
    are the 256 byte symbols in byte order, then one token per learned merge,
    then filler names up to id 128000; ids from 128000 on are the Llama 3
    special tokens at their real ids and reserved names elsewhere."""
    from .gguf import SPECIAL_TOKENS
    from .tokenizer import BYTE_ENCODER, SPECIAL_BASE
    merges = train_bpe(_BPE_CORPUS, n_merges)
    toks = [chr(BYTE_ENCODER[b]) for b in range(256)]
    seen = set(toks)
    for a, b in merges:
        if a + b not in seen:
            toks.append(a + b)
            seen.add(a + b)
    if len(toks) > min(vocab, SPECIAL_BASE):
        raise ValueError(f"vocabulary of {vocab} ids is too small for {len(toks)} byte and merge tokens")
    toks += [f"<|synthetic_{i}|>" for i in range(len(toks), min(vocab, SPECIAL_BASE))]
    toks += [SPECIAL_TOKENS.get(i, f"<|reserved_special_token_{i - SPECIAL_BASE}|>")
             for i in range(SPECIAL_BASE, vocab)]
    return toks, [f"{a} {b}" for a, b in merges]
