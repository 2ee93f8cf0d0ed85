"""TransformerBlock / LlamaInference driven through an IKernelFactory, call for call.

Reference: src/main/java/com/arturskowronski/llama3babylon/hat/TransformerBlock.java:130-217
and LlamaInference.java:117-164.  This is the reference's own orchestration
(host buffers, per-head KV gather, one kernel call per operation) with the
kernels supplied by a factory -- the drop-in path of `CudaKernelFactory`.
It exists to show the per-kernel operators are interchangeable with the
reference's; the fast path is the fused device-resident decode
(`inference.LlamaInference`).
"""
from __future__ import annotations

import numpy as np

from .config import LlamaConfig
from .kernels import IKernelFactory

f32 = np.float32


class FactoryTransformerBlock:
    def __init__(self, cfg: LlamaConfig, weights: dict, layer: int, factory: IKernelFactory, acc=None):
        self.cfg = cfg
        p = f"blk.{layer}."
        g = lambda n: np.ascontiguousarray(weights[p + n])
        self.attn_norm, self.ffn_norm = g("attn_norm.weight").astype(f32), g("ffn_norm.weight").astype(f32)
        self.wq, self.wk, self.wv, self.wo = g("attn_q.weight"), g("attn_k.weight"), g("attn_v.weight"), g("attn_output.weight")
        self.w1, self.w2, self.w3 = g("ffn_gate.weight"), g("ffn_down.weight"), g("ffn_up.weight")
        self.rms, self.gemv, self.rope = factory.createRMSNorm(acc), factory.createGEMV(acc), factory.createRoPE(acc)
        self.attn, self.softmax, self.silu = factory.createAttention(acc), factory.createSoftmax(acc), factory.createSiLU(acc)
        c = cfg
        self.q, self.k, self.v = np.zeros(c.q_dim, f32), np.zeros(c.kv_dim, f32), np.zeros(c.kv_dim, f32)
        self.att_out = np.zeros(c.q_dim, f32)
        self.q_head, self.head_out = np.zeros(c.head_dim, f32), np.zeros(c.head_dim, f32)
        self.k_head = np.zeros(c.max_seq * c.head_dim, f32)
        self.v_head = np.zeros(c.max_seq * c.head_dim, f32)
        self.scores = np.zeros(c.max_seq, f32)
        self.f1, self.f3, self.fo = np.zeros(c.hidden, f32), np.zeros(c.hidden, f32), np.zeros(c.dim, f32)

    def forward(self, x: np.ndarray, pos: int, k_cache: np.ndarray, v_cache: np.ndarray) -> None:
        c = self.cfg
        hd, kvd = c.head_dim, c.kv_dim
        residual = x.copy()                                                   # :139
        self.rms.apply(x, self.attn_norm, c.dim)                              # :142
        self.gemv.apply(self.wq, x, self.q, c.q_dim, c.dim)                   # :145
        self.gemv.apply(self.wk, x, self.k, kvd, c.dim)                       # :146
        self.gemv.apply(self.wv, x, self.v, kvd, c.dim)                       # :147
        self.rope.apply(self.q, pos, c.n_heads, hd, c.rope_theta)             # :150
        self.rope.apply(self.k, pos, c.n_kv_heads, hd, c.rope_theta)          # :151
        k_cache[pos * kvd:(pos + 1) * kvd] = self.k                           # :158-162
        v_cache[pos * kvd:(pos + 1) * kvd] = self.v
        seq = pos + 1
        kv_mul = c.n_heads // c.n_kv_heads
        kc = k_cache[:seq * kvd].reshape(seq, c.n_kv_heads, hd)
        vc = v_cache[:seq * kvd].reshape(seq, c.n_kv_heads, hd)
        for h in range(c.n_heads):                                           # :165-192
            kvh = h // kv_mul
            self.q_head[:] = self.q[h * hd:(h + 1) * hd]
            self.k_head[:seq * hd] = kc[:, kvh].ravel()
            self.v_head[:seq * hd] = vc[:, kvh].ravel()
            self.attn.computeScores(self.q_head, self.k_head, self.scores, seq, hd)
            self.softmax.apply(self.scores, seq)
            self.attn.computeValues(self.scores, self.v_head, self.head_out, seq, hd)
            self.att_out[h * hd:(h + 1) * hd] = self.head_out
        self.gemv.apply(self.wo, self.att_out, x, c.dim, c.q_dim)             # :195
        x += residual                                                         # :198 (float32 add)
        residual = x.copy()                                                   # :201
        self.rms.apply(x, self.ffn_norm, c.dim)                               # :204
        self.gemv.apply(self.w1, x, self.f1, c.hidden, c.dim)                 # :207
        self.gemv.apply(self.w3, x, self.f3, c.hidden, c.dim)                 # :208
        self.silu.apply(self.f1, c.hidden)                                    # :209
        self.f1 *= self.f3                                                    # :210
        self.gemv.apply(self.w2, self.f1, self.fo, c.dim, c.hidden)           # :211
        x[:] = residual + self.fo                                             # :214-216


class FactoryLlamaInference:
    """LlamaInference.forward through per-kernel factory calls (host buffers)."""

    def __init__(self, cfg: LlamaConfig, weights: dict, factory: IKernelFactory, acc=None):
        self.cfg = cfg
        self.emb = np.ascontiguousarray(weights["token_embd.weight"])
        self.out_norm = np.ascontiguousarray(weights["output_norm.weight"], f32)
        self.blocks = [FactoryTransformerBlock(cfg, weights, l, factory, acc) for l in range(cfg.n_layers)]
        self.rms, self.gemv = factory.createRMSNorm(acc), factory.createGEMV(acc)
        self.k_cache = [np.zeros(cfg.max_seq * cfg.kv_dim, f32) for _ in range(cfg.n_layers)]
        self.v_cache = [np.zeros(cfg.max_seq * cfg.kv_dim, f32) for _ in range(cfg.n_layers)]
        self.x = np.zeros(cfg.dim, f32)
        self.logits = np.zeros(cfg.vocab, f32)

    def forward(self, token: int, pos: int) -> np.ndarray:
        self.x[:] = self.emb[token].astype(f32)                              # :122-140
        for l, b in enumerate(self.blocks):                                   # :143-145
            b.forward(self.x, pos, self.k_cache[l], self.v_cache[l])
        self.rms.apply(self.x, self.out_norm, self.cfg.dim)                  # :148
        self.gemv.apply(self.emb, self.x, self.logits, self.cfg.vocab, self.cfg.dim)  # :151-156
        return self.logits.copy()                                            # :159-162
