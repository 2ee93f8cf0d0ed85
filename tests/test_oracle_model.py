"""The oracle's model-level glue (TransformerBlock.forward / LlamaInference
forward + generate) against an independent float64 numpy restatement, on the
small configuration.  CPU only."""
import numpy as np
import pytest


def np_forward_f64(cfg, w, tokens):
    """Float64 restatement of LlamaInference.forward over a token sequence;
    returns the logits of every position."""
    f = lambda a: np.asarray(a, np.float64)
    kc = np.zeros((cfg.n_layers, len(tokens), cfg.n_kv_heads, cfg.head_dim))
    vc = np.zeros_like(kc)
    hd, kvm = cfg.head_dim, cfg.n_heads // cfg.n_kv_heads
    freq = 1.0 / cfg.rope_theta ** (np.arange(0, hd, 2) / hd)

    def norm(x, g):
        return x / np.sqrt(np.mean(x * x) + cfg.rms_eps) * g

    def rope(v, pos, nh):
        v = v.reshape(nh, hd // 2, 2).copy()
        a = pos * freq
        c, s = np.cos(a), np.sin(a)
        v0, v1 = v[..., 0].copy(), v[..., 1].copy()
        v[..., 0], v[..., 1] = v0 * c - v1 * s, v0 * s + v1 * c
        return v.reshape(-1)

    out = []
    for pos, t in enumerate(tokens):
        x = f(w["token_embd.weight"][t])
        for l in range(cfg.n_layers):
            p = f"blk.{l}."
            xn = norm(x, f(w[p + "attn_norm.weight"]))
            q = rope(f(w[p + "attn_q.weight"]) @ xn, pos, cfg.n_heads)
            k = rope(f(w[p + "attn_k.weight"]) @ xn, pos, cfg.n_kv_heads)
            v = f(w[p + "attn_v.weight"]) @ xn
            kc[l, pos] = k.reshape(cfg.n_kv_heads, hd)
            vc[l, pos] = v.reshape(cfg.n_kv_heads, hd)
            att = np.zeros(cfg.n_heads * hd)
            for h in range(cfg.n_heads):
                K, V = kc[l, :pos + 1, h // kvm], vc[l, :pos + 1, h // kvm]
                s = K @ q[h * hd:(h + 1) * hd] / np.sqrt(hd)
                e = np.exp(s - s.max())
                att[h * hd:(h + 1) * hd] = (e / e.sum()) @ V
            x = x + f(w[p + "attn_output.weight"]) @ att
            xn = norm(x, f(w[p + "ffn_norm.weight"]))
            g, u = f(w[p + "ffn_gate.weight"]) @ xn, f(w[p + "ffn_up.weight"]) @ xn
            x = x + f(w[p + "ffn_down.weight"]) @ (g / (1 + np.exp(-g)) * u)
        out.append(f(w["token_embd.weight"]) @ norm(x, f(w["output_norm.weight"])))
    return np.array(out)


def test_oracle_forward_matches_f64(oracle, tiny_weights):
    cfg, w = tiny_weights
    om = oracle.OracleModel(cfg, w)
    toks = [3, 17, 999, 0, 512]
    ref = np_forward_f64(cfg, w, toks)
    for pos, t in enumerate(toks):
        lg = om.forward(t, pos)
        err = np.abs(lg - ref[pos]).max() / np.abs(ref[pos]).max()
        assert err < 1e-4, (pos, err)


def test_oracle_generate_is_prefill_then_greedy(oracle, tiny_weights):
    cfg, w = tiny_weights
    prompt = [5, 6, 7, 8]
    om = oracle.OracleModel(cfg, w)
    gen = om.generate(prompt, 6, stop=())
    # Restate LlamaInference.generate (LlamaInference.java:180-217) step by step.
    om2 = oracle.OracleModel(cfg, w)
    for i, t in enumerate(prompt):
        lg = om2.forward(t, i)
    toks = [oracle.argmax(lg)]
    while len(toks) < 6:
        lg = om2.forward(toks[-1], len(prompt) + len(toks) - 1)
        toks.append(oracle.argmax(lg))
    assert list(gen) == toks


def test_oracle_generate_stops_on_stop_token(oracle, tiny_weights):
    cfg, w = tiny_weights
    om = oracle.OracleModel(cfg, w)
    free = om.generate([1, 2, 3], 5, stop=())
    om2 = oracle.OracleModel(cfg, w)
    stop = int(free[1])
    stopped = om2.generate([1, 2, 3], 5, stop=(stop,))
    # The stop token is emitted, then generation ends (LlamaInference.java:201).
    first = list(free).index(stop)
    assert list(stopped) == list(free[:first + 1])


def test_oracle_gemv_close_to_f64(oracle):
    rng = np.random.default_rng(0)
    W = (rng.standard_normal((300, 2048)) * 0.02).astype(np.float16)
    x = rng.standard_normal(2048).astype(np.float32)
    y = oracle.gemv_f16(W, x)
    ref = W.astype(np.float64) @ x.astype(np.float64)
    assert np.abs(y - ref).max() < 1e-4


def test_oracle_f32_storage_mode_matches_f16(oracle, tiny_weights):
    """WeightStorageModeComparisonTest (integration/WeightStorageModeComparisonTest.java:23-84)
    asserts that F16, F16_FAST and F32 storage give bit-identical logits: the
    F32 mode widens the same F16 values exactly and the GEMV sums the same
    products in the same order.  Checked on the synthetic model."""
    cfg, w = tiny_weights
    m16 = oracle.OracleModel(cfg, w)
    m32 = oracle.OracleModel(cfg, w, f32=True)
    for pos, t in enumerate([5, 77, 3, 900]):
        assert np.array_equal(m16.forward(t, pos), m32.forward(t, pos))
    w32 = {k: (v.astype(np.float32) if v.dtype == np.float16 else v) for k, v in w.items()}
    m32b = oracle.OracleModel(cfg, w32, f32=True)  # F32 tensors as given
    m16.forward(5, 0)
    assert np.array_equal(m16.forward(6, 1), (m32b.forward(5, 0), m32b.forward(6, 1))[1])
