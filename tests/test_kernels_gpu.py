"""GPU parity of every per-kernel operator (the CudaKernelFactory surface)
against the oracle and the reference's known answers.  Calls go through the
C ABI of libllamacuda.so."""
import math

import numpy as np
import pytest

from parity import assert_kernel_close, max_rel_err

pytestmark = pytest.mark.gpu
f32 = np.float32


@pytest.fixture(scope="module")
def factory(acc):
    from llamahat import CudaKernelFactory
    f = CudaKernelFactory()
    return f, acc


# ------------------------------------------------------- known answers

def test_known_answer_gemv(factory, golden):
    f, acc = factory
    g = f.createGEMV(acc)
    c = golden["gemv_f32_4x3"]
    y = np.zeros(4, f32)
    g.apply(np.array(c["matrix"], f32), np.array(c["vector"], f32), y, 4, 3)
    np.testing.assert_allclose(y, c["expected"], atol=c["tol"], rtol=0)
    c = golden["gemv_f16_2x4"]
    y = np.zeros(2, f32)
    g.apply(np.array(c["matrix"], np.float16), np.array(c["vector"], f32), y, 2, 4)
    np.testing.assert_allclose(y, c["expected"], atol=c["tol"], rtol=0)


def test_known_answer_rmsnorm(factory, golden):
    f, acc = factory
    k = f.createRMSNorm(acc)
    c = golden["rmsnorm_simple"]
    x = np.array(c["input"], f32)
    k.apply(x, np.array(c["weight"], f32), 4)
    assert abs(float(np.mean(x.astype(np.float64) ** 2)) - 1.0) <= c["tol"]
    c = golden["rmsnorm_weights"]
    x = np.array(c["input"], f32)
    k.apply(x, np.array(c["weight"], f32), 2)
    np.testing.assert_allclose(x, c["expected"], atol=c["tol"], rtol=0)


def test_known_answer_rope(factory, golden):
    f, acc = factory
    c = golden["rope_2x4_pos1"]
    x = np.array(c["input"], f32)
    f.createRoPE(acc).apply(x, c["pos"], c["num_heads"], c["head_dim"], c["theta"])
    np.testing.assert_allclose(x, c["expected"], atol=c["tol"], rtol=0)


@pytest.mark.parametrize("cid", ["silu_3", "silu_ramp_3", "silu_ramp_64", "silu_ramp_2048", "silu_ramp_8192"])
def test_known_answer_silu(factory, golden, cid):
    f, acc = factory
    c = golden[cid]
    x = np.array(c["input"], f32)
    f.createSiLU(acc).apply(x, x.size)
    np.testing.assert_allclose(x, c["expected"], atol=c["tol"], rtol=0)
    # exp is evaluated in double like (float)Math.exp: results match bit for bit.
    assert np.array_equal(x, np.array(c["expected"], f32))


def test_known_answer_softmax(factory, golden):
    f, acc = factory
    s = f.createSoftmax(acc)
    c = golden["softmax_values"]
    x = np.array(c["input"], f32)
    s.apply(x, 5)
    np.testing.assert_allclose(x, c["expected"], atol=c["tol"], rtol=0)
    assert abs(float(x.sum()) - 1.0) <= 1e-4
    x = np.array(golden["softmax_monotonic"]["input"], f32)
    s.apply(x, 4)
    assert all(x[i] < x[i + 1] for i in range(3))
    x = np.array(golden["softmax_stable"]["input"], f32)
    s.apply(x, 3)
    assert np.all(np.isfinite(x)) and abs(float(x.sum()) - 1.0) <= 1e-4
    c = golden["softmax_row"]
    x = np.array(c["input"], f32)
    s.applyRow(x, 3, 4)
    assert abs(float(x[3:7].sum()) - 1.0) <= 1e-4 and np.all(x[:3] == 0) and np.all(x[7:] == 0)


def test_known_answer_attention(factory, golden):
    f, acc = factory
    a, s = f.createAttention(acc), f.createSoftmax(acc)
    c = golden["attention_uniform"]
    hd, sl = c["head_dim"], c["seq_len"]
    sc = np.zeros(sl, f32)
    a.computeScores(np.array(c["query"], f32), np.array(c["keys"], f32), sc, sl, hd)
    np.testing.assert_allclose(sc, c["expected_scores"], atol=c["tol"], rtol=0)
    s.apply(sc, sl)
    np.testing.assert_allclose(sc, c["expected_probs"], atol=c["tol"], rtol=0)
    out = np.zeros(hd, f32)
    a.computeValues(sc, np.array(c["values"], f32), out, sl, hd)
    np.testing.assert_allclose(out, c["expected_out"], atol=c["tol"], rtol=0)


@pytest.mark.parametrize("cid", ["argmax_positive", "argmax_negative", "argmax_mixed", "argmax_last", "argmax_single"])
def test_known_answer_argmax(acc, golden, cid):
    from llamahat.inference import LlamaInference
    c = golden[cid]
    assert LlamaInference.argmax(np.array(c["values"], f32)) == c["expected_index"]


def test_f16_exact_values(factory, golden):
    f, acc = factory
    c = golden["f16_exact"]
    W = np.array(c["bits"], np.uint16).reshape(-1, 1)
    y = np.zeros(W.shape[0], f32)
    f.createGEMV(acc).apply(W, np.ones(1, f32), y, W.shape[0], 1)
    assert list(y) == c["values"]


# ------------------------------------------------------- seeded parity

GEMV_SHAPES = [(2048, 2048), (512, 2048), (8192, 2048), (2048, 8192), (128256, 2048),
               (1, 256), (3, 300), (7, 768), (100, 16384), (33, 4096), (5, 2048), (1000, 512)]


@pytest.mark.parametrize("rows,cols", GEMV_SHAPES)
def test_gemv_f16_parity(factory, oracle, rows, cols):
    f, acc = factory
    rng = np.random.default_rng(rows * 7 + cols)
    W = (rng.standard_normal((rows, cols), dtype=np.float32) * 0.02).astype(np.float16)
    x = rng.standard_normal(cols, dtype=np.float32)
    y = np.zeros(rows, f32)
    f.createGEMV(acc).apply(W, x, y, rows, cols)
    assert_kernel_close(y, oracle.gemv_f16(W, x))


def test_gemv_device_buffers(factory, oracle):
    torch = pytest.importorskip("torch")
    f, acc = factory
    rng = np.random.default_rng(5)
    W = (rng.standard_normal((4096, 2048), dtype=np.float32) * 0.02).astype(np.float16)
    x = rng.standard_normal(2048, dtype=np.float32)
    dW, dx = torch.from_numpy(W).cuda(), torch.from_numpy(x).cuda()
    dy = torch.zeros(4096, dtype=torch.float32, device="cuda")
    f.createGEMV(acc).apply(dW, dx, dy, 4096, 2048)
    acc.synchronize()
    assert_kernel_close(dy.cpu().numpy(), oracle.gemv_f16(W, x))


@pytest.mark.parametrize("batch", [1, 8, 64])
def test_gemv_batched_parity(factory, oracle, batch):
    f, acc = factory
    rng = np.random.default_rng(batch)
    rows, cols = 1024, 2048
    W = (rng.standard_normal((rows, cols), dtype=np.float32) * 0.02).astype(np.float16)
    X = rng.standard_normal((batch, cols), dtype=np.float32)
    Y = np.zeros((batch, rows), f32)
    f.createGEMV(acc).apply_batched(W, X, Y, rows, cols, batch)
    for b in range(batch):
        assert_kernel_close(Y[b], oracle.gemv_f16(W, X[b]))


def test_gemv_f32_parity(factory, oracle):
    f, acc = factory
    rng = np.random.default_rng(9)
    W = rng.standard_normal((777, 333), dtype=np.float32)
    x = rng.standard_normal(333, dtype=np.float32)
    y = np.zeros(777, f32)
    f.createGEMV(acc).apply(W, x, y, 777, 333)
    assert_kernel_close(y, oracle.gemv_f32(W, x))


@pytest.mark.parametrize("rows,width", [(1, 2048), (64, 2048), (4096, 2048), (3, 1000), (1, 2)])
def test_rmsnorm_parity(factory, oracle, rows, width):
    f, acc = factory
    rng = np.random.default_rng(rows + width)
    x = rng.standard_normal((rows, width), dtype=np.float32)
    w = (1 + 0.01 * rng.standard_normal(width)).astype(f32)
    ref = np.stack([oracle.rmsnorm(x[r], w) for r in range(rows)])
    k = f.createRMSNorm(acc)
    if rows == 1:
        y = x[0].copy()
        k.apply(y, w, width)
    else:
        y = x.copy()
        k.apply_rows(y, w, rows, width, 1e-5)
    assert_kernel_close(y, ref)


@pytest.mark.parametrize("n_heads", [32, 8])
def test_rope_parity(factory, oracle, n_heads):
    f, acc = factory
    rng = np.random.default_rng(n_heads)
    k = f.createRoPE(acc)
    for pos in [0, 1, 47, 2047, int(rng.integers(0, 8192)), 8191]:
        v = rng.standard_normal(n_heads * 64, dtype=np.float32)
        ref = oracle.rope(v, pos, n_heads, 64, 500000.0)
        y = v.copy()
        k.apply(y, pos, n_heads, 64, 500000.0)
        assert_kernel_close(y, ref, tol=1e-6)


def test_rope_rows_parity(factory, oracle):
    f, acc = factory
    rng = np.random.default_rng(3)
    rows = 64
    v = rng.standard_normal((rows, 32 * 64), dtype=np.float32)
    pos = rng.integers(0, 8192, rows).astype(np.int32)
    ref = np.stack([oracle.rope(v[r], int(pos[r]), 32, 64, 500000.0) for r in range(rows)])
    y = v.copy()
    f.createRoPE(acc).apply_rows(y, pos, rows, 32, 64, 500000.0)
    assert_kernel_close(y, ref, tol=1e-6)
    assert np.mean(y == ref) > 0.999


@pytest.mark.parametrize("rows", [1, 64, 4096])
def test_swiglu_parity(factory, oracle, rows):
    f, acc = factory
    rng = np.random.default_rng(rows)
    g = rng.standard_normal((rows, 8192), dtype=np.float32)
    u = rng.standard_normal((rows, 8192), dtype=np.float32)
    y = g.copy()
    f.createSiLU(acc).swiglu(y, u, g.size)
    ref = oracle.swiglu(g.ravel(), u.ravel()).reshape(rows, 8192)
    assert np.array_equal(y, ref)


@pytest.mark.parametrize("rows,width", [(1, 128), (64, 1024), (1, 8192), (4096, 8192), (2, 20000), (3, 1)])
def test_softmax_parity(factory, oracle, rows, width):
    f, acc = factory
    rng = np.random.default_rng(rows * 3 + width)
    x = (rng.standard_normal((rows, width), dtype=np.float32) * 2.0).astype(f32)
    ref = np.stack([oracle.softmax(x[r]) for r in range(rows)])
    y = x.copy()
    s = f.createSoftmax(acc)
    if rows == 1:
        s.apply(y[0], width)
    else:
        s.apply_rows(y, rows, width)
    assert_kernel_close(y, ref)


@pytest.mark.parametrize("seq_len", [1, 4, 47, 1000, 2048])
def test_attention_scores_values_bit_exact(factory, oracle, seq_len):
    f, acc = factory
    rng = np.random.default_rng(seq_len)
    q = rng.standard_normal(64, dtype=np.float32)
    K = rng.standard_normal((seq_len, 64), dtype=np.float32)
    V = rng.standard_normal((seq_len, 64), dtype=np.float32)
    a = f.createAttention(acc)
    sc = np.zeros(seq_len, f32)
    a.computeScores(q, K, sc, seq_len, 64)
    ref = oracle.attn_scores(q, K, seq_len, 64)
    assert np.array_equal(sc, ref)
    p = oracle.softmax(ref)
    out = np.zeros(64, f32)
    a.computeValues(p, V, out, seq_len, 64)
    assert np.array_equal(out, oracle.attn_values(p, V, seq_len, 64))


@pytest.mark.parametrize("batch,seq", [(1, 1), (1, 47), (1, 128), (1, 1024), (1, 8192), (4, 300), (64, 128),
                                       (64, 1024), (64, 8192)])
def test_attention_decode_parity(factory, oracle, batch, seq):
    """Fused GQA decode attention (32 q / 8 kv heads) vs the reference's per-head loop
    (TransformerBlock.java:153-192 with Attention.java:32-61), including the
    attention workload's 64-sequence batches at 1024 and 8192 cached positions
    (the throughput path with split merges); there a sample of sequences, the
    first and last among them, is checked."""
    f, acc = factory
    rng = np.random.default_rng(batch * 1000 + seq)
    nh, nkv, hd = 32, 8, 64
    max_seq = seq + 3
    q = rng.standard_normal((batch, nh * hd), dtype=np.float32)
    K = rng.standard_normal((batch, max_seq, nkv, hd), dtype=np.float32)
    V = rng.standard_normal((batch, max_seq, nkv, hd), dtype=np.float32)
    lens = np.array([seq - (b % 3) if seq > 3 else seq for b in range(batch)], np.int32)
    out = np.zeros((batch, nh * hd), f32)
    f.createAttention(acc).decode(q, K, V, out, lens, batch, nh, nkv, hd, max_seq * nkv * hd, hd, nkv * hd)
    assert np.isfinite(out).all()
    check = range(batch) if batch * seq <= 64 * 128 else sorted({0, 1, 2, 17, 33, 50, batch - 2, batch - 1})
    for b in check:
        ref = oracle.gqa_attention(q[b], K[b], V[b], int(lens[b]), nh, nkv, hd)
        assert_kernel_close(out[b], ref)
        if batch == 1 and seq <= 64:
            # One split: the reference's loop order, bit for bit.
            assert np.array_equal(out[b], ref)


def test_argmax_large_with_ties(acc):
    from llamahat.inference import LlamaInference
    rng = np.random.default_rng(1)
    v = rng.standard_normal(128256).astype(f32)
    v[77777] = 9.0
    v[99999] = 9.0
    v[100] = 9.0
    assert LlamaInference.argmax(v) == 100
    v[0] = np.nan
    assert LlamaInference.argmax(v) == 0
    v[0] = -np.inf
    v[5] = np.nan
    assert LlamaInference.argmax(v) == 100
