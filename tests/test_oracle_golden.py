"""The CPU oracle against the reference's own known-answer tests (golden
vectors transcribed in tests/golden/known_answers.json).  CPU only."""
import math

import numpy as np
import pytest

f32 = np.float32


def test_gemv_f32_4x3(oracle, golden):
    c = golden["gemv_f32_4x3"]
    W = np.array(c["matrix"], f32).reshape(c["rows"], c["cols"])
    y = oracle.gemv_f32(W, np.array(c["vector"], f32))
    np.testing.assert_allclose(y, c["expected"], atol=c["tol"], rtol=0)


def test_gemv_f16_2x4(oracle, golden):
    c = golden["gemv_f16_2x4"]
    W = np.array(c["matrix"], np.float16).reshape(c["rows"], c["cols"])
    y = oracle.gemv_f16(W, np.array(c["vector"], f32))
    np.testing.assert_allclose(y, c["expected"], atol=c["tol"], rtol=0)


def test_rmsnorm_simple(oracle, golden):
    c = golden["rmsnorm_simple"]
    x = oracle.rmsnorm(np.array(c["input"], f32), np.array(c["weight"], f32))
    ms = f32(0)
    for v in x:
        ms = f32(ms + f32(v * v))
    assert abs(float(ms) / len(x) - c["expected_mean_of_squares"]) <= c["tol"]


@pytest.mark.parametrize("cid", ["rmsnorm_weights", "rope_2x4_pos1", "silu_3", "silu_ramp_3", "silu_ramp_64",
                                 "silu_ramp_2048", "silu_ramp_8192", "softmax_values"])
def test_elementwise_known_answers(oracle, golden, cid):
    c = golden[cid]
    x = np.array(c["input"], f32)
    if c["kernel"] == "rmsnorm":
        y = oracle.rmsnorm(x, np.array(c["weight"], f32))
    elif c["kernel"] == "rope":
        y = oracle.rope(x, c["pos"], c["num_heads"], c["head_dim"], c["theta"])
    elif c["kernel"] == "silu":
        y = oracle.silu(x)
    else:
        y = oracle.softmax(x)
    np.testing.assert_allclose(y, c["expected"], atol=c["tol"], rtol=0)


def test_silu_ramps_bit_exact(oracle, golden):
    # The Java expression evaluated in binary32 must be reproduced exactly.
    for n in (3, 64, 2048, 8192):
        c = golden[f"silu_ramp_{n}"]
        y = oracle.silu(np.array(c["input"], f32))
        assert np.array_equal(y, np.array(c["expected"], f32))


def test_softmax_properties(oracle, golden):
    y = oracle.softmax(np.array(golden["softmax_sums_to_one"]["input"], f32))
    assert abs(float(y.sum(dtype=np.float64)) - 1.0) <= 1e-4
    y = oracle.softmax(np.array(golden["softmax_monotonic"]["input"], f32))
    assert all(y[i] < y[i + 1] for i in range(len(y) - 1))
    y = oracle.softmax(np.array(golden["softmax_stable"]["input"], f32))
    assert np.all(np.isfinite(y)) and abs(float(y.sum()) - 1.0) <= 1e-4
    c = golden["softmax_row"]
    y = oracle.softmax_row(np.array(c["input"], f32), c["row_offset"], c["row_size"])
    o, n = c["row_offset"], c["row_size"]
    assert abs(float(y[o:o + n].sum()) - 1.0) <= c["tol"]
    assert np.all(y[:o] == 0) and np.all(y[o + n:] == 0)


def test_attention_uniform(oracle, golden):
    c = golden["attention_uniform"]
    hd, sl = c["head_dim"], c["seq_len"]
    s = oracle.attn_scores(np.array(c["query"], f32), np.array(c["keys"], f32), sl, hd)
    np.testing.assert_allclose(s, c["expected_scores"], atol=c["tol"], rtol=0)
    p = oracle.softmax(s)
    np.testing.assert_allclose(p, c["expected_probs"], atol=c["tol"], rtol=0)
    o = oracle.attn_values(p, np.array(c["values"], f32), sl, hd)
    np.testing.assert_allclose(o, c["expected_out"], atol=c["tol"], rtol=0)


def test_f16_exact_values(oracle, golden):
    c = golden["f16_exact"]
    for v, b in zip(c["values"], c["bits"]):
        assert oracle.f16_to_f32(b) == v


def test_f16_all_bit_patterns(oracle):
    # Float.float16ToFloat is the exact IEEE widening: compare every pattern.
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    got = np.array([oracle.f16_to_f32(int(b)) for b in bits[::97]], f32)
    r = ref[::97]
    nan = np.isnan(r)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), r[~nan].view(np.uint32))


@pytest.mark.parametrize("cid", ["argmax_positive", "argmax_negative", "argmax_mixed", "argmax_last", "argmax_single"])
def test_argmax(oracle, golden, cid):
    c = golden[cid]
    assert oracle.argmax(np.array(c["values"], f32)) == c["expected_index"]


def test_argmax_ties_and_nan(oracle):
    assert oracle.argmax(np.array([1, 5, 5, 2], f32)) == 1
    assert oracle.argmax(np.array([np.nan, 5, 7], f32)) == 0      # strict '>' never beats NaN
    assert oracle.argmax(np.array([1, np.nan, 7, 7], f32)) == 2


def test_rope_interleaved_not_half_split(oracle):
    # Pairs are (v[i], v[i+1]) (RoPE.java:46-49): a vector with only v[1] set
    # must only move within the first pair.
    v = np.zeros(8, f32)
    v[1] = 1.0
    y = oracle.rope(v, 3, 1, 8, 500000.0)
    assert np.all(y[2:] == 0) and y[0] != 0
    assert y[0] == f32(-math.sin(3.0)) and y[1] == f32(math.cos(3.0))
