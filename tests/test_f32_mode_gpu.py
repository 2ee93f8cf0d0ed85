"""WeightStorageMode.F32 on the GPU (H/WeightStorageMode.java,
H/LlamaInference.java:102-108): projections and embedding stored as fp32 and
multiplied by fp32-weight GEMVs (K/GEMV.java:34-43), checked against the
oracle's F32 storage mode -- logits within 1e-2 and the kernel gate, greedy
tokens identical wherever the oracle's top-2 margin exceeds 1e-2.  Calls go
through the C ABI."""
import numpy as np
import pytest

from parity import LOGITS_ABS_TOL, MARGIN, assert_kernel_close, top2_margin

pytestmark = pytest.mark.gpu


def _f32_weights(w, seed):
    """The F16 projections plus a perturbation below F16 resolution, so the
    fp32 values are not representable in F16 (a true F32 GGUF)."""
    rng = np.random.default_rng(seed)
    out = {}
    for k, v in w.items():
        if v.dtype == np.float16:
            a = v.astype(np.float32)
            out[k] = a + (rng.standard_normal(a.shape).astype(np.float32) * np.float32(1e-5))
        else:
            out[k] = v
    return out


def _follow(om, prompt, gen):
    """Tokens agree with the oracle's argmax along the GPU's path until a near-tie."""
    logits = None
    for pos, t in enumerate(prompt):
        logits = om.forward(int(t), pos)
    checked = 0
    for i, t in enumerate(gen):
        if top2_margin(logits) <= MARGIN:
            break
        assert int(t) == int(np.argmax(logits)), f"token {i}: gpu {t} oracle {int(np.argmax(logits))}"
        checked += 1
        if i + 1 < len(gen):
            logits = om.forward(int(t), len(prompt) + i)
    return checked


def test_f32_mode_tiny_f16_values(acc, tiny_weights, oracle):
    """F16 tensors uploaded in F32 mode are widened exactly: the F32 path
    computes the F16 path's values (WeightStorageModeComparisonTest)."""
    from llamahat import CudaModel, LlamaInference, WeightStorageMode
    cfg, w = tiny_weights
    model = CudaModel(cfg, w, acc=acc, weight_mode=WeightStorageMode.F32)
    inf = LlamaInference(model)
    om = oracle.OracleModel(cfg, w, f32=True)
    for pos, t in enumerate([3, 17, 999, 0, 512, 5, 700, 1]):
        g, r = inf.forward(t, pos), om.forward(t, pos)
        assert np.abs(g - r).max() <= LOGITS_ABS_TOL
        assert_kernel_close(g, r)
    prompt = [11, 22, 33, 44, 55]
    gen = LlamaInference(model).generate(prompt, 16, stopTokens=())
    assert len(gen) == 16
    assert _follow(oracle.OracleModel(cfg, w, f32=True), prompt, gen) >= 8


def test_f32_mode_tiny_true_f32_tensors(acc, tiny_weights, oracle):
    """F32 tensors (not F16-representable) as LlamaModel.mapTensor accepts them."""
    from llamahat import CudaModel, LlamaInference, WeightStorageMode
    cfg, w16 = tiny_weights
    w = _f32_weights(w16, 5)
    model = CudaModel(cfg, w, acc=acc, weight_mode=WeightStorageMode.F32)
    inf = LlamaInference(model)
    om = oracle.OracleModel(cfg, w, f32=True)
    om16 = oracle.OracleModel(cfg, w16)
    for pos, t in enumerate([7, 70, 700, 77]):
        g, r = inf.forward(t, pos), om.forward(t, pos)
        assert np.abs(g - r).max() <= LOGITS_ABS_TOL
        assert_kernel_close(g, r)
        # the perturbation is visible: the F16 oracle differs from the F32 one
        r16 = om16.forward(t, pos)
        assert not np.array_equal(r16, r)
    prompt = [9, 8, 7]
    gen = LlamaInference(model).generate(prompt, 12, stopTokens=())
    assert _follow(oracle.OracleModel(cfg, w, f32=True), prompt, gen) >= 6


def test_f32_mode_stop_token_and_stream(acc, tiny_weights, oracle):
    from llamahat import CudaModel, LlamaInference, WeightStorageMode
    cfg, w = tiny_weights
    model = CudaModel(cfg, w, acc=acc, weight_mode=WeightStorageMode.F32)
    prompt = [101, 202, 303]
    free = oracle.OracleModel(cfg, w, f32=True).generate(prompt, 10, stop=())
    stop = int(free[3])
    first = list(free).index(stop)
    seen = []
    gen = LlamaInference(model).generate(prompt, 10, stopTokens={stop}, onToken=lambda t, i: seen.append((i, t)))
    assert list(gen) == list(free[:first + 1])
    assert seen == list(enumerate(gen))


def test_f32_mode_gguf_load(acc, tiny_weights, tmp_path):
    from llamahat import CudaModel, LlamaInference, WeightStorageMode
    from llamahat.gguf import write_gguf
    cfg, w = tiny_weights
    path = str(tmp_path / "tiny32.gguf")
    write_gguf(path, cfg, _f32_weights(w, 9))
    loaded = CudaModel(gguf_path=path, acc=acc, max_seq=cfg.max_seq, weight_mode=WeightStorageMode.F32)
    direct = CudaModel(cfg, _f32_weights(w, 9), acc=acc, weight_mode=WeightStorageMode.F32)
    assert np.array_equal(LlamaInference(loaded).forward(42, 0), LlamaInference(direct).forward(42, 0))


def test_f32_mode_limits(acc, tiny_weights):
    from llamahat import Batch, CudaModel, IllegalArgumentError, LlamaCudaError, Session, WeightStorageMode
    cfg, w = tiny_weights
    model = CudaModel(cfg, w, acc=acc, weight_mode=WeightStorageMode.F32)
    with pytest.raises(LlamaCudaError, match="F16 weights"):
        Batch(model, 2)                      # the batch engine runs on F16 weights
    with pytest.raises(LlamaCudaError):
        Session(model).enable_trace(16)      # the trace belongs to the fused F16 kernel
    with pytest.raises(IllegalArgumentError):
        Session(model).forward(cfg.vocab, 0)  # token outside the vocabulary
    assert WeightStorageMode.fromString("fast") is WeightStorageMode.F16_FAST
    with pytest.raises(ValueError):
        WeightStorageMode.fromString("bf16")


def test_f32_mode_llama_1b_one_layer(acc, oracle):
    """Llama-3.2-1B shapes, one layer, random F16 weights widened to fp32."""
    from llamahat import LLAMA_3_2_1B, CudaModel, LlamaInference, WeightStorageMode
    from llamahat.synth import synth_prompt, synth_weights
    cfg = LLAMA_3_2_1B.with_(n_layers=1, max_seq=64)
    w = synth_weights(cfg, seed=1234)
    model = CudaModel(cfg, w, acc=acc, weight_mode=WeightStorageMode.F32)
    prompt = [int(t) for t in synth_prompt(16, seed=1234)]
    gen = LlamaInference(model).generate(prompt, 8, stopTokens=())
    assert len(gen) == 8
    om = oracle.OracleModel(cfg, w, f32=True)
    assert _follow(om, prompt, gen) >= 4
    inf = LlamaInference(model)
    for pos, t in enumerate(prompt + [int(x) for x in gen[:-1]]):
        g = inf.forward(t, pos)
    r = oracle.OracleModel(cfg, w, f32=True)
    for pos, t in enumerate(prompt + [int(x) for x in gen[:-1]]):
        rr = r.forward(t, pos)
    assert np.abs(g - rr).max() <= LOGITS_ABS_TOL
    assert_kernel_close(g, rr)
