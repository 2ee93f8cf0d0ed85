"""GPU parity of multi-sequence serving (lc_batch_*): every sequence of a
batch must get LlamaInference.generate's result (H/LlamaInference.java
:180-217) -- checked against the oracle's greedy path: tokens identical
wherever the oracle's top-2 logit margin exceeds 1e-2, logits within 1e-2.
Calls go through the C ABI."""
import numpy as np
import pytest

from parity import LOGITS_ABS_TOL, MARGIN, top2_margin

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny(acc, tiny_weights):
    from llamahat import CudaModel
    cfg, w = tiny_weights
    return cfg, w, CudaModel(cfg, w, acc=acc)


def follow_oracle(om, prompt, gen, max_new):
    """Runs the oracle along the GPU's token path; returns the number of
    generated tokens checked.  Each GPU token must be the oracle's argmax
    unless the oracle's top-2 margin there is <= MARGIN (then the paths may
    legitimately part and the check stops).  The oracle overwrites its KV
    cache from position 0, so one OracleModel serves every sequence."""
    logits = None
    for pos, t in enumerate(prompt):
        logits = om.forward(int(t), pos)
    for i, t in enumerate(gen):
        if top2_margin(logits) <= MARGIN:
            return i
        assert int(t) == int(np.argmax(logits)), f"token {i}: gpu {t} oracle {int(np.argmax(logits))}"
        if i + 1 < len(gen):
            logits = om.forward(int(t), len(prompt) + i)
    return len(gen)


def test_batch_matches_oracle_tiny(tiny, oracle):
    from llamahat import Batch
    cfg, w, model = tiny
    om = oracle.OracleModel(cfg, w)
    rng = np.random.default_rng(3)
    lens = [1, 5, 9, 2, 16]
    prompts = [rng.integers(0, cfg.vocab, n).astype(np.int32) for n in lens]
    b = Batch(model, 8)
    outs = b.generate(prompts, 12, stop=())
    checked = 0
    for p, g in zip(prompts, outs):
        assert len(g) == 12
        checked += follow_oracle(om, p, g, 12)
    assert checked >= 30  # most of the path is compared
    # logits of the last position of each sequence (its last generated token's forward)
    for s, (p, g) in enumerate(zip(prompts, outs)):
        for pos, t in enumerate(list(p) + list(g[:-1])):
            r = om.forward(int(t), pos)
        if len(p) + len(g) - 1 == max(len(q) for q in prompts) + 11:  # ran to the last step
            assert np.abs(b.logits(s) - r).max() <= LOGITS_ABS_TOL


def test_batch_prefill_matches_oracle_tiny(tiny, oracle):
    """Prompts of more than 64 tokens in all run as one prefill (row-tiled
    tcgen05 products, causal prefill attention); the sequences still follow
    the oracle, with logits within tolerance."""
    from llamahat import Batch
    cfg, w, model = tiny
    om = oracle.OracleModel(cfg, w)
    rng = np.random.default_rng(17)
    lens = [20, 3, 64, 1, 37, 9, 70, 12]  # 216 prompt tokens, one longer than a query block
    prompts = [rng.integers(0, cfg.vocab, n).astype(np.int32) for n in lens]
    b = Batch(model, 8)
    outs = b.generate(prompts, 6, stop=())
    checked = 0
    for p, g in zip(prompts, outs):
        assert len(g) == 6
        checked += follow_oracle(om, p, g, 6)
    assert checked >= 30
    for s, (p, g) in enumerate(zip(prompts, outs)):
        for pos, t in enumerate(list(p) + list(g[:-1])):
            r = om.forward(int(t), pos)
        assert np.abs(b.logits(s) - r).max() <= LOGITS_ABS_TOL


def test_batch_prefill_agrees_with_stepwise(tiny):
    """The same prompts through the prefill path (more than 64 tokens in
    all) and position by position (one sequence at a time) give the same
    greedy tokens."""
    from llamahat import Batch
    cfg, w, model = tiny
    rng = np.random.default_rng(23)
    prompts = [rng.integers(0, cfg.vocab, 40).astype(np.int32) for _ in range(4)]
    b = Batch(model, 4)
    together = b.generate(prompts, 8, stop=())   # 160 rows: prefill
    for p, g in zip(prompts, together):
        alone = b.generate([p], 8, stop=())[0]   # 40 rows: position by position
        assert list(g) == list(alone)


def test_batch_agrees_with_single_sequence_path(tiny):
    """The batch engine (tcgen05 products) and the fused single-sequence
    kernel give the same greedy tokens on the same prompts."""
    from llamahat import Batch, Session
    cfg, w, model = tiny
    prompts = [[11, 22, 33, 44, 55, 66, 77, 88], [101, 202, 303], [9, 8, 7, 6]]
    outs = Batch(model, 4).generate(prompts, 16, stop=())
    for p, g in zip(prompts, outs):
        assert list(g) == list(Session(model).generate(p, 16, stop=()))


def test_batch_stop_tokens(tiny, oracle):
    from llamahat import Batch
    cfg, w, model = tiny
    prompt = [101, 202, 303]
    free = oracle.OracleModel(cfg, w).generate(prompt, 10, stop=())
    stop = int(free[2])
    outs = Batch(model, 2).generate([prompt, prompt], 10, stop={stop})
    first = list(free).index(stop)
    for g in outs:
        assert list(g) == list(free[:first + 1])


def test_batch_reuse_and_sizes(tiny):
    """A batch object serves calls of different sizes; results do not depend
    on the other sequences of the call."""
    from llamahat import Batch
    cfg, w, model = tiny
    b = Batch(model, 64)
    rng = np.random.default_rng(9)
    prompts = [rng.integers(0, cfg.vocab, 4).astype(np.int32) for _ in range(64)]
    full = b.generate(prompts, 6, stop=())
    one = b.generate(prompts[17:18], 6, stop=())
    assert list(one[0]) == list(full[17])
    five = b.generate(prompts[:5], 6, stop=())
    for i in range(5):
        assert list(five[i]) == list(full[i])
    t, d, n = b.last_ms()
    assert t > 0 and d > 0 and n == 4 + 6 - 1


def test_batch_rejects_bad_arguments(tiny):
    from llamahat import Batch, IllegalArgumentError
    cfg, w, model = tiny
    b = Batch(model, 2)
    with pytest.raises(IllegalArgumentError):
        b.generate([[1], [2], [3]], 4)               # more sequences than max_batch
    with pytest.raises(IllegalArgumentError):
        b.generate([[1, cfg.vocab]], 4)              # token out of range
    with pytest.raises(IllegalArgumentError):
        b.generate([[1] * cfg.max_seq], 2)           # past max_seq
    with pytest.raises(IllegalArgumentError):
        Batch(model, 65)
    assert len(b.generate([[1, 2]], 3, stop=())[0]) == 3  # still usable


def test_batch_1b_matches_oracle(acc, oracle):
    """Llama-3.2-1B shapes (random weights), 4 sequences: the first
    generated tokens follow the oracle."""
    from llamahat import Batch, CudaModel
    from llamahat.config import LLAMA_3_2_1B
    from llamahat.synth import synth_weights
    cfg = LLAMA_3_2_1B.with_(max_seq=256)
    w = synth_weights(cfg, seed=1234)
    model = CudaModel(cfg, w, acc=acc)
    om = oracle.OracleModel(cfg, w)
    prompts = [[128000, 9906, 11], [1, 2, 3, 4, 5], [77777], [500, 600]]
    outs = Batch(model, 4).generate(prompts, 4, stop=())
    checked = sum(follow_oracle(om, p, g, 4) for p, g in zip(prompts, outs))
    assert checked >= 8


def test_batch_1b_prefill_matches_oracle(acc, oracle):
    """Llama-3.2-1B shapes (random weights), prompts of 129 tokens in all, so
    they run as one prefill pass at the real dimensions: row-tiled tcgen05
    products over all prompt rows, the causal prefill attention and K/V
    written at (sequence, position).  The reference prefills token by token
    (H/LlamaInference.java:186-193); every sequence must still follow the
    oracle's greedy path and end with logits within 1e-2 of the oracle's."""
    from llamahat import Batch, CudaModel
    from llamahat.config import LLAMA_3_2_1B
    from llamahat.synth import synth_weights
    cfg = LLAMA_3_2_1B.with_(max_seq=256)
    w = synth_weights(cfg, seed=1234)
    model = CudaModel(cfg, w, acc=acc)
    om = oracle.OracleModel(cfg, w)
    rng = np.random.default_rng(4321)
    lens = [32, 40, 7, 50]  # 129 prompt rows
    prompts = [rng.integers(0, 128000, n).astype(np.int32) for n in lens]
    max_new = 8
    b = Batch(model, 4)
    outs = b.generate(prompts, max_new, stop=())
    checked = 0
    for s, (p, g) in enumerate(zip(prompts, outs)):
        assert len(g) == max_new
        logits = None
        for pos, t in enumerate(p):
            logits = om.forward(int(t), pos)
        full = True
        for i, t in enumerate(g):
            if top2_margin(logits) <= MARGIN:
                full = False
                break
            assert int(t) == int(np.argmax(logits)), f"seq {s} token {i}: gpu {t} oracle {int(np.argmax(logits))}"
            checked += 1
            if i + 1 < len(g):
                logits = om.forward(int(t), len(p) + i)
        if full:
            # logits that chose the last token (its forward at len(p) + max_new - 2)
            assert np.abs(b.logits(s) - logits).max() <= LOGITS_ABS_TOL
    assert checked >= 16
