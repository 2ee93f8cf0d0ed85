"""Chat path on the GPU: streaming generation (lc_generate_stream: the fused
kernel publishes each greedy token to mapped host memory while the launch
runs) and LlamaInference.chat (LlamaInference.java:227-247) over a GGUF file
carrying the synthetic tokenizer, checked against the oracle's generate plus
the host tokenizer."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny_model(acc, tiny_weights):
    from llamahat import CudaModel
    cfg, w = tiny_weights
    return cfg, w, CudaModel(cfg, w, acc=acc)


@pytest.fixture(scope="module")
def chat_setup(acc, tmp_path_factory):
    """TINY dimensions with the full 128256-id vocabulary, so that the
    Llama 3 special tokens exist, written as GGUF with the tokenizer."""
    from llamahat import LlamaInference
    from llamahat.config import TINY
    from llamahat.gguf import write_gguf
    from llamahat.synth import synth_weights
    cfg = TINY.with_(vocab=128256)
    w = synth_weights(cfg, seed=11)
    path = str(tmp_path_factory.mktemp("chat") / "chat.gguf")
    write_gguf(path, cfg, w)
    return cfg, w, LlamaInference(path, acc=acc, max_seq=cfg.max_seq)


def test_stream_delivers_every_token_in_order(tiny_model):
    from llamahat import Session
    cfg, w, model = tiny_model
    s = Session(model)
    prompt = [11, 22, 33, 44, 55]
    got = []
    out = s.generate(prompt, 24, stop=(), on_token=lambda t, i: got.append((t, i)))
    assert [i for _, i in got] == list(range(len(out)))
    assert [t for t, _ in got] == list(out) and len(out) == 24
    # identical to the launch without streaming
    assert list(Session(model).generate(prompt, 24, stop=())) == list(out)


def test_stream_with_stop_token(tiny_model, oracle):
    from llamahat import Session
    cfg, w, model = tiny_model
    prompt = [101, 202, 303]
    free = oracle.OracleModel(cfg, w).generate(prompt, 12, stop=())
    stop = int(free[3])
    got = []
    out = Session(model).generate(prompt, 12, stop=(stop,), on_token=lambda t, i: got.append(t))
    first = list(free).index(stop)
    assert list(out) == list(free[:first + 1]) == got


def test_stream_callback_error_is_raised_after_the_launch(tiny_model):
    from llamahat import Session
    cfg, w, model = tiny_model
    s = Session(model)
    calls = []

    def cb(t, i):
        calls.append(i)
        if i == 2:
            raise KeyError("stop here")

    with pytest.raises(KeyError):
        s.generate([1, 2, 3], 10, stop=(), on_token=cb)
    assert calls == [0, 1, 2]  # later tokens are not passed on after the error
    assert len(s.generate([1, 2, 3], 10, stop=())) == 10  # the session stays usable


def test_chat_matches_oracle(chat_setup, oracle):
    from llamahat.tokenizer import ChatFormat, Message, Role
    cfg, w, inf = chat_setup
    assert inf.tokenizer is not None and inf.tokenizer.vocabularySize() == cfg.vocab
    text = inf.chat("You are a helpful assistant.", "Say hi", 12)
    cf = ChatFormat(inf.tokenizer)
    prompt = cf.encodeDialogPrompt([Message(Role.SYSTEM, "You are a helpful assistant."),
                                    Message(Role.USER, "Say hi")])
    ref = oracle.OracleModel(cfg, w).generate(prompt, 12, stop=sorted(cf.getStopTokens()))
    kept = []
    for t in ref:
        if int(t) in cf.getStopTokens():
            break
        kept.append(int(t))
    assert text == inf.tokenizer.decode(kept)


def test_chat_streams_text(chat_setup):
    cfg, w, inf = chat_setup
    pieces = []
    text = inf.chat(None, "Tell a joke about programming", 10, onText=pieces.append)
    assert "".join(pieces) == text
    assert text == inf.chat("", "Tell a joke about programming", 10)  # empty system prompt = none


def test_chat_needs_a_tokenizer(tiny_model):
    from llamahat import IllegalStateError, LlamaInference
    cfg, w, model = tiny_model
    with pytest.raises(IllegalStateError):
        LlamaInference(model).chat(None, "hi", 4)


def test_gguf_without_tokenizer_is_rejected_by_path(tiny_model, tmp_path, acc):
    """LlamaInference's constructor reads the tokenizer from the GGUF
    metadata (LlamaInference.java:97-99) and fails without one."""
    from llamahat import IllegalArgumentError, LlamaInference
    from llamahat.gguf import write_gguf
    cfg, w, model = tiny_model
    path = str(tmp_path / "notok.gguf")
    write_gguf(path, cfg, w, tokenizer=False)
    with pytest.raises(IllegalArgumentError, match="Expected gpt2"):
        LlamaInference(path, acc=acc, max_seq=cfg.max_seq)
