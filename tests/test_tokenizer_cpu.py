"""Tokenizer and chat template of the chat path (H/Tokenizer.java,
H/ChatFormat.java), host side only.

Pinned three ways: hand-derived known answers of the Java pattern and merge
loop; an independent byte-level BPE (HuggingFace `tokenizers`, given the
reference's pattern string verbatim in its own regex engine) on the
synthetic vocabulary; and the round-trip and template properties the
reference's TokenizerIntegrationTest checks with the real vocabulary."""
import numpy as np
import pytest

from llamahat import IllegalArgumentError, IllegalStateError
from llamahat.synth import synth_tokenizer, train_bpe
from llamahat.tokenizer import (_PATTERN, BYTE_DECODER, BYTE_ENCODER, ChatFormat, Message, Role, StreamDecoder,
                                Tokenizer, java_strip)

# Tokenizer.java:16-18, as written in the Java source.
JAVA_PATTERN = ("(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\\r\\n\\p{L}\\p{N}]?\\p{L}+|"
                "\\p{N}{1,3}| ?[^\\s\\p{L}\\p{N}]+[\\r\\n]*|\\s*[\\r\\n]+|\\s+(?!\\S)|\\s+")

TEXTS = [
    "Hello, world!",
    "You are a helpful assistant.",
    "Tell a joke about programming",
    "It's THE end; they'LL see.\n\n  next\tline  ",
    "héllo wörld 😀 12345678 ÷× ß",
    "a\r\n\r\nb   c!!!\n",
    "   leading and trailing   ",
    "",
]


@pytest.fixture(scope="module")
def synth():
    toks, merges = synth_tokenizer(128256)
    return toks, merges, Tokenizer(toks, merges)


def _byte_tokenizer(words, specials=True):
    """Byte symbols at ids 0..255, then `words` (merge results) in order."""
    toks = [chr(BYTE_ENCODER[b]) for b in range(256)] + list(words)
    if specials:
        toks += [f"<|pad_{i}|>" for i in range(len(toks), 128000)]
        toks += ["<|begin_of_text|>", "<|end_of_text|>", "<|r2|>", "<|r3|>", "<|r4|>", "<|r5|>",
                 "<|start_header_id|>", "<|end_header_id|>", "<|eom_id|>", "<|eot_id|>"]
    return toks


def test_byte_map():
    """Tokenizer.java:221-245: a bijection; printable Latin-1 maps to itself,
    the rest to 256.. in byte order (space -> U+0120, newline -> U+010A)."""
    assert sorted(BYTE_ENCODER) == list(range(256))
    assert len(set(BYTE_ENCODER.values())) == 256
    assert BYTE_ENCODER[ord("A")] == ord("A") and BYTE_ENCODER[0xAE] == 0xAE
    assert BYTE_ENCODER[0] == 256 and BYTE_ENCODER[ord(" ")] == 0x120 and BYTE_ENCODER[ord("\n")] == 0x10A
    assert BYTE_ENCODER[0xAD] == 0x143 and max(BYTE_ENCODER.values()) == 0x143
    assert all(BYTE_DECODER[v] == k for k, v in BYTE_ENCODER.items())


@pytest.mark.parametrize("text,chunks", [
    ("Hello, world!", ["Hello", ",", " world", "!"]),
    ("I'm here, they'LL go", ["I", "'m", " here", ",", " they", "'LL", " go"]),
    ("abc 12345", ["abc", " ", "123", "45"]),
    ("  hi", [" ", " hi"]),
    ("a\n\nb", ["a", "\n\n", "b"]),
    ("x!!!\n", ["x", "!!!\n"]),
    ("end   ", ["end", "   "]),
    ("\u00a0word", ["\u00a0word"]),       # no-break space is not \s in Java: it prefixes the letters
    ("tab\u2003x", ["tab", "\u2003x"]),   # nor is an em space
])
def test_pretokenizer_java_semantics(text, chunks):
    assert [m.group() for m in _PATTERN.finditer(text)] == chunks


def test_merge_loop_known_answers():
    """Tokenizer.java:130-162: lowest rank first, every occurrence left to
    right without overlap; rules naming unknown tokens are ignored; bytes
    without a symbol are dropped."""
    words = ["ll", "ell", "hell", "hello"]
    toks = _byte_tokenizer(words, specials=False)
    merges = ["l l", "e ll", "h ell", "hell o", "q z"]  # "q z": no "qz" token -> ignored
    tk = Tokenizer(toks, merges)
    ids = {w: 256 + i for i, w in enumerate(words)}
    assert tk.encode("hello") == [ids["hello"]]
    assert tk.encode("hellllo") == [ids["hell"], ids["ll"], ord("o")]
    assert tk.encode("lll") == [ids["ll"], ord("l")]
    assert tk.encode("qz") == [ord("q"), ord("z")]
    # A vocabulary without the symbol of byte 'x' drops it (Tokenizer.java:120-123).
    toks2 = list(toks)
    toks2[ord("x")] = "<|no_x|>"
    assert Tokenizer(toks2, merges).encode("xhellox") == [ids["hello"]]
    # A later merge rule for the same pair wins the rank (map put semantics).
    tk3 = Tokenizer(toks, ["e ll", "l l", "e ll"])
    assert tk3.merge_ranks[(ord("e"), ids["ll"])] == 2


def test_matches_independent_bpe(synth):
    """Same ids as HuggingFace's byte-level BPE with the reference's pattern
    string (Oniguruma) on texts whose whitespace is ASCII."""
    tokenizers = pytest.importorskip("tokenizers")
    toks, merges, tk = synth
    bpe = tokenizers.models.BPE(vocab={t: i for i, t in enumerate(toks)},
                                merges=[tuple(m.split(" ", 1)) for m in merges], ignore_merges=False)
    hf = tokenizers.Tokenizer(bpe)
    hf.pre_tokenizer = tokenizers.pre_tokenizers.Sequence([
        tokenizers.pre_tokenizers.Split(tokenizers.Regex(JAVA_PATTERN), behavior="isolated", invert=False),
        tokenizers.pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    rng = np.random.default_rng(3)
    alphabet = list("abcdefghijklmnopqrstuvwxyz ETAOIN,.!?'\n\t0123456789éü😀")
    random_texts = ["".join(rng.choice(alphabet, size=int(rng.integers(1, 80)))) for _ in range(200)]
    for t in TEXTS + random_texts:
        assert tk.encode(t) == hf.encode(t).ids, repr(t)


def test_round_trip(synth):
    """TokenizerIntegrationTest.testEncodeDecodeRoundTrip, on more texts."""
    _, _, tk = synth
    for t in TEXTS:
        assert tk.decode(tk.encode(t)) == t
    assert len(tk.encode("Hello, world!")) < len("Hello, world!")  # merges apply


def test_decode_rules(synth):
    toks, merges, tk = synth
    # Special tokens decode to their text; ids outside the vocabulary are skipped.
    assert tk.decode([128000, -5, 10 ** 9, ord("h"), ord("i")]) == "<|begin_of_text|>hi"
    assert tk.decodeToken(128009) == "<|eot_id|>"
    # A unit outside the byte map contributes its own UTF-8; a supplementary
    # character in a token string is two lone surrogates -> "??".
    toks2 = list(toks)
    toks2[1000] = "€"
    toks2[1001] = "\U0001F600"
    tk2 = Tokenizer(toks2, merges)
    assert tk2.decode([1000]) == "€"
    assert tk2.decode([1001]) == "??"
    # Malformed UTF-8 becomes U+FFFD.
    assert tk.decode([0xE2, ord("a")]) == "\ufffda"  # id b is the symbol of byte b: a lone lead byte
    assert tk.isSpecialToken(128000) and not tk.isSpecialToken(127999) and not tk.isSpecialToken(128256)
    assert tk.vocabularySize() == 128256
    sp = tk.getSpecialTokens()
    assert sp["<|begin_of_text|>"] == 128000 and sp["<|end_of_text|>"] == 128001
    assert sp["<|start_header_id|>"] == 128006 and sp["<|end_header_id|>"] == 128007 and sp["<|eot_id|>"] == 128009


def test_stream_decoder(synth):
    """Pieces of whole characters whose concatenation is decode(all)."""
    _, _, tk = synth
    for t in TEXTS:
        ids = tk.encode(t)
        sd = StreamDecoder(tk)
        pieces = [sd.feed(i) for i in ids] + [sd.flush()]
        assert "".join(pieces) == tk.decode(ids) == t
    # the 4-byte emoji arrives as four byte tokens: nothing until the last
    ids = tk.encode("😀")
    assert len(ids) == 4
    sd = StreamDecoder(tk)
    assert [sd.feed(i) for i in ids] == ["", "", "", "😀"]


def test_from_gguf_metadata_errors(synth):
    toks, merges, _ = synth
    with pytest.raises(IllegalArgumentError, match="Expected gpt2"):
        Tokenizer.fromGGUFMetadata({"tokenizer.ggml.model": "llama", "tokenizer.ggml.tokens": toks,
                                    "tokenizer.ggml.merges": merges})
    with pytest.raises(IllegalArgumentError):
        Tokenizer.fromGGUFMetadata({"tokenizer.ggml.model": "gpt2", "tokenizer.ggml.tokens": toks})
    with pytest.raises(IllegalArgumentError, match="without a space"):
        Tokenizer(toks, ["ab"])
    tk = Tokenizer.fromGGUFMetadata({"tokenizer.ggml.model": "gpt2", "tokenizer.ggml.tokens": toks,
                                     "tokenizer.ggml.merges": merges})
    assert tk.encode("Hello, world!") == Tokenizer(toks, merges).encode("Hello, world!")


def test_java_strip():
    assert java_strip(" \t\n\x0b\f\r\x1c\x1f hi \u2003\u2028") == "hi"
    assert java_strip("\u00a0hi\u202f") == "\u00a0hi\u202f"  # no-break spaces are not whitespace in Java
    assert java_strip("") == "" and java_strip("   ") == ""


def test_chat_format(synth):
    """ChatFormat.java:37-62 and TokenizerIntegrationTest.testChatFormatProducesExpectedTokens."""
    _, _, tk = synth
    cf = ChatFormat(tk)
    dialog = [Message(Role.SYSTEM, "You are a helpful assistant."), Message(Role.USER, "  Tell a joke about programming\n")]
    ids = cf.encodeDialogPrompt(dialog)
    assert ids[0] == 128000 and 128006 in ids and 128007 in ids
    assert tk.decode(ids) == ("<|begin_of_text|><|start_header_id|>system<|end_header_id|>\nYou are a helpful "
                              "assistant.<|eot_id|><|start_header_id|>user<|end_header_id|>\nTell a joke about "
                              "programming<|eot_id|><|start_header_id|>assistant<|end_header_id|>\n")
    head = cf.encodeHeader(Message(Role.USER, "x"))
    assert head == [128006] + tk.encode("user") + [128007] + tk.encode("\n")
    assert cf.encodeMessage(Message(Role.ASSISTANT, " ok ")) == cf.encodeHeader(Message(Role.ASSISTANT, "")) + \
        tk.encode("ok") + [128009]
    assert cf.getStopTokens() == {128001, 128009}
    assert str(Role.SYSTEM) == "system" and Role("tool").name == "tool"


def test_chat_format_needs_special_tokens():
    toks = _byte_tokenizer([], specials=False)
    with pytest.raises(IllegalStateError, match="begin_of_text"):
        ChatFormat(Tokenizer(toks, []))


def test_train_bpe_deterministic():
    text = "low lower lowest newer newest wide wider widest"
    m1, m2 = train_bpe(text, 50), train_bpe(text, 50)
    assert m1 == m2 and len(m1) > 3
    toks = [chr(BYTE_ENCODER[b]) for b in range(256)]
    for a, b in m1:
        if a + b not in toks:
            toks.append(a + b)
    tk = Tokenizer(toks, [f"{a} {b}" for a, b in m1])
    for w in text.split():
        assert tk.decode(tk.encode(w)) == w
    assert len(tk.encode(" lowest")) < len(" lowest")


def test_gguf_tokenizer_metadata(tmp_path):
    """write_gguf stores the synthetic tokenizer; fromGGUFMetadata reads it back."""
    from llamahat.config import LlamaConfig
    from llamahat.gguf import read_gguf, write_gguf
    from llamahat.synth import synth_weights
    cfg = LlamaConfig(dim=64, hidden=128, n_layers=1, n_heads=2, n_kv_heads=1, head_dim=32, vocab=1000, max_seq=32)
    w = synth_weights(cfg, seed=3)
    path = str(tmp_path / "tok.gguf")
    write_gguf(path, cfg, w, tokenizer=True)
    meta, _ = read_gguf(path)
    tk = Tokenizer.fromGGUFMetadata(meta)
    toks, merges = synth_tokenizer(1000)
    assert tk.vocabulary == toks and meta["tokenizer.ggml.merges"] == merges
    assert tk.decode(tk.encode("Say hi")) == "Say hi"
    with pytest.raises(ValueError):
        write_gguf(path, cfg, w, tokenizer=(toks[:10], merges))


def test_gguf_f32_projections_round_trip(tmp_path):
    """F32 projection tensors are written as GGML type F32 and read back
    bit-exact (LlamaModel.mapTensor's F32 branch); other dtypes are refused."""
    from llamahat.config import LlamaConfig
    from llamahat.gguf import read_gguf, write_gguf
    from llamahat.synth import synth_weights
    cfg = LlamaConfig(dim=64, hidden=128, n_layers=1, n_heads=2, n_kv_heads=1, head_dim=32, vocab=1000, max_seq=32)
    w = {k: (v.astype(np.float32) + np.float32(1e-5)) if v.dtype == np.float16 else v
         for k, v in synth_weights(cfg, seed=4).items()}
    path = str(tmp_path / "f32.gguf")
    write_gguf(path, cfg, w)
    _, t = read_gguf(path)
    for k, v in w.items():
        assert t[k].dtype == np.float32 and np.array_equal(np.asarray(t[k]).reshape(v.shape), v), k
    bad = dict(w)
    bad["output_norm.weight"] = bad["output_norm.weight"].astype(np.float16)
    with pytest.raises(TypeError):
        write_gguf(path, cfg, bad)
