"""Byte-level BPE tokenizer and the Llama 3 Instruct chat template.

Mirrors H/Tokenizer.java and H/ChatFormat.java of the reference
(H/ = src/main/java/com/arturskowronski/llama3babylon/hat/): the same
vocabulary and merge tables read from GGUF metadata, the same
pre-tokenisation pattern, the same greedy lowest-rank merge loop and the same
decode rules, so that the ids fed to the decode kernel are the ids the Java
host would feed.

Java regex semantics, restated for the `regex` module:
  * `\\s` / `\\S` in java.util.regex is ASCII only ([ \\t\\n\\x0B\\f\\r]); the
    pattern below spells that class out.
  * `(?i:...)` without UNICODE_CASE folds ASCII letters only; the contraction
    alternatives spell out both cases.
  * `\\p{L}` / `\\p{N}` are the Unicode general categories in both engines.
"""
from __future__ import annotations

import codecs
import unicodedata
from dataclasses import dataclass

import regex

from ._lib import IllegalArgumentError, IllegalStateError

_WS = r"[ \t\n\x0B\f\r]"
_NWS = r"[^ \t\n\x0B\f\r]"
# Tokenizer.java:16-18 (LLAMA_3_PATTERN) under Java's default flags.
LLAMA_3_PATTERN = (
    r"'[sS]|'[tT]|'[rR][eE]|'[vV][eE]|'[mM]|'[lL][lL]|'[dD]"
    r"|[^\r\n\p{L}\p{N}]?\p{L}+"
    r"|\p{N}{1,3}"
    r"| ?[^ \t\n\x0B\f\r\p{L}\p{N}]+[\r\n]*"
    rf"|{_WS}*[\r\n]+"
    rf"|{_WS}+(?!{_NWS})"
    rf"|{_WS}+"
)
_PATTERN = regex.compile(LLAMA_3_PATTERN)

SPECIAL_BASE = 128000  # Tokenizer.java:89-92: ids from here on are special tokens


def bytes_to_unicode() -> dict[int, int]:
    """GPT-2 byte -> code point map (Tokenizer.java:221-245): printable
    Latin-1 bytes map to themselves, the other 68 bytes to 256, 257, ... in
    byte order."""
    keep = list(range(ord("!"), ord("~") + 1)) + list(range(0xA1, 0xAD)) + list(range(0xAE, 0x100))
    table = {b: b for b in keep}
    n = 0
    for b in range(256):
        if b not in table:
            table[b] = 256 + n
            n += 1
    return table


BYTE_ENCODER = bytes_to_unicode()
BYTE_DECODER = {v: k for k, v in BYTE_ENCODER.items()}


def _java_char_utf8(cp: int) -> bytes:
    """UTF-8 bytes of one Java `char` (a UTF-16 unit): a lone surrogate
    encodes as '?' (String.getBytes replaces malformed input)."""
    if 0xD800 <= cp <= 0xDFFF:
        return b"?"
    return chr(cp).encode("utf-8")


class Tokenizer:
    """Tokenizer.java: encode / encodeAsList / decode / decodeToken /
    isSpecialToken / getSpecialTokens / vocabularySize."""

    def __init__(self, vocabulary: list[str], merges: list[str]):
        self.vocabulary = list(vocabulary)
        self.token_to_index: dict[str, int] = {}
        for i, t in enumerate(self.vocabulary):  # Tokenizer.java:61-64: a later duplicate wins
            self.token_to_index[t] = i
        self.merges: dict[tuple[int, int], int] = {}
        self.merge_ranks: dict[tuple[int, int], int] = {}
        for rank, rule in enumerate(merges):  # Tokenizer.java:67-86
            rule = str(rule)
            sp = rule.find(" ")
            if sp < 0:  # substring(0, -1) throws in the reference
                raise IllegalArgumentError(-1, f"merge rule without a space: {rule!r}")
            first, second = rule[:sp], rule[sp + 1:]
            a, b = self.token_to_index.get(first), self.token_to_index.get(second)
            m = self.token_to_index.get(first + second)
            if a is not None and b is not None and m is not None:
                self.merges[(a, b)] = m
                self.merge_ranks[(a, b)] = rank
        self.special_tokens = {self.vocabulary[i]: i for i in range(SPECIAL_BASE, len(self.vocabulary))}
        # One token per byte, or None when the vocabulary lacks that byte's
        # symbol (Tokenizer.java:119-123 then drops the byte).
        self._byte_ids = [self.token_to_index.get(chr(BYTE_ENCODER[b])) for b in range(256)]

    @staticmethod
    def fromGGUFMetadata(metadata: dict) -> "Tokenizer":
        """Tokenizer.java:47-95."""
        model = metadata.get("tokenizer.ggml.model")
        if model != "gpt2":
            raise IllegalArgumentError(-1, f"Expected gpt2 tokenizer model, got: {model}")
        tokens = metadata.get("tokenizer.ggml.tokens")
        merges = metadata.get("tokenizer.ggml.merges")
        if tokens is None or merges is None:  # a NullPointerException in the reference
            raise IllegalArgumentError(-1, "GGUF metadata lacks tokenizer.ggml.tokens or tokenizer.ggml.merges")
        return Tokenizer([str(t) for t in tokens], [str(m) for m in merges])

    from_gguf_metadata = fromGGUFMetadata

    # ---------------------------------------------------------------- encode
    def encode(self, text: str) -> list[int]:
        return self.encodeAsList(text)

    def encodeAsList(self, text: str) -> list[int]:
        """Tokenizer.java:102-110: pre-tokenise, then BPE each chunk."""
        out: list[int] = []
        for m in _PATTERN.finditer(text):
            out.extend(self._encode_chunk(m.group()))
        return out

    encode_as_list = encodeAsList

    def _encode_chunk(self, chunk: str) -> list[int]:
        """Tokenizer.java:112-165: byte symbols, then repeatedly merge every
        occurrence (left to right, non-overlapping) of the adjacent pair with
        the lowest merge rank until no pair has a rank."""
        ids = [t for t in (self._byte_ids[b] for b in chunk.encode("utf-8")) if t is not None]
        ranks = self.merge_ranks
        while len(ids) >= 2:
            best, best_rank = None, None
            for pair in zip(ids, ids[1:]):
                r = ranks.get(pair)
                if r is not None and (best_rank is None or r < best_rank):
                    best, best_rank = pair, r
            if best is None:
                break
            merged = self.merges[best]
            a, b = best
            nxt: list[int] = []
            i, n = 0, len(ids)
            while i < n:
                if i < n - 1 and ids[i] == a and ids[i + 1] == b:
                    nxt.append(merged)
                    i += 2
                else:
                    nxt.append(ids[i])
                    i += 1
            ids = nxt
        return ids

    # ---------------------------------------------------------------- decode
    def decode_bytes(self, tokens) -> bytes:
        """The byte string Tokenizer.decode builds (Tokenizer.java:171-197):
        ids outside the vocabulary are skipped; each UTF-16 unit of the joined
        token strings maps back through the byte decoder, or -- when it has no
        byte (special-token text outside the map) -- to its own UTF-8 bytes.

        The reference sizes its byte buffer to the string length and grows it
        only for unmapped units, so a string such as an unmapped unit whose
        bytes exactly fill the buffer followed by a mapped one throws
        ArrayIndexOutOfBoundsException there; this restatement returns the
        bytes instead."""
        vocab = self.vocabulary
        out = bytearray()
        for t in tokens:
            t = int(t)
            if 0 <= t < len(vocab):
                for ch in _utf16_units(vocab[t]):
                    b = BYTE_DECODER.get(ch)
                    out += bytes((b,)) if b is not None else _java_char_utf8(ch)
        return bytes(out)

    def decode(self, tokens) -> str:
        """Tokenizer.java:171-199; malformed UTF-8 becomes U+FFFD, as
        new String(bytes, UTF_8) does."""
        return self.decode_bytes(tokens).decode("utf-8", errors="replace")

    def decodeToken(self, token_id: int) -> str:
        return self.decode([token_id])

    decode_token = decodeToken

    def isSpecialToken(self, token_id: int) -> bool:
        return SPECIAL_BASE <= token_id < len(self.vocabulary)

    is_special_token = isSpecialToken

    def getSpecialTokens(self) -> dict[str, int]:
        return dict(self.special_tokens)

    def vocabularySize(self) -> int:
        return len(self.vocabulary)

    vocabulary_size = vocabularySize


def _utf16_units(s: str):
    """The UTF-16 code units of `s` (what String.charAt walks)."""
    for c in s:
        cp = ord(c)
        if cp >= 0x10000:
            cp -= 0x10000
            yield 0xD800 + (cp >> 10)
            yield 0xDC00 + (cp & 0x3FF)
        else:
            yield cp


class StreamDecoder:
    """Incremental text of a token stream: feed ids as they arrive, get the
    newly completed characters.  The concatenation of all pieces (plus
    `flush()`) equals Tokenizer.decode of the whole list."""

    def __init__(self, tokenizer: Tokenizer):
        self.tokenizer = tokenizer
        self._dec = codecs.getincrementaldecoder("utf-8")(errors="replace")

    def feed(self, token_id: int) -> str:
        return self._dec.decode(self.tokenizer.decode_bytes([token_id]))

    def flush(self) -> str:
        return self._dec.decode(b"", final=True)


# ---------------------------------------------------------------- chat format

def _java_is_whitespace(c: str) -> bool:
    """Character.isWhitespace: space / line / paragraph separators except the
    no-break spaces, plus \\t \\n \\x0B \\f \\r and the four C0 separators."""
    if c in "\t\n\x0b\f\r\x1c\x1d\x1e\x1f":
        return True
    if c in "\u00a0\u2007\u202f":
        return False
    return unicodedata.category(c) in ("Zs", "Zl", "Zp")


def java_strip(s: str) -> str:
    """String.strip(): removes leading and trailing Character.isWhitespace."""
    i, j = 0, len(s)
    while i < j and _java_is_whitespace(s[i]):
        i += 1
    while j > i and _java_is_whitespace(s[j - 1]):
        j -= 1
    return s[i:j]


@dataclass(frozen=True)
class Role:
    """ChatFormat.Role (ChatFormat.java:66-73)."""
    name: str

    def __str__(self) -> str:
        return self.name


Role.SYSTEM = Role("system")
Role.USER = Role("user")
Role.ASSISTANT = Role("assistant")


@dataclass(frozen=True)
class Message:
    """ChatFormat.Message (ChatFormat.java:64)."""
    role: Role
    content: str


class ChatFormat:
    """Llama 3 Instruct template (ChatFormat.java:12-62):
    <|begin_of_text|> then, per message, <|start_header_id|>role<|end_header_id|>
    "\\n" content.strip() <|eot_id|>, then the open assistant header."""

    Message = Message
    Role = Role

    def __init__(self, tokenizer: Tokenizer):
        self.tokenizer = tokenizer
        special = tokenizer.getSpecialTokens()

        def need(name: str) -> int:
            if name not in special:  # unboxing null throws in the reference
                raise IllegalStateError(-8, f"vocabulary lacks the special token {name}")
            return special[name]

        self.begin_of_text = need("<|begin_of_text|>")
        self.start_header = need("<|start_header_id|>")
        self.end_header = need("<|end_header_id|>")
        self.end_of_turn = need("<|eot_id|>")
        self.end_of_text = need("<|end_of_text|>")
        self.stop_tokens = frozenset({self.end_of_text, self.end_of_turn})

    def getStopTokens(self) -> frozenset[int]:
        return self.stop_tokens

    def encodeHeader(self, message: Message) -> list[int]:
        t = [self.start_header]
        t += self.tokenizer.encodeAsList(message.role.name)
        t.append(self.end_header)
        t += self.tokenizer.encodeAsList("\n")
        return t

    def encodeMessage(self, message: Message) -> list[int]:
        t = self.encodeHeader(message)
        t += self.tokenizer.encodeAsList(java_strip(message.content))
        t.append(self.end_of_turn)
        return t

    def encodeDialogPrompt(self, dialog) -> list[int]:
        t = [self.begin_of_text]
        for m in dialog:
            t += self.encodeMessage(m)
        t += self.encodeHeader(Message(Role.ASSISTANT, ""))
        return t

    get_stop_tokens = getStopTokens
    encode_header = encodeHeader
    encode_message = encodeMessage
    encode_dialog_prompt = encodeDialogPrompt
