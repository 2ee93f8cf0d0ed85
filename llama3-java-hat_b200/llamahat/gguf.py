"""GGUF v3 writer and reader for synthetic Llama models.

The writer produces files the reference's loader accepts
(GGUFReader.java:57-123, LlamaModel.java:74-86): general.architecture =
"llama", F16 projection tensors (F32 when the arrays given are fp32, as
LlamaModel.mapTensor reads them in WeightStorageMode.F32), F32 norm tensors,
tied embeddings (no
output.weight), 32-byte alignment, and -- when the vocabulary is the full
128256 ids -- the tokenizer metadata LlamaInference's constructor reads
(Tokenizer.java:47-95, ChatFormat.java:22-29): a gpt2 tokenizer model,
128256 token strings (byte symbols, learned merges, the Llama-3 special
tokens at their ids) and the merge rules.
"""
from __future__ import annotations

import struct

import numpy as np

from .config import LlamaConfig
from .synth import tensor_specs

GGUF_MAGIC = 0x46554747
T_U32, T_I32, T_F32, T_STRING, T_ARRAY = 4, 5, 6, 8, 9
SPECIAL_TOKENS = {
    128000: "<|begin_of_text|>",
    128001: "<|end_of_text|>",
    128006: "<|start_header_id|>",
    128007: "<|end_header_id|>",
    128008: "<|eom_id|>",
    128009: "<|eot_id|>",
}


def _s(b: bytearray, s: str) -> None:
    e = s.encode()
    b += struct.pack("<Q", len(e)) + e


def _kv(b: bytearray, key: str, t: int, v) -> None:
    _s(b, key)
    b += struct.pack("<I", t)
    if t == T_STRING:
        _s(b, v)
    elif t == T_U32:
        b += struct.pack("<I", v)
    elif t == T_I32:
        b += struct.pack("<i", v)
    elif t == T_F32:
        b += struct.pack("<f", v)
    elif t == T_ARRAY:
        et, items = v
        b += struct.pack("<IQ", et, len(items))
        for it in items:
            if et == T_STRING:
                _s(b, it)
            else:
                raise ValueError("only string arrays are written")
    else:
        raise ValueError(t)


def write_gguf(path: str, cfg: LlamaConfig, weights: dict[str, np.ndarray], alignment: int = 32,
               tokenizer=None) -> None:
    """Writes a GGUF v3 file.  `tokenizer`: None -> the synthetic tokenizer
    (llamahat.synth.synth_tokenizer) when the vocabulary is the full 128256
    ids, else none; True / False force it on / off; or a (token strings,
    merge rules) pair."""
    specs = tensor_specs(cfg)
    kv = bytearray()
    n_kv = 0

    def add(key, t, v):
        nonlocal n_kv
        _kv(kv, key, t, v)
        n_kv += 1

    add("general.architecture", T_STRING, "llama")
    add("general.name", T_STRING, "synthetic-llama")
    add("general.alignment", T_U32, alignment)
    add("llama.embedding_length", T_U32, cfg.dim)
    add("llama.feed_forward_length", T_U32, cfg.hidden)
    add("llama.block_count", T_U32, cfg.n_layers)
    add("llama.attention.head_count", T_U32, cfg.n_heads)
    add("llama.attention.head_count_kv", T_U32, cfg.n_kv_heads)
    add("llama.context_length", T_U32, cfg.max_seq)
    add("llama.rope.freq_base", T_F32, cfg.rope_theta)
    add("llama.attention.layer_norm_rms_epsilon", T_F32, cfg.rms_eps)
    if tokenizer is None:
        tokenizer = cfg.vocab >= 128256
    if tokenizer is True:
        from .synth import synth_tokenizer
        tokenizer = synth_tokenizer(cfg.vocab)
    if tokenizer:
        toks, merges = tokenizer
        if len(toks) != cfg.vocab:
            raise ValueError(f"{len(toks)} token strings for a vocabulary of {cfg.vocab}")
        add("tokenizer.ggml.model", T_STRING, "gpt2")
        add("tokenizer.ggml.tokens", T_ARRAY, (T_STRING, list(toks)))
        add("tokenizer.ggml.merges", T_ARRAY, (T_STRING, list(merges)))

    info = bytearray()
    offsets = []
    off = 0
    for name, shape, kind in specs:
        a = weights[name]
        nbytes = a.size * a.dtype.itemsize
        _s(info, name)
        dims = tuple(reversed(shape))  # GGUF lists ne0 (innermost) first
        info += struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        ttype = 1 if a.dtype == np.float16 else 0  # GGML F16 or F32, as given
        info += struct.pack("<I", ttype) + struct.pack("<Q", off)
        offsets.append(off)
        off += (nbytes + alignment - 1) // alignment * alignment

    header = struct.pack("<IIQQ", GGUF_MAGIC, 3, len(specs), n_kv)
    meta_end = len(header) + len(kv) + len(info)
    data_start = (meta_end + alignment - 1) // alignment * alignment
    with open(path, "wb") as f:
        f.write(header)
        f.write(kv)
        f.write(info)
        f.write(b"\0" * (data_start - meta_end))
        pos = 0
        for (name, shape, kind), o in zip(specs, offsets):
            if o > pos:
                f.write(b"\0" * (o - pos))
                pos = o
            a = np.ascontiguousarray(weights[name])
            want = (np.float16, np.float32) if kind == "proj" else (np.float32,)
            if a.dtype not in want:
                raise TypeError(f"{name}: expected {' or '.join(np.dtype(t).name for t in want)}, got {a.dtype}")
            f.write(a.tobytes())
            pos += a.nbytes


def read_gguf(path: str) -> tuple[dict, dict[str, np.ndarray]]:
    """Returns (metadata, tensors) with tensors as read-only memmap views."""
    mm = np.memmap(path, mode="r", dtype=np.uint8)
    buf = memoryview(mm)
    o = 0

    def u(fmt):
        nonlocal o
        v = struct.unpack_from(fmt, buf, o)
        o += struct.calcsize(fmt)
        return v[0]

    def s():
        n = u("<Q")
        nonlocal o
        r = bytes(buf[o:o + n]).decode()
        o += n
        return r

    scalar = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<B", 10: "<Q", 11: "<q", 12: "<d"}

    def val(t):
        if t == T_STRING:
            return s()
        if t == T_ARRAY:
            et, n = u("<I"), u("<Q")
            return [val(et) for _ in range(n)]
        return u(scalar[t])

    if u("<I") != GGUF_MAGIC:
        raise IOError("Not a GGUF file or wrong magic")
    u("<I")
    n_t, n_kv = u("<Q"), u("<Q")
    meta = {}
    for _ in range(n_kv):
        k = s()
        meta[k] = val(u("<I"))
    infos = []
    for _ in range(n_t):
        name = s()
        nd = u("<I")
        dims = [u("<Q") for _ in range(nd)]
        t = u("<I")
        off = u("<Q")
        infos.append((name, dims, t, off))
    al = int(meta.get("general.alignment", 32))
    start = (o + al - 1) // al * al
    tensors = {}
    for name, dims, t, off in infos:
        n = int(np.prod(dims))
        dt = np.float16 if t == 1 else np.float32
        a = np.frombuffer(mm, dtype=dt, count=n, offset=start + off)
        tensors[name] = a.reshape(tuple(reversed(dims)))
    return meta, tensors
