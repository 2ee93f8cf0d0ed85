"""Device-resident model and the LlamaInference mirror.

Reference: src/main/java/com/arturskowronski/llama3babylon/hat/LlamaInference.java
  ctor :58-100, forward(token, pos) :117-164, generate(prompt, maxNew[, stop]) :173-217,
  argmax :252-262.

`LlamaInference` keeps the reference's call surface.  Weights are uploaded
to the GPU once (`CudaModel`); each `forward` is one launch of the fused decode
kernel; `generate` runs the whole prefill + greedy loop in one launch and
copies back only the generated token ids.
"""
from __future__ import annotations

import ctypes
import weakref

import numpy as np

from . import _lib
from .config import LlamaConfig, WeightStorageMode
from .kernels import Accelerator, _addr, default_accelerator

EOS_TOKEN = 128001  # LlamaInference.java:174


class CudaModel:
    """Weights in HBM (one arena) plus the prepared decode kernel."""

    def __init__(self, cfg: LlamaConfig | None = None, weights: dict | None = None, gguf_path: str | None = None,
                 acc: Accelerator | None = None, max_seq: int = 0,
                 weight_mode: WeightStorageMode = WeightStorageMode.F16):
        self.acc = acc or default_accelerator()
        self.weight_mode = weight_mode
        lib = _lib.load()
        h = ctypes.c_void_p()
        if gguf_path is not None:
            _lib.check(lib.lc_model_load_gguf_mode(self.acc.handle, gguf_path.encode(), max_seq,
                                                   weight_mode.device_mode, ctypes.byref(h)))
            c = _lib.LcConfig()
            _lib.check(lib.lc_model_get_config(h, ctypes.byref(c)))
            self.cfg = LlamaConfig.from_lc(c)
        else:
            if cfg is None or weights is None:
                raise ValueError("need cfg and weights, or gguf_path")
            self.cfg = cfg
            lc = cfg.to_lc()
            lc.weight_mode = weight_mode.device_mode
            _lib.check(lib.lc_model_create(self.acc.handle, ctypes.byref(lc), ctypes.byref(h)))
        self.handle = h
        self.gguf_path = gguf_path
        self._fin = weakref.finalize(self, lib.lc_model_destroy, h)
        if gguf_path is None:
            for name, a in weights.items():
                self.upload(name, a)
            _lib.check(lib.lc_model_finalize(h))

    def upload(self, name: str, a) -> None:
        lib = _lib.load()
        if isinstance(a, np.ndarray):
            dtype = 1 if a.dtype in (np.float16, np.uint16) else 0
            a = np.ascontiguousarray(a)
            _lib.check(lib.lc_model_upload_tensor(self.handle, name.encode(), a.ctypes.data, a.size, dtype))
        else:  # torch tensor (host or device)
            dtype = 1 if str(a.dtype) in ("torch.float16", "torch.int16") else 0
            _lib.check(lib.lc_model_upload_tensor(self.handle, name.encode(), a.contiguous().data_ptr(), a.numel(), dtype))

    def close(self) -> None:
        self._fin()


class Session:
    """One decoding sequence: device KV cache + activations."""

    def __init__(self, model: CudaModel):
        self.model = model
        lib = _lib.load()
        h = ctypes.c_void_p()
        _lib.check(lib.lc_session_create(model.handle, ctypes.byref(h)))
        self.handle = h
        self._fin = weakref.finalize(self, lib.lc_session_destroy, h)

    def forward(self, token: int, pos: int, logits=None) -> tuple[np.ndarray | None, int]:
        lib = _lib.load()
        am = np.zeros(1, np.int32)
        lp = None if logits is None else _addr(logits, "f32", self.model.cfg.vocab, True)
        _lib.check(lib.lc_forward(self.handle, int(token), int(pos), lp, am.ctypes.data))
        return logits, int(am[0])

    def generate(self, prompt, max_new: int, stop=(EOS_TOKEN,), on_token=None) -> np.ndarray:
        """Prefill + greedy decode in one launch.  `on_token(token, index)`,
        when given, is called for each generated id in order while the launch
        runs (lc_generate_stream); an exception it raises is re-raised here
        after the launch ends."""
        lib = _lib.load()
        p = np.ascontiguousarray(np.asarray(prompt, dtype=np.int32))
        st = np.ascontiguousarray(np.asarray(sorted(stop) if stop else [], dtype=np.int32))
        out = np.zeros(max(max_new, 1), np.int32)
        n = np.zeros(1, np.int32)
        stp = st.ctypes.data if st.size else None
        if on_token is None:
            _lib.check(lib.lc_generate(self.handle, p.ctypes.data, p.size, int(max_new), stp, st.size,
                                       out.ctypes.data, n.ctypes.data))
        else:
            errors = []

            def relay(token, index, _user):
                if errors:
                    return
                try:
                    on_token(int(token), int(index))
                except BaseException as e:  # raised again once the C call returns
                    errors.append(e)

            cb = _lib.TOKEN_CALLBACK(relay)
            _lib.check(lib.lc_generate_stream(self.handle, p.ctypes.data, p.size, int(max_new), stp, st.size,
                                              cb, None, out.ctypes.data, n.ctypes.data))
            if errors:
                raise errors[0]
        return out[: int(n[0])].copy()

    def decode(self, token: int, start_pos: int, n_steps: int, out=None) -> np.ndarray:
        lib = _lib.load()
        o = out if out is not None else np.zeros(n_steps, np.int32)
        _lib.check(lib.lc_decode(self.handle, int(token), int(start_pos), int(n_steps), _addr(o, "i32", n_steps, True)))
        return o

    def enable_trace(self, words_per_cta: int) -> None:
        """Phase trace of the fused kernel (see lc_session_enable_trace)."""
        _lib.check(_lib.load().lc_session_enable_trace(self.handle, int(words_per_cta)))

    def read_trace(self) -> np.ndarray:
        """[grid][words_per_cta] uint64 %globaltimer stamps (0 = not written)."""
        lib = _lib.load()
        g, w = ctypes.c_int32(), ctypes.c_int32()
        _lib.check(lib.lc_session_read_trace(self.handle, None, 0, ctypes.byref(g), ctypes.byref(w)))
        out = np.zeros((g.value, w.value), np.uint64)
        if out.size:
            _lib.check(lib.lc_session_read_trace(self.handle, out.ctypes.data, out.size, None, None))
        return out

    def last_ms(self) -> float:
        v = ctypes.c_float()
        _lib.check(_lib.load().lc_session_last_ms(self.handle, ctypes.byref(v)))
        return float(v.value)

    def close(self) -> None:
        self._fin()


class Batch:
    """Up to 64 independent sequences decoded in lockstep (serving): each
    sequence gets LlamaInference.generate's computation, every weight matrix
    is read once per step for all of them."""

    def __init__(self, model: CudaModel, max_batch: int):
        self.model = model
        lib = _lib.load()
        h = ctypes.c_void_p()
        _lib.check(lib.lc_batch_create(model.handle, int(max_batch), ctypes.byref(h)))
        self.handle = h
        self.max_batch = int(max_batch)
        self._fin = weakref.finalize(self, lib.lc_batch_destroy, h)

    def generate(self, prompts, max_new: int, stop=(EOS_TOKEN,)) -> list[np.ndarray]:
        """Greedy tokens per sequence (stop token included, as generate)."""
        lib = _lib.load()
        ps = [np.asarray(p, dtype=np.int32).ravel() for p in prompts]
        lens = np.array([p.size for p in ps], np.int32)
        flat = np.ascontiguousarray(np.concatenate(ps) if ps else np.zeros(0, np.int32))
        st = np.ascontiguousarray(np.asarray(sorted(stop) if stop else [], dtype=np.int32))
        out = np.zeros((len(ps), max(int(max_new), 1)), np.int32)
        _lib.check(lib.lc_batch_generate(self.handle, len(ps), flat.ctypes.data, lens.ctypes.data, int(max_new),
                                         st.ctypes.data if st.size else None, st.size, out.ctypes.data))
        res = []
        for row in out:
            k = int(np.argmax(row < 0)) if (row < 0).any() else row.size
            res.append(row[:k].copy())
        return res

    def last_ms(self) -> tuple[float, float, int]:
        """(device ms of the whole call, ms from the last prompt position on, positions run)."""
        t, d, n = ctypes.c_float(), ctypes.c_float(), ctypes.c_int32()
        _lib.check(_lib.load().lc_batch_last_ms(self.handle, ctypes.byref(t), ctypes.byref(d), ctypes.byref(n)))
        return float(t.value), float(d.value), int(n.value)

    def logits(self, seq: int) -> np.ndarray:
        """Logits of sequence `seq` at the last position of the last generate."""
        out = np.zeros(self.model.cfg.vocab, np.float32)
        _lib.check(_lib.load().lc_batch_logits(self.handle, int(seq), out.ctypes.data))
        return out

    def close(self) -> None:
        self._fin()


class LlamaInference:
    """Mirror of LlamaInference (LlamaInference.java): forward / generate /
    chat / argmax.

    Given a GGUF path, the constructor also builds the tokenizer and chat
    format from the file's metadata, as the reference's does
    (LlamaInference.java:97-99), and fails the same way when the metadata has
    no gpt2 tokenizer.  Given a CudaModel, `tokenizer` may be passed in (or is
    read from the model's GGUF file when it came from one); without one,
    chat() raises IllegalStateError."""

    def __init__(self, model: CudaModel | str, acc: Accelerator | None = None, max_seq: int = 0,
                 tokenizer=None, weightMode: WeightStorageMode = WeightStorageMode.F16):
        from .tokenizer import ChatFormat, Tokenizer
        path = model if isinstance(model, str) else getattr(model, "gguf_path", None)
        if tokenizer is None and path is not None:
            from .gguf import read_gguf
            meta, _ = read_gguf(path)
            if isinstance(model, str) or meta.get("tokenizer.ggml.model") is not None:
                tokenizer = Tokenizer.fromGGUFMetadata(meta)
        self.model = model if isinstance(model, CudaModel) else CudaModel(gguf_path=model, acc=acc, max_seq=max_seq,
                                                                          weight_mode=weightMode)
        self.session = Session(self.model)
        self.cfg = self.model.cfg
        self.tokenizer = tokenizer
        self.chatFormat = ChatFormat(tokenizer) if tokenizer is not None else None

    def forward(self, token: int, pos: int) -> np.ndarray:
        """Logits [vocab] for `token` at `pos` (LlamaInference.java:117-164)."""
        logits = np.empty(self.cfg.vocab, np.float32)
        self.session.forward(token, pos, logits)
        return logits

    def generate(self, promptTokens, maxNewTokens: int, stopTokens=frozenset({EOS_TOKEN}), onToken=None) -> np.ndarray:
        """Greedy generation (LlamaInference.java:173-217).  `onToken(token,
        index)` streams each generated id while the launch runs."""
        return self.session.generate(promptTokens, maxNewTokens, tuple(stopTokens), on_token=onToken)

    def chat(self, systemPrompt: str | None, userPrompt: str, maxNewTokens: int, onText=None) -> str:
        """LlamaInference.chat (LlamaInference.java:227-247): the Instruct
        template around the prompts, greedy generation that stops at
        <|end_of_text|> or <|eot_id|>, and the decoded text of the tokens
        before the first stop token.  `onText(piece)` receives that text as it
        is generated, in pieces of whole characters whose concatenation is the
        returned string."""
        from .tokenizer import Message, Role, StreamDecoder
        if self.chatFormat is None:
            raise _lib.IllegalStateError(_lib.LC_ERR_STATE, "no tokenizer: load from a GGUF file or pass tokenizer=")
        dialog = []
        if systemPrompt:
            dialog.append(Message(Role.SYSTEM, systemPrompt))
        dialog.append(Message(Role.USER, userPrompt))
        prompt = self.chatFormat.encodeDialogPrompt(dialog)
        stop = self.chatFormat.getStopTokens()
        on_token = None
        if onText is not None:
            dec = StreamDecoder(self.tokenizer)
            ended = [False]

            def on_token(token, _index):
                if ended[0] or token in stop:
                    ended[0] = True
                    return
                piece = dec.feed(token)
                if piece:
                    onText(piece)
        generated = self.session.generate(prompt, maxNewTokens, tuple(stop), on_token=on_token)
        kept = []
        for t in generated:
            if int(t) in stop:
                break
            kept.append(int(t))
        if onText is not None:
            tail = dec.flush()
            if tail:
                onText(tail)
        return self.tokenizer.decode(kept)

    @staticmethod
    def argmax(values) -> int:
        """First index of the maximum (LlamaInference.java:252-262), computed on the GPU."""
        from .kernels import argmax as _am
        return _am(np.ascontiguousarray(np.asarray(values, dtype=np.float32)))
