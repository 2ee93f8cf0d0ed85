"""Row-sharded lm_head over N GPUs (one process per GPU).

The lm_head GEMV (H/LlamaInference.java:151-156: logits = W_out . x, W_out
[vocab][dim]) splits by rows: rank r of N owns rows [lo_r, hi_r), computes
that slice of the logits, and the ranks exchange either the slices (an
all-gather of vocab floats per sequence) or only their local argmax
candidates (an all-reduce of one packed 64-bit key per sequence).  The
packed key orders by value, then by the lowest index, so the all-reduce
(max) returns exactly LlamaInference.argmax (first maximum, :252-262).
"""
from __future__ import annotations

import numpy as np


def shard_rows(vocab: int, world: int, rank: int, align: int = 16) -> tuple[int, int]:
    """Rows [lo, hi) of rank `rank`: contiguous slices in rank order, each a
    multiple of `align` rows except the last, which takes the remainder."""
    per = -(-vocab // world)
    per = -(-per // align) * align
    lo = min(vocab, rank * per)
    hi = min(vocab, lo + per)
    return lo, hi


def argmax_key(values: np.ndarray, offset: int = 0) -> np.ndarray:
    """Packed keys of the row-wise first maximum of `values` [B][n]:
    order-preserving float bits above the inverted global index.  NaNs never
    win, except that a NaN at global index 0 makes the key the largest one
    (LlamaInference.argmax returns 0 then: nothing compares greater)."""
    v = np.asarray(values, np.float32)
    B = v.shape[0]
    keys = np.zeros(B, np.uint64)
    for b in range(B):
        row = v[b]
        if offset == 0 and row.size and np.isnan(row[0]):
            keys[b] = np.uint64(0xFFFFFFFFFFFFFFFF)
            continue
        ok = ~np.isnan(row)
        if not ok.any():
            continue
        i = int(np.flatnonzero(row == row[ok].max())[0])
        bits = np.frombuffer(np.float32(row[i]).tobytes(), np.uint32)[0]
        bits = (~bits & 0xFFFFFFFF) if bits & 0x80000000 else (bits | 0x80000000)
        keys[b] = (np.uint64(bits) << np.uint64(32)) | np.uint64((~(offset + i)) & 0xFFFFFFFF)
    return keys


def key_index(keys: np.ndarray) -> np.ndarray:
    """Global index of packed keys (0 for an empty key, as argmax of no number)."""
    k = np.asarray(keys, np.uint64)
    idx = (~(k & np.uint64(0xFFFFFFFF))) & np.uint64(0xFFFFFFFF)
    return np.where(k == 0, 0, idx.astype(np.int64)).astype(np.int64)


def gather_logits(slices: list[np.ndarray], vocab: int) -> np.ndarray:
    """Full logits [B][vocab] from the rank-ordered slices."""
    return np.concatenate(slices, axis=1)[:, :vocab]


KEYX_HANDLE_BYTES = 64


class PeerKeyExchange:
    """All-reduce (max) of packed argmax keys over NVLink peer memory
    (lc_keyx_*): each rank stores its keys into every rank's mailbox and
    waits, bounded, for the others' flags -- no library collective.

    `gather_handles(handle: bytes) -> list[bytes]` returns every rank's
    mailbox handle in rank order; by default torch.distributed's
    all_gather_object on the default process group (any backend).
    Collective: every rank constructs it, calls allreduce the same number of
    times in the same order, and closes it after a barrier."""

    def __init__(self, acc, world: int, rank: int, max_batch: int = 64, gather_handles=None):
        import ctypes
        from . import _lib
        self.acc, self.world, self.rank, self.max_batch = acc, int(world), int(rank), int(max_batch)
        lib = _lib.load()
        h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(KEYX_HANDLE_BYTES)
        _lib.check(lib.lc_keyx_create(acc.handle, self.world, self.rank, self.max_batch, ctypes.byref(h), buf))
        self.handle = h
        try:
            mine = bytes(buf.raw)
            if gather_handles is None:
                gather_handles = _torch_gather_handles
            hs = gather_handles(mine) if self.world > 1 else [mine]
            if len(hs) != self.world or any(len(x) != KEYX_HANDLE_BYTES for x in hs):
                raise ValueError("gather_handles must return world handles of 64 bytes in rank order")
            allh = ctypes.create_string_buffer(b"".join(hs), KEYX_HANDLE_BYTES * self.world)
            _lib.check(lib.lc_keyx_open(h, allh))
        except BaseException:
            lib.lc_keyx_destroy(h)
            self.handle = None
            raise

    def allreduce(self, keys, batch: int | None = None) -> None:
        """keys: device tensor of int64 / uint64 packed keys [batch]; in
        place, enqueued on the accelerator's stream."""
        from . import _lib
        n = int(batch if batch is not None else keys.numel())
        _lib.check(_lib.load().lc_keyx_allreduce(self.handle, keys.data_ptr(), n))

    def close(self) -> None:
        from . import _lib
        if self.handle is not None:
            _lib.load().lc_keyx_destroy(self.handle)
            self.handle = None


def _torch_gather_handles(mine: bytes) -> list[bytes]:
    import torch.distributed as dist
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, mine)
    return out

