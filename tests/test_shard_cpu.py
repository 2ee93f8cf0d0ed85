"""Host logic of the row-sharded lm_head (llamahat/shard.py) on 2 gloo ranks
(CPU): slices gathered in rank order rebuild the unsharded logits, and the
max-all-reduce of packed argmax keys returns LlamaInference.argmax
(H/LlamaInference.java:252-262) -- first maximum across shard boundaries,
NaNs never winning.  The products are numpy stand-ins; the GPU product is
covered by tests/test_gemm_gpu.py."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from llamahat.shard import argmax_key, gather_logits, key_index, shard_rows

VOCAB, DIM, B = 1000, 64, 4
SIGN = np.uint64(1 << 63)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _problem():
    rng = np.random.default_rng(11)
    W = rng.standard_normal((VOCAB, DIM)).astype(np.float32)
    x = rng.standard_normal((B, DIM)).astype(np.float32)
    logits = (x.astype(np.float64) @ W.astype(np.float64).T).astype(np.float32)
    lo0, hi0 = shard_rows(VOCAB, 2, 0)
    logits[1, 7] = logits[1, hi0 + 3] = np.float32(1e6)   # tie across the shard boundary: index 7 wins
    logits[2, :] = np.nan
    logits[2, hi0 + 5] = np.float32(-3.0)                  # the only number sits in rank 1's shard
    return logits


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = _problem()
        lo, hi = shard_rows(VOCAB, world, rank)
        mine = np.ascontiguousarray(full[:, lo:hi])
        # A: all-gather the slices (padded to the largest slice)
        per = shard_rows(VOCAB, world, 0)[1]
        pad = np.zeros((B, per), np.float32)
        pad[:, : hi - lo] = mine
        out = [torch.zeros(B, per) for _ in range(world)]
        dist.all_gather(out, torch.from_numpy(pad))
        slices = [o.numpy()[:, : shard_rows(VOCAB, world, r)[1] - shard_rows(VOCAB, world, r)[0]]
                  for r, o in enumerate(out)]
        gathered = gather_logits(slices, VOCAB)
        # B: max-all-reduce of packed keys (sign bit flipped: int64 order)
        keys = argmax_key(mine, offset=lo) ^ SIGN
        t = torch.from_numpy(keys.view(np.int64).copy())
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        idx = key_index(t.numpy().view(np.uint64) ^ SIGN)
        q.put((rank, gathered, idx))
    finally:
        dist.destroy_process_group()


def test_shard_rows_cover_vocab():
    for world in (1, 2, 4, 8):
        spans = [shard_rows(128256, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == 128256
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        assert all((hi - lo) % 16 == 0 for lo, hi in spans)


def test_two_rank_gather_and_argmax():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    full = _problem()
    ref_idx = []
    for b in range(B):
        row = full[b]
        best = 0  # LlamaInference.argmax: first index whose value is greater than every earlier one
        for i in range(1, VOCAB):
            if row[i] > row[best]:
                best = i
        ref_idx.append(best)
    assert ref_idx[1] == 7 and ref_idx[2] == 0  # tie across shards; NaN at index 0
    for rank, gathered, idx in res:
        np.testing.assert_array_equal(np.nan_to_num(gathered, nan=7.0), np.nan_to_num(full, nan=7.0))
        assert list(idx) == ref_idx
