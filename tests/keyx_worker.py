"""One rank of the peer key-exchange check (run under torch.distributed.run
by tests/test_keyx_gpu.py, one process per GPU; gloo carries only the
mailbox handles and the host-side checks).

Checks, on every rank:
  * lc_keyx_allreduce returns the unsigned maximum of all ranks' keys, for
    batches 1, 7, 64 and 300 back-to-back calls (slot parity alternation);
  * keys produced by the lm_head slice product (lc_gemm_f16_tiled_argmax on
    this rank's rows) reduce to the key of the best rank's slice;
  * a rank that skips a call makes the others' bounded wait give up: the
    context reports LC_ERR_TIMEOUT and stays usable.
Exits 0 when all hold."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "llama3-java-hat_b200")]

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def keys_of(seed: int, n: int) -> np.ndarray:
    g = np.random.default_rng(seed)
    return g.integers(0, 2**63, size=n, dtype=np.int64).view(np.uint64) | (g.integers(0, 2, size=n).astype(np.uint64) << np.uint64(63))


def main() -> int:
    import llamahat
    from llamahat import CudaKernelFactory, DeviceTimeoutError
    from llamahat.shard import PeerKeyExchange, shard_rows
    rank, ws, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    torch.cuda.set_device(local)
    acc = llamahat.Accelerator(local)
    x = PeerKeyExchange(acc, ws, rank, max_batch=64)
    try:
        # 1. plain keys, several batches, many calls in a row
        calls = [(1, 1), (7, 2), (64, 3)] + [(64, 100 + i) for i in range(300)]
        dev = []
        for B, seed in calls:
            k = torch.from_numpy(keys_of(seed * 31 + rank, B).view(np.int64).copy()).cuda()
            x.allreduce(k, B)
            dev.append(k)
        acc.synchronize()
        for (B, seed), k in zip(calls, dev):
            want = np.max(np.stack([keys_of(seed * 31 + r, B) for r in range(ws)]), axis=0)
            got = k.cpu().numpy().view(np.uint64)
            assert np.array_equal(got, want), f"rank {rank}: batch {B} seed {seed}"
        # 2. keys from this rank's lm_head slice
        V, D, B = 4096, 2048, 5
        lo, hi = shard_rows(V, ws, rank)
        torch.manual_seed(7)
        W = (torch.randn(V, D) * 0.02).half()
        X = torch.randn(B, D)
        gemv = CudaKernelFactory().createGEMV(acc)
        n = hi - lo
        Wt = torch.empty(n * D, dtype=torch.int16, device="cuda")
        gemv.tile(W[lo:hi].contiguous().view(torch.int16).cuda().view(-1), Wt, n, D)
        Y = torch.empty(B, n, device="cuda")
        K = torch.zeros(B, dtype=torch.int64, device="cuda")
        gemv.apply_batched_tiled_argmax(Wt, X.cuda(), Y, n, D, B, lo, K)
        acc.synchronize()
        mine = K.cpu().numpy().view(np.uint64).copy()
        everyone = [None] * ws
        dist.all_gather_object(everyone, mine)
        x.allreduce(K, B)
        acc.synchronize()
        got = K.cpu().numpy().view(np.uint64)
        assert np.array_equal(got, np.max(np.stack(everyone), axis=0)), f"rank {rank}: lm_head keys"
        idx = (~(got & np.uint64(0xFFFFFFFF))) & np.uint64(0xFFFFFFFF)
        assert all(0 <= int(i) < V for i in idx)
        # 3. rank ws-1 skips one call: the others' waits give up, bounded
        dist.barrier()
        k = torch.ones(4, dtype=torch.int64, device="cuda")
        if rank != ws - 1:
            x.allreduce(k, 4)
            try:
                acc.synchronize()
                raise AssertionError(f"rank {rank}: expected a timeout")
            except DeviceTimeoutError:
                pass
            acc.synchronize()  # the context stays usable
        dist.barrier()
    finally:
        dist.barrier()
        x.close()
        dist.destroy_process_group()
    print(f"rank {rank}: ok", flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
