"""Peer-memory argmax-key all-reduce (lc_keyx_*), the exchange of the lm_head
row shard.  One GPU: the single-rank path and argument errors.  Two GPUs or
more: tests/keyx_worker.py under torch.distributed.run (one process per GPU)
checks the reduction, keys from the lm_head slice product and a bounded wait
that gives up."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_single_rank(acc):
    import torch
    from llamahat import IllegalArgumentError
    from llamahat.shard import PeerKeyExchange
    x = PeerKeyExchange(acc, 1, 0, max_batch=8)
    try:
        ref = np.array([5, 2**63 + 7, 0, 123], dtype=np.uint64)
        k = torch.from_numpy(ref.view(np.int64).copy()).cuda()
        for _ in range(3):  # epochs 1..3, both slot parities
            x.allreduce(k, 4)
        acc.synchronize()
        assert np.array_equal(k.cpu().numpy().view(np.uint64), ref)
        with pytest.raises(IllegalArgumentError):
            x.allreduce(torch.zeros(9, dtype=torch.int64, device="cuda"), 9)  # past max_batch
    finally:
        x.close()
    with pytest.raises(IllegalArgumentError):
        PeerKeyExchange(acc, 9, 0)  # world past LC_KEYX_MAX_WORLD
    with pytest.raises(IllegalArgumentError):
        PeerKeyExchange(acc, 2, 2)  # rank outside the world


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_ranks_over_nvlink():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}", os.path.join(ROOT, "tests", "keyx_worker.py")]
    r = subprocess.run(["timeout", "-k", "30", "300"] + cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count(": ok") == 2
