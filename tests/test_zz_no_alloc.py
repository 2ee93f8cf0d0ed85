"""lc_attention_decode_static: GQA decode attention that allocates no device
memory (its scratch is a static device array inside the library), for hosts
that cannot call cudaMalloc where they run attention -- e.g. a host whose GPU
memory belongs to its own pool allocator, or a decode loop that cannot afford
cudaFree's device-wide synchronisation.

The test calls it through the C ABI, twice in a row with different shapes,
and compares each result with the allocating entry point lc_attention_decode
on the same device buffers.  It runs last (file name) and needs nothing set
up by other tests."""
import ctypes

import numpy as np
import pytest

from parity import assert_kernel_close

pytestmark = pytest.mark.gpu


def _case(torch, seed, batch, seq):
    g = torch.Generator(device="cuda").manual_seed(seed)
    nh, nkv, hd = 32, 8, 64
    max_seq = seq + 5
    q = torch.randn(batch, nh * hd, device="cuda", generator=g)
    k = torch.randn(batch, max_seq, nkv, hd, device="cuda", generator=g)
    v = torch.randn(batch, max_seq, nkv, hd, device="cuda", generator=g)
    lens = torch.tensor([max(1, seq - (b % 4)) for b in range(batch)], dtype=torch.int32, device="cuda")
    strides = (max_seq * nkv * hd, hd, nkv * hd)
    return q, k, v, lens, (nh, nkv, hd), strides


def _run(lib, acc, fn, q, k, v, lens, heads, strides, torch):
    from llamahat import _lib
    out = torch.full_like(q, float("nan"))
    nh, nkv, hd = heads
    rc = fn(acc.handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lens.data_ptr(), q.shape[0], nh,
            nkv, hd, *strides)
    _lib.check(rc)
    acc.synchronize()
    return out.cpu().numpy()


def test_static_scratch_matches_allocating_entry_point():
    torch = pytest.importorskip("torch")
    import llamahat
    from llamahat import _lib
    lib = _lib.load()
    acc = llamahat.Accelerator(0)
    # Two calls in a row with different plans (many splits, then a batch):
    # the second must not see the first call's leftovers in the shared array.
    for seed, batch, seq in ((1, 1, 3000), (2, 6, 700), (3, 1, 3000)):
        q, k, v, lens, heads, strides = _case(torch, seed, batch, seq)
        ref = _run(lib, acc, lib.lc_attention_decode, q, k, v, lens, heads, strides, torch)
        got = _run(lib, acc, lib.lc_attention_decode_static, q, k, v, lens, heads, strides, torch)
        assert np.isfinite(got).all()
        assert_kernel_close(got, ref)
        assert np.array_equal(got, ref)  # same kernel and plan: identical bits


def test_static_scratch_limits_are_errors():
    torch = pytest.importorskip("torch")
    import llamahat
    from llamahat import _lib
    lib = _lib.load()
    acc = llamahat.Accelerator(0)
    q, k, v, lens, (nh, nkv, hd), strides = _case(torch, 4, 1, 64)
    out = torch.zeros_like(q)
    # More sequences than the static limit.
    big = torch.ones(2048, dtype=torch.int32, device="cuda")
    rc = lib.lc_attention_decode_static(acc.handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                        big.data_ptr(), 2048, nh, nkv, hd, *strides)
    assert rc == _lib.LC_ERR_INVALID_ARG and "static-scratch limit" in _lib.last_error()
    # A plan larger than the 8 MiB array (1024 sequences x 8192 positions).
    lens_big = torch.full((1024,), 8192, dtype=torch.int32, device="cuda")
    rc = lib.lc_attention_decode_static(acc.handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                        lens_big.data_ptr(), 1024, nh, nkv, hd, *strides)
    assert rc == _lib.LC_ERR_INVALID_ARG and "8 MiB" in _lib.last_error()
    # Host buffers are refused (staging them would allocate).
    hq = np.zeros(nh * hd, np.float32)
    rc = lib.lc_attention_decode_static(acc.handle, hq.ctypes.data, k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                        lens.data_ptr(), 1, nh, nkv, hd, *strides)
    assert rc == _lib.LC_ERR_INVALID_ARG
