"""lc_attention_decode_static: GQA decode attention that allocates no device
memory (its scratch is a static device array inside the library), for hosts
that cannot call cudaMalloc where they run attention -- e.g. a host whose GPU
memory belongs to its own pool allocator, or a decode loop that cannot afford
cudaFree's device-wide synchronisation.

The tests call it through the C ABI, several times in a row with different
shapes, and compare each result with the oracle's per-head loop
(TransformerBlock.java:153-192) and, bit for bit, with the allocating entry
point lc_attention_decode on the same buffers.  Lengths are passed in device
memory, in host memory, and in device memory written on the context stream
just before the call.  The file runs last (file name) and needs nothing set
up by other tests."""
import numpy as np
import pytest

from parity import assert_kernel_close

pytestmark = pytest.mark.gpu

NH, NKV, HD = 32, 8, 64


def _case(torch, seed, batch, seq):
    g = torch.Generator(device="cuda").manual_seed(seed)
    max_seq = seq + 5
    q = torch.randn(batch, NH * HD, device="cuda", generator=g)
    k = torch.randn(batch, max_seq, NKV, HD, device="cuda", generator=g)
    v = torch.randn(batch, max_seq, NKV, HD, device="cuda", generator=g)
    lens = torch.tensor([max(1, seq - (b % 4)) for b in range(batch)], dtype=torch.int32, device="cuda")
    strides = (max_seq * NKV * HD, HD, NKV * HD)
    return q, k, v, lens, strides


def _call(acc, fn, q, k, v, lens_ptr, batch, strides, torch):
    from llamahat import _lib
    out = torch.full_like(q, float("nan"))
    rc = fn(acc.handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lens_ptr, batch, NH, NKV, HD,
            *strides)
    _lib.check(rc)
    acc.synchronize()
    return out.cpu().numpy()


def _check_oracle(oracle, got, q, k, v, lens):
    qn, kn, vn = q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy()
    for b in range(qn.shape[0]):
        ref = oracle.gqa_attention(qn[b], kn[b], vn[b], int(lens[b]), NH, NKV, HD)
        assert_kernel_close(got[b], ref)


def test_static_scratch_matches_oracle_and_allocating_entry_point(oracle):
    torch = pytest.importorskip("torch")
    import llamahat
    from llamahat import _lib
    lib = _lib.load()
    acc = llamahat.Accelerator(0)
    # Calls in a row with different plans (many splits, then a batch, then
    # many splits again): no call may see an earlier call's leftovers in the
    # shared array.  Odd cases pass the lengths in host memory.
    for i, (seed, batch, seq) in enumerate(((1, 1, 3000), (2, 6, 700), (3, 1, 3000), (5, 3, 64))):
        q, k, v, lens, strides = _case(torch, seed, batch, seq)
        hl = np.ascontiguousarray(lens.cpu().numpy())
        ref = _call(acc, lib.lc_attention_decode, q, k, v, lens.data_ptr(), batch, strides, torch)
        lp = hl.ctypes.data if i % 2 else lens.data_ptr()
        got = _call(acc, lib.lc_attention_decode_static, q, k, v, lp, batch, strides, torch)
        assert np.isfinite(got).all()
        assert np.array_equal(got, ref)  # same kernel and plan: identical bits
        _check_oracle(oracle, got, q, k, v, hl)
    # Host lengths with the multi-split shape, straight after a device-length call.
    q, k, v, lens, strides = _case(torch, 6, 1, 3000)
    hl = np.ascontiguousarray(lens.cpu().numpy())
    got = _call(acc, lib.lc_attention_decode_static, q, k, v, hl.ctypes.data, 1, strides, torch)
    ref = _call(acc, lib.lc_attention_decode, q, k, v, lens.data_ptr(), 1, strides, torch)
    assert np.array_equal(got, ref)
    _check_oracle(oracle, got, q, k, v, hl)


def test_static_scratch_sees_lengths_written_on_the_context_stream(oracle):
    """Lengths produced by work queued on the context stream just before the
    call (here: a long sleep kernel, then a copy of the real lengths over
    lengths of 1) must be the ones the split plan is sized for."""
    torch = pytest.importorskip("torch")
    import llamahat
    from llamahat import _lib
    lib = _lib.load()
    acc = llamahat.Accelerator(0)
    q, k, v, lens, strides = _case(torch, 7, 2, 3000)
    real = lens.clone()
    lens.fill_(1)
    torch.cuda.synchronize()
    ctx_stream = torch.cuda.ExternalStream(acc.stream, device=torch.device("cuda", 0))
    out = torch.full_like(q, float("nan"))
    with torch.cuda.stream(ctx_stream):
        torch.cuda._sleep(50_000_000)  # tens of milliseconds of GPU time on the context stream
        lens.copy_(real)
    rc = lib.lc_attention_decode_static(acc.handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                        lens.data_ptr(), 2, NH, NKV, HD, *strides)
    _lib.check(rc)
    acc.synchronize()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    _check_oracle(oracle, got, q, k, v, real.cpu().numpy())


def test_static_scratch_limits_are_errors():
    torch = pytest.importorskip("torch")
    import llamahat
    from llamahat import _lib
    lib = _lib.load()
    acc = llamahat.Accelerator(0)
    q, k, v, lens, strides = _case(torch, 4, 1, 64)
    out = torch.zeros_like(q)
    # More sequences than the static limit.
    big = torch.ones(2048, dtype=torch.int32, device="cuda")
    rc = lib.lc_attention_decode_static(acc.handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                        big.data_ptr(), 2048, NH, NKV, HD, *strides)
    assert rc == _lib.LC_ERR_INVALID_ARG and "static-scratch limit" in _lib.last_error()
    # A plan larger than the 8 MiB array (1024 sequences x 8192 positions).
    lens_big = torch.full((1024,), 8192, dtype=torch.int32, device="cuda")
    rc = lib.lc_attention_decode_static(acc.handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                        lens_big.data_ptr(), 1024, NH, NKV, HD, *strides)
    assert rc == _lib.LC_ERR_INVALID_ARG and "8 MiB" in _lib.last_error()
    # Host q/k/v/out are refused (staging them would allocate).
    hq = np.zeros(NH * HD, np.float32)
    rc = lib.lc_attention_decode_static(acc.handle, hq.ctypes.data, k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                        lens.data_ptr(), 1, NH, NKV, HD, *strides)
    assert rc == _lib.LC_ERR_INVALID_ARG
    # The context stays usable after the rejected calls.
    hl = np.ascontiguousarray(lens.cpu().numpy())
    rc = lib.lc_attention_decode_static(acc.handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                        hl.ctypes.data, 1, NH, NKV, HD, *strides)
    assert rc == _lib.LC_OK
    acc.synchronize()
    assert torch.isfinite(out).all()
