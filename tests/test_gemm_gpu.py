"""GPU parity of the tcgen05 batched product (lc_gemm_f16_tiled) against the
oracle's sequential GEMV (K/GEMV.java:66-91), one activation row at a time,
plus the tiled weight layout it reads.  Calls go through the C ABI."""
import numpy as np
import pytest

from parity import assert_kernel_close, max_rel_err

pytestmark = pytest.mark.gpu
f32 = np.float32


@pytest.fixture(scope="module")
def gemv(acc):
    from llamahat import CudaKernelFactory
    return CudaKernelFactory().createGEMV(acc)


def _tiled(gemv, W):
    import torch
    rows, cols = W.shape
    Wt = torch.empty(rows * cols, dtype=torch.int16, device="cuda")
    gemv.tile(np.ascontiguousarray(W.view(np.uint16)), Wt, rows, cols)
    return Wt


def test_weights_tile_layout(gemv):
    """lc_weights_tile writes element (r, c) at the tiled offset
    ((r/8 * ncb + c/w) * 8w + (c%w)/8 * 64 + (r%8) * 8 + c%8)."""
    rows, cols = 24, 4096 + 64 * 3  # w = largest multiple of 64 <= 2048 dividing cols
    w = max(k for k in range(64, 2049, 64) if cols % k == 0)
    W = (np.arange(rows * cols, dtype=np.uint32) % 60000).astype(np.uint16).reshape(rows, cols)
    t = _tiled(gemv, W.view(np.float16)).cpu().numpy().view(np.uint16)
    r = np.arange(rows)[:, None]
    c = np.arange(cols)[None, :]
    off = ((r // 8) * (cols // w) + c // w) * 8 * w + ((c % w) // 8) * 64 + (r % 8) * 8 + c % 8
    assert np.array_equal(t[off], W)


@pytest.mark.parametrize("rows,cols,batch", [
    (16, 64, 1), (48, 128, 3), (64, 192, 5),          # small, odd batch, cols not a power of two
    (2048, 2048, 1), (2048, 2048, 8), (2048, 2048, 64),  # q / o projection
    (512, 2048, 8), (3072, 2048, 64),                   # k / v, fused qkv
    (2048, 8192, 64),                                   # down projection: split K
    (4112, 2048, 64),                                   # rows not a multiple of the N block
    (2048, 2048, 1000), (512, 8192, 300),               # many row tiles (prefill products)
])
def test_gemm_parity(gemv, oracle, rows, cols, batch):
    rng = np.random.default_rng(rows * 7 + cols + batch)
    W = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float16)
    X = rng.standard_normal((batch, cols)).astype(f32)
    X[0, : cols // 2] *= 1e-3  # rows with a wide dynamic range
    Wt = _tiled(gemv, W)
    Y = np.full((batch, rows), np.nan, f32)
    gemv.apply_batched_tiled(Wt, X, Y, rows, cols, batch)
    check = range(batch) if rows * cols * batch <= 2048 * 2048 * 8 else [0, batch // 2, batch - 1]
    for b in check:
        assert_kernel_close(Y[b], oracle.gemv_f16(W, X[b]))
    # every row, against the float64 product
    ref = X.astype(np.float64) @ W.astype(np.float64).T
    assert max_rel_err(Y, ref) <= 1e-3


def test_gemm_device_buffers_and_repeat(gemv, oracle):
    """Device X / Y; repeated calls give identical bits (the split sums are
    added in a fixed order)."""
    import torch
    rows, cols, batch = 2048, 8192, 32
    rng = np.random.default_rng(5)
    W = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float16)
    X = rng.standard_normal((batch, cols)).astype(f32)
    Wt = _tiled(gemv, W)
    dX = torch.from_numpy(X).cuda()
    dY = torch.empty((batch, rows), dtype=torch.float32, device="cuda")
    gemv.apply_batched_tiled(Wt, dX, dY, rows, cols, batch)
    gemv.acc.synchronize()
    y1 = dY.cpu().numpy().copy()
    gemv.apply_batched_tiled(Wt, dX, dY, rows, cols, batch)
    gemv.acc.synchronize()
    assert np.array_equal(y1, dY.cpu().numpy())
    assert_kernel_close(y1[3], oracle.gemv_f16(W, X[3]))


@pytest.mark.parametrize("batch,offset", [(1, 0), (5, 1000), (64, 64128)])
def test_gemm_argmax_keys(gemv, oracle, batch, offset):
    """Packed argmax keys of the logits epilogue: the first maximum of each
    row (LlamaInference.argmax), global index = offset + column; a planted tie
    resolves to the lower column."""
    rows, cols = 4096, 2048
    rng = np.random.default_rng(batch + offset)
    W = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float16)
    W[1000] = W[3000]  # identical rows: equal logits, column 1000 must win
    X = rng.standard_normal((batch, cols)).astype(f32)
    X[0] = W[3000].astype(f32) * 50  # make row 1000 / 3000 the maximum of sequence 0
    Wt = _tiled(gemv, W)
    Y = np.zeros((batch, rows), f32)
    keys = np.zeros(batch, np.uint64)
    gemv.apply_batched_tiled_argmax(Wt, X, Y, rows, cols, batch, offset, keys)
    idx = (~(keys & np.uint64(0xFFFFFFFF))) & np.uint64(0xFFFFFFFF)
    for b in range(batch):
        first = int(np.argmax(Y[b]))  # numpy: first maximum of the GPU logits
        assert int(idx[b]) == offset + first
    assert int(idx[0]) == offset + 1000
    assert_kernel_close(Y[0], oracle.gemv_f16(W, X[0]))
    # without logits
    k2 = np.zeros(batch, np.uint64)
    gemv.apply_batched_tiled_argmax(Wt, X, None, rows, cols, batch, offset, k2)
    assert np.array_equal(keys, k2)


def test_gemm_rejects_bad_shapes(gemv):
    from llamahat import IllegalArgumentError
    W = np.zeros(64 * 64, np.float16)
    X = np.zeros(64 * 65, f32)
    Y = np.zeros(65 * 64, f32)
    with pytest.raises(IllegalArgumentError):
        big = np.zeros(16385 * 64, f32)
        gemv.apply_batched_tiled(W, big, big.copy(), 64, 64, 16385)  # batch past the row limit
    with pytest.raises(IllegalArgumentError):
        gemv.apply_batched_tiled(W, X, Y, 24, 64, 1)   # rows % 16
    with pytest.raises(IllegalArgumentError):
        gemv.apply_batched_tiled(W, X, Y, 64, 48, 1)   # cols % 64
