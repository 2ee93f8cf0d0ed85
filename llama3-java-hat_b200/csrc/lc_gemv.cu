// lc_gemv.cu -- standalone streaming F16 GEMV (batch 1), y = W x.
//
// Persistent grid of one CTA per SM; each CTA streams a contiguous row range
// of W through the shared-memory ring (lc_stream.cuh) and writes its rows of
// y.  HBM-bound: algorithmic bytes = rows*cols*2 + cols*4 + rows*4.
#include "lc_internal.h"
#include "lc_stream.cuh"

namespace lc {

constexpr int kGemvYsCap = 4096;  // floats of per-row partials per CTA

template <int V>
__global__ void __launch_bounds__(kStreamThreads, 1)
    stream_gemv_kernel(const __half* __restrict__ W, const float* __restrict__ x, float* __restrict__ y, int rows,
                       int cols, int nseg, int* err, unsigned long long timeout_ns) {
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ int s_stop;
    // Launched with programmatic stream serialisation: the next kernel may
    // be scheduled now, and nothing here (weights, x, y) is touched before
    // the predecessor has completed.
    griddep_launch();
    griddep_wait();
    Ring ring;
    ring.buf = smem;
    ring.full = reinterpret_cast<uint64_t*>(smem + (size_t)kStages * Geo<V>::kStageBytes);
    ring.empty = ring.full + kStages;
    float* ys = reinterpret_cast<float*>(ring.empty + kStages);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int r0, r1;
    job_range(rows, 1, gridDim.x, blockIdx.x, &r0, &r1);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&ring.full[s], 1);
            mbar_init(&ring.empty[s], kConsumerWarps);
        }
        s_stop = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        if (lane == 0) {
            Producer pr;
            pr.policy = l2_policy_evict_first();
            pr.stream_rows<V>(ring, W, cols, nseg, r0, r1, err, &s_stop, timeout_ns);
            pr.drain(ring, err);
        }
        return;
    }

    float xr[8 * V];
    load_slice_f32<V>(x + (warp % nseg) * Geo<V>::kSegCols, xr);
    Consumer cs;
    const bool ok = cs.consume_rows<V>(ring, nseg, r0, r1, xr, ys, err, timeout_ns);
    if (!ok) *reinterpret_cast<volatile int*>(&s_stop) = 1;
    named_bar_sync(kConsumerBar, kConsumerThreads);
    if (!ok) return;
    for (int k = threadIdx.x; k < r1 - r0; k += kConsumerThreads) {
        float s = ys[k * nseg];
        for (int g = 1; g < nseg; ++g) s += ys[k * nseg + g];
        y[r0 + k] = s;
    }
}

static int pick_nseg(int cols) {
    for (int nseg = 1; nseg <= 8; nseg *= 2) {
        if (cols % nseg) continue;
        const int S = cols / nseg;
        if (S <= 2048 && S % 256 == 0) return nseg;
    }
    return 0;
}

bool stream_gemv_supported(const void* W, const void* x, int rows, int cols) {
    if (rows < 1 || cols < 256) return false;
    if (pick_nseg(cols) == 0) return false;
    if ((reinterpret_cast<uintptr_t>(W) & 15) || (reinterpret_cast<uintptr_t>(x) & 15)) return false;
    return true;
}

template <int V>
static cudaError_t launch_v(const uint16_t* W, const float* x, float* y, int rows, int cols, int nseg, int num_sms,
                            int* err, cudaStream_t st) {
    const size_t smem = (size_t)kStages * Geo<V>::kStageBytes + 2 * kStages * sizeof(uint64_t) +
                        (size_t)kGemvYsCap * sizeof(float);
    // Per-device attribute; cheap enough to set on every launch.
    cudaError_t e =
        cudaFuncSetAttribute(stream_gemv_kernel<V>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    long long grid = num_sms;
    // Rows per CTA must fit the partial-sum buffer: ceil(rows/grid) <= cap_rows.
    const long long cap_rows = kGemvYsCap / nseg;
    const long long need = (rows + cap_rows - 1) / cap_rows;
    if (need > grid) grid = need;
    if (grid > rows) grid = rows;
    return launch_ex(stream_gemv_kernel<V>, dim3((unsigned)grid), dim3(kStreamThreads), smem, st, true,
                     reinterpret_cast<const __half*>(W), x, y, rows, cols, nseg, err, 2000000000ull);
}

cudaError_t launch_stream_gemv(const uint16_t* W, const float* x, float* y, int rows, int cols, int num_sms, int* err,
                               cudaStream_t st) {
    const int nseg = pick_nseg(cols);
    const int V = cols / nseg / 256;
    switch (V) {
        case 1: return launch_v<1>(W, x, y, rows, cols, nseg, num_sms, err, st);
        case 2: return launch_v<2>(W, x, y, rows, cols, nseg, num_sms, err, st);
        case 3: return launch_v<3>(W, x, y, rows, cols, nseg, num_sms, err, st);
        case 4: return launch_v<4>(W, x, y, rows, cols, nseg, num_sms, err, st);
        case 5: return launch_v<5>(W, x, y, rows, cols, nseg, num_sms, err, st);
        case 6: return launch_v<6>(W, x, y, rows, cols, nseg, num_sms, err, st);
        case 7: return launch_v<7>(W, x, y, rows, cols, nseg, num_sms, err, st);
        case 8: return launch_v<8>(W, x, y, rows, cols, nseg, num_sms, err, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace lc
