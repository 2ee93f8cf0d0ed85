// lc_stream.cuh -- the weight-streaming engine shared by the standalone GEMV
// and the fused decode kernel.
//
// A CTA owns a contiguous row range of each weight matrix it works on.  One
// producer thread streams that range, stage by stage, from HBM into a ring of
// shared-memory stages with 1-D bulk async copies (cp.async.bulk, completion
// as mbarrier transaction bytes, L2 evict-first).  Eight consumer warps dot
// each stage with the activation vector held in registers and release the
// stage.  The producer never waits for activations, only for free stages, so
// weight traffic keeps flowing while the consumers synchronise with the rest
// of the grid.
//
// Stage geometry.  A "segment" is S = 256*V consecutive columns of one row
// (one warp, 32 lanes x V 16-byte vectors).  A row of `cols` columns is
// nseg = cols / S segments (nseg in {1,2,4,8}); a stage holds 8 segments =
// 8/nseg whole rows, so consumer warp w always works on segment w % nseg of
// row w / nseg and keeps the matching slice of the activation in registers.
#pragma once

#include "lc_common.cuh"

namespace lc {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kStreamThreads = kConsumerThreads + 32;  // + producer warp
constexpr int kStages = 6;
constexpr uint32_t kConsumerBar = 1;  // named barrier id for consumer warps

template <int V>
struct Geo {
    static constexpr int kSegCols = 256 * V;
    static constexpr int kSegBytes = kSegCols * 2;
    static constexpr int kStageBytes = 8 * kSegBytes;
};

// Rows of a job owned by `rank` (0..G-1) when rows are dealt in units of
// `unit` rows (2 keeps RoPE / SwiGLU pairs together).  Ranks below the
// remainder get one extra unit.
__host__ __device__ inline void job_range(int rows, int unit, int G, int rank, int* r0, int* r1) {
    const int P = rows / unit;
    const int base = P / G, ext = P % G;
    const int start = rank * base + (rank < ext ? rank : ext);
    const int cnt = base + (rank < ext ? 1 : 0);
    *r0 = start * unit;
    *r1 = (start + cnt) * unit;
}

// Running rotation so that the extra units of consecutive jobs land on
// different CTAs and the bytes per CTA even out over a decode step.
struct Rotation {
    int shift = 0;
    __host__ __device__ int rank(int cta, int G) const { return (cta + shift) % G; }
    __host__ __device__ void advance(int rows, int unit, int G) {
        const int ext = (rows / unit) % G;
        shift = (shift - ext % G + G) % G;
    }
};

struct Ring {
    uint8_t* buf;
    uint64_t* full;
    uint64_t* empty;
};

// ------------------------------------------------------------- producer --

struct Producer {
    uint32_t it = 0;  // stages issued so far
    uint64_t policy;
    bool aborted = false;

    // Streams rows [r0, r1) of W (cols columns) into the ring.  `stop` is a
    // shared flag the consumers raise when they leave early.
    template <int V>
    __device__ __forceinline__ bool stream_rows(const Ring& ring, const __half* W, int cols, int nseg, int r0, int r1,
                                                volatile int* err, volatile int* stop, uint64_t timeout_ns) {
        const int srows = 8 / nseg;
        for (int r = r0; r < r1; r += srows) {
            const int n = min(srows, r1 - r);
            const uint32_t slot = it % kStages;
            const uint32_t par = ((it / kStages) & 1u) ^ 1u;
            if (!mbar_try_wait(&ring.empty[slot], par)) {
                const uint64_t deadline = globaltimer_ns() + timeout_ns;
                bool ok = false;
                for (uint32_t k = 1;; ++k) {
                    if (mbar_try_wait(&ring.empty[slot], par)) {
                        ok = true;
                        break;
                    }
                    if ((k & 63u) == 0u) {
                        if (*stop != 0 || *err != 0) break;
                        if (globaltimer_ns() > deadline) {
                            atomicCAS(const_cast<int*>(err), 0, (int)kDevTimeoutEmpty);
                            break;
                        }
                    }
                }
                if (!ok) {
                    aborted = true;
                    return false;
                }
            }
            const uint32_t bytes = (uint32_t)n * (uint32_t)cols * 2u;
            mbar_arrive_expect_tx(&ring.full[slot], bytes);
            bulk_g2s(ring.buf + (size_t)slot * Geo<V>::kStageBytes, W + (size_t)r * (size_t)cols, bytes,
                     &ring.full[slot], policy);
            ++it;
        }
        return true;
    }

    // Before the CTA exits: wait until every issued copy has landed, so no
    // bulk copy is still writing into shared memory of a finished CTA.
    __device__ __forceinline__ void drain(const Ring& ring, volatile int* err) {
        const uint32_t first = it > (uint32_t)kStages ? it - (uint32_t)kStages : 0u;
        for (uint32_t k = first; k < it; ++k) {
            const uint32_t slot = k % kStages;
            const uint32_t par = (k / kStages) & 1u;
            const uint64_t deadline = globaltimer_ns() + 200000000ull;  // copies land in microseconds
            while (!mbar_try_wait(&ring.full[slot], par)) {
                if (globaltimer_ns() > deadline) {
                    atomicCAS(const_cast<int*>(err), 0, (int)kDevTimeoutDrain);
                    break;
                }
            }
        }
    }
};

// ------------------------------------------------------------- consumer --

struct Consumer {
    uint32_t it = 0;  // stages consumed so far

    // Dots rows [r0, r1) of a job (cols = nseg*S) with the warp's activation
    // slice xr; the per-(row, segment) partial of warp-reduced fp32 sums goes
    // to ys[(row - r0) * nseg + seg].  Returns false on timeout / error.
    uint64_t wait_ns = 0;  // time spent waiting for stages (diagnostics, thread 0)
    bool timing = false;

    template <int V>
    __device__ __forceinline__ bool consume_rows(const Ring& ring, int nseg, int r0, int r1, const float (&xr)[8 * V],
                                                 float* ys, volatile int* err, uint64_t timeout_ns) {
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        const int srows = 8 / nseg;
        const int my_row = warp / nseg, my_seg = warp % nseg;
        uint32_t slot = it % kStages, par = (it / kStages) & 1u;
        // Compact loop body (one stage per iteration, nothing unrolled across
        // stages): the decode kernel holds five copies of it and instruction
        // fetch, not arithmetic, is what a bigger body costs.
#pragma unroll 1
        for (int r = r0; r < r1; r += srows) {
            if (timing) {
                const uint64_t t0 = globaltimer_ns();
                if (!mbar_wait_bounded(&ring.full[slot], par, err, t0 + timeout_ns, kDevTimeoutFull)) return false;
                wait_ns += globaltimer_ns() - t0;
            } else if (!mbar_try_wait(&ring.full[slot], par) &&
                       !mbar_wait_bounded(&ring.full[slot], par, err, globaltimer_ns() + timeout_ns, kDevTimeoutFull)) {
                return false;
            }
            if (r + my_row < r1) {
                const uint8_t* base = ring.buf + (size_t)slot * Geo<V>::kStageBytes +
                                      (size_t)(my_row * nseg + my_seg) * Geo<V>::kSegBytes + (size_t)lane * 16;
                uint4 wv[V];
#pragma unroll
                for (int v = 0; v < V; ++v) wv[v] = *reinterpret_cast<const uint4*>(base + v * 512);
                float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll
                for (int v = 0; v < V; ++v) {
                    const __half2* h2 = reinterpret_cast<const __half2*>(&wv[v]);
                    const float2 t0 = __half22float2(h2[0]), t1 = __half22float2(h2[1]);
                    const float2 t2 = __half22float2(h2[2]), t3 = __half22float2(h2[3]);
                    a0 = fmaf(t0.y, xr[v * 8 + 1], fmaf(t0.x, xr[v * 8 + 0], a0));
                    a1 = fmaf(t1.y, xr[v * 8 + 3], fmaf(t1.x, xr[v * 8 + 2], a1));
                    a2 = fmaf(t2.y, xr[v * 8 + 5], fmaf(t2.x, xr[v * 8 + 4], a2));
                    a3 = fmaf(t3.y, xr[v * 8 + 7], fmaf(t3.x, xr[v * 8 + 6], a3));
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&ring.empty[slot]);  // weights are in registers now
                float acc = warp_sum((a0 + a1) + (a2 + a3));
                if (lane == 0) ys[(r - r0 + my_row) * nseg + my_seg] = acc;
            } else {
                __syncwarp();
                if (lane == 0) mbar_arrive(&ring.empty[slot]);
            }
            ++it;
            if (++slot == (uint32_t)kStages) {
                slot = 0;
                par ^= 1u;
            }
        }
        return true;
    }
};

// Lane's columns of a segment: v*256 + lane*8 + j.
template <int V>
__device__ __forceinline__ void load_slice_f32(const float* src, float (&xr)[8 * V]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int v = 0; v < V; ++v) {
        const float4 a = __ldcg(reinterpret_cast<const float4*>(src + v * 256 + lane * 8));
        const float4 b = __ldcg(reinterpret_cast<const float4*>(src + v * 256 + lane * 8 + 4));
        xr[v * 8 + 0] = a.x; xr[v * 8 + 1] = a.y; xr[v * 8 + 2] = a.z; xr[v * 8 + 3] = a.w;
        xr[v * 8 + 4] = b.x; xr[v * 8 + 5] = b.y; xr[v * 8 + 6] = b.z; xr[v * 8 + 7] = b.w;
    }
}

template <int V>
__device__ __forceinline__ void load_slice_f16(const __half* src, float (&xr)[8 * V]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int v = 0; v < V; ++v) {
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(src + v * 256 + lane * 8));
        float f[8];
        unpack_h8(w, f);
#pragma unroll
        for (int j = 0; j < 8; ++j) xr[v * 8 + j] = f[j];
    }
}

// RMSNorm of a full vector held as the warp's slices (dim == S): every warp
// computes the same sum of squares in the same order, so every warp of every
// CTA holds bit-identical normalised values.  x*invRms*w as RMSNorm.java:43,48.
template <int V>
__device__ __forceinline__ void rmsnorm_slice(float (&xr)[8 * V], const float* __restrict__ w, int dim, float eps) {
    const int lane = threadIdx.x & 31;
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < 8 * V; ++k) ss = fmaf(xr[k], xr[k], ss);
    ss = warp_sum(ss);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)dim), eps)));
#pragma unroll
    for (int v = 0; v < V; ++v) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(w + v * 256 + lane * 8));
        const float4 b = __ldg(reinterpret_cast<const float4*>(w + v * 256 + lane * 8 + 4));
        const float wv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) xr[v * 8 + j] = __fmul_rn(__fmul_rn(xr[v * 8 + j], inv), wv[j]);
    }
}

}  // namespace lc
