// lc_gemm.cu -- batched GEMV / skinny GEMM on the tcgen05 tensor cores.
//
// Y[s][n] = sum_k A[s][k] * W[n][k] for B <= 64 activation rows s (decode
// batch: one row per sequence), W F16 in the tiled layout of lc_internal.h,
// fp32 results through a fused epilogue (residual add, RoPE + KV-cache
// write, SwiGLU, logits + argmax).  It is the IGEMV product
// (K/IGEMV.java:34-68) for many activation vectors at once.
//
// Precision.  A is fp32.  Each row is split into f16 hi and lo parts under a
// power-of-two row scale 2^e with max_k |A[s][k]| * 2^e in [2^14, 2^15):
// A * 2^e = hi + lo to 2^-22 relative, the subtraction being exact.  The 128
// MMA rows hold (hi, lo) of the 64 sequences interleaved (row 2s = hi(s),
// row 2s+1 = lo(s)), so one tcgen05.mma (M = 128, N = N block, K = 16) does
// both halves and D lanes 2s, 2s+1 sum to the product (adjacent lanes of one
// warp: a shuffle).  Products of f16 values are exact; accumulation is fp32.
//
// Work unit = (N block of nblk rows, K split).  Units are dealt round-robin
// over a grid of at most one CTA per SM.  Warp roles (320 threads):
//   warp 0     streams the unit's weight blocks: per 64-column chunk and
//              8-row tile one 1 KB 1-D bulk copy (the tile's 8 octets of the
//              chunk are contiguous in the tiled layout) into a 4-stage ring;
//   warp 1     allocates 512 TMEM columns (two 256-column accumulators);
//              lane 0 issues the MMAs of each chunk and commits them to the
//              stage's "empty" barrier, and each unit to its accumulator;
//   warps 2-5  epilogue: TMEM lane quarter warp % 4, 16 columns per load;
//   warps 6-9  load the unit's A chunks (fp32, L2) and write hi / lo in the
//              canonical K-major layout, then arrive on the stage.
// With kspl > 1 every unit writes its partial sums; the last unit of an N
// block (ticket) adds them in split order (deterministic) and runs the
// epilogue.  Every wait is bounded (error word + LC_ERR_TIMEOUT); TMEM is
// released and in-flight copies and MMAs are drained on every path.
#include "lc_internal.h"
#include "lc_tcgen05.cuh"

namespace lc {
namespace {

constexpr int kThreads = 320;
constexpr int kStages = 4;
constexpr int kKC = 64;                   // columns per stage
constexpr int kABytes = 128 * kKC * 2;    // 16 KB: 128 MMA rows
constexpr int kMaxN = 256;
constexpr int kWBytes = kMaxN * kKC * 2;  // 32 KB
constexpr int kStageBytes = kABytes + kWBytes;
constexpr int kTmemCols = 512;
constexpr uint32_t kBarEpi = 1;           // named barrier of the 128 epilogue threads
constexpr int kEpiT0 = 64, kLoadT0 = 192; // first thread of the epilogue / loader warps

struct Bars {
    uint64_t wfull[kStages];  // weight bytes landed (producer arrive + tx)
    uint64_t afull[kStages];  // A chunk written (4 loader warps)
    uint64_t empty[kStages];  // MMAs of the stage done (tcgen05.commit)
    uint64_t dfull[2];        // accumulator complete (tcgen05.commit)
    uint64_t dempty[2];       // accumulator read out (epilogue)
    uint64_t drain;           // all MMAs of the CTA done
    uint32_t tmem;
    int flag;
    uint32_t rmax[kGemmMaxB];
    unsigned long long best[kGemmMaxB];
};
constexpr int kSmemBytes = kStages * kStageBytes + (int)sizeof(Bars);

// Row scale of the hi / lo split (same rule as the fused decode kernel).
__device__ __forceinline__ int row_exp(float m) {
    if (!(m > 0.0f)) return 0;
    int e = 14 - (((__float_as_int(m) >> 23) & 0xff) - 127);
    return e < -126 ? -126 : (e > 126 ? 126 : e);
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// RoPE of one interleaved pair (RoPE.java:42-49): angle pos * freq in float,
// cos / sin in double rounded to float, products and sums not contracted.
__device__ __forceinline__ void rope2(float& v0, float& v1, int pos, float freq) {
    double sd, cd;
    sincos((double)__fmul_rn((float)pos, freq), &sd, &cd);
    const float s = (float)sd, c = (float)cd, a = v0, b = v1;
    v0 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    v1 = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
}

// Epilogue of output columns n..n+3 (n % 4 == 0) of row s.
__device__ __forceinline__ void apply4(const GemmParams& p, Bars* bs, int s, int n, float (&y)[4]) {
    switch (p.op) {
        case kGemmStore:
            *reinterpret_cast<float4*>(p.y + (size_t)s * p.ldy + n) = make_float4(y[0], y[1], y[2], y[3]);
            break;
        case kGemmResid: {
            // o-proj / down-proj output plus the residual (TransformerBlock.java:195-198, 211-216)
            float4* dst = reinterpret_cast<float4*>(p.y + (size_t)s * p.ldy + n);
            float4 x = *dst;
            x.x = __fadd_rn(y[0], x.x);
            x.y = __fadd_rn(y[1], x.y);
            x.z = __fadd_rn(y[2], x.z);
            x.w = __fadd_rn(y[3], x.w);
            *dst = x;
            break;
        }
        case kGemmQKV: {
            const int pos = p.pos[s];
            if (n < p.qdim + p.kvd) {
                const int i = (n < p.qdim ? n : n - p.qdim) & (kGemmHeadDim - 1);
                rope2(y[0], y[1], pos, p.rope_freq[i >> 1]);
                rope2(y[2], y[3], pos, p.rope_freq[(i >> 1) + 1]);
            }
            const float4 v = make_float4(y[0], y[1], y[2], y[3]);
            if (n < p.qdim) {
                *reinterpret_cast<float4*>(p.q + (size_t)s * p.qdim + n) = v;
            } else {
                const bool isk = n < p.qdim + p.kvd;
                const int rr = n - p.qdim - (isk ? 0 : p.kvd);
                float* base = isk ? p.kcache : p.vcache;
                float* dst = base + (size_t)s * p.kv_seq_stride + (size_t)(rr / kGemmHeadDim) * p.kv_head_stride +
                             (size_t)pos * kGemmHeadDim + (rr & (kGemmHeadDim - 1));
                *reinterpret_cast<float4*>(dst) = v;
            }
            break;
        }
        case kGemmSwiGLU: {
            // rows 4m..4m+3 = gate 2m, up 2m, gate 2m+1, up 2m+1 (TransformerBlock.java:207-210)
            const float h0 = __fmul_rn(silu_ref(y[0]), y[1]);
            const float h1 = __fmul_rn(silu_ref(y[2]), y[3]);
            *reinterpret_cast<float2*>(p.h + (size_t)s * p.ldh + (n >> 1)) = make_float2(h0, h1);
            const float m = fmaxf(fabsf(h0), fabsf(h1));
            if (m > 0.0f) atomicMax(&bs->rmax[s], __float_as_uint(m));
            break;
        }
        default: {  // kGemmLogits
            if (p.logits)
                *reinterpret_cast<float4*>(p.logits + (size_t)s * p.ldl + n) = make_float4(y[0], y[1], y[2], y[3]);
            unsigned long long k = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                unsigned long long kj = 0;
                if (y[j] == y[j]) kj = argmax_key(y[j], n + j);
                else if (n + j == 0) kj = ~0ull;  // NaN at index 0: LlamaInference.argmax returns 0
                k = kj > k ? kj : k;
            }
            if (k) atomicMax(&bs->best[s], k);
            break;
        }
    }
}

__device__ __forceinline__ bool wait_warp(uint64_t* bar, uint32_t par, const GemmParams& p, int code) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0)
        ok = mbar_wait_bounded(bar, par, p.err, globaltimer_ns() + p.timeout_ns, code) ? 1 : 0;
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ GemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    Bars* bs = reinterpret_cast<Bars*>(smem + kStages * kStageBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, G = gridDim.x;
    const int krange = p.K / p.kspl, nchunk = krange / kKC, ncb = p.K / p.cbw;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bs->wfull[s], 1);
            mbar_init(&bs->afull[s], 4);
            mbar_init(&bs->empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&bs->dfull[a], 1);
            mbar_init(&bs->dempty[a], 1);
        }
        mbar_init(&bs->drain, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(&bs->tmem, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bs->tmem;

    if (warp == 0) {
        // ---------------------------------------------------- weight stream --
        const uint64_t policy = l2_policy_evict_first();
        uint32_t it = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < p.units && ok; u += G) {
            const int nbi = u / p.kspl, ks = u % p.kspl, n0 = nbi * p.nblk;
            const int ntile = min(p.nblk, p.N - n0) >> 3;
            for (int c = 0; c < nchunk; ++c, ++it) {
                const uint32_t slot = it % kStages, par = ((it / kStages) & 1u) ^ 1u;
                if (!wait_warp(&bs->empty[slot], par, p, kDevTimeoutEmpty)) {
                    ok = false;
                    break;
                }
                const int kc = ks * krange + c * kKC, cb = kc / p.cbw, o0 = (kc % p.cbw) >> 3;
                if (lane == 0) mbar_arrive_expect_tx(&bs->wfull[slot], (uint32_t)ntile * 1024u);
                __syncwarp();
                uint8_t* dst = smem + slot * kStageBytes + kABytes;
                for (int t = lane; t < ntile; t += 32) {
                    const __half* src = p.W + (((size_t)(n0 >> 3) + t) * ncb + cb) * (size_t)(8 * p.cbw) + o0 * 64;
                    bulk_g2s(dst + t * 1024, src, 1024u, &bs->wfull[slot], policy);
                }
            }
        }
        // Every issued copy lands before the CTA may exit.
        if (lane == 0) {
            const uint32_t first = it > (uint32_t)kStages ? it - kStages : 0u;
            for (uint32_t k = first; k < it; ++k)
                mbar_wait_bounded(&bs->wfull[k % kStages], (k / kStages) & 1u, p.err, globaltimer_ns() + 200000000ull,
                                  kDevTimeoutDrain);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------- MMA --
        if (lane == 0) {
            uint32_t it = 0;
            int j = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < p.units && ok; u += G, ++j) {
                const int a = j & 1, n0 = (u / p.kspl) * p.nblk, nb = min(p.nblk, p.N - n0);
                if (!mbar_wait_bounded(&bs->dempty[a], ((j >> 1) & 1) ^ 1, p.err,
                                       globaltimer_ns() + p.timeout_ns, kDevTimeoutFull)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(a * kMaxN);
                const uint32_t idesc = tc_idesc_f16_f32(128, nb);
                for (int c = 0; c < nchunk; ++c, ++it) {
                    const uint32_t slot = it % kStages, par = (it / kStages) & 1u;
                    const uint64_t dl = globaltimer_ns() + p.timeout_ns;
                    if (!mbar_wait_bounded(&bs->wfull[slot], par, p.err, dl, kDevTimeoutFull) ||
                        !mbar_wait_bounded(&bs->afull[slot], par, p.err, dl, kDevTimeoutFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t ab = smem_u32(smem + slot * kStageBytes), wb = ab + kABytes;
#pragma unroll
                    for (int k = 0; k < kKC / 16; ++k)
                        tc_mma_f16(d, tc_desc_kmajor(ab + k * 256, 128, 1024), tc_desc_kmajor(wb + k * 256, 128, 1024),
                                   idesc, (c | k) != 0 ? 1u : 0u);
                    tc_commit(&bs->empty[slot]);
                }
                if (ok) tc_commit(&bs->dfull[a]);
            }
            // Every MMA issued by this thread completes before TMEM is released.
            tc_commit(&bs->drain);
            mbar_wait_bounded(&bs->drain, 0, p.err, globaltimer_ns() + 200000000ull, kDevTimeoutDrain);
        }
    } else if (warp < 6) {
        // -------------------------------------------------------- epilogue --
        const int et = threadIdx.x - kEpiT0, q4 = warp & 3, r = q4 * 32 + lane, s = r >> 1;
        const bool lead = (r & 1) == 0 && s < p.B;
        const float unscale = s < p.B ? __int_as_float((127 - row_exp(__ldg(p.rowmax + s))) << 23) : 0.0f;
        int j = 0;
        for (int u = blockIdx.x; u < p.units; u += G, ++j) {
            const int a = j & 1, nbi = u / p.kspl, ks = u % p.kspl, n0 = nbi * p.nblk, nb = min(p.nblk, p.N - n0);
            if (et < kGemmMaxB) {
                bs->rmax[et] = 0u;
                bs->best[et] = 0ull;
            }
            bool got = mbar_wait_bounded(&bs->dfull[a], (j >> 1) & 1, p.err, globaltimer_ns() + p.timeout_ns,
                                         kDevTimeoutFull);
            if (bar_red_or(kBarEpi, 128, !got)) break;  // uniform exit
            tc_fence_after();
            for (int c0 = 0; c0 < nb; c0 += 16) {
                uint32_t v[16];
                tmem_ld16(tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(a * kMaxN + c0), v);
                tmem_wait_ld(v);
                float y[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float x = __uint_as_float(v[i]);
                    const float o = __shfl_xor_sync(0xffffffffu, x, 1);
                    y[i] = (x + o) * unscale;  // even lanes: hi + lo
                }
                if (lead) {
                    if (p.kspl == 1) {
#pragma unroll
                        for (int qd = 0; qd < 4; ++qd) {
                            float y4[4] = {y[4 * qd], y[4 * qd + 1], y[4 * qd + 2], y[4 * qd + 3]};
                            apply4(p, bs, s, n0 + c0 + 4 * qd, y4);
                        }
                    } else {
                        float4* dst = reinterpret_cast<float4*>(p.part + ((size_t)ks * p.B + s) * p.N + n0 + c0);
#pragma unroll
                        for (int qd = 0; qd < 4; ++qd)
                            dst[qd] = make_float4(y[4 * qd], y[4 * qd + 1], y[4 * qd + 2], y[4 * qd + 3]);
                    }
                }
            }
            tc_fence_before();
            named_bar_sync(kBarEpi, 128);
            if (et == 0) mbar_arrive(&bs->dempty[a]);
            if (p.kspl > 1) {
                // The last split of this N block adds the partials in split order.
                __threadfence();
                named_bar_sync(kBarEpi, 128);
                if (et == 0) bs->flag = atomicAdd(p.tickets + nbi, 1u) == (uint32_t)(p.kspl - 1) ? 1 : 0;
                named_bar_sync(kBarEpi, 128);
                if (*reinterpret_cast<volatile int*>(&bs->flag)) {
                    __threadfence();
                    const int nq = nb >> 2;
                    for (int i = et; i < p.B * nq; i += 128) {
                        const int ss = i / nq, n = n0 + 4 * (i % nq);
                        float4 acc = __ldcg(reinterpret_cast<const float4*>(p.part + (size_t)ss * p.N + n));
                        for (int k = 1; k < p.kspl; ++k) {
                            const float4 t =
                                __ldcg(reinterpret_cast<const float4*>(p.part + ((size_t)k * p.B + ss) * p.N + n));
                            acc.x += t.x;
                            acc.y += t.y;
                            acc.z += t.z;
                            acc.w += t.w;
                        }
                        float y4[4] = {acc.x, acc.y, acc.z, acc.w};
                        apply4(p, bs, ss, n, y4);
                    }
                    if (et == 0) p.tickets[nbi] = 0u;
                }
            }
            named_bar_sync(kBarEpi, 128);
            if (et < p.B) {
                if (p.op == kGemmSwiGLU && bs->rmax[et]) atomicMax(p.hmax + et, bs->rmax[et]);
                if (p.op == kGemmLogits && bs->best[et]) atomicMax(p.best + et, bs->best[et]);
            }
            named_bar_sync(kBarEpi, 128);
        }
    } else {
        // ---------------------------------------------------------- A loader --
        const int lt = threadIdx.x - kLoadT0;
        const int items = ((p.B + 3) >> 2) * 64;  // (4 sequences x 8 octets x hi / lo) blocks
        uint32_t it = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < p.units && ok; u += G) {
            const int ks = u % p.kspl;
            for (int c = 0; c < nchunk; ++c, ++it) {
                const uint32_t slot = it % kStages, par = ((it / kStages) & 1u) ^ 1u;
                if (!wait_warp(&bs->empty[slot], par, p, kDevTimeoutEmpty)) {
                    ok = false;
                    break;
                }
                const int kc = ks * krange + c * kKC;
                uint8_t* ab = smem + slot * kStageBytes;
                for (int i = lt; i < items; i += 128) {
                    // 8 consecutive items = rows 0..7 of one core matrix (128 B)
                    const int part = i & 1, sl = (i >> 1) & 3, o = (i >> 3) & 7, s4 = i >> 6, s = 4 * s4 + sl;
                    if (s < p.B) {
                        const float4* src = reinterpret_cast<const float4*>(p.A + (size_t)s * p.lda + kc + 8 * o);
                        const float4 x0 = __ldcg(src), x1 = __ldcg(src + 1);
                        const float sc = __int_as_float((127 + row_exp(__ldg(p.rowmax + s))) << 23);
                        const float f[8] = {x0.x * sc, x0.y * sc, x0.z * sc, x0.w * sc,
                                            x1.x * sc, x1.y * sc, x1.z * sc, x1.w * sc};
                        uint32_t w[4];
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const __half2 hh = __floats2half2_rn(f[2 * k], f[2 * k + 1]);
                            if (part == 0) {
                                w[k] = *reinterpret_cast<const uint32_t*>(&hh);
                            } else {
                                const float2 hf = __half22float2(hh);
                                w[k] = pack_h2(f[2 * k] - hf.x, f[2 * k + 1] - hf.y);
                            }
                        }
                        *reinterpret_cast<uint4*>(ab + s4 * 1024 + o * 128 + (2 * sl + part) * 16) =
                            make_uint4(w[0], w[1], w[2], w[3]);
                    }
                }
                fence_async_shared();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bs->afull[slot]);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

__global__ void rowmax_kernel(const float* __restrict__ A, int lda, int K, float* __restrict__ out) {
    const float* a = A + (size_t)blockIdx.x * lda;
    float m = 0.0f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) m = fmaxf(m, fabsf(a[k]));
    m = warp_max(m);
    __shared__ float red[8];
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
        out[blockIdx.x] = m;
    }
}

}  // namespace

bool gemm_plan(GemmParams* p, int num_sms) {
    if (p->B < 1 || p->B > kGemmMaxB || p->N < 16 || p->N % 16 || p->K < kKC || p->K % kKC || p->cbw < kKC ||
        p->cbw % kKC || p->K % p->cbw || p->lda % 4)
        return false;
    const int G = num_sms > 0 ? num_sms : 1;
    double best = 1e300;
    for (int nblk = kMaxN; nblk >= 16; nblk -= 16) {
        const int nbk = (p->N + nblk - 1) / nblk;
        for (int kspl = 1; kspl <= 32; kspl *= 2) {
            if (p->K % (kspl * kKC)) continue;
            const int krange = p->K / kspl, units = nbk * kspl, waves = (units + G - 1) / G;
            // Per-CTA time of the slowest wave in bytes: weights (HBM), A (L2,
            // cheaper), a fixed cost per unit (pipeline fill, epilogue) and
            // the partial round trip of split units.
            double cost = waves * ((double)nblk * krange * 2 + 0.35 * p->B * krange * 4 + 64 * 1024);
            if (kspl > 1) cost += 0.5 * (double)kspl * p->B * nblk * 4 + 32 * 1024;
            if (cost < best * 0.999) {
                best = cost;
                p->nblk = nblk;
                p->kspl = kspl;
                p->units = units;
            }
        }
    }
    return true;
}

size_t gemm_part_bytes(const GemmParams& p) {
    return p.kspl > 1 ? (size_t)p.kspl * p.B * p.N * sizeof(float) : 0;
}

int gemm_tile_width(int cols) {
    if (cols % kKC) return 0;
    int best = kKC;
    for (int w = kKC; w <= 2048 && w <= cols; w += kKC)
        if (cols % w == 0) best = w;
    return best;
}

cudaError_t gemm_prepare() {
    return cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
}

cudaError_t launch_gemm(const GemmParams& p, int num_sms, cudaStream_t st) {
    const int grid = p.units < num_sms ? p.units : num_sms;
    gemm_kernel<<<grid, kThreads, kSmemBytes, st>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_rowmax(const float* A, int lda, int K, int B, float* rowmax, cudaStream_t st) {
    rowmax_kernel<<<B, 256, 0, st>>>(A, lda, K, rowmax);
    return cudaGetLastError();
}

}  // namespace lc
