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
// over a grid of at most one CTA per SM.  A is split once per product
// (launch_gemm_split, or fused into the producing kernel) into the MMA's
// K-major layout in global memory, so both operands reach shared memory as
// 1-D bulk copies.  Warp roles (192 threads):
//   warp 0     lane 0, per 64-column chunk: one TMA box of the weights (a 4-D
//              tensor map over the tiled layout: 8 octets x nblk/8 tiles,
//              landing in the MMA's K-major core-matrix order) and one box
//              of the pre-split activations (3-D map), into a ring of 4..12
//              stages (fewer, larger stages for wide N blocks: about 190 KB
//              in flight);
//   warp 1     allocates 512 TMEM columns (two 256-column accumulators);
//              lane 0 issues the MMAs of each chunk, commits them to the
//              stage's "empty" barrier, and each unit to its accumulator;
//   warps 2-5  epilogue: TMEM lane quarter warp % 4, 16 columns per load.
// With kspl > 1 every unit writes its partial sums and a second, fully
// parallel kernel adds them in split order (deterministic) and runs the
// epilogue.  Every wait is bounded (error word + LC_ERR_TIMEOUT); TMEM is
// released and in-flight copies and MMAs are drained on every path.
#include <cudaTypedefs.h>

#include "lc_internal.h"
#include "lc_tcgen05.cuh"

namespace lc {
namespace {

constexpr int kThreads = 192;
constexpr int kMaxStages = 12;
constexpr int kRingBytes = 200 * 1024;
constexpr int kKC = 64;                   // columns per stage
constexpr int kABytes = 128 * kKC * 2;    // 16 KB: 128 MMA rows (only the used row groups are copied)
constexpr int kMaxN = 256;
constexpr int kTmemCols = 512;
constexpr uint32_t kBarEpi = 1;           // named barrier of the 128 epilogue threads
constexpr int kEpiT0 = 64;                // first epilogue thread

struct Bars {
    uint64_t full[kMaxStages];   // weight and activation bytes landed (producer arrive + tx)
    uint64_t empty[kMaxStages];  // MMAs of the stage done (tcgen05.commit)
    uint64_t dfull[2];        // accumulator complete (tcgen05.commit)
    uint64_t dempty[2];       // accumulator read out (epilogue)
    uint64_t drain;           // all MMAs of the CTA done
    uint32_t tmem;
    unsigned long long best[kGemmMaxB];
};
constexpr int kSmemMax = kRingBytes + (int)sizeof(Bars);

// RoPE of one interleaved pair (RoPE.java:42-49): angle pos * freq in float,
// cos / sin in double rounded to float, products and sums not contracted.
__device__ __forceinline__ void rope2(float& v0, float& v1, int pos, float freq) {
    double sd, cd;
    sincos((double)__fmul_rn((float)pos, freq), &sd, &cd);
    const float s = (float)sd, c = (float)cd, a = v0, b = v1;
    v0 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    v1 = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
}

// Epilogue of output columns n..n+3 (n % 4 == 0) of row s.  Returns the
// argmax key of the four logits (kGemmLogits; 0 otherwise).
__device__ __forceinline__ unsigned long long apply4(const GemmParams& p, int s, int n, float (&y)[4]) {
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
                const int seq = p.row_seq ? p.row_seq[s] : s;
                float* dst = base + (size_t)seq * p.kv_seq_stride + (size_t)(rr / kGemmHeadDim) * p.kv_head_stride +
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
            break;
        }
        default: {  // kGemmLogits
            if (p.logits)
                *reinterpret_cast<float4*>(p.logits + (size_t)s * p.ldl + n) = make_float4(y[0], y[1], y[2], y[3]);
            unsigned long long k = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                unsigned long long kj = 0;
                if (n + j >= p.n_valid) break;
                if (y[j] == y[j]) kj = argmax_key(y[j], p.idx_offset + n + j);
                else if (p.idx_offset + n + j == 0) kj = ~0ull;  // NaN at index 0: LlamaInference.argmax returns 0
                k = kj > k ? kj : k;
            }
            return k;
        }
    }
    return 0ull;
}

// Unit u -> (K split, row tile, N block): the split varies fastest, then the
// row tile, so consecutive CTAs share an N block of weights (L2 reuse when
// there are several row tiles).
struct Unit {
    int ks, mt, nbi;
};
__device__ __forceinline__ Unit unit_of(const GemmParams& p, int u) {
    const int rest = u / p.kspl;
    return Unit{u % p.kspl, rest % p.mtiles, rest / p.mtiles};
}

__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ GemmParams p,
                                                           const __grid_constant__ CUtensorMap wmap,
                                                           const __grid_constant__ CUtensorMap amap) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int NS = p.stages, SB = p.stage_bytes;
    Bars* bs = reinterpret_cast<Bars*>(smem + NS * SB);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, G = gridDim.x;
    const int krange = p.K / p.kspl, nchunk = krange / kKC;
    const int nrg = p.mtiles > 1 ? 16 : (p.B + 3) >> 2;  // activation row groups per box

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&bs->full[s], 1);
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
        // ------------------------------------------------------ copy stream --
        if (lane == 0) {
            const uint64_t wpol = l2_policy_evict_first(), apol = l2_policy_evict_last();
            const uint32_t tx = (uint32_t)(p.nblk * kKC * 2 + nrg * 1024);  // full boxes, out-of-range rows zero-filled
            // Weights never depend on an earlier kernel: the first stages'
            // weight boxes go out before the wait for the predecessor (whose
            // results the activation boxes carry).
            const int u0 = blockIdx.x;
            const int pre = u0 < p.units ? min(NS, nchunk) : 0;
            const Unit U0 = unit_of(p, u0);
            {
                const int ks = U0.ks, g0 = (U0.nbi * p.nblk) >> 3;
                for (int c = 0; c < pre; ++c) {
                    const int kc = ks * krange + c * kKC;
                    mbar_arrive_expect_tx(&bs->full[c], tx);
                    tma_load_4d(smem + c * SB + kABytes, &wmap, 0, (kc % p.cbw) >> 3, kc / p.cbw, g0, &bs->full[c],
                                wpol);
                }
            }
            griddep_wait();
            for (int c = 0; c < pre; ++c)
                tma_load_3d(smem + c * SB, &amap, 0, (U0.ks * krange + c * kKC) >> 3, U0.mt * 16, &bs->full[c], apol);
            uint32_t it = (uint32_t)pre, slot = (uint32_t)(pre % NS), par = pre == NS ? 0u : 1u;
            bool ok = true;
            for (int u = blockIdx.x; u < p.units && ok; u += G) {
                const Unit U = unit_of(p, u);
                const int ks = U.ks, g0 = (U.nbi * p.nblk) >> 3;
                for (int c = (u == u0 ? pre : 0); c < nchunk; ++c) {
                    if (!mbar_wait_bounded(&bs->empty[slot], par, p.err, globaltimer_ns() + p.timeout_ns,
                                           kDevTimeoutEmpty)) {
                        ok = false;
                        break;
                    }
                    const int kc = ks * krange + c * kKC;
                    uint8_t* st = smem + slot * SB;
                    mbar_arrive_expect_tx(&bs->full[slot], tx);
                    tma_load_4d(st + kABytes, &wmap, 0, (kc % p.cbw) >> 3, kc / p.cbw, g0, &bs->full[slot], wpol);
                    tma_load_3d(st, &amap, 0, kc >> 3, U.mt * 16, &bs->full[slot], apol);
                    ++it;
                    if (++slot == (uint32_t)NS) {
                        slot = 0;
                        par ^= 1u;
                    }
                }
            }
            // Every issued copy lands before the CTA may exit.
            const uint32_t first = it > (uint32_t)NS ? it - NS : 0u;
            for (uint32_t k = first; k < it; ++k)
                mbar_wait_bounded(&bs->full[k % NS], (k / NS) & 1u, p.err, globaltimer_ns() + 200000000ull,
                                  kDevTimeoutDrain);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------- MMA --
        if (lane == 0) {
            uint32_t slot = 0, par = 0;
            int j = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < p.units && ok; u += G, ++j) {
                const int a = j & 1, n0 = unit_of(p, u).nbi * p.nblk, nb = min(p.nblk, p.N - n0);
                if (!mbar_wait_bounded(&bs->dempty[a], ((j >> 1) & 1) ^ 1, p.err, globaltimer_ns() + p.timeout_ns,
                                       kDevTimeoutFull)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(a * kMaxN);
                const uint32_t idesc = tc_idesc_f16_f32(128, nb);
                for (int c = 0; c < nchunk; ++c) {
                    if (!mbar_wait_bounded(&bs->full[slot], par, p.err, globaltimer_ns() + p.timeout_ns,
                                           kDevTimeoutFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t ab = smem_u32(smem + slot * SB), wb = ab + kABytes;
#pragma unroll
                    for (int k = 0; k < kKC / 16; ++k)
                        tc_mma_f16(d, tc_desc_kmajor(ab + k * 256, 128, 1024), tc_desc_kmajor(wb + k * 256, 128, 1024),
                                   idesc, (c | k) != 0 ? 1u : 0u);
                    tc_commit(&bs->empty[slot]);
                    if (++slot == (uint32_t)NS) {
                        slot = 0;
                        par ^= 1u;
                    }
                }
                if (ok) tc_commit(&bs->dfull[a]);
            }
            // Every MMA issued by this thread completes before TMEM is released.
            tc_commit(&bs->drain);
            mbar_wait_bounded(&bs->drain, 0, p.err, globaltimer_ns() + 200000000ull, kDevTimeoutDrain);
        }
    } else {
        // -------------------------------------------------------- epilogue --
        griddep_wait();  // unscale and the epilogue's outputs belong to the predecessor's stream order
        const int et = threadIdx.x - kEpiT0, q4 = warp & 3, r = q4 * 32 + lane, sl = r >> 1;
        // With one row tile a lane's row is the same in every unit: its best
        // key over all the CTA's units goes out once, after the last unit
        // (one global atomic per row and CTA).
        const bool carry = p.mtiles == 1;
        unsigned long long kcarry = 0ull;
        bool done_all = true;
        int j = 0;
        for (int u = blockIdx.x; u < p.units; u += G, ++j) {
            // Dependents may launch once every CTA is in its last epilogue
            // (earlier, their blocks would compete with the weight stream).
            if (u + G >= p.units) griddep_launch();
            const Unit U = unit_of(p, u);
            const int a = j & 1, ks = U.ks, n0 = U.nbi * p.nblk, nb = min(p.nblk, p.N - n0);
            const int s = U.mt * kGemmMaxB + sl;  // activation row of this lane pair
            const bool lead = (r & 1) == 0 && s < p.B;
            const float unscale = s < p.B ? __ldcg(p.unscale + s) : 0.0f;
            if (et < kGemmMaxB) bs->best[et] = 0ull;
            bool got = mbar_wait_bounded(&bs->dfull[a], (j >> 1) & 1, p.err, globaltimer_ns() + p.timeout_ns,
                                         kDevTimeoutFull);
            if (bar_red_or(kBarEpi, 128, !got)) {  // uniform exit
                done_all = false;
                break;
            }
            tc_fence_after();
            // Each row's keys come from one lead lane of the CTA (TMEM lane
            // pair 2s, 2s + 1): its best key stays in a register.
            unsigned long long kb = 0ull;
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
                    if (p.kspl == 1 && p.op == kGemmLogits) {
                        // Logits of the 16 columns, then one packed key for the
                        // chunk: its maximum (NaN never wins, padding columns
                        // excluded) at the lowest column holding it -- the
                        // largest of the 16 per-column keys -- except that a
                        // NaN at global index 0 wins outright
                        // (LlamaInference.argmax returns 0 then).
                        const int nc = n0 + c0;
                        if (p.logits) {
                            float4* lo4 = reinterpret_cast<float4*>(p.logits + (size_t)s * p.ldl + nc);
#pragma unroll
                            for (int qd = 0; qd < 4; ++qd)
                                lo4[qd] = make_float4(y[4 * qd], y[4 * qd + 1], y[4 * qd + 2], y[4 * qd + 3]);
                        }
                        float m = -INFINITY;
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            if (nc + i < p.n_valid) m = fmaxf(m, y[i]);
                        int fi = -1;
#pragma unroll
                        for (int i = 15; i >= 0; --i)
                            if (nc + i < p.n_valid && y[i] == m) fi = i;
                        unsigned long long k = fi >= 0 ? argmax_key(m, p.idx_offset + nc + fi) : 0ull;
                        if (p.idx_offset + nc == 0 && y[0] != y[0]) k = ~0ull;
                        kb = k > kb ? k : kb;
                    } else if (p.kspl == 1) {
#pragma unroll
                        for (int qd = 0; qd < 4; ++qd) {
                            float y4[4] = {y[4 * qd], y[4 * qd + 1], y[4 * qd + 2], y[4 * qd + 3]};
                            const unsigned long long k = apply4(p, s, n0 + c0 + 4 * qd, y4);
                            kb = k > kb ? k : kb;
                        }
                    } else {
                        float4* dst = reinterpret_cast<float4*>(p.part + ((size_t)ks * p.B + s) * p.N + n0 + c0);
#pragma unroll
                        for (int qd = 0; qd < 4; ++qd)
                            dst[qd] = make_float4(y[4 * qd], y[4 * qd + 1], y[4 * qd + 2], y[4 * qd + 3]);
                    }
                }
            }
            if (carry) kcarry = kb > kcarry ? kb : kcarry;
            else if (lead && kb) bs->best[sl] = kb;
            tc_fence_before();
            named_bar_sync(kBarEpi, 128);
            if (et == 0) mbar_arrive(&bs->dempty[a]);
            named_bar_sync(kBarEpi, 128);
            if (!carry && et < kGemmMaxB && U.mt * kGemmMaxB + et < p.B && p.op == kGemmLogits && bs->best[et])
                atomicMax(p.best + U.mt * kGemmMaxB + et, bs->best[et]);
            named_bar_sync(kBarEpi, 128);
        }
        if (carry && done_all && p.op == kGemmLogits && (r & 1) == 0 && sl < p.B && kcarry)
            atomicMax(p.best + sl, kcarry);
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// Split-K results: y = the partial sums of the kspl splits added in split
// order (deterministic), then the epilogue.  One (row, 4 columns) item per
// thread; a row's items are consecutive, so the argmax keys of a warp are
// merged before one atomic per row and warp.
__global__ void __launch_bounds__(256) gemm_reduce_kernel(const __grid_constant__ GemmParams p) {
    griddep_launch();
    griddep_wait();
    const int nq = p.N >> 2;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const bool live = i < (long long)p.B * nq;
    int s = 0;
    unsigned long long k = 0ull;
    if (live) {
        s = (int)(i / nq);
        const int n = (int)(i % nq) * 4;
        const float* src = p.part + (size_t)s * p.N + n;
        const size_t stride = (size_t)p.B * p.N;
        // Up to 8 splits' loads in flight at once (one L2 round trip instead
        // of one per split), added in split order.
        float4 acc = __ldcg(reinterpret_cast<const float4*>(src));
        for (int k0 = 1; k0 < p.kspl; k0 += 8) {
            float4 t[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (k0 + j < p.kspl) t[j] = __ldcg(reinterpret_cast<const float4*>(src + (k0 + j) * stride));
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (k0 + j < p.kspl) {
                    acc.x += t[j].x;
                    acc.y += t[j].y;
                    acc.z += t[j].z;
                    acc.w += t[j].w;
                }
            }
        }
        float y4[4] = {acc.x, acc.y, acc.z, acc.w};
        k = apply4(p, s, n, y4);
    }
    if (p.op == kGemmLogits) {
        // lanes of one row are contiguous: reduce per (warp, row) segment
        const int lane = threadIdx.x & 31;
        const int s0 = __shfl_sync(0xffffffffu, s, 0);
        const bool uniform = __all_sync(0xffffffffu, s == s0);
        if (uniform) {
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, k, o);
                k = k2 > k ? k2 : k;
            }
            if (lane == 0 && k) atomicMax(p.best + s0, k);
        } else if (live && k) {
            atomicMax(p.best + s, k);
        }
    }
}

// One activation row per CTA: max |A[s][k]|, the row scale 2^e with
// max * 2^e in [2^14, 2^15), then hi = f16(a * 2^e), lo = f16(a * 2^e - hi)
// into the pre-split layout (MMA rows 2 (s % 4) and 2 (s % 4) + 1 of row
// group s / 4).
__global__ void __launch_bounds__(256) split_rows_kernel(const float* __restrict__ A, int lda, int K,
                                                         uint8_t* __restrict__ As, float* __restrict__ unscale) {
    griddep_launch();
    griddep_wait();
    const int s = blockIdx.x;
    const float* a = A + (size_t)s * lda;
    float m = 0.0f;
    for (int k = threadIdx.x * 4; k < K; k += 256 * 4) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(a + k));
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    m = warp_max(m);
    __shared__ float red[8];
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < 8; ++w) m = fmaxf(m, red[w]);
    const int e = split_row_exp(m);
    const float sc = pow2f(e);
    if (threadIdx.x == 0) unscale[s] = pow2f(-e);
    for (int o = threadIdx.x; o < (K >> 3); o += 256) {
        const float4 x0 = __ldcg(reinterpret_cast<const float4*>(a + 8 * o));
        const float4 x1 = __ldcg(reinterpret_cast<const float4*>(a + 8 * o + 4));
        const float f[8] = {x0.x * sc, x0.y * sc, x0.z * sc, x0.w * sc, x1.x * sc, x1.y * sc, x1.z * sc, x1.w * sc};
        uint4* d = reinterpret_cast<uint4*>(As + split_offset(s, o, K));
        split_octet(f, d[0], d[1]);
    }
}

}  // namespace

bool gemm_plan(GemmParams* p, int num_sms) {
    if (p->B < 1 || p->N < 16 || p->N % 16 || p->K < kKC || p->K % kKC || p->cbw < kKC || p->cbw % kKC ||
        p->K % p->cbw)
        return false;
    const int G = num_sms > 0 ? num_sms : 1;
    p->mtiles = (p->B + kGemmMaxB - 1) / kGemmMaxB;
    if (p->mtiles > 1) {
        // Many row tiles (prefill): the product is compute- and L2-bound;
        // widest N blocks, whole K per unit.
        p->nblk = kMaxN;
        p->kspl = 1;
        p->units = p->mtiles * ((p->N + kMaxN - 1) / kMaxN);
        p->stage_bytes = kABytes + kMaxN * kKC * 2;
        p->stages = kRingBytes / p->stage_bytes;
        return true;
    }
    const int nrg = (p->B + 3) / 4;
    double best = 1e300;
    for (int nblk = kMaxN; nblk >= 16; nblk -= 16) {
        const int nbk = (p->N + nblk - 1) / nblk;
        const int sb = kABytes + nblk * kKC * 2;
        int stages = kRingBytes / sb;
        if (stages > kMaxStages) stages = kMaxStages;
        // Weight bytes in flight per SM; below ~96 KB the stream is latency-bound.
        const double inflight = (double)stages * nblk * kKC * 2;
        const double bw = inflight < 96.0 * 1024 ? inflight / (96.0 * 1024) : 1.0;
        for (int kspl = 1; kspl <= 32; kspl *= 2) {
            if (p->K % (kspl * kKC)) continue;
            const int krange = p->K / kspl, units = nbk * kspl, waves = (units + G - 1) / G;
            // Per-CTA time of the slowest wave in bytes: weights (HBM), the
            // pre-split activations (L2, cheaper), a fixed cost per unit
            // (pipeline fill, epilogue) and the partial round trip of splits.
            double cost = waves * (((double)nblk * krange * 2 + 0.5 * nrg * krange * 16) / bw + 96 * 1024);
            // Split K: partials written and read back by the reduce kernel
            // (spread over the SMs) plus its launch.
            if (kspl > 1) cost += 3.0 * (double)kspl * p->B * p->N * 4 / G + 128 * 1024;
            if (cost < best * 0.999) {
                best = cost;
                p->nblk = nblk;
                p->kspl = kspl;
                p->units = units;
                p->stages = stages;
                p->stage_bytes = sb;
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
    return cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
}

namespace {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }
    return fn;
}
}  // namespace

cudaError_t gemm_make_wmap(CUtensorMap* out, const GemmParams& p) {
    auto enc = encode_fn();
    if (!enc || ((uintptr_t)p.W & 15)) return cudaErrorInvalidValue;
    // Element (i, o, cb, g) = half i of octet o of tile (g, cb): the tiled layout.
    const int ncb = p.K / p.cbw;
    const int rows = p.rows_mem > 0 ? p.rows_mem : p.N;  // rows stored; the rest of the last box reads zeros
    cuuint64_t dims[4] = {64, (cuuint64_t)(p.cbw / 8), (cuuint64_t)ncb, (cuuint64_t)(rows / 8)};
    cuuint64_t strides[3] = {128, (cuuint64_t)p.cbw * 16, (cuuint64_t)ncb * p.cbw * 16};
    cuuint32_t box[4] = {64, kKC / 8, 1, (cuuint32_t)(p.nblk / 8)};
    cuuint32_t es[4] = {1, 1, 1, 1};
    CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, const_cast<__half*>(p.W), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t gemm_make_amap(CUtensorMap* out, const GemmParams& p) {
    auto enc = encode_fn();
    if (!enc || ((uintptr_t)p.As & 15)) return cudaErrorInvalidValue;
    const int nrg = (p.B + 3) / 4;  // row groups stored; a box past them reads zeros
    cuuint64_t dims[3] = {64, (cuuint64_t)(p.K / 8), (cuuint64_t)nrg};
    cuuint64_t strides[2] = {128, (cuuint64_t)(p.K / 8) * 128};
    cuuint32_t box[3] = {64, kKC / 8, (cuuint32_t)(nrg < 16 ? nrg : 16)};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<uint8_t*>(p.As), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t launch_gemm(const GemmParams& p, const CUtensorMap& wmap, const CUtensorMap& amap, int num_sms,
                        cudaStream_t st, bool pdl) {
    if (p.stages < 2 || p.stages > kMaxStages || p.stages * p.stage_bytes > kRingBytes || p.nblk % 16 ||
        p.nblk > kMaxN || p.units < 1)
        return cudaErrorInvalidValue;
    const int grid = p.units < num_sms ? p.units : num_sms;
    const int smem = p.stages * p.stage_bytes + (int)sizeof(Bars);
    cudaError_t e = launch_ex(gemm_kernel, dim3(grid), dim3(kThreads), (size_t)smem, st, pdl, p, wmap, amap);
    if (e != cudaSuccess || p.kspl == 1) return e;
    const long long items = (long long)p.B * (p.N >> 2);
    return launch_ex(gemm_reduce_kernel, dim3((unsigned)((items + 255) / 256)), dim3(256), 0, st, pdl, p);
}

cudaError_t launch_gemm_split(const float* A, int lda, int K, int B, uint8_t* As, float* unscale, cudaStream_t st,
                              bool pdl) {
    return launch_ex(split_rows_kernel, dim3(B), dim3(256), 0, st, pdl, A, lda, K, As, unscale);
}

}  // namespace lc
