// lc_attention.cuh -- one unit of GQA split-KV decode attention.
//
// A unit is (sequence, kv head, split of positions [t0, t1)).  It serves the
// kv_mul = n_heads / n_kv query heads that share the kv head (GQA, 4:1 for
// Llama-3.2-1B; TransformerBlock.java:165-168).  256 threads cooperate through
// named barrier 1 (the consumer warps of the fused decode kernel, or the whole
// CTA of the standalone launch).
//
// With a single split the unit reproduces the reference loop order exactly:
// sequential score dot products (Attention.java:36-40), max, exp in double,
// sequential sum, p = e * (1/sum) (Softmax.java:30-50), sequential weighted
// values (Attention.java:54-60) -- bit-identical to the Java kernels for the
// same q, K and V.  With several splits each unit writes a partial
// (max, sum, unnormalised output) and the last unit to finish (ticket on a
// completion counter) merges them (flash-decoding combine).
#pragma once

#include "lc_common.cuh"

namespace lc {

constexpr int kAttnHeadDim = 64;

// Units of more than kAttnExactMax positions take the throughput path.
constexpr int kAttnExactMax = 64;

// Shared-memory floats a unit needs: q, scores, (max, sum) per head and a
// flag word, then the cross-warp value partials of the throughput path.
__host__ __device__ inline int attn_unit_smem_floats(int kv_mul, int tmax) {
    return kv_mul * kAttnHeadDim + kv_mul * tmax + 2 * kv_mul + 4 + 8 * kv_mul * kAttnHeadDim;
}

// Partial record per (split, head): [m, l, o[64]].
constexpr int kAttnPartStride = kAttnHeadDim + 2;

// Scores, softmax and weighted values of one unit.  nsplit == 1 writes the
// normalised output of the kv_mul heads to out[h * 64 + i]; otherwise the
// partial record of (split, h) goes to part[(split * kv_mul + h) * stride].
// Ends with the unit's stores issued (no barrier after them).
__device__ __forceinline__ void attention_core(const float* __restrict__ q, const float* __restrict__ K,
                                               const float* __restrict__ Vc, int64_t pos_stride, int t0, int t1,
                                               int nsplit, int split, float* __restrict__ out,
                                               float* __restrict__ part, int part_stride, float scale, int kv_mul,
                                               int tmax, float* sm) {
    constexpr int HD = kAttnHeadDim;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int T = t1 - t0;
    float* qs = sm;
    float* sc = qs + kv_mul * HD;
    float* st = sc + kv_mul * tmax;

    for (int i = tid; i < kv_mul * HD; i += 256) qs[i] = __ldcg(q + i);
    named_bar_sync(1, 256);

    // Scores: consecutive threads take the kv_mul heads of one position.
    for (int idx = tid; idx < T * kv_mul; idx += 256) {
        const int h = idx % kv_mul, tt = idx / kv_mul;
        const float4* kr = reinterpret_cast<const float4*>(K + (int64_t)(t0 + tt) * pos_stride);
        const float* qh = qs + h * HD;
        float sum = 0.0f;
#pragma unroll
        for (int c = 0; c < HD / 4; ++c) {
            const float4 k4 = __ldcg(kr + c);
            sum = __fadd_rn(sum, __fmul_rn(qh[4 * c + 0], k4.x));
            sum = __fadd_rn(sum, __fmul_rn(qh[4 * c + 1], k4.y));
            sum = __fadd_rn(sum, __fmul_rn(qh[4 * c + 2], k4.z));
            sum = __fadd_rn(sum, __fmul_rn(qh[4 * c + 3], k4.w));
        }
        sc[h * tmax + tt] = __fmul_rn(sum, scale);
    }
    named_bar_sync(1, 256);

    // Per head: max, e = exp(s - max), sum.
    for (int h = warp; h < kv_mul; h += 8) {
        float* e = sc + h * tmax;
        float m = -INFINITY;
        for (int t = lane; t < T; t += 32) m = fmaxf(m, e[t]);
        m = warp_max(m);
        for (int t = lane; t < T; t += 32) e[t] = exp_via_double_nl(__fsub_rn(e[t], m));
        __syncwarp();
        float l = 0.0f;
        if (nsplit == 1) {
            if (lane == 0)
                for (int t = 0; t < T; ++t) l = __fadd_rn(l, e[t]);
            l = __shfl_sync(0xffffffffu, l, 0);
        } else {
            for (int t = lane; t < T; t += 32) l += e[t];
            l = warp_sum(l);
        }
        if (lane == 0) {
            st[2 * h] = m;
            st[2 * h + 1] = l;
        }
    }
    named_bar_sync(1, 256);

    // Weighted values: thread per (head, dim), sequential over positions.
    for (int hi = tid; hi < kv_mul * HD; hi += 256) {
        const int h = hi / HD, i = hi % HD;
        const float* e = sc + h * tmax;
        const float* vcol = Vc + (int64_t)t0 * pos_stride + i;
        float acc = 0.0f;
        if (nsplit == 1) {
            const float inv = __fdiv_rn(1.0f, st[2 * h + 1]);
#pragma unroll 4
            for (int t = 0; t < T; ++t)
                acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(e[t], inv), __ldcg(vcol + (int64_t)t * pos_stride)));
            out[h * HD + i] = acc;
        } else {
#pragma unroll 4
            for (int t = 0; t < T; ++t) acc = fmaf(e[t], __ldcg(vcol + (int64_t)t * pos_stride), acc);
            float* pp = part + ((int64_t)split * kv_mul + h) * part_stride;
            pp[2 + i] = acc;
            if (i == 0) {
                pp[0] = st[2 * h];
                pp[1] = st[2 * h + 1];
            }
        }
    }
}

// Throughput form of attention_core for units of more than kAttnExactMax
// positions: the same results up to float rounding (exp in float, sums in a
// tree order), with K and V rows read once, fully coalesced.  Scores: each
// warp takes 4 positions at a time, 8 lanes per position holding 8 of the
// 64 dimensions, a 3-step shuffle per head.  Softmax: one warp per head.
// Values: warps take positions t = warp (mod 8), each lane 2 dimensions of
// every head; the 8 warp partials are added in shared memory.
template <int KVM>
__device__ __forceinline__ void attention_core_fast(const float* __restrict__ q, const float* __restrict__ K,
                                                    const float* __restrict__ Vc, int64_t pos_stride, int t0,
                                                    int t1, int nsplit, int split, float* __restrict__ out,
                                                    float* __restrict__ part, int part_stride, float scale,
                                                    int tmax, float* sm) {
    constexpr int HD = kAttnHeadDim, MAXH = KVM, kv_mul = KVM;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 3, sub = lane & 7;
    const int T = t1 - t0;
    float* qs = sm;
    float* sc = qs + kv_mul * HD;
    float* st = sc + kv_mul * tmax;
    float* red = st + 2 * kv_mul + 4;  // [8 warps][kv_mul][64]

    for (int i = tid; i < kv_mul * HD; i += 256) qs[i] = __ldcg(q + i);
    named_bar_sync(1, 256);
    float qr[MAXH][8];
#pragma unroll
    for (int h = 0; h < MAXH; ++h)
#pragma unroll
        for (int j = 0; j < 8; ++j) qr[h][j] = h < kv_mul ? qs[h * HD + 8 * sub + j] : 0.0f;

    // Scores, four rounds of 32 positions in flight per warp pass.
    constexpr int R = 4;
    for (int base = warp * 4; base < T; base += 32 * R) {
        float4 a[R], b[R];
        bool ok[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int t = base + 32 * r + g;
            ok[r] = t < T;
            if (ok[r]) {
                const float4* kr = reinterpret_cast<const float4*>(K + (int64_t)(t0 + t) * pos_stride) + 2 * sub;
                a[r] = __ldcg(kr);
                b[r] = __ldcg(kr + 1);
            } else {
                a[r] = b[r] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int t = base + 32 * r + g;
#pragma unroll
            for (int h = 0; h < MAXH; ++h) {
                if (h < kv_mul) {
                    float d = qr[h][0] * a[r].x;
                    d = fmaf(qr[h][1], a[r].y, d);
                    d = fmaf(qr[h][2], a[r].z, d);
                    d = fmaf(qr[h][3], a[r].w, d);
                    d = fmaf(qr[h][4], b[r].x, d);
                    d = fmaf(qr[h][5], b[r].y, d);
                    d = fmaf(qr[h][6], b[r].z, d);
                    d = fmaf(qr[h][7], b[r].w, d);
                    d += __shfl_xor_sync(0xffffffffu, d, 1);
                    d += __shfl_xor_sync(0xffffffffu, d, 2);
                    d += __shfl_xor_sync(0xffffffffu, d, 4);
                    if (sub == 0 && ok[r]) sc[h * tmax + t] = d * scale;
                }
            }
        }
    }
    named_bar_sync(1, 256);

    // Per head: max, e = exp(s - max), sum.
    for (int h = warp; h < kv_mul; h += 8) {
        float* e = sc + h * tmax;
        float m = -INFINITY;
        for (int t = lane; t < T; t += 32) m = fmaxf(m, e[t]);
        m = warp_max(m);
        float l = 0.0f;
        for (int t = lane; t < T; t += 32) {
            const float v = expf(e[t] - m);
            e[t] = v;
            l += v;
        }
        l = warp_sum(l);
        if (lane == 0) {
            st[2 * h] = m;
            st[2 * h + 1] = l;
        }
    }
    named_bar_sync(1, 256);

    // Weighted values.
    float2 acc[MAXH];
#pragma unroll
    for (int h = 0; h < MAXH; ++h) acc[h] = make_float2(0.f, 0.f);
#pragma unroll 8
    for (int t = warp; t < T; t += 8) {
        const float2 v = __ldcg(reinterpret_cast<const float2*>(Vc + (int64_t)(t0 + t) * pos_stride) + lane);
#pragma unroll
        for (int h = 0; h < MAXH; ++h) {
            if (h < kv_mul) {
                const float p = sc[h * tmax + t];
                acc[h].x = fmaf(p, v.x, acc[h].x);
                acc[h].y = fmaf(p, v.y, acc[h].y);
            }
        }
    }
#pragma unroll
    for (int h = 0; h < MAXH; ++h)
        if (h < kv_mul) reinterpret_cast<float2*>(red + (warp * kv_mul + h) * HD)[lane] = acc[h];
    named_bar_sync(1, 256);
    for (int hi = tid; hi < kv_mul * HD; hi += 256) {
        const int h = hi / HD, i = hi % HD;
        float o = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) o += red[(w * kv_mul + h) * HD + i];
        if (nsplit == 1) {
            out[h * HD + i] = o * (1.0f / st[2 * h + 1]);
        } else {
            float* pp = part + ((int64_t)split * kv_mul + h) * part_stride;
            pp[2 + i] = o;
            if (i == 0) {
                pp[0] = st[2 * h];
                pp[1] = st[2 * h + 1];
            }
        }
    }
}

// Standalone unit: attention_core (attention_core_fast<KVM>, when KVM =
// kv_mul > 0, for units of more than kAttnExactMax positions and for every
// unit of a sequence with several splits), then with several splits the last
// unit to finish (ticket on *cnt) merges the partials into out.
template <int KVM>
__device__ __forceinline__ void attention_unit(const float* __restrict__ q, const float* __restrict__ K,
                                               const float* __restrict__ Vc, int64_t pos_stride, int t0, int t1,
                                               int nsplit, int split, float* __restrict__ out,
                                               float* __restrict__ part, uint32_t* cnt, float scale, int kv_mul,
                                               int tmax, float* sm) {
    constexpr int HD = kAttnHeadDim;
    const int tid = threadIdx.x;
    // The exact (Java-order) path only where its result is the whole answer:
    // one split of at most kAttnExactMax positions.  Several splits are
    // merged anyway, so they take the throughput path.
    if (KVM > 0 && (tmax > kAttnExactMax || nsplit > 1))
        attention_core_fast<(KVM > 0 ? KVM : 1)>(q, K, Vc, pos_stride, t0, t1, nsplit, split, out, part,
                                                 kAttnPartStride, scale, tmax, sm);
    else
        attention_core(q, K, Vc, pos_stride, t0, t1, nsplit, split, out, part, kAttnPartStride, scale, kv_mul, tmax, sm);
    volatile int* flag = reinterpret_cast<volatile int*>(sm + kv_mul * HD + kv_mul * tmax + 2 * kv_mul);
    if (nsplit > 1) {
        __threadfence();
        named_bar_sync(1, 256);
        if (tid == 0) {
            const uint32_t ticket = atomicAdd(cnt, 1u);
            *flag = (ticket == (uint32_t)(nsplit - 1)) ? 1 : 0;
        }
        named_bar_sync(1, 256);
        if (*flag) {
            __threadfence();
            // Loads of 8 splits at a time in flight (the merge is otherwise a
            // chain of dependent L2 round trips); the sums still run in split
            // order.
            constexpr int C = 8;
            for (int hi = tid; hi < kv_mul * HD; hi += 256) {
                const int h = hi / HD, i = hi % HD;
                const float* p0 = part + (int64_t)h * kAttnPartStride;
                const int64_t sstride = (int64_t)kv_mul * kAttnPartStride;
                float M = -INFINITY;
                for (int s0 = 0; s0 < nsplit; s0 += C) {
                    float m[C];
#pragma unroll
                    for (int j = 0; j < C; ++j) m[j] = s0 + j < nsplit ? __ldcg(p0 + (s0 + j) * sstride) : -INFINITY;
#pragma unroll
                    for (int j = 0; j < C; ++j) M = fmaxf(M, m[j]);
                }
                float L = 0.0f, O = 0.0f;
                for (int s0 = 0; s0 < nsplit; s0 += C) {
                    float m[C], l[C], o[C];
#pragma unroll
                    for (int j = 0; j < C; ++j) {
                        if (s0 + j < nsplit) {
                            const float* pp = p0 + (s0 + j) * sstride;
                            m[j] = __ldcg(pp);
                            l[j] = __ldcg(pp + 1);
                            o[j] = __ldcg(pp + 2 + i);
                        }
                    }
#pragma unroll
                    for (int j = 0; j < C; ++j) {
                        if (s0 + j < nsplit) {
                            const float w = exp_via_double(__fsub_rn(m[j], M));
                            L = fmaf(l[j], w, L);
                            O = fmaf(o[j], w, O);
                        }
                    }
                }
                out[h * HD + i] = __fdiv_rn(O, L);
            }
            if (tid == 0) atomicExch(cnt, 0u);
        }
    }
    named_bar_sync(1, 256);
}

}  // namespace lc
