// lc_kernels.cu -- standalone sm_100a kernels behind the per-kernel operators
// of the C ABI (the IKernelFactory surface): generic GEMV, RMSNorm, RoPE,
// SiLU / SwiGLU, softmax, attention scores/values, fused GQA split-KV decode
// attention and argmax.
//
// Numerics follow the reference's plain-Java kernels: binary32 arithmetic,
// exp/sin/cos evaluated in double and rounded to float where the Java code
// writes (float)Math.*, explicit round-to-nearest intrinsics (__fmul_rn /
// __fadd_rn) where the Java expression order must not be contracted into an
// FMA.  Reductions run as trees where the reference is sequential; that order
// difference is the only deviation.
#include "lc_internal.h"

namespace lc {

// ------------------------------------------------------------------ GEMV --

// Warp per row, any shape and alignment.  Lane-strided fp32 partial sums then
// a shuffle tree.  Used for shapes the streaming GEMV does not take.
template <typename WT>
__global__ void gemv_generic_kernel(const WT* __restrict__ W, const float* __restrict__ x, float* __restrict__ y,
                                    int rows, int cols) {
    const int lane = threadIdx.x & 31;
    const int warps = (gridDim.x * blockDim.x) >> 5;
    for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
        const WT* w = W + (size_t)r * (size_t)cols;
        float acc = 0.0f;
        for (int c = lane; c < cols; c += 32) {
            float wv;
            if constexpr (sizeof(WT) == 2) wv = __half2float(__ushort_as_half(w[c]));
            else wv = w[c];
            acc = fmaf(wv, x[c], acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) y[r] = acc;
    }
}

void launch_gemv_generic_f16(const uint16_t* W, const float* x, float* y, int rows, int cols, cudaStream_t st) {
    int blocks = (rows + 7) / 8;
    if (blocks > 148 * 16) blocks = 148 * 16;
    gemv_generic_kernel<uint16_t><<<blocks, 256, 0, st>>>(W, x, y, rows, cols);
}

void launch_gemv_generic_f32(const float* W, const float* x, float* y, int rows, int cols, cudaStream_t st) {
    int blocks = (rows + 7) / 8;
    if (blocks > 148 * 16) blocks = 148 * 16;
    gemv_generic_kernel<float><<<blocks, 256, 0, st>>>(W, x, y, rows, cols);
}

// Batched F16 GEMV on CUDA cores: one warp per (row, group of up to 8
// sequences).  X rows are read through L1; W row re-read once per group.
__global__ void gemv_batched_kernel(const uint16_t* __restrict__ W, const float* __restrict__ X, float* __restrict__ Y,
                                    int rows, int cols, int batch) {
    const int lane = threadIdx.x & 31;
    const int groups = (batch + 7) / 8;
    const long long total = (long long)rows * groups;
    const long long warps = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long t = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < total; t += warps) {
        const int r = (int)(t / groups);
        const int b0 = (int)(t % groups) * 8;
        const int nb = min(8, batch - b0);
        const uint16_t* w = W + (size_t)r * (size_t)cols;
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
        for (int c = lane; c < cols; c += 32) {
            float wv = __half2float(__ushort_as_half(w[c]));
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (j < nb) acc[j] = fmaf(wv, X[(size_t)(b0 + j) * cols + c], acc[j]);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float s = warp_sum(acc[j]);
            if (lane == 0 && j < nb) Y[(size_t)(b0 + j) * rows + r] = s;
        }
    }
}

void launch_gemv_batched_f16(const uint16_t* W, const float* X, float* Y, int rows, int cols, int batch,
                             cudaStream_t st) {
    long long work = (long long)rows * ((batch + 7) / 8);
    long long blocks = (work + 7) / 8;
    if (blocks > 148 * 32) blocks = 148 * 32;
    gemv_batched_kernel<<<(int)blocks, 256, 0, st>>>(W, X, Y, rows, cols, batch);
}

// --------------------------------------------------------------- RMSNorm --

template <int NT>
LC_DEV float block_sum(float v, float* red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[w] = v;
    __syncthreads();
    float s = 0.0f;
    if (threadIdx.x == 0) {
        for (int i = 0; i < NT / 32; ++i) s += red[i];
        red[32] = s;
    }
    __syncthreads();
    s = red[32];
    __syncthreads();
    return s;
}

// One CTA per row: sum of squares (tree), invRms exactly as RMSNorm.java:43,
// then x*invRms*w left to right (RMSNorm.java:48).  In place.
__global__ void rmsnorm_rows_kernel(float* __restrict__ x, const float* __restrict__ w, int width, float eps) {
    griddep_launch();  // programmatic dependent launch: the next kernel may be scheduled now,
    griddep_wait();    // and nothing here is touched before the predecessor has completed
    __shared__ float red[33];
    float* row = x + (size_t)blockIdx.x * (size_t)width;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < width; i += 256) {
        float v = row[i];
        ss = fmaf(v, v, ss);
    }
    ss = block_sum<256>(ss, red);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)width), eps)));
    for (int i = threadIdx.x; i < width; i += 256) row[i] = __fmul_rn(__fmul_rn(row[i], inv), w[i]);
}

void launch_rmsnorm_rows(float* x, const float* w, int rows, int width, float eps, cudaStream_t st) {
    launch_ex(rmsnorm_rows_kernel, dim3(rows), dim3(256), 0, st, true, x, w, width, eps);
}

// ------------------------------------------------------------------ RoPE --

// Thread per (row, head, pair).  freq[] is computed on the host in double
// exactly like RoPE.java:42; the angle is a float product (RoPE.java:43) and
// cos/sin are evaluated in double then rounded (RoPE.java:44-45).
// One CTA per row at a time.  The angle of pair j depends on (pos, j) only,
// so its cos / sin (double, rounded to float: RoPE.java:45-46) are computed
// once per row into shared memory and shared by all heads; the rotation keeps
// the reference's uncontracted expressions, so results stay bit-identical.
__global__ void __launch_bounds__(256) rope_rows_kernel(float* __restrict__ vec, const int32_t* __restrict__ pos,
                                                        int rows, int num_heads, int head_dim, RopeFreq fq) {
    griddep_launch();  // programmatic dependent launch: the next kernel may be scheduled now,
    griddep_wait();    // and nothing here is touched before the predecessor has completed
    __shared__ float2 cs[256];  // (cos, sin) per pair index; head_dim <= 512
    const int half = head_dim >> 1, width = num_heads * head_dim;
    const bool vec4 = (head_dim % 4 == 0) && ((reinterpret_cast<uintptr_t>(vec) & 15) == 0);
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {
        const float p = (float)pos[r];
        for (int j = threadIdx.x; j < half; j += blockDim.x) {
            double sd, cd;
            sincos((double)__fmul_rn(p, fq.f[j]), &sd, &cd);
            cs[j] = make_float2((float)cd, (float)sd);
        }
        __syncthreads();
        float* v = vec + (size_t)r * width;
        if (vec4) {
            for (int q = threadIdx.x; q < width / 4; q += blockDim.x) {
                float4 x = reinterpret_cast<float4*>(v)[q];
                const int j = ((4 * q) % head_dim) >> 1;
                const float2 c0 = cs[j], c1 = cs[j + 1];
                const float4 o = make_float4(__fsub_rn(__fmul_rn(x.x, c0.x), __fmul_rn(x.y, c0.y)),
                                             __fadd_rn(__fmul_rn(x.x, c0.y), __fmul_rn(x.y, c0.x)),
                                             __fsub_rn(__fmul_rn(x.z, c1.x), __fmul_rn(x.w, c1.y)),
                                             __fadd_rn(__fmul_rn(x.z, c1.y), __fmul_rn(x.w, c1.x)));
                reinterpret_cast<float4*>(v)[q] = o;
            }
        } else {
            for (int t = threadIdx.x; t < width / 2; t += blockDim.x) {
                const int j = t % half;
                const float2 c = cs[j];
                const float v0 = v[2 * t], v1 = v[2 * t + 1];
                v[2 * t] = __fsub_rn(__fmul_rn(v0, c.x), __fmul_rn(v1, c.y));
                v[2 * t + 1] = __fadd_rn(__fmul_rn(v0, c.y), __fmul_rn(v1, c.x));
            }
        }
        __syncthreads();  // cs is rewritten for the next row
    }
}

void launch_rope_rows(float* vec, const int32_t* pos, int rows, int num_heads, int head_dim, const RopeFreq& fq,
                      cudaStream_t st) {
    const int blocks = rows < 148 * 8 ? rows : 148 * 8;
    launch_ex(rope_rows_kernel, dim3(blocks < 1 ? 1 : blocks), dim3(256), 0, st, true, vec, pos, rows, num_heads, head_dim, fq);
}

// ----------------------------------------------------------- SiLU/SwiGLU --

__global__ void silu_kernel(float* __restrict__ x, long long n) {
    griddep_launch();  // programmatic dependent launch: the next kernel may be scheduled now,
    griddep_wait();    // and nothing here is touched before the predecessor has completed
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        x[i] = silu_ref(x[i]);
}

// g = silu(g) * u : SiLU.java:36-39 then TransformerBlock.elementWiseMul.
__global__ void swiglu_kernel(float* __restrict__ g, const float* __restrict__ u, long long n) {
    griddep_launch();  // programmatic dependent launch: the next kernel may be scheduled now,
    griddep_wait();    // and nothing here is touched before the predecessor has completed
    const long long stride = (long long)gridDim.x * blockDim.x;
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const bool vec4 = ((reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(u)) & 15) == 0;
    if (vec4) {
        const long long n4 = n >> 2;
        for (long long k = i; k < n4; k += stride) {
            float4 a = reinterpret_cast<float4*>(g)[k];
            const float4 b = __ldg(reinterpret_cast<const float4*>(u) + k);
            a.x = __fmul_rn(silu_ref(a.x), b.x);
            a.y = __fmul_rn(silu_ref(a.y), b.y);
            a.z = __fmul_rn(silu_ref(a.z), b.z);
            a.w = __fmul_rn(silu_ref(a.w), b.w);
            reinterpret_cast<float4*>(g)[k] = a;
        }
        for (long long k = (n4 << 2) + i; k < n; k += stride) g[k] = __fmul_rn(silu_ref(g[k]), u[k]);
    } else {
        for (; i < n; i += stride) g[i] = __fmul_rn(silu_ref(g[i]), u[i]);
    }
}

static int ew_blocks(long long n) {
    long long b = (n + 1023) / 1024;
    if (b > 148 * 8) b = 148 * 8;
    return b < 1 ? 1 : (int)b;
}

void launch_silu(float* x, long long n, cudaStream_t st) { launch_ex(silu_kernel, dim3(ew_blocks(n)), dim3(256), 0, st, true, x, n); }

void launch_swiglu(float* g, const float* u, long long n, cudaStream_t st) {
    launch_ex(swiglu_kernel, dim3(ew_blocks(n)), dim3(256), 0, st, true, g, u, n);
}

// --------------------------------------------------------------- Softmax --

// Softmax.java:28-51 per row: m = max, e_i = exp(x_i - m), sum, inv = 1/sum,
// x_i = e_i * inv.  exp is the precise float expf (within 2 ulp of the
// reference's double exp rounded to float) and the sum is a tree, so results
// match the reference to summation order and those ulps.  The row is read
// once and written once.

// Rows of up to 32 * EPL floats: one warp per row, EPL floats per lane.
template <int EPL>
__global__ void __launch_bounds__(256) softmax_rows_warp_kernel(float* __restrict__ x, int rows, int width) {
    griddep_launch();  // programmatic dependent launch: the next kernel may be scheduled now,
    griddep_wait();    // and nothing here is touched before the predecessor has completed
    const int lane = threadIdx.x & 31;
    const long long r = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (r >= rows) return;
    float* row = x + (size_t)r * (size_t)width;
    float v[EPL];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < EPL; ++k) {
        const int i = lane + 32 * k;
        v[k] = i < width ? row[i] : -INFINITY;
        m = fmaxf(m, v[k]);
    }
    m = warp_max(m);
    float l = 0.0f;
#pragma unroll
    for (int k = 0; k < EPL; ++k) {
        v[k] = (lane + 32 * k < width) ? expf(__fsub_rn(v[k], m)) : 0.0f;
        l += v[k];
    }
    l = warp_sum(l);
    const float inv = __fdiv_rn(1.0f, l);
#pragma unroll
    for (int k = 0; k < EPL; ++k) {
        const int i = lane + 32 * k;
        if (i < width) row[i] = __fmul_rn(v[k], inv);
    }
}

// Rows of up to 256 * EPT floats: one CTA per row, EPT floats per thread.
template <int EPT>
__global__ void __launch_bounds__(256) softmax_rows_kernel(float* __restrict__ x, int width) {
    griddep_launch();  // programmatic dependent launch: the next kernel may be scheduled now,
    griddep_wait();    // and nothing here is touched before the predecessor has completed
    __shared__ float red[8];
    float* row = x + (size_t)blockIdx.x * (size_t)width;
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float v[EPT];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
        const int i = threadIdx.x + k * 256;
        v[k] = i < width ? row[i] : -INFINITY;
        m = fmaxf(m, v[k]);
    }
    m = warp_max(m);
    if (lane == 0) red[w] = m;
    __syncthreads();
    m = red[0];
#pragma unroll
    for (int k = 1; k < 8; ++k) m = fmaxf(m, red[k]);
    float l = 0.0f;
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
        v[k] = (threadIdx.x + k * 256 < width) ? expf(__fsub_rn(v[k], m)) : 0.0f;
        l += v[k];
    }
    l = warp_sum(l);
    __syncthreads();  // red reused
    if (lane == 0) red[w] = l;
    __syncthreads();
    float L = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) L += red[k];
    const float inv = __fdiv_rn(1.0f, L);
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
        const int i = threadIdx.x + k * 256;
        if (i < width) row[i] = __fmul_rn(v[k], inv);
    }
}

// Rows wider than the register budget: max pass, exp-sum pass, write pass.
__global__ void __launch_bounds__(256) softmax_rows_wide_kernel(float* __restrict__ x, int width) {
    griddep_launch();  // programmatic dependent launch: the next kernel may be scheduled now,
    griddep_wait();    // and nothing here is touched before the predecessor has completed
    __shared__ float red[8];
    float* row = x + (size_t)blockIdx.x * (size_t)width;
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float m = -INFINITY;
    for (int i = threadIdx.x; i < width; i += 256) m = fmaxf(m, row[i]);
    m = warp_max(m);
    if (lane == 0) red[w] = m;
    __syncthreads();
    m = red[0];
    for (int k = 1; k < 8; ++k) m = fmaxf(m, red[k]);
    float l = 0.0f;
    for (int i = threadIdx.x; i < width; i += 256) l += expf(__fsub_rn(row[i], m));
    l = warp_sum(l);
    __syncthreads();
    if (lane == 0) red[w] = l;
    __syncthreads();
    float L = 0.0f;
    for (int k = 0; k < 8; ++k) L += red[k];
    const float inv = __fdiv_rn(1.0f, L);
    for (int i = threadIdx.x; i < width; i += 256) row[i] = __fmul_rn(expf(__fsub_rn(row[i], m)), inv);
}

void launch_softmax_rows(float* x, int rows, int width, cudaStream_t st) {
    const unsigned wgrid = (unsigned)((rows + 7) / 8);
    if (width <= 128) launch_ex(softmax_rows_warp_kernel<4>, dim3(wgrid), dim3(256), 0, st, true, x, rows, width);
    else if (width <= 256) launch_ex(softmax_rows_warp_kernel<8>, dim3(wgrid), dim3(256), 0, st, true, x, rows, width);
    else if (width <= 512) launch_ex(softmax_rows_warp_kernel<16>, dim3(wgrid), dim3(256), 0, st, true, x, rows, width);
    else if (width <= 1024) launch_ex(softmax_rows_warp_kernel<32>, dim3(wgrid), dim3(256), 0, st, true, x, rows, width);
    else if (width <= 4096) launch_ex(softmax_rows_kernel<16>, dim3(rows), dim3(256), 0, st, true, x, width);
    else if (width <= 8192) launch_ex(softmax_rows_kernel<32>, dim3(rows), dim3(256), 0, st, true, x, width);
    else launch_ex(softmax_rows_wide_kernel, dim3(rows), dim3(256), 0, st, true, x, width);
}

// ---------------------------------------------- attention scores / values --

// Thread per position: sequential dot product in the reference order, then
// the scale (Attention.java:33-41).  Bit-identical to the Java loop.
__global__ void attn_scores_kernel(const float* __restrict__ q, const float* __restrict__ keys,
                                   float* __restrict__ scores, int seq_len, int head_dim, float scale) {
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < seq_len; t += gridDim.x * blockDim.x) {
        const float* k = keys + (size_t)t * head_dim;
        float sum = 0.0f;
        for (int i = 0; i < head_dim; ++i) sum = __fadd_rn(sum, __fmul_rn(q[i], k[i]));
        scores[t] = __fmul_rn(sum, scale);
    }
}

// Thread per output dimension: sequential sum over positions in the reference
// order (Attention.java:54-60).  Bit-identical to the Java loop.
__global__ void attn_values_kernel(const float* __restrict__ p, const float* __restrict__ values,
                                   float* __restrict__ out, int seq_len, int head_dim) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < head_dim; i += gridDim.x * blockDim.x) {
        float sum = 0.0f;
        for (int t = 0; t < seq_len; ++t) sum = __fadd_rn(sum, __fmul_rn(p[t], values[(size_t)t * head_dim + i]));
        out[i] = sum;
    }
}

void launch_attn_scores(const float* q, const float* keys, float* scores, int seq_len, int head_dim, float scale,
                        cudaStream_t st) {
    int blocks = (seq_len + 255) / 256;
    if (blocks < 1) blocks = 1;
    if (blocks > 148 * 8) blocks = 148 * 8;
    attn_scores_kernel<<<blocks, 256, 0, st>>>(q, keys, scores, seq_len, head_dim, scale);
}

void launch_attn_values(const float* p, const float* values, float* out, int seq_len, int head_dim,
                        cudaStream_t st) {
    int blocks = (head_dim + 63) / 64;
    attn_values_kernel<<<blocks, 64, 0, st>>>(p, values, out, seq_len, head_dim);
}

// ---------------------------------------------------------------- argmax --

// Single CTA: each thread scans its strided indices in increasing order with
// strict '>' (first occurrence), then candidates merge by (value desc, index
// asc).  NaNs never win; values[0] == NaN yields 0 as in the Java loop.
__global__ void argmax_kernel(const float* __restrict__ v, int n, int32_t* __restrict__ out) {
    __shared__ float bv_s[32];
    __shared__ int bi_s[32];
    float bv = -INFINITY;
    int bi = -1;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float x = v[i];
        if (x == x && (bi < 0 || x > bv)) {
            bv = x;
            bi = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
        int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_merge(bv, bi, v2, i2);
    }
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        bv_s[w] = bv;
        bi_s[w] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float B = bv_s[0];
        int I = bi_s[0];
        for (int k = 1; k < (int)(blockDim.x >> 5); ++k) argmax_merge(B, I, bv_s[k], bi_s[k]);
        const float v0 = v[0];
        *out = (v0 != v0 || I < 0) ? 0 : I;
    }
}

void launch_argmax(const float* v, int n, int32_t* out, cudaStream_t st) { argmax_kernel<<<1, 1024, 0, st>>>(v, n, out); }

}  // namespace lc
