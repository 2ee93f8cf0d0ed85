// lc_f32.cu -- decode with fp32 weights: WeightStorageMode.F32
// (H/WeightStorageMode.java; H/LlamaInference.java:102-108 maps every
// projection and the embedding to an F32Array).  One forward of
// LlamaInference.forward (H/LlamaInference.java:117-164) is a sequence of
// launches on the context stream: the embedding row, per layer the
// TransformerBlock.forward steps (H/TransformerBlock.java:130-217) -- RMSNorm,
// the q/k/v GEMV over the stacked [Wq; Wk; Wv], RoPE, the KV-cache write, GQA
// attention, the o GEMV added to the residual, RMSNorm, the stacked gate/up
// GEMV, SwiGLU, the down GEMV added to the residual -- then the final RMSNorm,
// the lm_head GEMV and the greedy argmax into the token list.  The GEMV is
// GEMV.apply(F32Array, ...) (K/GEMV.java:34-43) with a deterministic order:
// a warp per output row, lane partial sums of float4 columns, a shuffle tree.
// Positions and sequence lengths are read from device arrays (pos[i] = i,
// len[i] = i + 1), so the launches need no host data per step.
#include "lc_internal.h"

namespace lc {

namespace {

__global__ void f16_to_f32_kernel(const __half* __restrict__ src, float* __restrict__ dst, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        dst[i] = __half2float(src[i]);
}

// x = embedding row of tokens[pos] (H/LlamaInference.java:133-137); a token
// outside the vocabulary records kDevBadToken and embeds row 0.
__global__ void embed_f32_kernel(const float* __restrict__ emb, const int32_t* __restrict__ tokens, int pos,
                                 int vocab, int dim, float* __restrict__ x, int* err) {
    int t = tokens[pos];
    if (t < 0 || t >= vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicCAS(err, 0, (int)kDevBadToken);
        t = 0;
    }
    const float* row = emb + (size_t)t * dim;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x) x[i] = row[i];
}

constexpr int kGemvThreads = 256;

// y[r] (+)= sum_c W[r][c] * x[c] for rows r of a row-major fp32 matrix; x
// (cols floats, a multiple of 4) staged in shared memory, one warp per row.
__global__ void __launch_bounds__(kGemvThreads) gemv_f32_rows_kernel(const float* __restrict__ W,
                                                                     const float* __restrict__ x, float* y, int rows,
                                                                     int cols, int accumulate) {
    extern __shared__ float4 xs4[];
    const int n4 = cols / 4;
    for (int i = threadIdx.x; i < n4; i += blockDim.x) xs4[i] = reinterpret_cast<const float4*>(x)[i];
    __syncthreads();
    const int lane = threadIdx.x & 31, wpb = blockDim.x / 32;
    for (int r = blockIdx.x * wpb + (threadIdx.x >> 5); r < rows; r += gridDim.x * wpb) {
        const float4* w4 = reinterpret_cast<const float4*>(W + (size_t)r * cols);
        float a0 = 0.f, a1 = 0.f;
        int c = lane;
        for (; c + 32 < n4; c += 64) {
            const float4 u = __ldcs(w4 + c), v = __ldcs(w4 + c + 32), p = xs4[c], q = xs4[c + 32];
            a0 = fmaf(u.x, p.x, fmaf(u.y, p.y, fmaf(u.z, p.z, fmaf(u.w, p.w, a0))));
            a1 = fmaf(v.x, q.x, fmaf(v.y, q.y, fmaf(v.z, q.z, fmaf(v.w, q.w, a1))));
        }
        if (c < n4) {
            const float4 u = __ldcs(w4 + c), p = xs4[c];
            a0 = fmaf(u.x, p.x, fmaf(u.y, p.y, fmaf(u.z, p.z, fmaf(u.w, p.w, a0))));
        }
        float a = warp_sum(a0 + a1);
        if (lane == 0) y[r] = accumulate ? y[r] + a : a;
    }
}

// The rotated k and the v of this position into the head-major caches of one
// layer ([n_kv][max_seq][head_dim]; TransformerBlock.java:158-162).
__global__ void kv_store_f32_kernel(const float* __restrict__ k, const float* __restrict__ v, float* kc, float* vc,
                                    int pos, int kvd, int head_dim, int max_seq) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < kvd; i += gridDim.x * blockDim.x) {
        const size_t o = ((size_t)(i / head_dim) * max_seq + pos) * head_dim + i % head_dim;
        kc[o] = k[i];
        vc[o] = v[i];
    }
}

cudaError_t gemv_f32(const float* W, const float* x, float* y, int rows, int cols, bool accumulate, int num_sms,
                     cudaStream_t st) {
    const int wpb = kGemvThreads / 32;
    int blocks = (rows + wpb - 1) / wpb;
    const int cap = num_sms * 8;
    if (blocks > cap) blocks = cap;
    gemv_f32_rows_kernel<<<blocks, kGemvThreads, (size_t)cols * 4, st>>>(W, x, y, rows, cols, accumulate ? 1 : 0);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_f16_to_f32(const __half* src, float* dst, long long n, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    const long long blocks = (n + 255) / 256;
    f16_to_f32_kernel<<<(int)(blocks < 4096 ? blocks : 4096), 256, 0, st>>>(src, dst, n);
    return cudaGetLastError();
}

bool f32_supported(int dim, int hidden, int qdim, const char** why) {
    if (dim % 4 || hidden % 4 || qdim % 4) return *why = "fp32 weights need dimensions that are multiples of 4", false;
    if (hidden > 16384 || dim > 16384 || qdim > 16384)
        return *why = "fp32 weights implement GEMV inputs of at most 16384 columns", false;
    return true;
}

cudaError_t f32_prepare() {
    return cudaFuncSetAttribute(gemv_f32_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 16384 * 4);
}

cudaError_t f32_forward(const F32Step& f, int pos, bool logits, bool store_token, cudaStream_t st) {
    const int dim = f.dim, hidden = f.hidden, hd = f.head_dim;
    const int qdim = f.n_heads * hd, kvd = f.n_kv * hd;
    float* q = f.qkv;
    float* k = f.qkv + qdim;
    float* v = k + kvd;
    cudaError_t e;
#define F32_CK(x)                        \
    do {                                 \
        if ((e = (x)) != cudaSuccess) return e; \
    } while (0)
    embed_f32_kernel<<<(dim + 255) / 256, 256, 0, st>>>(f.tok_emb, f.tokens, pos, f.vocab, dim, f.x, f.err);
    F32_CK(cudaGetLastError());
    const AttnPlan plan = plan_attention(1, f.n_heads, f.n_kv, hd, pos + 1, f.num_sms);
    if (attention_scratch_bytes(plan) > f.attn_scratch_bytes) return cudaErrorInvalidValue;
    for (int l = 0; l < f.n_layers; ++l) {
        const F32Layer& L = f.layers[l];
        float* kc = f.kcache + (size_t)l * f.n_kv * f.max_seq * hd;
        float* vc = f.vcache + (size_t)l * f.n_kv * f.max_seq * hd;
        F32_CK(cudaMemcpyAsync(f.xb, f.x, (size_t)dim * 4, cudaMemcpyDeviceToDevice, st));   // :139-142
        launch_rmsnorm_rows(f.xb, L.attn_norm, 1, dim, f.eps, st);
        F32_CK(gemv_f32(L.wqkv, f.xb, f.qkv, qdim + 2 * kvd, dim, false, f.num_sms, st));       // :145-147
        launch_rope_rows(q, f.posv + pos, 1, f.n_heads, hd, f.rope, st);  // :150
        launch_rope_rows(k, f.posv + pos, 1, f.n_kv, hd, f.rope, st);     // :151
        kv_store_f32_kernel<<<(kvd + 255) / 256, 256, 0, st>>>(k, v, kc, vc, pos, kvd, hd, f.max_seq);
        F32_CK(cudaGetLastError());
        F32_CK(launch_attention_decode(plan, q, kc, vc, f.att, f.lenv + pos, 0, (int64_t)f.max_seq * hd, hd,
                                       f.attn_scratch, st));                                     // :164-192
        F32_CK(gemv_f32(L.wo, f.att, f.x, dim, qdim, true, f.num_sms, st));                     // :195-198
        F32_CK(cudaMemcpyAsync(f.xb, f.x, (size_t)dim * 4, cudaMemcpyDeviceToDevice, st));       // :201-204
        launch_rmsnorm_rows(f.xb, L.ffn_norm, 1, dim, f.eps, st);
        F32_CK(gemv_f32(L.wgu, f.xb, f.gu, 2 * hidden, dim, false, f.num_sms, st));            // :207-208
        launch_swiglu(f.gu, f.gu + hidden, hidden, st);  // :209-210
        F32_CK(gemv_f32(L.wdown, f.gu, f.x, dim, hidden, true, f.num_sms, st));                 // :211-216
    }
    if (!logits) return cudaSuccess;
    F32_CK(cudaMemcpyAsync(f.xb, f.x, (size_t)dim * 4, cudaMemcpyDeviceToDevice, st));
    launch_rmsnorm_rows(f.xb, f.out_norm, 1, dim, f.eps, st);  // :148
    F32_CK(gemv_f32(f.lm, f.xb, f.logits, f.vocab, dim, false, f.num_sms, st));                 // :151-156
    if (store_token) launch_argmax(f.logits, f.vocab, f.tokens + pos + 1, st);                  // :196-205
#undef F32_CK
    return cudaGetLastError();
}

}  // namespace lc
