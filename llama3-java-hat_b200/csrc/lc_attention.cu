// lc_attention.cu -- standalone fused GQA decode attention (split-KV).
//
// Grid: batch x n_kv x max_splits CTAs of 256 threads; CTA (b, h, s) is one
// attention unit (lc_attention.cuh).  Units past a sequence's own split count
// return at once.  Partials and completion counters live in caller-provided
// scratch; the counters are cleared on the stream before each launch.
#include "lc_attention.cuh"
#include "lc_internal.h"

namespace lc {

constexpr int kAttnTmax = 1024;  // positions per split at most

AttnPlan plan_attention(int batch, int n_heads, int n_kv, int head_dim, int max_len, int num_sms) {
    AttnPlan p;
    p.batch = batch;
    p.n_heads = n_heads;
    p.n_kv = n_kv;
    p.head_dim = head_dim;
    // Aim for about two units per SM; each split at least 64 positions.
    long long pairs = (long long)batch * n_kv;
    long long want = (2LL * num_sms + pairs - 1) / pairs;
    if (want < 1) want = 1;
    long long T = (max_len + want - 1) / want;
    if (T < 64) T = 64;
    if (T > kAttnTmax) T = kAttnTmax;
    p.split_len = (int)T;
    p.max_splits = (int)((max_len + T - 1) / T);
    if (p.max_splits < 1) p.max_splits = 1;
    return p;
}

size_t attention_scratch_bytes(const AttnPlan& p) {
    const int kv_mul = p.n_heads / p.n_kv;
    size_t parts = (size_t)p.batch * p.n_kv * p.max_splits * kv_mul * kAttnPartStride * sizeof(float);
    size_t cnts = (size_t)p.batch * p.n_kv * sizeof(uint32_t);
    return ((parts + 255) / 256) * 256 + cnts;
}

template <int KVM>
__global__ void __launch_bounds__(256) attention_decode_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                               const float* __restrict__ v, float* __restrict__ out,
                                                               const int32_t* __restrict__ seq_len, int n_heads,
                                                               int n_kv, int64_t seq_stride, int64_t head_stride,
                                                               int64_t pos_stride, int split_len, int max_splits,
                                                               float* part, uint32_t* cnt, float scale) {
    extern __shared__ float sm[];
    griddep_launch();
    griddep_wait();
    const int s = blockIdx.x % max_splits;
    const int h = (blockIdx.x / max_splits) % n_kv;
    const int b = blockIdx.x / (max_splits * n_kv);
    const int kv_mul = n_heads / n_kv;
    const int len = seq_len[b];
    const int nsplit = (len + split_len - 1) / split_len;
    float* o = out + ((int64_t)b * n_heads + (int64_t)h * kv_mul) * kAttnHeadDim;
    if (len <= 0) {
        if (s == 0)
            for (int i = threadIdx.x; i < kv_mul * kAttnHeadDim; i += 256) o[i] = 0.0f;
        return;
    }
    if (s >= nsplit) return;
    const int t0 = s * split_len;
    const int t1 = min(len, t0 + split_len);
    const float* qh = q + ((int64_t)b * n_heads + (int64_t)h * kv_mul) * kAttnHeadDim;
    const float* kb = k + (int64_t)b * seq_stride + (int64_t)h * head_stride;
    const float* vb = v + (int64_t)b * seq_stride + (int64_t)h * head_stride;
    float* pb = part + ((int64_t)b * n_kv + h) * max_splits * kv_mul * kAttnPartStride;
    attention_unit<KVM>(qh, kb, vb, pos_stride, t0, t1, nsplit, s, o, pb, cnt + (int64_t)b * n_kv + h, scale, kv_mul,
                   split_len, sm);
}

cudaError_t launch_attention_decode(const AttnPlan& p, const float* q, const float* k, const float* v, float* out,
                                    const int32_t* seq_len, int64_t seq_stride, int64_t head_stride,
                                    int64_t pos_stride, void* scratch, cudaStream_t st, bool pdl) {
    const int kv_mul = p.n_heads / p.n_kv;
    size_t parts = (size_t)p.batch * p.n_kv * p.max_splits * kv_mul * kAttnPartStride * sizeof(float);
    parts = ((parts + 255) / 256) * 256;
    float* part = reinterpret_cast<float*>(scratch);
    uint32_t* cnt = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(scratch) + parts);
    // The merging unit leaves each counter at zero; a PDL launch (graph
    // replays of a prepared plan) relies on that, other launches clear them.
    cudaError_t e = pdl ? cudaSuccess : cudaMemsetAsync(cnt, 0, (size_t)p.batch * p.n_kv * sizeof(uint32_t), st);
    if (e != cudaSuccess) return e;
    const size_t smem = (size_t)attn_unit_smem_floats(kv_mul, p.split_len) * sizeof(float);
    const float scale = 1.0f / (float)sqrt((double)p.head_dim);  // Attention.java:33
    const long long grid = (long long)p.batch * p.n_kv * p.max_splits;
    // The throughput path is compiled for 1, 2, 4 and 8 query heads per kv
    // head (register arrays sized at compile time); other ratios use the
    // exact path at every length.
    auto run = [&](auto kern) -> cudaError_t {
        if (smem > 48 * 1024) {
            cudaError_t a = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (a != cudaSuccess) return a;
        }
        return launch_ex(kern, dim3((unsigned)grid), dim3(256), smem, st, pdl, q, k, v, out, seq_len, p.n_heads, p.n_kv,
                         seq_stride, head_stride, pos_stride, p.split_len, p.max_splits, part, cnt, scale);
    };
    switch (kv_mul) {
        case 1: e = run(attention_decode_kernel<1>); break;
        case 2: e = run(attention_decode_kernel<2>); break;
        case 4: e = run(attention_decode_kernel<4>); break;
        case 8: e = run(attention_decode_kernel<8>); break;
        default: e = run(attention_decode_kernel<0>); break;
    }
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace lc
