// lc_batch.cu -- greedy decode of up to 64 independent sequences in lockstep
// (multi-sequence serving).  The reference serves one sequence per
// LlamaInference (H/LlamaInference.java:173-217); a batch gives every
// sequence exactly that computation, with each weight matrix read once per
// step for all of them.
//
// One step = one position of every sequence:
//   per layer  norm_split(x, attn_norm)  -> QKV GEMM (RoPE; q; K/V cache at pos[s])
//              -> attention units (lc_attention.cuh; positions 0..pos[s])
//              -> split(att) -> O GEMM (+ residual into x)
//              -> norm_split(x, ffn_norm) -> gate/up GEMM (SwiGLU into h)
//              -> split(h)   -> down GEMM (+ residual into x)
//   then       norm_split(x, out_norm) -> lm_head GEMM (logits, argmax key per
//              sequence) -> step_end (next token, position + 1)
// The GEMMs are the tcgen05 kernel of lc_gemm.cu.  The step is captured once
// per batch size as two CUDA graphs (with and without the lm_head, which
// prompt positions before the last do not need) and replayed per position;
// positions and tokens live on the device, so a generate call is one stream
// of graph launches and one read-back at the end.
#include "lc_attention.cuh"
#include "lc_internal.h"
#include "lc_tcgen05.cuh"

namespace lc {
namespace {

constexpr int kNormThreads = 256;

// x[s] = embedding row of the sequence's token at pos[s] when emb != null
// (LlamaInference.java:122-140), then RMSNorm(x[s]) * w (RMSNorm.java:35-50:
// invRms = 1 / sqrt(ss / n + eps), x * invRms * w) split into the GEMM's
// A operand.  best[s] (when given) is cleared for the lm_head that follows.
// Row s of the output reads activation row in_rows[s] (in_rows null: s); the
// embedded token is tok[s * tok_stride + pos[s]] (pos null: + 0).
__global__ void __launch_bounds__(kNormThreads) norm_split_kernel(
    float* __restrict__ x, int dim, const float* __restrict__ w, float eps, const __half* __restrict__ emb,
    const int32_t* __restrict__ tok, int tok_stride, const int32_t* __restrict__ pos,
    const int32_t* __restrict__ in_rows, uint8_t* __restrict__ As, float* __restrict__ unscale,
    unsigned long long* __restrict__ best) {
    extern __shared__ float ys[];  // dim floats
    __shared__ float red[kNormThreads / 32];
    griddep_launch();
    griddep_wait();
    const int s = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float* xs = x + (size_t)(in_rows ? in_rows[s] : s) * dim;
    if (emb) {
        const __half* e = emb + (size_t)tok[(size_t)s * tok_stride + (pos ? pos[s] : 0)] * dim;
        for (int i = tid; i < dim; i += kNormThreads) xs[i] = __half2float(e[i]);
    }
    float ss = 0.0f;
    for (int i = tid; i < dim; i += kNormThreads) ss = fmaf(xs[i], xs[i], ss);
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int k = 0; k < kNormThreads / 32; ++k) tot += red[k];
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)dim), eps)));
    float m = 0.0f;
    for (int i = tid; i < dim; i += kNormThreads) {
        const float y = __fmul_rn(__fmul_rn(xs[i], inv), w[i]);
        ys[i] = y;
        m = fmaxf(m, fabsf(y));
    }
    m = warp_max(m);
    __syncthreads();  // red reused; ys complete
    if (lane == 0) red[warp] = m;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kNormThreads / 32; ++k) m = fmaxf(m, red[k]);
    const int e = split_row_exp(m);
    const float sc = pow2f(e);
    if (tid == 0) {
        unscale[s] = pow2f(-e);
        if (best) best[s] = 0ull;
    }
    for (int o = tid; o < (dim >> 3); o += kNormThreads) {
        float f[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) f[k] = ys[8 * o + k] * sc;
        uint4* d = reinterpret_cast<uint4*>(As + split_offset(s, o, dim));
        split_octet(f, d[0], d[1]);
    }
}

// The argmax of each sequence's logits becomes its next token when the
// position was its last prompt token or a generated one (LlamaInference
// .java:196-205: first maximum; 0 when nothing compares greater, e.g. NaN
// logits); every sequence advances one position.
__global__ void step_end_kernel(int B, int32_t* __restrict__ pos, int32_t* __restrict__ seqlen,
                                int32_t* __restrict__ tok, int tok_stride, const int32_t* __restrict__ n_prompt,
                                const unsigned long long* __restrict__ best, int lm) {
    griddep_launch();
    griddep_wait();
    const int s = threadIdx.x;
    if (s >= B) return;
    const int p = pos[s];
    if (lm && p + 1 >= n_prompt[s]) {
        const unsigned long long k = best[s];
        tok[(size_t)s * tok_stride + p + 1] = k ? argmax_key_index(k) : 0;
    }
    pos[s] = p + 1;
    seqlen[s] = p + 2;
}

// Causal attention of a prompt (prefill): CTA = (sequence, kv head, block
// of kPrefillQBlock query positions).  K rows [0, end of the block) are
// staged in shared memory with a padded stride (lane j reads row j: no bank
// conflicts), V rows unpadded; each warp takes (query position, query head)
// pairs: scores with lanes over key positions, softmax by warp reductions
// (exp in float), values with lanes over dimensions.  Same arithmetic as the
// decode units up to float rounding (Attention.java:32-61, Softmax.java:28-51
// per head, positions 0..t).
constexpr int kPrefillMaxLen = 256;
constexpr int kPrefillQBlock = 64;
constexpr int kKPad = kAttnHeadDim + 1;

// Floats of the padded K rows, rounded up so that V starts 16-byte aligned.
__host__ __device__ inline size_t prefill_k_floats(int rows) { return ((size_t)rows * kKPad + 3) / 4 * 4; }

__host__ __device__ inline size_t prefill_attn_smem(int rows) {
    return (prefill_k_floats(rows) + (size_t)rows * kAttnHeadDim + 8 * kAttnHeadDim) * sizeof(float);
}

__global__ void __launch_bounds__(256) prefill_attention_kernel(const float* __restrict__ q,
                                                                const float* __restrict__ kcache,
                                                                const float* __restrict__ vcache,
                                                                float* __restrict__ att,
                                                                const int32_t* __restrict__ seq_start, int n_heads,
                                                                int n_kv, int nqb, int64_t kv_seq_stride,
                                                                int64_t kv_head_stride, float scale) {
    constexpr int HD = kAttnHeadDim;
    extern __shared__ float smf[];
    griddep_launch();
    griddep_wait();
    const int qb = blockIdx.x % nqb, kvh = (blockIdx.x / nqb) % n_kv, s = blockIdx.x / (nqb * n_kv);
    const int r0 = seq_start[s], P = seq_start[s + 1] - r0;
    const int t0 = qb * kPrefillQBlock;
    if (t0 >= P) return;
    const int t1 = min(P, t0 + kPrefillQBlock);  // queries [t0, t1), keys [0, t1)
    const int kv_mul = n_heads / n_kv, qdim = n_heads * HD;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* Ks = smf;
    float* Vs = Ks + prefill_k_floats(t1);  // 16-byte aligned: float4 stores below
    float* qs = Vs + (size_t)t1 * HD + warp * HD;
    const float* Kb = kcache + (size_t)s * kv_seq_stride + (size_t)kvh * kv_head_stride;
    const float* Vb = vcache + (size_t)s * kv_seq_stride + (size_t)kvh * kv_head_stride;
    for (int i = threadIdx.x; i < t1 * (HD / 4); i += 256) {
        const int t = i / (HD / 4), c = (i % (HD / 4)) * 4;
        const float4 kk = __ldcg(reinterpret_cast<const float4*>(Kb + (size_t)t * HD + c));
        const float4 vv = __ldcg(reinterpret_cast<const float4*>(Vb + (size_t)t * HD + c));
        float* kd = Ks + t * kKPad + c;
        kd[0] = kk.x;
        kd[1] = kk.y;
        kd[2] = kk.z;
        kd[3] = kk.w;
        *reinterpret_cast<float4*>(Vs + t * HD + c) = vv;
    }
    __syncthreads();
    constexpr int MJ = kPrefillMaxLen / 32;
    for (int pr = warp; pr < (t1 - t0) * kv_mul; pr += 8) {
        const int t = t0 + pr / kv_mul, h = kvh * kv_mul + pr % kv_mul;
        const float* qr = q + (size_t)(r0 + t) * qdim + h * HD;
        qs[2 * lane] = __ldcg(qr + 2 * lane);
        qs[2 * lane + 1] = __ldcg(qr + 2 * lane + 1);
        __syncwarp();
        float sc[MJ];
        float mx = -INFINITY;
#pragma unroll
        for (int m = 0; m < MJ; ++m) {
            const int j = lane + 32 * m;
            sc[m] = -INFINITY;
            if (32 * m <= t && j <= t) {
                const float* kr = Ks + j * kKPad;
                float d = 0.0f;
#pragma unroll 16
                for (int i = 0; i < HD; ++i) d = fmaf(qs[i], kr[i], d);
                sc[m] = d * scale;
                mx = fmaxf(mx, sc[m]);
            }
        }
        mx = warp_max(mx);
        float l = 0.0f;
#pragma unroll
        for (int m = 0; m < MJ; ++m) {
            const float e = (lane + 32 * m <= t) ? expf(sc[m] - mx) : 0.0f;
            sc[m] = e;
            l += e;
        }
        l = warp_sum(l);
        float2 o = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int m = 0; m < MJ; ++m) {
            if (32 * m <= t) {
                const int jn = min(32, t + 1 - 32 * m);
                for (int jj = 0; jj < jn; ++jj) {
                    const float e = __shfl_sync(0xffffffffu, sc[m], jj);
                    const float2 v = *reinterpret_cast<const float2*>(Vs + (32 * m + jj) * HD + 2 * lane);
                    o.x = fmaf(e, v.x, o.x);
                    o.y = fmaf(e, v.y, o.y);
                }
            }
        }
        const float inv = 1.0f / l;
        *reinterpret_cast<float2*>(att + (size_t)(r0 + t) * qdim + h * HD + 2 * lane) = make_float2(o.x * inv, o.y * inv);
        __syncwarp();  // qs reused
    }
}

enum { kJobQKV = 0, kJobO = 1, kJobGU = 2, kJobDN = 3 };

}  // namespace

struct BatchEngine {
    BatchModel m;
    int max_batch = 0, sms = 0;
    cudaStream_t st = nullptr;
    int* err = nullptr;
    int tok_stride = 0, ldl = 0, kmax = 0;
    float *x = nullptr, *q = nullptr, *att = nullptr, *h = nullptr, *logits = nullptr, *unscale = nullptr;
    float *kcache = nullptr, *vcache = nullptr, *rope = nullptr, *part = nullptr;
    uint8_t* As = nullptr;
    unsigned long long* best = nullptr;
    int32_t *pos = nullptr, *seqlen = nullptr, *tok = nullptr, *nprompt = nullptr;
    size_t part_bytes = 0, attn_bytes = 0;
    void* attn_scratch = nullptr;
    // per batch size: GEMM plans, tensor maps, graphs
    int gB = 0;
    AttnPlan aplan;
    std::vector<GemmParams> gp;  // 4 per layer, then the lm_head
    std::vector<CUtensorMap> wmap;
    CUtensorMap amap_dim, amap_qdim, amap_hidden;
    cudaGraphExec_t g_lm = nullptr, g_nolm = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr, ev2 = nullptr;
    float total_ms = 0.0f, decode_ms = 0.0f;
    int steps_run = 0;
    bool used_prefill = false;
    // prefill: one row per prompt token of a call
    int pcap = 0;
    float *px = nullptr, *pq = nullptr, *patt = nullptr, *ph = nullptr, *punscale = nullptr;
    uint8_t* pAs = nullptr;
    int32_t *prow = nullptr;  // [4][pcap]: token, position, sequence of each row; then seq_start[n + 1], last row[n]
    std::vector<CUtensorMap> pwmap;  // weight maps of the prefill products (N blocks of 256 rows)
    bool pattn_ready = false;
};

namespace {

template <class T>
cudaError_t dalloc(T** p, size_t n) {
    return cudaMalloc(reinterpret_cast<void**>(p), (n ? n : 1) * sizeof(T));
}

size_t kv_floats_per_seq(const BatchModel& m) {
    return (size_t)m.n_layers * m.n_kv * m.max_seq * m.head_dim;
}

cudaError_t enqueue_step(BatchEngine* e, int B, bool lm) {
    const BatchModel& m = e->m;
    const int qdim = m.n_heads * m.head_dim;
    const size_t layer_kv = (size_t)m.n_kv * m.max_seq * m.head_dim;
    const int64_t seq_stride = (int64_t)kv_floats_per_seq(m), head_stride = (int64_t)m.max_seq * m.head_dim;
    cudaError_t ce = cudaSuccess;
    // Every launch of the step is a programmatic dependent of the one before
    // (each kernel waits for its predecessor before touching its results).
    constexpr bool pdl = true;
    auto norm = [&](const float* w, const __half* emb, unsigned long long* best) {
        return launch_ex(norm_split_kernel, dim3(B), dim3(kNormThreads), (size_t)m.dim * 4, e->st, pdl, e->x, m.dim,
                         w, m.eps, emb, (const int32_t*)e->tok, e->tok_stride, (const int32_t*)e->pos,
                         (const int32_t*)nullptr, e->As, e->unscale, best);
    };
    for (int l = 0; l < m.n_layers && ce == cudaSuccess; ++l) {
        const LayerW& L = m.layers[l];
        const int j = 4 * l;
        ce = norm(L.attn_norm, l == 0 ? m.tok_emb : nullptr, nullptr);
        if (ce == cudaSuccess) ce = launch_gemm(e->gp[j + kJobQKV], e->wmap[j + kJobQKV], e->amap_dim, e->sms, e->st, pdl);
        if (ce == cudaSuccess)
            ce = launch_attention_decode(e->aplan, e->q, e->kcache + l * layer_kv, e->vcache + l * layer_kv, e->att,
                                         e->seqlen, seq_stride, head_stride, m.head_dim, e->attn_scratch, e->st, pdl);
        if (ce == cudaSuccess) ce = launch_gemm_split(e->att, qdim, qdim, B, e->As, e->unscale, e->st, pdl);
        if (ce == cudaSuccess) ce = launch_gemm(e->gp[j + kJobO], e->wmap[j + kJobO], e->amap_qdim, e->sms, e->st, pdl);
        if (ce == cudaSuccess) ce = norm(L.ffn_norm, nullptr, nullptr);
        if (ce == cudaSuccess) ce = launch_gemm(e->gp[j + kJobGU], e->wmap[j + kJobGU], e->amap_dim, e->sms, e->st, pdl);
        if (ce == cudaSuccess) ce = launch_gemm_split(e->h, m.hidden, m.hidden, B, e->As, e->unscale, e->st, pdl);
        if (ce == cudaSuccess)
            ce = launch_gemm(e->gp[j + kJobDN], e->wmap[j + kJobDN], e->amap_hidden, e->sms, e->st, pdl);
    }
    const int jl = 4 * m.n_layers;
    if (lm && ce == cudaSuccess) {
        ce = norm(m.out_norm, nullptr, e->best);
        if (ce == cudaSuccess) ce = launch_gemm(e->gp[jl], e->wmap[jl], e->amap_dim, e->sms, e->st, pdl);
    }
    if (ce == cudaSuccess) {
        ce = launch_ex(step_end_kernel, dim3(1), dim3(kGemmMaxB), 0, e->st, pdl, B, e->pos, e->seqlen, e->tok,
                       e->tok_stride, (const int32_t*)e->nprompt, (const unsigned long long*)e->best, lm ? 1 : 0);
    }
    return ce;
}

cudaError_t capture(BatchEngine* e, int B, bool lm, cudaGraphExec_t* out) {
    cudaGraph_t g = nullptr;
    cudaError_t ce = cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal);
    if (ce != cudaSuccess) return ce;
    cudaError_t ce2 = enqueue_step(e, B, lm);
    ce = cudaStreamEndCapture(e->st, &g);
    if (ce2 != cudaSuccess) ce = ce2;
    if (ce == cudaSuccess) ce = cudaGraphInstantiate(out, g, 0);
    if (g) cudaGraphDestroy(g);
    return ce;
}

// Plans, tensor maps, scratch and graphs for batch size B.
cudaError_t prepare(BatchEngine* e, int B) {
    if (e->gB == B) return cudaSuccess;
    if (e->g_lm) cudaGraphExecDestroy(e->g_lm);
    if (e->g_nolm) cudaGraphExecDestroy(e->g_nolm);
    e->g_lm = e->g_nolm = nullptr;
    e->gB = 0;
    const BatchModel& m = e->m;
    const int qdim = m.n_heads * m.head_dim, kvd = m.n_kv * m.head_dim;
    const size_t layer_kv = (size_t)m.n_kv * m.max_seq * m.head_dim;
    GemmParams base;
    memset(&base, 0, sizeof(base));
    base.cbw = m.dim;
    base.B = B;
    base.As = e->As;
    base.unscale = e->unscale;
    base.err = e->err;
    base.timeout_ns = 2000000000ull;
    e->gp.assign(4 * m.n_layers + 1, base);
    size_t part = 0;
    for (int j = 0; j < (int)e->gp.size(); ++j) {
        GemmParams& g = e->gp[j];
        const int l = j / 4, kind = j % 4;
        if (j == 4 * m.n_layers) {
            g.W = m.lm_head;
            g.N = (m.vocab + 15) / 16 * 16;
            g.rows_mem = (m.vocab + 7) / 8 * 8;
            g.K = m.dim;
            g.op = kGemmLogits;
            g.logits = e->logits;
            g.ldl = e->ldl;
            g.n_valid = m.vocab;
            g.best = e->best;
        } else {
            const LayerW& L = m.layers[l];
            if (kind == kJobQKV) {
                g.W = L.wqkv;
                g.N = qdim + 2 * kvd;
                g.K = m.dim;
                g.op = kGemmQKV;
                g.q = e->q;
                g.qdim = qdim;
                g.kvd = kvd;
                g.kcache = e->kcache + l * layer_kv;
                g.vcache = e->vcache + l * layer_kv;
                g.kv_seq_stride = (int64_t)kv_floats_per_seq(m);
                g.kv_head_stride = (int64_t)m.max_seq * m.head_dim;
                g.pos = e->pos;
                g.rope_freq = e->rope;
            } else if (kind == kJobO) {
                g.W = L.wo;
                g.N = m.dim;
                g.K = qdim;
                g.op = kGemmResid;
                g.y = e->x;
                g.ldy = m.dim;
            } else if (kind == kJobGU) {
                g.W = L.wgu;
                g.N = 2 * m.hidden;
                g.K = m.dim;
                g.op = kGemmSwiGLU;
                g.h = e->h;
                g.ldh = m.hidden;
            } else {
                g.W = L.wdown;
                g.N = m.dim;
                g.K = m.hidden;
                g.op = kGemmResid;
                g.y = e->x;
                g.ldy = m.dim;
            }
            g.rows_mem = g.N;
        }
        if (!gemm_plan(&g, e->sms)) return cudaErrorInvalidValue;
        part = std::max(part, gemm_part_bytes(g));
    }
    cudaError_t ce = cudaSuccess;
    if (part > e->part_bytes) {
        if (e->part) cudaFree(e->part);
        e->part = nullptr;
        e->part_bytes = 0;
        ce = cudaMalloc(&e->part, part);
        if (ce != cudaSuccess) return ce;
        e->part_bytes = part;
    }
    e->aplan = plan_attention(B, m.n_heads, m.n_kv, m.head_dim, m.max_seq, e->sms);
    const size_t ab = attention_scratch_bytes(e->aplan);
    if (ab > e->attn_bytes) {
        if (e->attn_scratch) cudaFree(e->attn_scratch);
        e->attn_scratch = nullptr;
        e->attn_bytes = 0;
        ce = cudaMalloc(&e->attn_scratch, ab);
        if (ce != cudaSuccess) return ce;
        e->attn_bytes = ab;
    }
    // The graph's attention launches rely on zero completion counters (the
    // merging unit leaves them at zero).
    ce = cudaMemset(e->attn_scratch, 0, e->attn_bytes);
    if (ce != cudaSuccess) return ce;
    e->wmap.resize(e->gp.size());
    for (size_t j = 0; j < e->gp.size(); ++j) {
        e->gp[j].part = e->part;
        ce = gemm_make_wmap(&e->wmap[j], e->gp[j]);
        if (ce != cudaSuccess) return ce;
    }
    GemmParams a = base;
    a.K = m.dim;
    if ((ce = gemm_make_amap(&e->amap_dim, a)) != cudaSuccess) return ce;
    a.K = qdim;
    if ((ce = gemm_make_amap(&e->amap_qdim, a)) != cudaSuccess) return ce;
    a.K = m.hidden;
    if ((ce = gemm_make_amap(&e->amap_hidden, a)) != cudaSuccess) return ce;
    if ((ce = gemm_prepare()) != cudaSuccess) return ce;
    if ((ce = capture(e, B, true, &e->g_lm)) != cudaSuccess) return ce;
    if ((ce = capture(e, B, false, &e->g_nolm)) != cudaSuccess) return ce;
    e->gB = B;
    return cudaSuccess;
}

}  // namespace

bool batch_supported(const BatchModel& m, const char** why) {
    const int qdim = m.n_heads * m.head_dim;
    if (m.head_dim != kGemmHeadDim || m.head_dim != kAttnHeadDim) return *why = "batched decode implements head_dim 64", false;
    if (m.dim % 64 || m.dim > 8192) return *why = "batched decode needs dim % 64 == 0 and dim <= 8192", false;
    if (qdim != m.dim) return *why = "batched decode needs n_heads * head_dim == dim", false;
    if (m.hidden % m.dim) return *why = "batched decode needs hidden to be a multiple of dim", false;
    if (m.n_heads % m.n_kv || m.n_heads / m.n_kv > 8) return *why = "batched decode implements n_heads / n_kv_heads in 1..8", false;
    return true;
}

BatchEngine* batch_create(const BatchModel& m, int max_batch, int num_sms, cudaStream_t st, int* err,
                          cudaError_t* ce_out) {
    BatchEngine* e = new BatchEngine();
    e->m = m;
    e->max_batch = max_batch;
    e->sms = num_sms;
    e->st = st;
    e->err = err;
    e->tok_stride = m.max_seq + 1;
    e->ldl = (m.vocab + 15) / 16 * 16;
    e->kmax = std::max(m.dim, m.hidden);
    const size_t MB = (size_t)max_batch, qdim = (size_t)m.n_heads * m.head_dim;
    cudaError_t ce = cudaSuccess;
    auto ok = [&](cudaError_t c) {
        if (ce == cudaSuccess) ce = c;
    };
    ok(dalloc(&e->x, MB * m.dim));
    ok(dalloc(&e->q, MB * qdim));
    ok(dalloc(&e->att, MB * qdim));
    ok(dalloc(&e->h, MB * m.hidden));
    ok(dalloc(&e->logits, MB * e->ldl));
    ok(dalloc(&e->unscale, MB));
    ok(dalloc(&e->As, gemm_split_bytes(max_batch, e->kmax)));
    ok(dalloc(&e->kcache, MB * kv_floats_per_seq(m)));
    ok(dalloc(&e->vcache, MB * kv_floats_per_seq(m)));
    ok(dalloc(&e->rope, (size_t)m.head_dim / 2));
    ok(dalloc(&e->best, MB));
    ok(dalloc(&e->pos, MB));
    ok(dalloc(&e->seqlen, MB));
    ok(dalloc(&e->nprompt, MB));
    ok(dalloc(&e->tok, MB * e->tok_stride));
    if (ce == cudaSuccess) ce = cudaMemcpy(e->rope, m.rope.f, (size_t)m.head_dim / 2 * 4, cudaMemcpyHostToDevice);
    // Rows of the pre-split operand past the batch are read by the MMA (and
    // ignored): start them as zeros.
    if (ce == cudaSuccess) ce = cudaMemset(e->As, 0, gemm_split_bytes(max_batch, e->kmax));
    if (ce == cudaSuccess) ce = cudaEventCreate(&e->ev0);
    if (ce == cudaSuccess) ce = cudaEventCreate(&e->ev1);
    if (ce == cudaSuccess) ce = cudaEventCreate(&e->ev2);
    if (ce != cudaSuccess) {
        batch_destroy(e);
        *ce_out = ce;
        return nullptr;
    }
    *ce_out = cudaSuccess;
    return e;
}

void batch_destroy(BatchEngine* e) {
    if (!e) return;
    if (e->st) cudaStreamSynchronize(e->st);
    if (e->g_lm) cudaGraphExecDestroy(e->g_lm);
    if (e->g_nolm) cudaGraphExecDestroy(e->g_nolm);
    void* bufs[] = {e->x,    e->q,      e->att,   e->h,      e->logits,   e->unscale, e->As,  e->kcache,
                    e->vcache, e->rope, e->best,  e->pos,    e->seqlen,   e->nprompt, e->tok, e->part,
                    e->attn_scratch, e->px, e->pq, e->patt, e->ph, e->punscale, e->pAs, e->prow};
    for (void* b : bufs)
        if (b) cudaFree(b);
    if (e->ev0) cudaEventDestroy(e->ev0);
    if (e->ev1) cudaEventDestroy(e->ev1);
    if (e->ev2) cudaEventDestroy(e->ev2);
    delete e;
}

int batch_max(const BatchEngine* e) { return e->max_batch; }
int batch_tok_stride(const BatchEngine* e) { return e->tok_stride; }

namespace {

// The prompts of a call as one row set: every prompt token is a row of the
// M-tiled products (the weights are read once per 64 rows instead of once
// per position), the causal attention runs per (sequence, kv head), and the
// lm_head runs once, on each sequence's last prompt token.  Leaves every
// sequence at position len_s with its first generated token in place.
cudaError_t prefill(BatchEngine* e, int n, const std::vector<int32_t>& tok_host, const std::vector<int32_t>& lens) {
    const BatchModel& m = e->m;
    const int qdim = m.n_heads * m.head_dim, kvd = m.n_kv * m.head_dim;
    const size_t layer_kv = (size_t)m.n_kv * m.max_seq * m.head_dim;
    int M = 0, maxlen = 0;
    for (int s = 0; s < n; ++s) {
        M += lens[s];
        maxlen = std::max(maxlen, lens[s]);
    }
    cudaError_t ce = cudaSuccess;
    if (M > e->pcap) {
        void* old[] = {e->px, e->pq, e->patt, e->ph, e->punscale, e->pAs, e->prow};
        for (void* b : old)
            if (b) cudaFree(b);
        e->px = e->pq = e->patt = e->ph = e->punscale = nullptr;
        e->pAs = nullptr;
        e->prow = nullptr;
        e->pcap = 0;
        const int cap = std::max(M, 1024);
        if ((ce = dalloc(&e->px, (size_t)cap * m.dim)) != cudaSuccess) return ce;
        if ((ce = dalloc(&e->pq, (size_t)cap * qdim)) != cudaSuccess) return ce;
        if ((ce = dalloc(&e->patt, (size_t)cap * qdim)) != cudaSuccess) return ce;
        if ((ce = dalloc(&e->ph, (size_t)cap * m.hidden)) != cudaSuccess) return ce;
        if ((ce = dalloc(&e->punscale, (size_t)cap)) != cudaSuccess) return ce;
        if ((ce = dalloc(&e->pAs, gemm_split_bytes(cap, e->kmax))) != cudaSuccess) return ce;
        if ((ce = dalloc(&e->prow, (size_t)3 * cap + 2 * kGemmMaxB + 2)) != cudaSuccess) return ce;
        e->pcap = cap;
    }
    // rows: token, position, sequence; then sequence starts and last rows
    std::vector<int32_t> rows((size_t)3 * e->pcap + 2 * kGemmMaxB + 2, 0);
    int32_t* rtok = rows.data();
    int32_t* rpos = rtok + e->pcap;
    int32_t* rseq = rpos + e->pcap;
    int32_t* sstart = rseq + e->pcap;
    int32_t* slast = sstart + kGemmMaxB + 1;
    std::vector<int32_t> pos_last(n), len1(n);
    for (int s = 0, r = 0; s < n; ++s) {
        sstart[s] = r;
        for (int t = 0; t < lens[s]; ++t, ++r) {
            rtok[r] = tok_host[(size_t)s * e->tok_stride + t];
            rpos[r] = t;
            rseq[r] = s;
        }
        slast[s] = r - 1;
        pos_last[s] = lens[s] - 1;
        len1[s] = lens[s];
        sstart[s + 1] = r;
    }
    const int32_t* d_tok = e->prow;
    const int32_t* d_pos = e->prow + e->pcap;
    const int32_t* d_seq = e->prow + 2 * e->pcap;
    const int32_t* d_start = e->prow + 3 * e->pcap;
    const int32_t* d_last = d_start + kGemmMaxB + 1;
    ce = cudaMemcpyAsync(e->prow, rows.data(), rows.size() * 4, cudaMemcpyHostToDevice, e->st);
    // the lm_head step below advances position len_s - 1 to len_s
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(e->pos, pos_last.data(), (size_t)n * 4, cudaMemcpyHostToDevice, e->st);
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(e->seqlen, len1.data(), (size_t)n * 4, cudaMemcpyHostToDevice, e->st);
    if (ce != cudaSuccess) return ce;

    // products of M rows (row tiles of 64, N blocks of 256, whole K per unit)
    GemmParams base;
    memset(&base, 0, sizeof(base));
    base.cbw = m.dim;
    base.B = M;
    base.As = e->pAs;
    base.unscale = e->punscale;
    base.err = e->err;
    base.timeout_ns = 2000000000ull;
    std::vector<GemmParams> gp(4 * m.n_layers, base);
    for (int j = 0; j < 4 * m.n_layers; ++j) {
        GemmParams& g = gp[j];
        const int l = j / 4, kind = j % 4;
        const LayerW& L = m.layers[l];
        if (kind == kJobQKV) {
            g.W = L.wqkv;
            g.N = qdim + 2 * kvd;
            g.K = m.dim;
            g.op = kGemmQKV;
            g.q = e->pq;
            g.qdim = qdim;
            g.kvd = kvd;
            g.kcache = e->kcache + l * layer_kv;
            g.vcache = e->vcache + l * layer_kv;
            g.kv_seq_stride = (int64_t)kv_floats_per_seq(m);
            g.kv_head_stride = (int64_t)m.max_seq * m.head_dim;
            g.pos = d_pos;
            g.row_seq = d_seq;
            g.rope_freq = e->rope;
        } else if (kind == kJobO) {
            g.W = L.wo;
            g.N = m.dim;
            g.K = qdim;
            g.op = kGemmResid;
            g.y = e->px;
            g.ldy = m.dim;
        } else if (kind == kJobGU) {
            g.W = L.wgu;
            g.N = 2 * m.hidden;
            g.K = m.dim;
            g.op = kGemmSwiGLU;
            g.h = e->ph;
            g.ldh = m.hidden;
        } else {
            g.W = L.wdown;
            g.N = m.dim;
            g.K = m.hidden;
            g.op = kGemmResid;
            g.y = e->px;
            g.ldy = m.dim;
        }
        g.rows_mem = g.N;
        if (!gemm_plan(&g, e->sms) || g.kspl != 1) return cudaErrorInvalidValue;
    }
    if (e->pwmap.size() != gp.size()) {
        e->pwmap.resize(gp.size());
        for (size_t j = 0; j < gp.size(); ++j)
            if ((ce = gemm_make_wmap(&e->pwmap[j], gp[j])) != cudaSuccess) return ce;
    }
    CUtensorMap a_dim, a_qdim, a_hidden;
    GemmParams a = base;
    a.K = m.dim;
    if ((ce = gemm_make_amap(&a_dim, a)) != cudaSuccess) return ce;
    a.K = qdim;
    if ((ce = gemm_make_amap(&a_qdim, a)) != cudaSuccess) return ce;
    a.K = m.hidden;
    if ((ce = gemm_make_amap(&a_hidden, a)) != cudaSuccess) return ce;
    const int nqb = (maxlen + kPrefillQBlock - 1) / kPrefillQBlock;
    const size_t asmem = prefill_attn_smem(std::min(maxlen, nqb * kPrefillQBlock));
    if (!e->pattn_ready) {
        ce = cudaFuncSetAttribute(prefill_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)prefill_attn_smem(kPrefillMaxLen));
        if (ce != cudaSuccess) return ce;
        e->pattn_ready = true;
    }
    const float scale = 1.0f / (float)sqrt((double)m.head_dim);  // Attention.java:33
    auto norm = [&](const float* w, const __half* emb) {
        return launch_ex(norm_split_kernel, dim3(M), dim3(kNormThreads), (size_t)m.dim * 4, e->st, false, e->px,
                         m.dim, w, m.eps, emb, d_tok, 1, (const int32_t*)nullptr, (const int32_t*)nullptr, e->pAs,
                         e->punscale, (unsigned long long*)nullptr);
    };
    for (int l = 0; l < m.n_layers && ce == cudaSuccess; ++l) {
        const LayerW& L = m.layers[l];
        const int j = 4 * l;
        ce = norm(L.attn_norm, l == 0 ? m.tok_emb : nullptr);
        if (ce == cudaSuccess) ce = launch_gemm(gp[j + kJobQKV], e->pwmap[j + kJobQKV], a_dim, e->sms, e->st);
        if (ce == cudaSuccess)
            ce = launch_ex(prefill_attention_kernel, dim3((unsigned)(n * m.n_kv * nqb)), dim3(256), asmem, e->st,
                           false, (const float*)e->pq, (const float*)(e->kcache + l * layer_kv),
                           (const float*)(e->vcache + l * layer_kv), e->patt, d_start, m.n_heads, m.n_kv, nqb,
                           (int64_t)kv_floats_per_seq(m), (int64_t)m.max_seq * m.head_dim, scale);
        if (ce == cudaSuccess) ce = launch_gemm_split(e->patt, qdim, qdim, M, e->pAs, e->punscale, e->st);
        if (ce == cudaSuccess) ce = launch_gemm(gp[j + kJobO], e->pwmap[j + kJobO], a_qdim, e->sms, e->st);
        if (ce == cudaSuccess) ce = norm(L.ffn_norm, nullptr);
        if (ce == cudaSuccess) ce = launch_gemm(gp[j + kJobGU], e->pwmap[j + kJobGU], a_dim, e->sms, e->st);
        if (ce == cudaSuccess) ce = launch_gemm_split(e->ph, m.hidden, m.hidden, M, e->pAs, e->punscale, e->st);
        if (ce == cudaSuccess) ce = launch_gemm(gp[j + kJobDN], e->pwmap[j + kJobDN], a_hidden, e->sms, e->st);
    }
    if (ce != cudaSuccess) return ce;
    // lm_head on the last prompt token of each sequence, then its first token
    const int jl = 4 * m.n_layers;
    ce = launch_ex(norm_split_kernel, dim3(n), dim3(kNormThreads), (size_t)m.dim * 4, e->st, false, e->px, m.dim,
                   m.out_norm, m.eps, (const __half*)nullptr, (const int32_t*)nullptr, 0, (const int32_t*)nullptr,
                   d_last, e->As, e->unscale, e->best);
    if (ce == cudaSuccess) ce = launch_gemm(e->gp[jl], e->wmap[jl], e->amap_dim, e->sms, e->st);
    if (ce == cudaSuccess)
        ce = launch_ex(step_end_kernel, dim3(1), dim3(kGemmMaxB), 0, e->st, false, n, e->pos, e->seqlen, e->tok,
                       e->tok_stride, (const int32_t*)e->nprompt, (const unsigned long long*)e->best, 1);
    return ce;
}

}  // namespace

cudaError_t batch_run(BatchEngine* e, int n, const std::vector<int32_t>& tok_host, const std::vector<int32_t>& lens,
                      int max_new, std::vector<int32_t>* tok_out) {
    cudaError_t ce = prepare(e, n);
    if (ce != cudaSuccess) return ce;
    std::vector<int32_t> zeros(n, 0), ones(n, 1);
    ce = cudaMemcpyAsync(e->tok, tok_host.data(), (size_t)n * e->tok_stride * 4, cudaMemcpyHostToDevice, e->st);
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(e->nprompt, lens.data(), (size_t)n * 4, cudaMemcpyHostToDevice, e->st);
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(e->pos, zeros.data(), (size_t)n * 4, cudaMemcpyHostToDevice, e->st);
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(e->seqlen, ones.data(), (size_t)n * 4, cudaMemcpyHostToDevice, e->st);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(e->st);  // host vectors go out of scope
    if (ce != cudaSuccess) return ce;
    int steps = 0, first_lm = 1 << 30, p_dec = 0, M = 0, maxlen = 0;
    for (int s = 0; s < n; ++s) {
        steps = std::max(steps, lens[s] + max_new - 1);
        first_lm = std::min(first_lm, lens[s] - 1);
        p_dec = std::max(p_dec, lens[s] - 1);
        M += lens[s];
        maxlen = std::max(maxlen, lens[s]);
    }
    // Prompts of more than one row tile (64 tokens) in all, up to
    // kPrefillMaxLen tokens each and kGemmMaxRows in all, run as one prefill;
    // otherwise prompt positions step one at a time.
    e->used_prefill = M > kGemmMaxB && maxlen <= kPrefillMaxLen && M <= kGemmMaxRows;
    ce = cudaEventRecord(e->ev0, e->st);
    if (e->used_prefill) {
        if (ce == cudaSuccess) ce = prefill(e, n, tok_host, lens);
        if (ce == cudaSuccess) ce = cudaEventRecord(e->ev1, e->st);
        for (int k = 0; k + 1 < max_new && ce == cudaSuccess; ++k) ce = cudaGraphLaunch(e->g_lm, e->st);
    } else {
        // the first token comes from position p_dec; the decode phase follows it
        for (int p = 0; p < steps && ce == cudaSuccess; ++p) {
            if (ce == cudaSuccess) ce = cudaGraphLaunch(p >= first_lm ? e->g_lm : e->g_nolm, e->st);
            if (p == p_dec && ce == cudaSuccess) ce = cudaEventRecord(e->ev1, e->st);
        }
    }
    if (ce == cudaSuccess) ce = cudaEventRecord(e->ev2, e->st);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(e->st);
    if (ce != cudaSuccess) return ce;
    cudaEventElapsedTime(&e->total_ms, e->ev0, e->ev2);
    cudaEventElapsedTime(&e->decode_ms, e->ev1, e->ev2);
    e->steps_run = steps;
    tok_out->resize((size_t)n * e->tok_stride);
    return cudaMemcpy(tok_out->data(), e->tok, (size_t)n * e->tok_stride * 4, cudaMemcpyDeviceToHost);
}

void batch_times(const BatchEngine* e, float* total_ms, float* decode_ms, int* steps) {
    *total_ms = e->total_ms;
    *decode_ms = e->decode_ms;
    *steps = e->steps_run;
}

cudaError_t batch_logits(const BatchEngine* e, int s, float* out) {
    return cudaMemcpy(out, e->logits + (size_t)s * e->ldl, (size_t)e->m.vocab * 4, cudaMemcpyDeviceToHost);
}

}  // namespace lc
