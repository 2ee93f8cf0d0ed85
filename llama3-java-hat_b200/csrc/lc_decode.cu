// lc_decode.cu -- the fused decode step: LlamaInference.forward
// (LlamaInference.java:117-164) with all 16 TransformerBlock.forward calls
// (TransformerBlock.java:130-217), the final RMSNorm, the lm_head GEMV and the
// greedy argmax, for `nsteps` consecutive positions, in ONE cooperative
// persistent launch (one CTA per SM).
//
// Phases of one position, separated by grid barriers:
//   QKV   rmsnorm(x, attn_norm) -> [Wq;Wk;Wv] GEMV -> RoPE(q,k) -> q buffer, KV-cache write
//   ATTN  GQA split-KV attention over positions 0..pos -> att
//   O     Wo GEMV + residual -> x
//   GU    rmsnorm(x, ffn_norm) -> [gate|up] GEMV -> silu(gate)*up -> h
//   DOWN  Wdown GEMV + residual -> x
//   LM    rmsnorm(x, out_norm) -> lm_head GEMV -> logits, per-CTA argmax
//   then every CTA merges the per-CTA argmax candidates into the next token.
//
// Weight bytes are >99.8% of the traffic.  Each CTA's producer thread streams
// the CTA's share of every weight matrix, in schedule order, into a 6-stage
// shared-memory ring with 1-D bulk copies; it only waits for free stages,
// never for a grid barrier, so HBM keeps streaming while the consumer warps
// synchronise.  Activations (x, q, att, h) are a few KB, read from L2 with
// .cg loads after each barrier; every warp recomputes the RMSNorm statistics
// of the full vector itself (bit-identical everywhere), so no barrier is
// spent on normalisation.
//
// Every wait is bounded (mbarrier phases, grid barrier): on timeout the
// kernel records an error code in p.err, all CTAs leave, the producer drains
// its in-flight copies, and the host reports LC_ERR_TIMEOUT.
#include "lc_attention.cuh"
#include "lc_internal.h"
#include "lc_stream.cuh"

namespace lc {

constexpr int kDecodeAttnTmax = 512;  // positions per attention split

__host__ __device__ inline bool lm_needed(const DecodeParams& p, int pos) {
    return !(p.skip_prefill_logits && pos + 1 < p.n_prompt);
}

// Split length for the attention phase at sequence length `seq`: about one
// unit per CTA, at least 64 positions, at most kDecodeAttnTmax.
__host__ __device__ inline int attn_split_len(int seq, int G, int n_kv) {
    int per = G / n_kv;
    if (per < 1) per = 1;
    int T = (seq + per - 1) / per;
    if (T < 64) T = 64;
    if (T > kDecodeAttnTmax) T = kDecodeAttnTmax;
    return T;
}

struct Shared {
    int stop;      // consumers -> producer: leave
    int flag;      // grid-barrier result broadcast
    int next;      // argmax broadcast
    int pad;
    float bv[kConsumerWarps];
    int bi[kConsumerWarps];
};

__device__ __forceinline__ bool grid_sync(const DecodeParams& p, uint32_t& target, Shared* sh) {
    named_bar_sync(kConsumerBar, kConsumerThreads);
    if (threadIdx.x == 0) {
        target += gridDim.x;
        __threadfence();
        atomicAdd(p.bar, 1u);
        int ok = 1;
        if (ld_acquire_gpu(p.bar) < target) {
            const uint64_t deadline = globaltimer_ns() + p.timeout_ns;
            for (uint32_t k = 1;; ++k) {
                if (ld_acquire_gpu(p.bar) >= target) break;
                if ((k & 15u) == 0u) {
                    if (*reinterpret_cast<volatile int*>(p.err) != 0) {
                        ok = 0;
                        break;
                    }
                    if (globaltimer_ns() > deadline) {
                        atomicCAS(p.err, 0, (int)kDevTimeoutGrid);
                        ok = 0;
                        break;
                    }
                }
                __nanosleep(32);
            }
        }
        __threadfence();
        *reinterpret_cast<volatile int*>(&sh->flag) = ok;
    }
    named_bar_sync(kConsumerBar, kConsumerThreads);
    return *reinterpret_cast<volatile int*>(&sh->flag) != 0;
}

// RoPE of one interleaved pair (RoPE.java:42-49) at position pos.
__device__ __forceinline__ void rope_pair(float& v0, float& v1, int pos, float freq) {
    const float val = __fmul_rn((float)pos, freq);
    double s, c;
    sincos((double)val, &s, &c);
    const float cf = (float)c, sf = (float)s;
    const float a = v0, b = v1;
    v0 = __fsub_rn(__fmul_rn(a, cf), __fmul_rn(b, sf));
    v1 = __fadd_rn(__fmul_rn(a, sf), __fmul_rn(b, cf));
}

// ------------------------------------------------------------- producer --

template <int V>
__device__ void run_producer(const DecodeParams& p, const Ring& ring, volatile int* stop) {
    constexpr int S = Geo<V>::kSegCols;
    const int G = gridDim.x, cta = blockIdx.x;
    const int qdim = p.n_heads * p.head_dim, kv_dim = p.n_kv * p.head_dim;
    const int qkv_rows = qdim + 2 * kv_dim;
    const int nseg_dim = p.dim / S, nseg_o = qdim / S, nseg_hid = p.hidden / S;
    Producer pr;
    pr.policy = l2_policy_evict_first();
    Rotation rot;
    volatile int* err = p.err;
    auto job = [&](const __half* W, int rows, int cols, int nseg) -> bool {
        int r0, r1;
        job_range(rows, 2, G, rot.rank(cta, G), &r0, &r1);
        rot.advance(rows, 2, G);
        return pr.stream_rows<V>(ring, W, cols, nseg, r0, r1, err, stop, p.timeout_ns);
    };
    bool go = true;
    for (int s = 0; s < p.nsteps && go; ++s) {
        const int pos = p.pos0 + s;
        for (int l = 0; l < p.n_layers && go; ++l) {
            const LayerW L = p.layers[l];
            go = job(L.wqkv, qkv_rows, p.dim, nseg_dim) && job(L.wo, p.dim, qdim, nseg_o) &&
                 job(L.wgu, 2 * p.hidden, p.dim, nseg_dim) && job(L.wdown, p.dim, p.hidden, nseg_hid);
        }
        if (go && lm_needed(p, pos)) go = job(p.lm_head, p.vocab, p.dim, nseg_dim);
    }
    pr.drain(ring, err);
}

// ------------------------------------------------------------- consumer --

// Control flow leaves the step loop only on a grid_sync() result, which is
// uniform across the CTA: a consumer warp whose stage wait timed out keeps
// walking the same named barriers as its siblings (its partial sums are
// garbage, the error word is set), so no warp is ever stranded at bar.sync.
template <int V>
__device__ void run_consumer(const DecodeParams& p, const Ring& ring, float* ys, Shared* sh) {
    constexpr int S = Geo<V>::kSegCols;
    const int G = gridDim.x, cta = blockIdx.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hd = p.head_dim;
    const int qdim = p.n_heads * hd, kv_dim = p.n_kv * hd, kv_mul = p.n_heads / p.n_kv;
    const int qkv_rows = qdim + 2 * kv_dim;
    const int nseg_dim = p.dim / S, nseg_o = qdim / S, nseg_hid = p.hidden / S;
    Consumer cs;
    Rotation rot;
    uint32_t target = 0;
    bool ok = true;
    int next = 0;
    int steps_done = 0;
    float xr[8 * V];

    for (int s = 0; s < p.nsteps && ok; ++s) {
        const int pos = p.pos0 + s;
        const int token = (s == 0 || pos < p.n_prompt) ? __ldcg(p.tokens + pos) : next;
        if (token < 0 || token >= p.vocab) {
            if (cta == 0 && tid == 0) atomicCAS(p.err, 0, (int)kDevBadToken);
            ok = false;
            break;
        }
        const __half* emb = p.tok_emb + (size_t)token * (size_t)p.dim;
        const int seq = pos + 1;

        for (int l = 0; l < p.n_layers && ok; ++l) {
            const LayerW L = p.layers[l];
            int r0, r1;

            // ---------------- QKV: TransformerBlock.java:139-162 ----------------
            if (l == 0) load_slice_f16<V>(emb, xr);
            else load_slice_f32<V>(p.x, xr);
            rmsnorm_slice<V>(xr, L.attn_norm, p.dim, p.eps);
            job_range(qkv_rows, 2, G, rot.rank(cta, G), &r0, &r1);
            rot.advance(qkv_rows, 2, G);
            cs.consume_rows<V>(ring, nseg_dim, r0, r1, xr, ys, p.err, p.timeout_ns);
            named_bar_sync(kConsumerBar, kConsumerThreads);
            for (int pr = tid; pr < (r1 - r0) / 2; pr += kConsumerThreads) {
                const int r = r0 + 2 * pr;
                float y0 = ys[2 * pr], y1 = ys[2 * pr + 1];
                if (r < qdim) {
                    rope_pair(y0, y1, pos, p.rope.f[(r % hd) >> 1]);
                    *reinterpret_cast<float2*>(p.qbuf + r) = make_float2(y0, y1);
                } else if (r < qdim + kv_dim) {
                    const int kr = r - qdim, kvh = kr / hd, i = kr % hd;
                    rope_pair(y0, y1, pos, p.rope.f[i >> 1]);
                    float* dst = p.kcache + (((size_t)l * p.n_kv + kvh) * p.max_seq + pos) * hd + i;
                    *reinterpret_cast<float2*>(dst) = make_float2(y0, y1);
                } else {
                    const int vr = r - qdim - kv_dim, kvh = vr / hd, i = vr % hd;
                    float* dst = p.vcache + (((size_t)l * p.n_kv + kvh) * p.max_seq + pos) * hd + i;
                    *reinterpret_cast<float2*>(dst) = make_float2(y0, y1);
                }
            }
            if (!(ok = grid_sync(p, target, sh))) break;

            // ---------------- ATTN: TransformerBlock.java:164-192 ----------------
            {
                const int T = attn_split_len(seq, G, p.n_kv);
                const int nsplit = (seq + T - 1) / T;
                const int units = p.n_kv * nsplit;
                for (int u = cta; u < units; u += G) {
                    const int kvh = u / nsplit, sp = u % nsplit;
                    const int t0 = sp * T, t1 = min(seq, t0 + T);
                    const size_t kvbase = ((size_t)l * p.n_kv + kvh) * p.max_seq * hd;
                    attention_unit(p.qbuf + (size_t)kvh * kv_mul * hd, p.kcache + kvbase, p.vcache + kvbase, hd, t0,
                                   t1, nsplit, sp, p.att + (size_t)kvh * kv_mul * hd,
                                   p.attn_part + (size_t)kvh * p.attn_max_splits * kv_mul * kAttnPartStride,
                                   p.attn_cnt + kvh, p.attn_scale, kv_mul, T, ys);
                }
            }
            if (!(ok = grid_sync(p, target, sh))) break;

            // ---------------- O + residual: TransformerBlock.java:195-198 ----------------
            load_slice_f32<V>(p.att + (warp % nseg_o) * S, xr);
            job_range(p.dim, 2, G, rot.rank(cta, G), &r0, &r1);
            rot.advance(p.dim, 2, G);
            cs.consume_rows<V>(ring, nseg_o, r0, r1, xr, ys, p.err, p.timeout_ns);
            named_bar_sync(kConsumerBar, kConsumerThreads);
            for (int k = tid; k < r1 - r0; k += kConsumerThreads) {
                const int r = r0 + k;
                float y = ys[k * nseg_o];
                for (int g = 1; g < nseg_o; ++g) y += ys[k * nseg_o + g];
                const float res = (l == 0) ? __half2float(emb[r]) : __ldcg(p.x + r);
                p.x[r] = __fadd_rn(y, res);
            }
            if (!(ok = grid_sync(p, target, sh))) break;

            // ---------------- GU + SwiGLU: TransformerBlock.java:201-210 ----------------
            load_slice_f32<V>(p.x, xr);
            rmsnorm_slice<V>(xr, L.ffn_norm, p.dim, p.eps);
            job_range(2 * p.hidden, 2, G, rot.rank(cta, G), &r0, &r1);
            rot.advance(2 * p.hidden, 2, G);
            cs.consume_rows<V>(ring, nseg_dim, r0, r1, xr, ys, p.err, p.timeout_ns);
            named_bar_sync(kConsumerBar, kConsumerThreads);
            for (int k = tid; k < (r1 - r0) / 2; k += kConsumerThreads)
                p.hbuf[r0 / 2 + k] = __fmul_rn(silu_ref(ys[2 * k]), ys[2 * k + 1]);
            if (!(ok = grid_sync(p, target, sh))) break;

            // ---------------- DOWN + residual: TransformerBlock.java:211-216 ----------------
            load_slice_f32<V>(p.hbuf + (warp % nseg_hid) * S, xr);
            job_range(p.dim, 2, G, rot.rank(cta, G), &r0, &r1);
            rot.advance(p.dim, 2, G);
            cs.consume_rows<V>(ring, nseg_hid, r0, r1, xr, ys, p.err, p.timeout_ns);
            named_bar_sync(kConsumerBar, kConsumerThreads);
            for (int k = tid; k < r1 - r0; k += kConsumerThreads) {
                const int r = r0 + k;
                float y = ys[k * nseg_hid];
                for (int g = 1; g < nseg_hid; ++g) y += ys[k * nseg_hid + g];
                p.x[r] = __fadd_rn(__ldcg(p.x + r), y);
            }
            if (!(ok = grid_sync(p, target, sh))) break;
        }
        if (!ok) break;

        bool stop_now = false;
        if (lm_needed(p, pos)) {
            // ---------------- LM head: LlamaInference.java:148-156 ----------------
            int r0, r1;
            load_slice_f32<V>(p.x, xr);
            rmsnorm_slice<V>(xr, p.out_norm, p.dim, p.eps);
            job_range(p.vocab, 2, G, rot.rank(cta, G), &r0, &r1);
            rot.advance(p.vocab, 2, G);
            cs.consume_rows<V>(ring, nseg_dim, r0, r1, xr, ys, p.err, p.timeout_ns);
            named_bar_sync(kConsumerBar, kConsumerThreads);
            float bv = -INFINITY;
            int bi = -1;
            for (int k = tid; k < r1 - r0; k += kConsumerThreads) {
                const float v = ys[k];
                p.logits[r0 + k] = v;
                if (v == v && (bi < 0 || v > bv)) {
                    bv = v;
                    bi = r0 + k;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
                const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
                argmax_merge(bv, bi, v2, i2);
            }
            if (lane == 0) {
                sh->bv[warp] = bv;
                sh->bi[warp] = bi;
            }
            named_bar_sync(kConsumerBar, kConsumerThreads);
            if (tid == 0) {
                float B = sh->bv[0];
                int I = sh->bi[0];
                for (int w = 1; w < kConsumerWarps; ++w) argmax_merge(B, I, sh->bv[w], sh->bi[w]);
                p.amax_val[cta] = B;
                p.amax_idx[cta] = I;
            }
            if (!(ok = grid_sync(p, target, sh))) break;
            // Every CTA merges the candidates (same result everywhere).
            if (warp == 0) {
                float B = -INFINITY;
                int I = -1;
                for (int c = lane; c < G; c += 32) argmax_merge(B, I, __ldcg(p.amax_val + c), __ldcg(p.amax_idx + c));
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float v2 = __shfl_xor_sync(0xffffffffu, B, o);
                    const int i2 = __shfl_xor_sync(0xffffffffu, I, o);
                    argmax_merge(B, I, v2, i2);
                }
                if (lane == 0) {
                    const float v0 = __ldcg(p.logits);
                    sh->next = (v0 != v0 || I < 0) ? 0 : I;
                }
            }
            named_bar_sync(kConsumerBar, kConsumerThreads);
            next = *reinterpret_cast<volatile int*>(&sh->next);
            if (pos + 1 >= p.n_prompt) {
                if (cta == 0 && tid == 0) p.tokens[pos + 1] = next;
                for (int k = 0; k < p.n_stop; ++k) stop_now |= (p.stop[k] == next);
            }
        }
        steps_done = s + 1;
        if (stop_now) break;
    }
    *reinterpret_cast<volatile int*>(&sh->stop) = 1;
    if (cta == 0 && tid == 0) *p.n_done = steps_done;
}

template <int V>
__global__ void __launch_bounds__(kStreamThreads, 1) decode_kernel(const __grid_constant__ DecodeParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ Shared sh;
    Ring ring;
    ring.buf = smem;
    ring.full = reinterpret_cast<uint64_t*>(smem + (size_t)kStages * Geo<V>::kStageBytes);
    ring.empty = ring.full + kStages;
    float* ys = reinterpret_cast<float*>(ring.empty + kStages);
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&ring.full[s], 1);
            mbar_init(&ring.empty[s], kConsumerWarps);
        }
        sh.stop = 0;
        sh.flag = 0;
        sh.next = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if ((threadIdx.x >> 5) == kConsumerWarps) {
        if ((threadIdx.x & 31) == 0) run_producer<V>(p, ring, &sh.stop);
        return;
    }
    run_consumer<V>(p, ring, ys, &sh);
}

// ---------------------------------------------------------------- host --

static int ys_floats_needed(const DecodeParams& p, int G, int S) {
    const int qdim = p.n_heads * p.head_dim, kv_dim = p.n_kv * p.head_dim;
    auto rows_per = [&](int rows) { return 2 * ((rows / 2 + G - 1) / G); };
    int need = rows_per(qdim + 2 * kv_dim) * (p.dim / S);
    need = max(need, rows_per(p.dim) * (qdim / S));
    need = max(need, rows_per(2 * p.hidden) * (p.dim / S));
    need = max(need, rows_per(p.dim) * (p.hidden / S));
    need = max(need, rows_per(p.vocab) * (p.dim / S));
    need = max(need, attn_unit_smem_floats(p.n_heads / p.n_kv, kDecodeAttnTmax));
    return need;
}

static const void* decode_fn(int V) {
    switch (V) {
        case 1: return (const void*)decode_kernel<1>;
        case 2: return (const void*)decode_kernel<2>;
        case 4: return (const void*)decode_kernel<4>;
        case 8: return (const void*)decode_kernel<8>;
        default: return nullptr;
    }
}

bool decode_plan(const DecodeParams& p, int num_sms, DecodeLaunch* out, const char** why) {
    const int qdim = p.n_heads * p.head_dim;
    if (p.head_dim != kAttnHeadDim) { *why = "fused decode needs head_dim == 64"; return false; }
    if (p.n_kv <= 0 || p.n_heads % p.n_kv != 0) { *why = "n_heads must be a multiple of n_kv_heads"; return false; }
    if (p.n_heads / p.n_kv > 8) { *why = "at most 8 query heads per kv head"; return false; }
    if (p.dim % 256 != 0 || p.dim > 2048) { *why = "fused decode needs dim a multiple of 256, at most 2048"; return false; }
    const int V = p.dim / 256;
    if (V != 1 && V != 2 && V != 4 && V != 8) { *why = "dim must be 256, 512, 1024 or 2048"; return false; }
    const int S = 256 * V;
    auto seg_ok = [&](int cols) { return cols % S == 0 && (cols / S) <= 8 && 8 % (cols / S) == 0; };
    if (qdim != p.dim) { *why = "n_heads*head_dim must equal dim"; return false; }
    if (!seg_ok(p.hidden)) { *why = "hidden must be dim times 1, 2, 4 or 8"; return false; }
    if (p.vocab % 2 != 0) { *why = "vocab must be even"; return false; }
    const int G = num_sms;
    out->grid = G;
    out->seg_vec = V;
    const size_t smem = (size_t)kStages * 16 * S + 2 * kStages * sizeof(uint64_t) +
                        (size_t)ys_floats_needed(p, G, S) * sizeof(float);
    if (smem > 227 * 1024) { *why = "shared memory plan exceeds 227 KB"; return false; }
    out->smem_bytes = (int)smem;
    return true;
}

cudaError_t decode_prepare(const DecodeLaunch& l) {
    const void* fn = decode_fn(l.seg_vec);
    if (!fn) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, l.smem_bytes);
    if (e != cudaSuccess) return e;
    int blocks = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, fn, kStreamThreads, l.smem_bytes);
    if (e != cudaSuccess) return e;
    if (blocks < 1) return cudaErrorCooperativeLaunchTooLarge;
    return cudaSuccess;
}

cudaError_t launch_decode(const DecodeParams& p, const DecodeLaunch& l, cudaStream_t st) {
    const void* fn = decode_fn(l.seg_vec);
    if (!fn) return cudaErrorInvalidValue;
    cudaError_t e = cudaMemsetAsync(p.bar, 0, sizeof(uint32_t), st);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)l.grid);
    cfg.blockDim = dim3(kStreamThreads);
    cfg.dynamicSmemBytes = (size_t)l.smem_bytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* args[] = {const_cast<DecodeParams*>(&p)};
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace lc
