// lc_internal.h -- declarations shared by the llamacuda translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <utility>
#include <cstring>
#include <vector>

#include "lc_common.cuh"

namespace lc {

// Host-precomputed RoPE inverse frequencies: f[j] = (float)(1/pow(theta, 2j/head_dim))
// (RoPE.java:42).  head_dim <= 512.
struct RopeFreq {
    float f[256];
};

void make_rope_freq(RopeFreq* out, float theta, int head_dim);

// ---- standalone kernels (lc_kernels.cu) ----
void launch_gemv_generic_f16(const uint16_t* W, const float* x, float* y, int rows, int cols, cudaStream_t st);
void launch_gemv_generic_f32(const float* W, const float* x, float* y, int rows, int cols, cudaStream_t st);
void launch_gemv_batched_f16(const uint16_t* W, const float* X, float* Y, int rows, int cols, int batch,
                             cudaStream_t st);
void launch_rmsnorm_rows(float* x, const float* w, int rows, int width, float eps, cudaStream_t st);
void launch_rope_rows(float* vec, const int32_t* pos, int rows, int num_heads, int head_dim, const RopeFreq& fq,
                      cudaStream_t st);
void launch_silu(float* x, long long n, cudaStream_t st);
void launch_swiglu(float* g, const float* u, long long n, cudaStream_t st);
void launch_softmax_rows(float* x, int rows, int width, cudaStream_t st);
void launch_attn_scores(const float* q, const float* keys, float* scores, int seq_len, int head_dim, float scale,
                        cudaStream_t st);
void launch_attn_values(const float* p, const float* values, float* out, int seq_len, int head_dim,
                        cudaStream_t st);
void launch_argmax(const float* v, int n, int32_t* out, cudaStream_t st);

// ---- streaming GEMV (lc_gemv.cu) ----
// True when the streaming kernel takes this shape and these pointers.
bool stream_gemv_supported(const void* W, const void* x, int rows, int cols);
cudaError_t launch_stream_gemv(const uint16_t* W, const float* x, float* y, int rows, int cols, int num_sms,
                               int* err, cudaStream_t st);

// ---- fused GQA decode attention (lc_attention.cu) ----
struct AttnPlan {
    int batch, n_heads, n_kv, head_dim;
    int split_len;  // positions per split (T)
    int max_splits; // splits per (sequence, kv head) upper bound
};
// Bytes of scratch the attention launch needs: partials + completion counters.
size_t attention_scratch_bytes(const AttnPlan& p);
AttnPlan plan_attention(int batch, int n_heads, int n_kv, int head_dim, int max_len, int num_sms);
// scratch: attention_scratch_bytes(p) bytes; counters inside are cleared by this call.
cudaError_t launch_attention_decode(const AttnPlan& p, const float* q, const float* k, const float* v, float* out,
                                    const int32_t* seq_len, int64_t seq_stride, int64_t head_stride,
                                    int64_t pos_stride, void* scratch, cudaStream_t st, bool pdl = false);

// Launch with optional programmatic stream serialisation.
template <typename... P, typename... A>
cudaError_t launch_ex(void (*kernel)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                      A&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<A>(args)...);
}

// ---- decode with fp32 weights, WeightStorageMode.F32 (lc_f32.cu) ----
struct F32Layer {
    const float* wqkv;   // [n_heads*head_dim + 2*kv_dim][dim]: q rows, then k, then v
    const float* wo;     // [dim][n_heads*head_dim]
    const float* wgu;    // [2*hidden][dim]: gate rows, then up rows
    const float* wdown;  // [dim][hidden]
    const float* attn_norm;
    const float* ffn_norm;
};
// Everything one fp32-weight forward touches (device pointers; `layers` is a
// host array).
struct F32Step {
    int dim, hidden, n_layers, n_heads, n_kv, head_dim, vocab, max_seq, num_sms;
    float eps;
    const float* tok_emb;   // [vocab][dim]
    const float* lm;        // [vocab][dim]: output.weight or the tied embedding
    const float* out_norm;
    const F32Layer* layers;
    RopeFreq rope;
    float *kcache, *vcache, *logits;  // the session's ([n_layers][n_kv][max_seq][head_dim] caches)
    int32_t* tokens;                  // token fed at each position; the argmax goes to tokens[pos + 1]
    int* err;
    float *x, *xb, *qkv, *att, *gu;   // scratch: dim, dim, q+k+v, n_heads*head_dim, 2*hidden
    const int32_t* posv;              // posv[i] = i
    const int32_t* lenv;              // lenv[i] = i + 1
    void* attn_scratch;
    size_t attn_scratch_bytes;
};
cudaError_t launch_f16_to_f32(const __half* src, float* dst, long long n, cudaStream_t st);
bool f32_supported(int dim, int hidden, int qdim, const char** why);
cudaError_t f32_prepare();
// Enqueues one forward at `pos` (token tokens[pos]); with `logits` the final
// norm, lm_head and, with `store_token`, the argmax into tokens[pos + 1].
cudaError_t f32_forward(const F32Step& f, int pos, bool logits, bool store_token, cudaStream_t st);

// ---- argmax-key all-reduce over peer memory (lc_keyx.cu) ----
constexpr int kKeyxMaxWorld = 8;
struct KeyxArgs {
    uint64_t* keys_mbox[kKeyxMaxWorld];   // key slots of rank p's mailbox (this rank's own included)
    uint32_t* flags_mbox[kKeyxMaxWorld];  // flags of rank p's mailbox
    uint64_t* keys;                       // [batch] this rank's keys in, the maximum over the ranks out
    int world, rank, batch, max_batch;
    uint32_t epoch;                       // call number, from 1, equal on every rank
    int* err;
    uint64_t timeout_ns;
};
// Byte offset of the flags in a mailbox ([2][world][max_batch] keys first).
inline size_t keyx_flags_offset(int world, int max_batch) {
    return ((size_t)2 * world * max_batch * sizeof(uint64_t) + 255) / 256 * 256;
}
size_t keyx_mailbox_bytes(int world, int max_batch);
cudaError_t launch_keyx(const KeyxArgs& a, cudaStream_t st, bool pdl);

// ---- fused decode step (lc_decode.cu) ----
//
// GEMV weights of the fused kernel live in HBM as row-group tiles: a tile is
// 8 consecutive rows x CB = dim consecutive columns, stored as
// [CB / 8 column octets][8 rows][8 halves] (16 * CB bytes, contiguous), and
// tile (g, cb) of a matrix with ncb = cols / CB column blocks starts at
// element (g * ncb + cb) * 8 * CB.  One 1-D bulk copy moves a tile into
// shared memory, where each 8x8 block of halves (128 contiguous bytes) is a
// core matrix of a K-major, no-swizzle tcgen05 descriptor, so tcgen05.cp
// moves the tile into tensor memory as it lies.  Rows are padded to a
// multiple of 8 with zeros.
struct LayerW {
    const __half* wqkv;   // tiled [dim + 2*kv_dim][dim]
    const __half* wo;     // tiled [dim][n_heads*head_dim]
    const __half* wgu;    // tiled [2*hidden][dim], row 2r = gate r, row 2r+1 = up r
    const __half* wdown;  // tiled [dim][hidden]
    const float* attn_norm;
    const float* ffn_norm;
};

// Element offset of (row, col) in the tiled layout of a matrix with `cols`
// columns and column-block width cb.
__host__ __device__ inline size_t tiled_offset(int64_t row, int64_t col, int64_t cols, int64_t cb) {
    const int64_t ncb = cols / cb;
    return (size_t)((((row >> 3) * ncb + col / cb) * 8 * cb) + ((col % cb) >> 3) * 64 + (row & 7) * 8 + (col & 7));
}

// Rewrites a row-major F16 matrix [rows][cols] into the tiled layout:
// source row r becomes row row0 + r * row_step of the destination matrix.
cudaError_t launch_tile_rows(const __half* src, __half* dst, int rows, int cols, int cb, int row0, int row_step,
                             cudaStream_t st);

constexpr int kMaxStop = 32;
constexpr int kMaxDecodeLayers = 64;  // layers the fused decode kernel takes (norm pointers in its parameters)
constexpr int kDecodePartStride = 68;  // words per attention partial: m, l, 0, 0, o[64]

struct DecodeParams {
    // model
    int dim, hidden, n_layers, n_heads, n_kv, head_dim, vocab, max_seq;
    float eps;
    float attn_scale;
    const __half* tok_emb;  // row-major [vocab][dim]
    const __half* lm_head;  // tiled [vocab rounded up to 8][dim]
    const float* out_norm;
    const LayerW* layers;   // device array [n_layers]
    const float* norm_w[2 * kMaxDecodeLayers];  // attn_norm of layer l at 2l, ffn_norm at 2l + 1
    RopeFreq rope;
    const float2* rope_cs;  // [max_seq][head_dim / 2] (sin, cos) of pos * freq, rounded like RoPE.java:44-46
    // session buffers (device)
    float* kcache;  // [n_layers][n_kv][max_seq][head_dim]
    float* vcache;
    float* logits;  // [vocab]
    int32_t* tokens;       // [max_seq + 1]: token fed at each position
    int* err;              // device error word
    int* n_done;           // steps completed
    // Exchange buffers: tagged 64-bit words (float bits | tag << 32); the
    // per-CTA flags say when to look, the tags say what is valid.
    uint64_t* xa;          // [dim]   x after the attention residual
    uint64_t* xb;          // [dim]   x after the FFN residual
    uint64_t* q;           // [n_heads*head_dim] rotated q of the current position
    uint64_t* kv;          // [2*kv_dim] rotated k, then v, of the current position
    uint64_t* att;         // [n_heads*head_dim] attention output (single split)
    uint64_t* part;        // [n_kv][attn_max_splits][kv_mul][kDecodePartStride] partials
    float* h;              // [hidden] silu(gate)*up (plain: published with a fence)
    uint64_t* amax;        // [grid][2] per-CTA argmax candidate (value, index bits)
    uint32_t* flags;       // [grid] latest exchange tag each CTA has published (a hint)
    uint32_t tag_base;     // launch epoch << 20; tags are tag_base + exchange + 1
    // launch
    int pos0, nsteps, n_prompt;
    int skip_prefill_logits;
    int n_stop;
    int32_t stop[kMaxStop];
    int attn_max_splits;   // splits per kv head upper bound (partials layout)
    unsigned long long timeout_ns;
    // Phase trace (debug): when non-null, consumer thread 0 of each CTA writes
    // %globaltimer stamps into trace[cta*trace_words + k].
    unsigned long long* trace;
    int trace_words;
    // Token stream (nullable; mapped host memory): CTA 0 writes generated
    // token i to stream[1 + i], then i + 1 to stream[0], with a system fence
    // between, so a host thread can poll the count while the launch runs.
    int32_t* stream;
    // Producer tile schedule of one position (decode_build_schedule): row
    // cta * sched_stride of `sched` lists the CTA's weight tiles in consumption
    // order as offsets from wbase in 256-byte units, the QKV..DN jobs of all
    // layers (sched_n[2 * cta] tiles) then the lm_head job (sched_n[2 * cta + 1]).
    const uint32_t* sched;
    const int* sched_n;
    int sched_stride;
    const uint8_t* wbase;
    // L2 prefetch window of the producer, in tiles ahead of the copies (0: off).
    int l2_prefetch_tiles;
};

struct DecodeLaunch {
    int grid;
    int smem_bytes;
    int ks;      // k-steps of 16 columns per consumer warp: dim / 128
    int stages;  // ring stages
};

// Splits per kv head the attention phase can use up to max_seq (partials
// layout of DecodeParams::part).
int decode_attn_max_splits(int max_seq, int grid, int n_kv);

// Host: the producer tile schedule of one position for a grid of G CTAs
// (DecodeParams::sched): p's model fields with host copies of the layer
// table in `layers`.  Fills rows of `stride` entries and per-CTA counts.
void decode_build_schedule(const DecodeParams& p, const LayerW* layers, int G, std::vector<uint32_t>* sched,
                           std::vector<int>* counts, int* stride);

// Validates the configuration against what the fused kernel implements and
// fills the launch shape.  Returns false with a message when unsupported.
bool decode_plan(const DecodeParams& p, int num_sms, DecodeLaunch* out, const char** why);
cudaError_t decode_prepare(const DecodeLaunch& l);  // sets the smem attribute once
cudaError_t launch_decode(const DecodeParams& p, const DecodeLaunch& l, cudaStream_t st);
// Same kernel built with the phase trace (p.trace must be set).
cudaError_t decode_prepare_traced(const DecodeLaunch& l);
cudaError_t launch_decode_traced(const DecodeParams& p, const DecodeLaunch& l, cudaStream_t st);

// ---- batched GEMM on tcgen05 (lc_gemm.cu) ----
//
// Y[s][n] = sum_k A[s][k] * W[n][k] for B <= 64 activation rows, W F16 in the
// tiled layout above (column-block width cbw).  A reaches the GEMM pre-split
// (launch_gemm_split or a fused producer): row s becomes f16 hi / lo parts
// under a power-of-two row scale, MMA rows 2s (hi) and 2s + 1 (lo), stored as
// [16 row groups of 8 MMA rows][K / 8 octets][8 rows][8 halves] (bytes
// ((s / 4) * (K / 8) + k / 8) * 128 + (2 * (s % 4) + part) * 16 + (k % 8) * 2),
// and unscale[s] = 2^-e.  The result goes through one of the fused epilogues.
enum GemmOp : int {
    kGemmStore = 0,   // y[s * ldy + n] = v
    kGemmResid = 1,   // y[s * ldy + n] += v (residual add, in place)
    kGemmQKV = 2,     // RoPE on q and k, q -> q[s][n], k / v -> the KV cache at pos[s]
    kGemmSwiGLU = 3,  // rows 4m..4m+3 = (gate, up) pairs: h[s][2m + j] = silu(g) * u
    kGemmLogits = 4,  // logits[s][n] (optional) and best[s] = packed (value, lowest index) argmax
};

constexpr int kGemmMaxB = 64;        // activation rows per row tile (one MMA of 128 hi / lo rows)
constexpr int kGemmMaxRows = 16384;  // activation rows of one product call (prefill)
constexpr int kGemmHeadDim = 64;  // head_dim of the kGemmQKV epilogue

// Bytes of the pre-split activations of B rows and K columns.
inline size_t gemm_split_bytes(int B, int K) { return (size_t)((B + 3) / 4) * (size_t)K * 16; }

struct GemmParams {
    const __half* W;  // tiled
    int N, K, cbw;    // rows, columns, column-block width (K % cbw == 0, cbw % 64 == 0)
    int rows_mem;     // rows stored in W (multiple of 8, <= N; 0: N)
    const uint8_t* As;      // pre-split activations
    const float* unscale;   // [B]
    int B;                  // activation rows; more than 64 run as tiles of 64 rows
    int nblk, kspl, units;  // N-block rows, K splits, row tiles * N-blocks * kspl
    int mtiles;             // row tiles of 64
    int stages, stage_bytes;
    float* part;             // [kspl][B][N] partial sums when kspl > 1
    int op;
    float* y;
    int ldy;
    // kGemmQKV
    float* q;
    int qdim, kvd;
    float* kcache;
    float* vcache;            // this layer's base: + s * kv_seq_stride + head * kv_head_stride + pos * 64
    int64_t kv_seq_stride, kv_head_stride;
    const int32_t* pos;       // [B]
    const int32_t* row_seq;   // [B] KV-cache sequence of each row (null: the row index)
    const float* rope_freq;   // [head_dim / 2]
    // kGemmSwiGLU
    float* h;
    int ldh;
    // kGemmLogits
    float* logits;
    int ldl;
    int n_valid;              // columns >= n_valid are padding (kGemmLogits)
    int idx_offset;           // global index of column 0 in the argmax keys (kGemmLogits)
    unsigned long long* best; // [B]
    int* err;
    uint64_t timeout_ns;
};

// Chooses nblk, kspl and the ring for a grid of `num_sms` CTAs; fills units
// and mtiles.  Returns false when the shape is unsupported (N % 16, K % 64,
// K % cbw, B < 1).
bool gemm_plan(GemmParams* p, int num_sms);
// Bytes of the partial-sum buffer p needs (0 when kspl == 1).
size_t gemm_part_bytes(const GemmParams& p);
cudaError_t gemm_prepare();  // sets the shared-memory attribute once
// TMA tensor maps: the tiled weights of p (box: nblk rows x 64 columns) and
// the pre-split activations of p.B rows (box: all row groups x 64 columns).
cudaError_t gemm_make_wmap(CUtensorMap* out, const GemmParams& p);
cudaError_t gemm_make_amap(CUtensorMap* out, const GemmParams& p);
// pdl: launched with programmatic stream serialisation (the kernels wait for
// their predecessor before touching its results; weight loads start early).
cudaError_t launch_gemm(const GemmParams& p, const CUtensorMap& wmap, const CUtensorMap& amap, int num_sms,
                        cudaStream_t st, bool pdl = false);
// A fp32 [B][lda] -> pre-split activations As and unscale[B].
cudaError_t launch_gemm_split(const float* A, int lda, int K, int B, uint8_t* As, float* unscale, cudaStream_t st,
                              bool pdl = false);
// Column-block width of the standalone tiled layout: the largest multiple of
// 64 up to 2048 dividing cols (0: cols % 64 != 0).
int gemm_tile_width(int cols);

// ---- multi-sequence greedy decode (lc_batch.cu) ----
struct BatchModel {
    int dim, hidden, n_layers, n_heads, n_kv, head_dim, vocab, max_seq;
    float eps;
    const __half* tok_emb;   // row-major [vocab][dim]
    const __half* lm_head;   // tiled, rows padded to a multiple of 8
    const float* out_norm;
    std::vector<LayerW> layers;  // host copy of the layer table (device pointers)
    RopeFreq rope;
};
struct BatchEngine;
bool batch_supported(const BatchModel& m, const char** why);
// Buffers for up to max_batch (1..64) sequences of up to m.max_seq positions.
BatchEngine* batch_create(const BatchModel& m, int max_batch, int num_sms, cudaStream_t st, int* err,
                          cudaError_t* ce);
void batch_destroy(BatchEngine* e);
int batch_max(const BatchEngine* e);
int batch_tok_stride(const BatchEngine* e);  // max_seq + 1
// Greedy generation of n sequences: tok_host [n][tok_stride] holds the
// prompts, lens their lengths (validated by the caller: tokens in range,
// lens[s] + max_new - 1 <= max_seq).  tok_out receives the token rows:
// prompt, then the generated tokens.
cudaError_t batch_run(BatchEngine* e, int n, const std::vector<int32_t>& tok_host, const std::vector<int32_t>& lens,
                      int max_new, std::vector<int32_t>* tok_out);
void batch_times(const BatchEngine* e, float* total_ms, float* decode_ms, int* steps);
cudaError_t batch_logits(const BatchEngine* e, int s, float* out);  // logits of the last lm_head step

// Argmax key: order-preserving float bits above the inverted index, so the
// largest key is the largest value with the lowest index.
__host__ __device__ inline unsigned long long argmax_key(float v, int idx) {
#ifdef __CUDA_ARCH__
    uint32_t b = __float_as_uint(v);
#else
    uint32_t b;
    memcpy(&b, &v, 4);
#endif
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | (uint32_t)(~(uint32_t)idx);
}
__host__ __device__ inline int argmax_key_index(unsigned long long k) { return (int)(~(uint32_t)(k & 0xffffffffu)); }

}  // namespace lc
