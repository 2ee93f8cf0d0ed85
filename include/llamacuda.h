/*
 * llamacuda.h -- C ABI of libllamacuda.so, the B200 (sm_100a) implementation of
 * the per-token Llama-3.2-1B decode path of ArturSkowronski/llama3-java-hat.
 *
 * Every entry point is plain C: opaque handles, plain pointers and sizes, an
 * int status (LC_OK == 0, negative on error, message via lc_last_error()).
 * No exception, C++ type or torch type crosses this boundary.  A Java 26 host
 * binds these symbols with java.lang.foreign downcall handles.
 *
 * Buffers: every float / half pointer argument of the per-kernel entry points
 * may be host memory (heap, pinned or an FFM MemorySegment address) or CUDA
 * device memory of the context's device.  Host buffers are staged through the
 * context: copied in, computed on the GPU, copied back, and the call returns
 * when the result is in place -- the blocking, in-place semantics of the
 * reference kernels.  When all buffers of a call are device memory the call
 * only enqueues work on the context's stream (lc_context_synchronize() waits).
 *
 * References below are file:line within the reference project, with
 *   K/ = src/main/java/com/arturskowronski/llama3babylon/hat/kernels/
 *   H/ = src/main/java/com/arturskowronski/llama3babylon/hat/
 */
#ifndef LLAMACUDA_H
#define LLAMACUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LLAMACUDA_ABI_VERSION 1

/* ------------------------------------------------------------ status ---- */
enum {
    LC_OK = 0,
    LC_ERR_INVALID_ARG = -1,  /* IllegalArgumentException in the reference */
    LC_ERR_CUDA = -2,         /* CUDA runtime / launch failure */
    LC_ERR_OUT_OF_MEMORY = -3,
    LC_ERR_NOT_FOUND = -4,    /* IOException "Tensor not found" (H/LlamaModel.java:129-132) */
    LC_ERR_SHAPE = -5,        /* IOException "Shape mismatch" (H/LlamaModel.java:249-252) */
    LC_ERR_IO = -6,           /* IOException on GGUF read (H/GGUFReader.java:57-66) */
    LC_ERR_TIMEOUT = -7,      /* a bounded device-side wait expired; the context stays usable */
    LC_ERR_STATE = -8,        /* IllegalStateException (e.g. model used before finalize) */
    LC_ERR_UNSUPPORTED = -9   /* configuration outside what the kernels implement */
};

/* Last error message of the calling thread ("" when none).  Copies at most
 * buf_len-1 bytes and NUL-terminates; returns the full message length. */
int lc_last_error(char* buf, size_t buf_len);
int lc_abi_version(void);

/* ----------------------------------------------------------- context ---- */
typedef struct lc_context lc_context;

int lc_device_count(int* count);
/* One context per GPU: device, stream, staging buffers. */
int lc_context_create(int device, lc_context** out);
int lc_context_destroy(lc_context* ctx);
int lc_context_synchronize(lc_context* ctx);
/* The context's cudaStream_t (as void*), for callers that time with events. */
void* lc_context_stream(lc_context* ctx);
int lc_context_sm_count(lc_context* ctx);

/* ---------------------------------------------- per-kernel operators ---- *
 * The IKernelFactory surface (K/IKernelFactory.java:9-40).  Same argument
 * meaning as the Java interfaces; in-place where the Java kernel is in place. */

/* IGEMV.apply(F16Array|F16Weights W, F32Array x, F32Array y, rows, cols)
 * K/IGEMV.java:34,50; K/GEMV.java:46-91.  W: raw IEEE-half bits, row-major
 * [rows][cols]; y[r] = sum_c f32(W[r,c]) * x[c] in fp32. */
int lc_gemv_f16(lc_context* ctx, const uint16_t* W, const float* x, float* y, int rows, int cols);

/* IGEMV.apply(F32Array W, ...) K/IGEMV.java:22; K/GEMV.java:34-43. */
int lc_gemv_f32(lc_context* ctx, const float* W, const float* x, float* y, int rows, int cols);

/* Batched F16 GEMV: Y[b][r] = sum_c W[r,c] * X[b][c] for b < batch (decode of
 * `batch` independent sequences against one weight matrix).  No reference
 * counterpart: the reference decodes one sequence at a time. */
int lc_gemv_f16_batched(lc_context* ctx, const uint16_t* W, const float* X, float* Y, int rows, int cols,
                        int batch);

/* Row-major F16 W [rows][cols] (host or device) -> Wt in the tiled layout the
 * tensor-core product reads: 8-row tiles of `w` columns (w = the largest
 * multiple of 64 up to 2048 dividing cols), [w/8 octets][8 rows][8 halves]
 * per tile.  rows % 8 == 0, cols % 64 == 0.  No reference counterpart (the
 * reference keeps W row-major: F16Weights, H/F16Weights.java:18-27). */
int lc_weights_tile(lc_context* ctx, const uint16_t* W, uint16_t* Wt, int rows, int cols);

/* The IGEMV product (K/IGEMV.java:34-68, sequential fp32 sums of
 * K/GEMV.java:66-91) for `batch` activation rows at once on the tcgen05
 * tensor cores: Y[b][r] = sum_c W[r][c] * X[b][c].  Wt: device memory from
 * lc_weights_tile; X [batch][cols], Y [batch][rows] fp32, host or device.
 * batch 1..16384 (up to 64 rows the weights stream once; more rows run as
 * tiles of 64, the prefill product), rows % 16 == 0, cols % 64 == 0.  Each X
 * row is split into f16 hi + lo parts under a power-of-two row scale (2^-22
 * relative), the products are exact and accumulate in fp32. */
int lc_gemm_f16_tiled(lc_context* ctx, const uint16_t* Wt, const float* X, float* Y, int rows, int cols, int batch);

/* lc_gemm_f16_tiled as a logits slice with its argmax: Y (may be NULL) as
 * above, and keys[b] = the packed argmax of Y[b] -- order-preserving float
 * bits in the high 32 bits, ~(index_offset + column) in the low 32, so the
 * largest key is the first maximum (LlamaInference.argmax,
 * H/LlamaInference.java:252-262; a NaN at global index 0 gives the largest
 * key, other NaNs never win).  Keys of row slices held by different GPUs
 * combine with an unsigned max (e.g. an all-reduce), which is how a
 * row-sharded lm_head finds the next token without gathering logits. */
int lc_gemm_f16_tiled_argmax(lc_context* ctx, const uint16_t* Wt, const float* X, float* Y, int rows, int cols,
                             int batch, int32_t index_offset, uint64_t* keys);

/* IRMSNorm.apply(x, weight, size) K/IRMSNorm.java:17; K/RMSNorm.java:35-50.
 * In place, eps = 1e-5f (K/RMSNorm.java:22). */
int lc_rmsnorm(lc_context* ctx, float* x, const float* weight, int size);

/* RMSNorm over `rows` independent rows of `width` (same math per row). */
int lc_rmsnorm_rows(lc_context* ctx, float* x, const float* weight, int rows, int width, float eps);

/* IRoPE.apply(vec, pos, numHeads, headDim, theta) K/IRoPE.java:19;
 * K/RoPE.java:36-52.  Interleaved pairs, in place. */
int lc_rope(lc_context* ctx, float* vec, int pos, int num_heads, int head_dim, float theta);

/* RoPE over `rows` vectors of num_heads*head_dim, row i at position pos[i]
 * (pos: host or device int32 array of `rows`). */
int lc_rope_rows(lc_context* ctx, float* vec, const int32_t* pos, int rows, int num_heads, int head_dim,
                 float theta);

/* ISiLU.apply(x, size) K/ISiLU.java:16; K/SiLU.java:32-40.  In place. */
int lc_silu(lc_context* ctx, float* x, int size);

/* Fused SwiGLU: gate[i] = silu(gate[i]) * up[i] for i < n -- SiLU followed by
 * TransformerBlock.elementWiseMul (H/TransformerBlock.java:209-210,240-244). */
int lc_swiglu(lc_context* ctx, float* gate, const float* up, int n);

/* ISoftmax.apply(x, size) K/ISoftmax.java:16; K/Softmax.java:28-51.  In place,
 * single kernel, the row is read once and written once. */
int lc_softmax(lc_context* ctx, float* x, int size);

/* ISoftmax.applyRow(x, rowOffset, rowSize) K/ISoftmax.java:26; K/Softmax.java:61-84. */
int lc_softmax_row(lc_context* ctx, float* x, int row_offset, int row_size);

/* Softmax over `rows` contiguous rows of `width`. */
int lc_softmax_rows(lc_context* ctx, float* x, int rows, int width);

/* IAttention.computeScores(q, keys, scores, seqLen, headDim) K/IAttention.java:19;
 * K/Attention.java:32-42.  keys: [seq_len][head_dim]. */
int lc_attn_scores(lc_context* ctx, const float* q, const float* keys, float* scores, int seq_len, int head_dim);

/* IAttention.computeValues(scores, values, out, seqLen, headDim) K/IAttention.java:30;
 * K/Attention.java:53-61.  values: [seq_len][head_dim]. */
int lc_attn_values(lc_context* ctx, const float* scores, const float* values, float* out, int seq_len,
                   int head_dim);

/* Fused GQA decode attention for one query token per sequence -- the per-head
 * loop of TransformerBlock.forward (H/TransformerBlock.java:164-192) in one
 * launch (split-KV flash decoding; partial results in device scratch owned by
 * the context).
 *   q:   [batch][n_heads][head_dim]
 *   k,v: cache of each sequence b at k + b*seq_stride; position t of kv head h
 *        at offset h*head_stride + t*pos_stride (floats).  The reference layout
 *        [max_seq][n_kv][head_dim] is pos_stride = n_kv*head_dim, head_stride = head_dim.
 *   seq_len: [batch] int32 (host or device), positions 0..seq_len[b]-1 attend.
 *   out: [batch][n_heads][head_dim]. */
int lc_attention_decode(lc_context* ctx, const float* q, const float* k, const float* v, float* out,
                        const int32_t* seq_len, int batch, int n_heads, int n_kv_heads, int head_dim,
                        int64_t seq_stride, int64_t head_stride, int64_t pos_stride);

/* lc_attention_decode without any device allocation.  No counterpart in the
 * reference.  For hosts that cannot call cudaMalloc at this point (device
 * memory owned by the host's own pool allocator, latency-critical loops that
 * cannot afford cudaFree's device-wide synchronisation, fixed device
 * footprint after load).  Same arguments and results as lc_attention_decode;
 * q, k, v and out must be device memory of the context's device; seq_len may
 * be host memory or device memory of the context's device (another GPU's:
 * LC_ERR_INVALID_ARG).  Scratch is a static 8 MiB device array per GPU (held
 * until exit); plans needing more, or batch > 1024, return LC_ERR_INVALID_ARG.
 * The first call on a device resolves the array's address (make it before
 * any stream capture).  All calls on a device share the array: calls that
 * overlap on the GPU race.  The lengths are read on the host to size the
 * split plan: with seq_len in device memory the call first waits for the
 * work already queued on the context stream (so lengths written there are
 * seen), then enqueues; with seq_len in host memory it only enqueues.  In
 * both cases it returns before the attention has run: synchronize the
 * context before reading out. */
int lc_attention_decode_static(lc_context* ctx, const float* q, const float* k, const float* v, float* out,
                               const int32_t* seq_len, int batch, int n_heads, int n_kv_heads, int head_dim,
                               int64_t seq_stride, int64_t head_stride, int64_t pos_stride);

/* lc_attention_decode with the split plan sized for max_len, an upper bound
 * of every seq_len[b] (positions past max_len are not attended).  seq_len is
 * not read on the host, so with device buffers the call only enqueues (it
 * can be captured in a CUDA graph); the first call of a context, or one with
 * a larger plan, allocates scratch. */
int lc_attention_decode_maxlen(lc_context* ctx, const float* q, const float* k, const float* v, float* out,
                               const int32_t* seq_len, int batch, int n_heads, int n_kv_heads, int head_dim,
                               int64_t seq_stride, int64_t head_stride, int64_t pos_stride, int max_len);

/* LlamaInference.argmax(values) H/LlamaInference.java:252-262: first index of
 * the maximum (ties -> lowest index; 0 when values[0] is NaN). */
int lc_argmax(lc_context* ctx, const float* values, int n, int32_t* out_index);

/* ------------------------------------------------------------- model ---- */
typedef struct lc_config {
    int32_t dim;        /* HIDDEN_SIZE 2048          (H/LlamaModel.java:30) */
    int32_t hidden;     /* INTERMEDIATE_SIZE 8192    (:31) */
    int32_t n_layers;   /* NUM_LAYERS 16             (:32) */
    int32_t n_heads;    /* NUM_HEADS 32              (:33) */
    int32_t n_kv_heads; /* NUM_KV_HEADS 8            (:34) */
    int32_t head_dim;   /* HEAD_DIM 64               (:35) */
    int32_t vocab;      /* VOCAB_SIZE 128256         (:36) */
    int32_t max_seq;    /* MAX_SEQ_LEN 2048          (:37) */
    float rope_theta;   /* 500000 (H/TransformerBlock.java:136) */
    float rms_eps;      /* 1e-5 (K/RMSNorm.java:22) */
    int32_t weight_mode; /* LC_WEIGHTS_F16 (0, default) or LC_WEIGHTS_F32 (1):
                            H/WeightStorageMode.java, chosen per model as
                            H/LlamaInference.java:58-62, 102-108 does */
    int32_t reserved[5];
} lc_config;

/* Weight storage modes (H/WeightStorageMode.java).  F16 and F16_FAST differ
 * only in the Java host's storage; on the GPU both keep the F16 weights
 * (tiled for the fused decode kernel).  F32 keeps the projections and the
 * embedding as fp32 (F16 tensors widened exactly, F32 tensors as given; twice
 * the memory) and decodes with fp32-weight GEMVs (K/GEMV.java:34-43).  The
 * multi-sequence batch (lc_batch_*) needs F16 weights. */
#define LC_WEIGHTS_F16 0
#define LC_WEIGHTS_F32 1

typedef struct lc_model lc_model;

/* Llama-3.2-1B constants of H/LlamaModel.java:30-37. */
void lc_config_llama32_1b(lc_config* out);

/* Allocates device storage for all weights (LlamaModel + the TransformerBlock
 * weight maps, H/TransformerBlock.java:87-96). */
int lc_model_create(lc_context* ctx, const lc_config* cfg, lc_model** out);

/* Uploads one tensor by its GGUF name ("token_embd.weight", "output.weight",
 * "output_norm.weight", "blk.N.attn_norm.weight", "blk.N.attn_q.weight", ...,
 * "blk.N.ffn_down.weight").  dtype: 0 = F32, 1 = F16 (raw half bits), the GGUF
 * type ids.  With LC_WEIGHTS_F16 projection weights must be F16
 * (H/LlamaModel.java:238-240); with LC_WEIGHTS_F32 they may be F16 or F32
 * (LlamaModel.mapTensor, :115-170).  Norms are F32 (F16 norms are widened);
 * n_elems must equal the expected element count (LC_ERR_SHAPE otherwise, as
 * H/LlamaModel.java:249-252). */
int lc_model_upload_tensor(lc_model* m, const char* name, const void* data, int64_t n_elems, int32_t dtype);

/* Checks that every tensor arrived (tied lm_head when "output.weight" is
 * absent, H/LlamaInference.java:69-72) and prepares the decode kernels. */
int lc_model_finalize(lc_model* m);

/* Reads a GGUF v3 file (H/GGUFReader.java:57-123, H/LlamaModel.java:74-86
 * validation) and uploads every tensor once; returns a finalized model.
 * max_seq <= 0 keeps the config default. */
int lc_model_load_gguf(lc_context* ctx, const char* path, int32_t max_seq, lc_model** out);

/* lc_model_load_gguf with a weight storage mode (LC_WEIGHTS_F16 or
 * LC_WEIGHTS_F32): the LlamaInference(ggufPath, factory, backend, weightMode)
 * constructor's choice, H/LlamaInference.java:58-62. */
int lc_model_load_gguf_mode(lc_context* ctx, const char* path, int32_t max_seq, int32_t weight_mode,
                            lc_model** out);

int lc_model_get_config(const lc_model* m, lc_config* out);
int lc_model_destroy(lc_model* m);

/* ----------------------------------------------------------- session ---- *
 * One decoding sequence: device-resident fp32 KV cache and activations, the
 * state LlamaInference owns per instance (H/LlamaInference.java:79-89). */
typedef struct lc_session lc_session;

int lc_session_create(lc_model* m, lc_session** out);
int lc_session_destroy(lc_session* s);

/* LlamaInference.forward(token, pos) H/LlamaInference.java:117-164: one decode
 * step.  logits (host or device, may be NULL) receives vocab floats;
 * argmax_out (may be NULL) receives the greedy token. */
int lc_forward(lc_session* s, int32_t token, int32_t pos, float* logits, int32_t* argmax_out);

/* LlamaInference.generate(prompt, maxNew, stopTokens) H/LlamaInference.java:173-217:
 * token-by-token prefill then greedy decode, all steps in one device launch.
 * out_tokens (host or device) receives up to max_new ids; *n_out the count.
 * prompt / stop may be host or device arrays. */
int lc_generate(lc_session* s, const int32_t* prompt, int32_t n_prompt, int32_t max_new, const int32_t* stop,
                int32_t n_stop, int32_t* out_tokens, int32_t* n_out);

/* Receives generated token number `index` (0-based) while the launch runs. */
typedef void (*lc_token_callback)(int32_t token, int32_t index, void* user);

/* lc_generate with streaming: the same single launch, but the kernel also
 * publishes each greedy token to mapped host memory as soon as it is chosen,
 * and the calling thread invokes on_token(token, index, user) for each one in
 * order while the launch is still running (the streaming callbacks of the
 * chat path around LlamaInference.chat, H/LlamaInference.java:227-247).
 * Every generated id, the stop token included, is passed exactly once before
 * the call returns; out_tokens / n_out are filled as by lc_generate. */
int lc_generate_stream(lc_session* s, const int32_t* prompt, int32_t n_prompt, int32_t max_new,
                       const int32_t* stop, int32_t n_stop, lc_token_callback on_token, void* user,
                       int32_t* out_tokens, int32_t* n_out);

/* Continues a sequence already holding positions 0..start_pos-1: feeds
 * `token` at start_pos and decodes n_steps greedy steps (positions
 * start_pos..start_pos+n_steps-1), writing the n_steps produced tokens to
 * out_tokens.  No stop tokens.  This is the device-resident decode loop that
 * lc_generate runs after the prompt. */
int lc_decode(lc_session* s, int32_t token, int32_t start_pos, int32_t n_steps, int32_t* out_tokens);

/* Phase trace of the fused decode kernel (diagnostics).  words_per_cta > 0
 * allocates a [grid][words_per_cta] uint64 buffer (0 frees it); while set,
 * every launch records %globaltimer stamps: per CTA, the first half holds
 * consumer marks (per layer: QKV start / consumed / barrier, attention done /
 * barrier, then start / consumed / barrier for O, gate-up and down; per
 * lm_head step: start / consumed / barrier / argmax), the second half one
 * producer mark per weight job (last stage issued).  Read with
 * lc_session_read_trace (grid and words_per_cta may be NULL). */
int lc_session_enable_trace(lc_session* s, int32_t words_per_cta);
int lc_session_read_trace(lc_session* s, uint64_t* out, int64_t n_words, int32_t* grid, int32_t* words_per_cta);

/* Device time of the last lc_generate / lc_decode / lc_forward launch in ms
 * (CUDA events on the session stream). */
int lc_session_last_ms(lc_session* s, float* ms);

/* ------------------------------------------------- multi-sequence batch ---
 * Greedy decode of up to 64 independent sequences in lockstep (serving).  No
 * reference counterpart: the reference serves one sequence per
 * LlamaInference (H/LlamaInference.java:173-217); each sequence of a batch
 * gets exactly that computation, with every weight matrix read once per
 * step for all sequences (tcgen05 tensor-core products).  A batch owns KV
 * caches for max_batch sequences of the model's max_seq positions. */
typedef struct lc_batch lc_batch;

int lc_batch_create(lc_model* m, int32_t max_batch, lc_batch** out);
int lc_batch_destroy(lc_batch* b);

/* LlamaInference.generate(prompt_s, max_new, stop) (H/LlamaInference.java
 * :180-217) for n_seqs sequences at once.  prompts: the prompts concatenated
 * (host), prompt_lens[n_seqs] >= 1; prompt_lens[s] + max_new - 1 <= max_seq.
 * out_tokens [n_seqs][max_new] (host) receives each sequence's generated
 * tokens, the stop token included; entries after a stop token are -1.
 * Synchronous. */
int lc_batch_generate(lc_batch* b, int32_t n_seqs, const int32_t* prompts, const int32_t* prompt_lens,
                      int32_t max_new, const int32_t* stop, int32_t n_stop, int32_t* out_tokens);

/* Device time of the last lc_batch_generate in ms: all steps, and the steps
 * from the last prompt position on (each of which yields one token per
 * sequence); steps = positions run. */
int lc_batch_last_ms(lc_batch* b, float* total_ms, float* decode_ms, int32_t* steps);

/* Logits (vocab floats, host) of sequence `seq` at the last position of the
 * last lc_batch_generate. */
int lc_batch_logits(lc_batch* b, int32_t seq, float* out);

/* ------------------------------------ lm_head row shard over N GPUs ---- */
/* The lm_head GEMV (H/LlamaInference.java:151-156) split by rows over N
 * GPUs, one process per GPU: each rank computes its logits slice and packed
 * argmax keys (lc_gemm_f16_tiled_argmax), then the ranks exchange only the
 * keys; the maximum key is LlamaInference.argmax (:252-262) of the full
 * logits.  lc_keyx does that exchange through NVLink peer memory: every
 * rank stores its keys into every rank's mailbox and waits, bounded, for
 * the others' flags (no library collective, no multicast).  No counterpart
 * in the reference, which runs on one device. */
typedef struct lc_keyx lc_keyx;
#define LC_KEYX_HANDLE_BYTES 64
#define LC_KEYX_MAX_WORLD 8

/* Allocates this rank's mailbox for up to max_batch keys per call and
 * writes its inter-process handle (LC_KEYX_HANDLE_BYTES bytes) to
 * handle_out; the host gathers the handles of all ranks in rank order. */
int lc_keyx_create(lc_context* ctx, int32_t world, int32_t rank, int32_t max_batch, lc_keyx** out,
                   void* handle_out);
/* Maps the other ranks' mailboxes: handles = world handles in rank order. */
int lc_keyx_open(lc_keyx* x, const void* handles);
/* In place: keys (device, [batch] uint64) becomes the maximum over the
 * ranks.  Collective: every rank makes the same calls in the same order.
 * Enqueue-only on the context's stream; a wait that gave up is reported by
 * lc_context_synchronize (LC_ERR_TIMEOUT). */
int lc_keyx_allreduce(lc_keyx* x, uint64_t* keys, int32_t batch);
/* After every rank's last lc_keyx_allreduce has completed (a barrier). */
int lc_keyx_destroy(lc_keyx* x);

#ifdef __cplusplus
}
#endif

#endif /* LLAMACUDA_H */
