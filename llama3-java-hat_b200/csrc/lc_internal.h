// lc_internal.h -- declarations shared by the llamacuda translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

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
                                    int64_t pos_stride, void* scratch, cudaStream_t st);

// ---- fused decode step (lc_decode.cu) ----
struct LayerW {
    const __half* wqkv;   // [dim + 2*kv_dim][dim]
    const __half* wo;     // [dim][n_heads*head_dim]
    const __half* wgu;    // [2*hidden][dim], row 2r = gate r, row 2r+1 = up r
    const __half* wdown;  // [dim][hidden]
    const float* attn_norm;
    const float* ffn_norm;
};

constexpr int kMaxStop = 32;

struct DecodeParams {
    // model
    int dim, hidden, n_layers, n_heads, n_kv, head_dim, vocab, max_seq;
    float eps;
    float attn_scale;
    const __half* tok_emb;
    const __half* lm_head;
    const float* out_norm;
    const LayerW* layers;  // device array [n_layers]
    RopeFreq rope;
    // session buffers (device)
    float* kcache;  // [n_layers][n_kv][max_seq][head_dim]
    float* vcache;
    float* x;       // [dim]
    float* qbuf;    // [n_heads*head_dim]
    float* att;     // [n_heads*head_dim]
    float* hbuf;    // [hidden]
    float* logits;  // [vocab]
    float* attn_part;      // attention partials
    uint32_t* attn_cnt;    // [n_kv] completion counters, self-resetting
    float* amax_val;       // [grid]
    int* amax_idx;         // [grid]
    int32_t* tokens;       // [max_seq + 1]: token fed at each position
    uint32_t* bar;         // grid barrier counter, zero at launch
    int* err;              // device error word
    int* n_done;           // steps completed
    // launch
    int pos0, nsteps, n_prompt;
    int skip_prefill_logits;
    int n_stop;
    int32_t stop[kMaxStop];
    int attn_max_splits;   // splits per kv head upper bound (partials layout)
    unsigned long long timeout_ns;
};

struct DecodeLaunch {
    int grid;
    int smem_bytes;
    int seg_vec;  // V: 256*V columns per segment
};

// Validates the configuration against what the fused kernel implements and
// fills the launch shape.  Returns false with a message when unsupported.
bool decode_plan(const DecodeParams& p, int num_sms, DecodeLaunch* out, const char** why);
cudaError_t decode_prepare(const DecodeLaunch& l);  // sets the smem attribute once
cudaError_t launch_decode(const DecodeParams& p, const DecodeLaunch& l, cudaStream_t st);

}  // namespace lc
