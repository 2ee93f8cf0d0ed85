/*
 * oracle.c -- CPU restatement of the reference's PlainJavaKernelFactory decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline /
 * reference arm may load it.  The product path never calls into it.
 *
 * The reference (ArturSkowronski/llama3-java-hat) is Java 26 + Babylon HAT and
 * cannot be compiled here (no JDK).  Every function below restates one Java
 * method with the same floating-point operation order:
 *   - float (binary32) arithmetic, round-to-nearest, no fused multiply-add
 *     (Java never contracts a*b+c); build with -ffp-contract=off, no -ffast-math;
 *   - (float)Math.exp/pow/sin/cos/sqrt are evaluated in double and cast to
 *     float, exactly as the Java expressions do;
 *   - Float.float16ToFloat is the exact IEEE half -> float widening.
 * Row-parallel (OpenMP) evaluation of GEMV rows and attention heads does not
 * change any result: each row / head keeps its own sequential order.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define OR_MAX_LAYERS 64

/* ---------------------------------------------------------------- F16 ---- */

/* Float.float16ToFloat (java.lang.Float): exact widening of an IEEE binary16
 * bit pattern, subnormals, infinities and NaN payloads included. */
float or_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = ((uint32_t)h >> 10) & 0x1fu;
    uint32_t m = (uint32_t)h & 0x3ffu;
    uint32_t bits;
    if (e == 0) {
        /* zero or subnormal: m * 2^-24, exact in binary32 */
        float f = (float)m * 5.9604644775390625e-8f;
        return sign ? -f : f;
    } else if (e == 31) {
        bits = sign | 0x7f800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static float g_f16_table[65536];
static int g_f16_table_ready = 0;

static void f16_table_init(void) {
    if (g_f16_table_ready) return;
    for (uint32_t i = 0; i < 65536u; ++i) g_f16_table[i] = or_f16_to_f32((uint16_t)i);
    g_f16_table_ready = 1;
}

void or_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int or_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* --------------------------------------------------------------- GEMV ---- */

/* GEMV.apply(F32Array matrix, F32Array vector, F32Array result, rows, cols)
 * kernels/GEMV.java:34-43: y[r] = sequential fp32 sum of W[r,c]*x[c]. */
void or_gemv_f32(const float* W, const float* x, float* y, int rows, int cols) {
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const float* w = W + (size_t)r * (size_t)cols;
        float sum = 0.0f;
        for (int c = 0; c < cols; ++c) sum += w[c] * x[c];
        y[r] = sum;
    }
}

/* GEMV.apply(F16Weights matrix, ...) kernels/GEMV.java:66-91 (also the F16Array
 * overload :46-63 and IGEMV defaults kernels/IGEMV.java:34-68, which compute
 * the same values): pass 1 widens the row to float, pass 2 is the sequential
 * fp32 dot product.  Four rows are interleaved for instruction-level
 * parallelism; every row still accumulates in column order. */
void or_gemv_f16(const uint16_t* W, const float* x, float* y, int rows, int cols) {
    f16_table_init();
    const int quads = rows / 4;
    #pragma omp parallel for schedule(static)
    for (int q = 0; q < quads; ++q) {
        const int r = q * 4;
        const uint16_t* w0 = W + (size_t)r * (size_t)cols;
        const uint16_t* w1 = w0 + cols;
        const uint16_t* w2 = w1 + cols;
        const uint16_t* w3 = w2 + cols;
        float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
        for (int c = 0; c < cols; ++c) {
            const float xc = x[c];
            s0 += g_f16_table[w0[c]] * xc;
            s1 += g_f16_table[w1[c]] * xc;
            s2 += g_f16_table[w2[c]] * xc;
            s3 += g_f16_table[w3[c]] * xc;
        }
        y[r] = s0; y[r + 1] = s1; y[r + 2] = s2; y[r + 3] = s3;
    }
    for (int r = quads * 4; r < rows; ++r) {
        const uint16_t* w = W + (size_t)r * (size_t)cols;
        float sum = 0.0f;
        for (int c = 0; c < cols; ++c) sum += g_f16_table[w[c]] * x[c];
        y[r] = sum;
    }
}

/* ------------------------------------------------------------ RMSNorm ---- */

/* RMSNorm.apply(input, weight, size) kernels/RMSNorm.java:35-50, EPSILON=1e-5f
 * (:22).  In place.  `eps` is exposed so model configs can state it; the
 * reference value is 1e-5f. */
void or_rmsnorm_eps(float* x, const float* w, int size, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < size; ++i) {
        float v = x[i];
        ss += v * v;
    }
    float inv_rms = 1.0f / (float)sqrt((double)(ss / (float)size + eps));
    for (int i = 0; i < size; ++i) x[i] = x[i] * inv_rms * w[i];
}

void or_rmsnorm(float* x, const float* w, int size) { or_rmsnorm_eps(x, w, size, 1e-5f); }

/* --------------------------------------------------------------- RoPE ---- */

/* RoPE.apply(vec, pos, numHeads, headDim, theta) kernels/RoPE.java:36-52:
 * interleaved pairs (v[i], v[i+1]), freq = (float)(1/pow(theta, i/headDim)),
 * angle = pos*freq in float, cos/sin in double then cast.  In place. */
void or_rope(float* vec, int pos, int num_heads, int head_dim, float theta) {
    for (int h = 0; h < num_heads; ++h) {
        int off = h * head_dim;
        for (int i = 0; i < head_dim; i += 2) {
            float freq = (float)(1.0 / pow((double)theta, (double)i / (double)head_dim));
            float val = (float)pos * freq;
            float c = (float)cos((double)val);
            float s = (float)sin((double)val);
            float v0 = vec[off + i];
            float v1 = vec[off + i + 1];
            vec[off + i] = v0 * c - v1 * s;
            vec[off + i + 1] = v0 * s + v1 * c;
        }
    }
}

/* --------------------------------------------------------------- SiLU ---- */

/* SiLU.apply(input, size) kernels/SiLU.java:32-40: x / (1 + (float)exp(-x)). */
void or_silu(float* x, int n) {
    for (int i = 0; i < n; ++i) {
        float v = x[i];
        x[i] = v / (1.0f + (float)exp((double)(-v)));
    }
}

/* SiLU followed by TransformerBlock.elementWiseMul (TransformerBlock.java:209-210,
 * :240-244): g[i] = silu(g[i]) * u[i]. */
void or_swiglu(float* g, const float* u, int n) {
    or_silu(g, n);
    for (int i = 0; i < n; ++i) g[i] = g[i] * u[i];
}

/* ------------------------------------------------------------ Softmax ---- */

/* Softmax.applyRow(input, rowOffset, rowSize) kernels/Softmax.java:61-84:
 * max pass, exp-and-sum pass (sequential), multiply by 1/sum.  In place. */
void or_softmax_row(float* x, int row_offset, int row_size) {
    float* r = x + row_offset;
    float mx = -INFINITY;
    for (int i = 0; i < row_size; ++i)
        if (r[i] > mx) mx = r[i];
    float sum = 0.0f;
    for (int i = 0; i < row_size; ++i) {
        float e = (float)exp((double)(r[i] - mx));
        r[i] = e;
        sum += e;
    }
    float inv = 1.0f / sum;
    for (int i = 0; i < row_size; ++i) r[i] = r[i] * inv;
}

/* Softmax.apply(input, size) kernels/Softmax.java:28-51 (same three passes). */
void or_softmax(float* x, int n) { or_softmax_row(x, 0, n); }

/* ---------------------------------------------------------- Attention ---- */

/* Attention.computeScores(q, keys, scores, seqLen, headDim)
 * kernels/Attention.java:32-42: scale = 1/(float)sqrt(headDim) applied after
 * the sequential dot product.  `key_stride` is the distance between positions
 * (the reference's gathered buffer has key_stride == headDim). */
void or_attn_scores_strided(const float* q, const float* keys, int key_stride, float* scores,
                            int seq_len, int head_dim) {
    float scale = 1.0f / (float)sqrt((double)head_dim);
    for (int t = 0; t < seq_len; ++t) {
        const float* k = keys + (size_t)t * (size_t)key_stride;
        float sum = 0.0f;
        for (int i = 0; i < head_dim; ++i) sum += q[i] * k[i];
        scores[t] = sum * scale;
    }
}

void or_attn_scores(const float* q, const float* keys, float* scores, int seq_len, int head_dim) {
    or_attn_scores_strided(q, keys, head_dim, scores, seq_len, head_dim);
}

/* Attention.computeValues(scores, values, out, seqLen, headDim)
 * kernels/Attention.java:53-61: out[i] = sequential sum over t of p[t]*V[t,i]. */
void or_attn_values_strided(const float* p, const float* values, int value_stride, float* out,
                            int seq_len, int head_dim) {
    for (int i = 0; i < head_dim; ++i) {
        float sum = 0.0f;
        for (int t = 0; t < seq_len; ++t) sum += p[t] * values[(size_t)t * (size_t)value_stride + i];
        out[i] = sum;
    }
}

void or_attn_values(const float* p, const float* values, float* out, int seq_len, int head_dim) {
    or_attn_values_strided(p, values, head_dim, out, seq_len, head_dim);
}

/* GQA decode attention for one token, as TransformerBlock.forward runs it
 * (TransformerBlock.java:164-192): for every q head h, kv head = h / (nh/nkv);
 * scores over positions 0..seq_len-1, softmax, weighted values.
 * q: [n_heads][head_dim]; kcache/vcache: position-major
 * [max_seq][n_kv_heads][head_dim] as the reference stores them (:158-162).
 * The reference first copies the head's keys into a contiguous buffer
 * (:175-182); reading them in place with a stride gives the same values. */
void or_gqa_attention(const float* q, const float* kcache, const float* vcache, float* out,
                      int seq_len, int n_heads, int n_kv_heads, int head_dim, float* scratch_scores) {
    const int kv_dim = n_kv_heads * head_dim;
    const int kv_mul = n_heads / n_kv_heads;
    #pragma omp parallel for schedule(static)
    for (int h = 0; h < n_heads; ++h) {
        float* sc = scratch_scores + (size_t)h * (size_t)seq_len;
        int kvh = h / kv_mul;
        or_attn_scores_strided(q + h * head_dim, kcache + kvh * head_dim, kv_dim, sc, seq_len, head_dim);
        or_softmax(sc, seq_len);
        or_attn_values_strided(sc, vcache + kvh * head_dim, kv_dim, out + h * head_dim, seq_len, head_dim);
    }
}

/* ------------------------------------------------------------- argmax ---- */

/* LlamaInference.argmax(values) LlamaInference.java:252-262: first index of
 * the maximum under strict '>' starting from values[0]. */
int or_argmax(const float* v, int n) {
    int idx = 0;
    float mx = v[0];
    for (int i = 1; i < n; ++i) {
        if (v[i] > mx) {
            mx = v[i];
            idx = i;
        }
    }
    return idx;
}

/* -------------------------------------------------------------- model ---- */

/* Host view of the model.  F16 tensors are raw bit patterns, row-major
 * [rows=out][cols=in], as LlamaModel maps them (LlamaModel.java:229-268). */
typedef struct {
    int dim, hidden, n_layers, n_heads, n_kv_heads, head_dim, vocab, max_seq;
    float rope_theta, rms_eps;
    const uint16_t* tok_emb;  /* [vocab][dim] */
    const float* out_norm;    /* [dim] */
    const uint16_t* out_w;    /* [vocab][dim]; == tok_emb when tied */
    const float* attn_norm[OR_MAX_LAYERS];
    const uint16_t* wq[OR_MAX_LAYERS];
    const uint16_t* wk[OR_MAX_LAYERS];
    const uint16_t* wv[OR_MAX_LAYERS];
    const uint16_t* wo[OR_MAX_LAYERS];
    const float* ffn_norm[OR_MAX_LAYERS];
    const uint16_t* wgate[OR_MAX_LAYERS];
    const uint16_t* wup[OR_MAX_LAYERS];
    const uint16_t* wdown[OR_MAX_LAYERS];
    /* WeightStorageMode.F32 (H/WeightStorageMode.java, LlamaInference.java:102-108):
     * when set, tok_emb, out_w and the seven projections point to fp32 data
     * (cast), multiplied by GEMV.apply(F32Array, ...) kernels/GEMV.java:34-43 and
     * embedded by the F32Array case of LlamaInference.java:133-137. */
    int f32;
} or_model;

/* The projection GEMV of the model's storage mode (TransformerBlock.java:219-226). */
static void or_gemv_w(const or_model* m, const uint16_t* W, const float* x, float* y, int rows, int cols) {
    if (m->f32) or_gemv_f32((const float*)(const void*)W, x, y, rows, cols);
    else or_gemv_f16(W, x, y, rows, cols);
}

/* Per-sequence state: the fp32 KV caches LlamaInference allocates
 * (LlamaInference.java:83-89) plus the block scratch buffers
 * (TransformerBlock.java:99-111). */
typedef struct {
    float* x;
    float* logits;
    float* kcache; /* [n_layers][max_seq][kv_dim] */
    float* vcache;
    float *q, *k, *v, *att, *resid, *g, *u, *f, *scores;
} or_state;

or_state* or_state_create(const or_model* m) {
    or_state* s = (or_state*)calloc(1, sizeof(or_state));
    if (!s) return NULL;
    size_t kv_dim = (size_t)m->n_kv_heads * (size_t)m->head_dim;
    size_t cache = (size_t)m->n_layers * (size_t)m->max_seq * kv_dim;
    s->x = (float*)calloc((size_t)m->dim, 4);
    s->logits = (float*)calloc((size_t)m->vocab, 4);
    s->kcache = (float*)calloc(cache, 4);
    s->vcache = (float*)calloc(cache, 4);
    s->q = (float*)calloc((size_t)m->n_heads * (size_t)m->head_dim, 4);
    s->k = (float*)calloc(kv_dim, 4);
    s->v = (float*)calloc(kv_dim, 4);
    s->att = (float*)calloc((size_t)m->n_heads * (size_t)m->head_dim, 4);
    s->resid = (float*)calloc((size_t)m->dim, 4);
    s->g = (float*)calloc((size_t)m->hidden, 4);
    s->u = (float*)calloc((size_t)m->hidden, 4);
    s->f = (float*)calloc((size_t)m->dim, 4);
    s->scores = (float*)calloc((size_t)m->n_heads * (size_t)m->max_seq, 4);
    if (!s->x || !s->logits || !s->kcache || !s->vcache || !s->q || !s->k || !s->v || !s->att ||
        !s->resid || !s->g || !s->u || !s->f || !s->scores) {
        return NULL;
    }
    return s;
}

void or_state_destroy(or_state* s) {
    if (!s) return;
    free(s->x); free(s->logits); free(s->kcache); free(s->vcache); free(s->q); free(s->k);
    free(s->v); free(s->att); free(s->resid); free(s->g); free(s->u); free(s->f); free(s->scores);
    free(s);
}

float* or_state_x(or_state* s) { return s->x; }
float* or_state_logits(or_state* s) { return s->logits; }
float* or_state_kcache(or_state* s) { return s->kcache; }
float* or_state_vcache(or_state* s) { return s->vcache; }

/* TransformerBlock.forward(x, pos, kCache, vCache) TransformerBlock.java:130-217. */
void or_block_forward(const or_model* m, int l, or_state* s, int pos) {
    const int dim = m->dim, hidden = m->hidden, nh = m->n_heads, nkv = m->n_kv_heads, hd = m->head_dim;
    const int kv_dim = nkv * hd;
    float* kc = s->kcache + (size_t)l * (size_t)m->max_seq * (size_t)kv_dim;
    float* vc = s->vcache + (size_t)l * (size_t)m->max_seq * (size_t)kv_dim;

    memcpy(s->resid, s->x, (size_t)dim * 4);                         /* :139 */
    or_rmsnorm_eps(s->x, m->attn_norm[l], dim, m->rms_eps);          /* :142 */
    or_gemv_w(m, m->wq[l], s->x, s->q, nh * hd, dim);                 /* :145 */
    or_gemv_w(m, m->wk[l], s->x, s->k, kv_dim, dim);                  /* :146 */
    or_gemv_w(m, m->wv[l], s->x, s->v, kv_dim, dim);                  /* :147 */
    or_rope(s->q, pos, nh, hd, m->rope_theta);                       /* :150 */
    or_rope(s->k, pos, nkv, hd, m->rope_theta);                      /* :151 */
    memcpy(kc + (size_t)pos * kv_dim, s->k, (size_t)kv_dim * 4);    /* :158-162 */
    memcpy(vc + (size_t)pos * kv_dim, s->v, (size_t)kv_dim * 4);
    or_gqa_attention(s->q, kc, vc, s->att, pos + 1, nh, nkv, hd, s->scores); /* :164-192 */
    or_gemv_w(m, m->wo[l], s->att, s->x, dim, nh * hd);               /* :195 */
    for (int i = 0; i < dim; ++i) s->x[i] = s->x[i] + s->resid[i];   /* :198, add() :234-238 */
    memcpy(s->resid, s->x, (size_t)dim * 4);                         /* :201 */
    or_rmsnorm_eps(s->x, m->ffn_norm[l], dim, m->rms_eps);           /* :204 */
    or_gemv_w(m, m->wgate[l], s->x, s->g, hidden, dim);               /* :207 */
    or_gemv_w(m, m->wup[l], s->x, s->u, hidden, dim);                 /* :208 */
    or_swiglu(s->g, s->u, hidden);                                   /* :209-210 */
    or_gemv_w(m, m->wdown[l], s->g, s->f, dim, hidden);               /* :211 */
    for (int i = 0; i < dim; ++i) s->x[i] = s->resid[i] + s->f[i];   /* :214-216 */
}

/* LlamaInference.forward(token, pos) LlamaInference.java:117-164.  Logits are
 * left in s->logits and copied to `logits_out` when it is not NULL. */
void or_forward(const or_model* m, or_state* s, int token, int pos, float* logits_out) {
    f16_table_init();
    if (m->f32) {
        const float* e = (const float*)(const void*)m->tok_emb + (size_t)token * (size_t)m->dim;
        for (int i = 0; i < m->dim; ++i) s->x[i] = e[i];               /* :133-137 */
    } else {
        const uint16_t* e = m->tok_emb + (size_t)token * (size_t)m->dim;
        for (int i = 0; i < m->dim; ++i) s->x[i] = g_f16_table[e[i]];    /* :122-132 */
    }
    for (int l = 0; l < m->n_layers; ++l) or_block_forward(m, l, s, pos); /* :143-145 */
    or_rmsnorm_eps(s->x, m->out_norm, m->dim, m->rms_eps);           /* :148 */
    or_gemv_w(m, m->out_w, s->x, s->logits, m->vocab, m->dim);         /* :151-156 */
    if (logits_out) memcpy(logits_out, s->logits, (size_t)m->vocab * 4); /* :159-162 */
}

/* LlamaInference.generate(prompt, maxNew, stopTokens) LlamaInference.java:180-217:
 * token-by-token prefill, first token from the last prefill logits, then greedy
 * decode until maxNew tokens or a stop token.  Returns the number generated. */
int or_generate(const or_model* m, or_state* s, const int* prompt, int n_prompt, int max_new,
                const int* stop, int n_stop, int* out) {
    if (n_prompt <= 0 || max_new <= 0) return 0;
    for (int i = 0; i < n_prompt; ++i) or_forward(m, s, prompt[i], i, NULL);
    int next = or_argmax(s->logits, m->vocab);
    out[0] = next;
    int generated = 1;
    for (;;) {
        if (generated >= max_new) break;
        int is_stop = 0;
        for (int j = 0; j < n_stop; ++j) is_stop |= (stop[j] == next);
        if (is_stop) break;
        or_forward(m, s, next, n_prompt + generated - 1, NULL);
        next = or_argmax(s->logits, m->vocab);
        out[generated++] = next;
    }
    return generated;
}
