// lc_api.cu -- the extern "C" surface of libllamacuda.so (include/llamacuda.h).
//
// Host-side runtime: contexts (device + stream + staging pool), host-buffer
// staging for the per-kernel operators, model weight storage and upload,
// sessions (device-resident KV cache and activations) and the launches of the
// fused decode kernel.  Nothing here computes model math on the CPU: every
// operator runs a CUDA kernel, and a missing or failing kernel is an error.
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <string>
#include <thread>
#include <vector>

#include "../../include/llamacuda.h"
#include "lc_attention.cuh"
#include "lc_internal.h"

using namespace lc;

// ------------------------------------------------------------ errors ----

static thread_local std::string g_last_error;

static int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

static int cuda_fail(cudaError_t e, const char* what) {
    return fail(e == cudaErrorMemoryAllocation ? LC_ERR_OUT_OF_MEMORY : LC_ERR_CUDA, "%s: %s (%s)", what,
                cudaGetErrorString(e), cudaGetErrorName(e));
}

#define CK(call, what)                                   \
    do {                                                 \
        cudaError_t _e = (call);                         \
        if (_e != cudaSuccess) return cuda_fail(_e, what); \
    } while (0)

extern "C" int lc_last_error(char* buf, size_t n) {
    if (buf && n) {
        size_t k = g_last_error.size() < n - 1 ? g_last_error.size() : n - 1;
        memcpy(buf, g_last_error.data(), k);
        buf[k] = 0;
    }
    return (int)g_last_error.size();
}

extern "C" int lc_abi_version(void) { return LLAMACUDA_ABI_VERSION; }

namespace lc {
void make_rope_freq(RopeFreq* out, float theta, int head_dim) {
    memset(out, 0, sizeof(*out));
    for (int i = 0; i < head_dim && i / 2 < 256; i += 2)
        out->f[i / 2] = (float)(1.0 / pow((double)theta, (double)i / (double)head_dim));  // RoPE.java:42
}
}  // namespace lc

// ----------------------------------------------------------- context ----

struct lc_context {
    int device = 0;
    int sms = 0;
    cudaStream_t stream = nullptr;
    std::vector<void*> pool;        // staging buffers, grow-only
    std::vector<size_t> pool_bytes;
    int* d_err = nullptr;           // device error word of standalone kernels
    void* attn_scratch = nullptr;
    size_t attn_scratch_bytes = 0;
    void* gemm_scratch = nullptr;   // row scales, pre-split activations, partial sums
    size_t gemm_scratch_bytes = 0;
    bool gemm_ready = false;        // shared-memory attribute of the GEMM kernel set
};

extern "C" int lc_device_count(int* count) {
    if (!count) return fail(LC_ERR_INVALID_ARG, "count is NULL");
    CK(cudaGetDeviceCount(count), "cudaGetDeviceCount");
    return LC_OK;
}

extern "C" int lc_context_create(int device, lc_context** out) {
    if (!out) return fail(LC_ERR_INVALID_ARG, "out is NULL");
    int n = 0;
    CK(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
    if (device < 0 || device >= n) return fail(LC_ERR_INVALID_ARG, "device %d out of range [0,%d)", device, n);
    CK(cudaSetDevice(device), "cudaSetDevice");
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    if (prop.major < 10) return fail(LC_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a", device, prop.major, prop.minor);
    lc_context* c = new lc_context();
    c->device = device;
    c->sms = prop.multiProcessorCount;
    cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&c->d_err, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(c->d_err, 0, sizeof(int));
    if (e != cudaSuccess) {
        delete c;
        return cuda_fail(e, "context setup");
    }
    *out = c;
    return LC_OK;
}

extern "C" int lc_context_destroy(lc_context* c) {
    if (!c) return LC_OK;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    for (void* p : c->pool) cudaFree(p);
    if (c->attn_scratch) cudaFree(c->attn_scratch);
    if (c->gemm_scratch) cudaFree(c->gemm_scratch);
    if (c->d_err) cudaFree(c->d_err);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
    return LC_OK;
}

static int check_device_error(lc_context* c) {
    int h = 0;
    CK(cudaMemcpy(&h, c->d_err, sizeof(int), cudaMemcpyDeviceToHost), "read device error word");
    if (h != 0) {
        cudaMemset(c->d_err, 0, sizeof(int));
        return fail(LC_ERR_TIMEOUT, "device-side wait gave up (code %d)", h);
    }
    return LC_OK;
}

extern "C" int lc_context_synchronize(lc_context* c) {
    if (!c) return fail(LC_ERR_INVALID_ARG, "context is NULL");
    CK(cudaSetDevice(c->device), "cudaSetDevice");
    CK(cudaStreamSynchronize(c->stream), "cudaStreamSynchronize");
    return check_device_error(c);
}

extern "C" void* lc_context_stream(lc_context* c) { return c ? (void*)c->stream : nullptr; }
extern "C" int lc_context_sm_count(lc_context* c) { return c ? c->sms : 0; }

// ------------------------------------------------------------ staging ----
//
// Host pointers are copied into pooled device buffers; device pointers of the
// context's device are used directly.  After the launch, staged outputs are
// copied back and the call synchronises.

namespace {

enum Dir { kIn, kOut, kInOut };

struct Stager {
    lc_context* c;
    int slot = 0;
    bool any_host = false;
    struct Back {
        void* host;
        void* dev;
        size_t bytes;
    };
    std::vector<Back> backs;
    int status = LC_OK;

    explicit Stager(lc_context* ctx) : c(ctx) {}

    bool is_device(const void* p, int* rc) {
        cudaPointerAttributes a;
        cudaError_t e = cudaPointerGetAttributes(&a, p);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) {
            if (a.type == cudaMemoryTypeDevice && a.device != c->device) {
                *rc = fail(LC_ERR_INVALID_ARG, "device pointer belongs to device %d, context is on %d", a.device, c->device);
            }
            return true;
        }
        return false;
    }

    void* buffer(size_t bytes) {
        if ((size_t)slot >= c->pool.size()) {
            c->pool.push_back(nullptr);
            c->pool_bytes.push_back(0);
        }
        if (c->pool_bytes[slot] < bytes) {
            if (c->pool[slot]) cudaFree(c->pool[slot]);
            c->pool[slot] = nullptr;
            c->pool_bytes[slot] = 0;
            size_t want = bytes < 256 ? 256 : bytes;
            if (cudaMalloc(&c->pool[slot], want) != cudaSuccess) {
                cudaGetLastError();
                return nullptr;
            }
            c->pool_bytes[slot] = want;
        }
        return c->pool[slot++];
    }

    // Returns the device pointer to hand to the kernel, or nullptr on error
    // (status set).
    void* arg(const void* p, size_t bytes, Dir d) {
        if (status != LC_OK) return nullptr;
        if (!p) {
            status = fail(LC_ERR_INVALID_ARG, "NULL buffer");
            return nullptr;
        }
        int rc = LC_OK;
        if (is_device(p, &rc)) {
            if (rc != LC_OK) status = rc;
            return rc == LC_OK ? const_cast<void*>(p) : nullptr;
        }
        any_host = true;
        void* dev = buffer(bytes);
        if (!dev) {
            status = fail(LC_ERR_OUT_OF_MEMORY, "staging buffer of %zu bytes", bytes);
            return nullptr;
        }
        if (d != kOut && bytes) {
            cudaError_t e = cudaMemcpyAsync(dev, p, bytes, cudaMemcpyHostToDevice, c->stream);
            if (e != cudaSuccess) {
                status = cuda_fail(e, "copy in");
                return nullptr;
            }
        }
        if (d != kIn) backs.push_back({const_cast<void*>(p), dev, bytes});
        return dev;
    }

    int finish(cudaError_t launch) {
        if (status != LC_OK) return status;
        if (launch != cudaSuccess) return cuda_fail(launch, "kernel launch");
        for (auto& b : backs) {
            if (!b.bytes) continue;
            cudaError_t e = cudaMemcpyAsync(b.host, b.dev, b.bytes, cudaMemcpyDeviceToHost, c->stream);
            if (e != cudaSuccess) return cuda_fail(e, "copy out");
        }
        if (any_host) {
            cudaError_t e = cudaStreamSynchronize(c->stream);
            if (e != cudaSuccess) return cuda_fail(e, "synchronize");
            return check_device_error(c);
        }
        return LC_OK;
    }
};

}  // namespace

#define CTX_CHECK(c)                                                        \
    do {                                                                    \
        if (!(c)) return fail(LC_ERR_INVALID_ARG, "context is NULL");       \
        cudaError_t _e = cudaSetDevice((c)->device);                        \
        if (_e != cudaSuccess) return cuda_fail(_e, "cudaSetDevice");       \
    } while (0)

// ------------------------------------------------------- per-kernel ops ----

extern "C" int lc_gemv_f16(lc_context* c, const uint16_t* W, const float* x, float* y, int rows, int cols) {
    CTX_CHECK(c);
    if (rows <= 0 || cols <= 0) return fail(LC_ERR_INVALID_ARG, "rows=%d cols=%d", rows, cols);
    Stager s(c);
    auto* dW = (const uint16_t*)s.arg(W, (size_t)rows * cols * 2, kIn);
    auto* dx = (const float*)s.arg(x, (size_t)cols * 4, kIn);
    auto* dy = (float*)s.arg(y, (size_t)rows * 4, kOut);
    if (s.status != LC_OK) return s.status;
    cudaError_t e;
    if (stream_gemv_supported(dW, dx, rows, cols)) {
        e = launch_stream_gemv(dW, dx, dy, rows, cols, c->sms, c->d_err, c->stream);
    } else {
        launch_gemv_generic_f16(dW, dx, dy, rows, cols, c->stream);
        e = cudaGetLastError();
    }
    return s.finish(e);
}

extern "C" int lc_gemv_f32(lc_context* c, const float* W, const float* x, float* y, int rows, int cols) {
    CTX_CHECK(c);
    if (rows <= 0 || cols <= 0) return fail(LC_ERR_INVALID_ARG, "rows=%d cols=%d", rows, cols);
    Stager s(c);
    auto* dW = (const float*)s.arg(W, (size_t)rows * cols * 4, kIn);
    auto* dx = (const float*)s.arg(x, (size_t)cols * 4, kIn);
    auto* dy = (float*)s.arg(y, (size_t)rows * 4, kOut);
    if (s.status != LC_OK) return s.status;
    launch_gemv_generic_f32(dW, dx, dy, rows, cols, c->stream);
    return s.finish(cudaGetLastError());
}

extern "C" int lc_gemv_f16_batched(lc_context* c, const uint16_t* W, const float* X, float* Y, int rows, int cols,
                                   int batch) {
    CTX_CHECK(c);
    if (rows <= 0 || cols <= 0 || batch <= 0) return fail(LC_ERR_INVALID_ARG, "rows=%d cols=%d batch=%d", rows, cols, batch);
    Stager s(c);
    auto* dW = (const uint16_t*)s.arg(W, (size_t)rows * cols * 2, kIn);
    auto* dX = (const float*)s.arg(X, (size_t)batch * cols * 4, kIn);
    auto* dY = (float*)s.arg(Y, (size_t)batch * rows * 4, kOut);
    if (s.status != LC_OK) return s.status;
    launch_gemv_batched_f16(dW, dX, dY, rows, cols, batch, c->stream);
    return s.finish(cudaGetLastError());
}

// Tensor-core batched product on tiled weights (lc_gemm.cu).
extern "C" int lc_weights_tile(lc_context* c, const uint16_t* W, uint16_t* Wt, int rows, int cols) {
    CTX_CHECK(c);
    if (rows <= 0 || cols <= 0 || rows % 8 || gemm_tile_width(cols) == 0)
        return fail(LC_ERR_INVALID_ARG, "rows=%d cols=%d (rows %% 8 == 0 and cols %% 64 == 0 required)", rows, cols);
    Stager s(c);
    auto* dW = (const __half*)s.arg(W, (size_t)rows * cols * 2, kIn);
    auto* dT = (__half*)s.arg(Wt, (size_t)rows * cols * 2, kOut);
    if (s.status != LC_OK) return s.status;
    if (((uintptr_t)dW | (uintptr_t)dT) & 15) return fail(LC_ERR_INVALID_ARG, "W and Wt must be 16-byte aligned");
    return s.finish(launch_tile_rows(dW, dT, rows, cols, gemm_tile_width(cols), 0, 1, c->stream));
}

static int gemm_tiled(lc_context* c, const uint16_t* Wt, const float* X, float* Y, int rows, int cols, int batch,
                      int idx_offset, uint64_t* keys) {
    CTX_CHECK(c);
    if (rows <= 0 || cols <= 0 || batch <= 0 || batch > kGemmMaxRows || rows % 16 || gemm_tile_width(cols) == 0)
        return fail(LC_ERR_INVALID_ARG, "rows=%d cols=%d batch=%d (rows %% 16 == 0, cols %% 64 == 0, batch 1..%d)",
                    rows, cols, batch, kGemmMaxRows);
    GemmParams g;
    memset(&g, 0, sizeof(g));
    g.N = rows;
    g.K = cols;
    g.cbw = gemm_tile_width(cols);
    g.B = batch;
    if (!gemm_plan(&g, c->sms)) return fail(LC_ERR_INVALID_ARG, "unsupported GEMM shape %d x %d", rows, cols);
    Stager s(c);
    auto* dW = (const __half*)s.arg(Wt, (size_t)rows * cols * 2, kIn);
    auto* dX = (const float*)s.arg(X, (size_t)batch * cols * 4, kIn);
    auto* dY = Y ? (float*)s.arg(Y, (size_t)batch * rows * 4, kOut) : nullptr;
    auto* dK = keys ? (unsigned long long*)s.arg(keys, (size_t)batch * 8, kOut) : nullptr;
    if (s.status != LC_OK) return s.status;
    if (((uintptr_t)dW | (uintptr_t)dX | (uintptr_t)dY) & 15) return fail(LC_ERR_INVALID_ARG, "buffers must be 16-byte aligned");
    const size_t off_a = ((size_t)batch * 4 + 255) / 256 * 256;  // row scales first
    const size_t off_p = off_a + ((gemm_split_bytes(batch, cols) + 255) / 256) * 256;
    const size_t need = off_p + gemm_part_bytes(g);
    if (c->gemm_scratch_bytes < need) {
        if (c->gemm_scratch) cudaFree(c->gemm_scratch);
        c->gemm_scratch = nullptr;
        c->gemm_scratch_bytes = 0;
        CK(cudaMalloc(&c->gemm_scratch, need), "GEMM scratch");
        CK(cudaMemset(c->gemm_scratch, 0, need), "GEMM scratch");
        c->gemm_scratch_bytes = need;
    }
    if (!c->gemm_ready) {
        CK(gemm_prepare(), "GEMM shared-memory attribute");
        c->gemm_ready = true;
    }
    uint8_t* base = (uint8_t*)c->gemm_scratch;
    float* unscale = (float*)base;
    uint8_t* As = base + off_a;
    g.W = dW;
    g.As = As;
    g.unscale = unscale;
    g.part = (float*)(base + off_p);
    if (dK) {
        g.op = kGemmLogits;
        g.logits = dY;
        g.ldl = rows;
        g.best = dK;
        g.idx_offset = idx_offset;
    } else {
        g.op = kGemmStore;
        g.y = dY;
        g.ldy = rows;
    }
    g.n_valid = rows;
    g.err = c->d_err;
    g.timeout_ns = 2000000000ull;
    CUtensorMap wmap, amap;
    if (gemm_make_wmap(&wmap, g) != cudaSuccess || gemm_make_amap(&amap, g) != cudaSuccess)
        return fail(LC_ERR_CUDA, "tensor map encoding failed");
    cudaError_t e = dK ? cudaMemsetAsync(dK, 0, (size_t)batch * 8, c->stream) : cudaSuccess;
    // Programmatic dependent launches: each kernel waits for its predecessor's
    // completion before touching its data (the product streams its weights
    // before that wait), so back-to-back calls overlap launch latency.
    if (e == cudaSuccess) e = launch_gemm_split(dX, cols, cols, batch, As, unscale, c->stream, true);
    if (e == cudaSuccess) e = launch_gemm(g, wmap, amap, c->sms, c->stream, true);
    return s.finish(e);
}

extern "C" int lc_gemm_f16_tiled(lc_context* c, const uint16_t* Wt, const float* X, float* Y, int rows, int cols,
                                 int batch) {
    if (!Y) return fail(LC_ERR_INVALID_ARG, "NULL buffer");
    return gemm_tiled(c, Wt, X, Y, rows, cols, batch, 0, nullptr);
}

extern "C" int lc_gemm_f16_tiled_argmax(lc_context* c, const uint16_t* Wt, const float* X, float* Y, int rows,
                                        int cols, int batch, int32_t index_offset, uint64_t* keys) {
    if (!keys) return fail(LC_ERR_INVALID_ARG, "NULL keys");
    if (index_offset < 0) return fail(LC_ERR_INVALID_ARG, "index_offset %d", index_offset);
    return gemm_tiled(c, Wt, X, Y, rows, cols, batch, index_offset, keys);
}

extern "C" int lc_rmsnorm_rows(lc_context* c, float* x, const float* w, int rows, int width, float eps) {
    CTX_CHECK(c);
    if (rows <= 0 || width <= 0) return fail(LC_ERR_INVALID_ARG, "rows=%d width=%d", rows, width);
    Stager s(c);
    auto* dx = (float*)s.arg(x, (size_t)rows * width * 4, kInOut);
    auto* dw = (const float*)s.arg(w, (size_t)width * 4, kIn);
    if (s.status != LC_OK) return s.status;
    launch_rmsnorm_rows(dx, dw, rows, width, eps, c->stream);
    return s.finish(cudaGetLastError());
}

extern "C" int lc_rmsnorm(lc_context* c, float* x, const float* w, int size) {
    return lc_rmsnorm_rows(c, x, w, 1, size, 1e-5f);  // RMSNorm.java:22
}

extern "C" int lc_rope_rows(lc_context* c, float* vec, const int32_t* pos, int rows, int num_heads, int head_dim,
                            float theta) {
    CTX_CHECK(c);
    if (rows <= 0 || num_heads <= 0 || head_dim <= 0 || (head_dim & 1) || head_dim > 512)
        return fail(LC_ERR_INVALID_ARG, "rows=%d num_heads=%d head_dim=%d", rows, num_heads, head_dim);
    Stager s(c);
    auto* dv = (float*)s.arg(vec, (size_t)rows * num_heads * head_dim * 4, kInOut);
    auto* dp = (const int32_t*)s.arg(pos, (size_t)rows * 4, kIn);
    if (s.status != LC_OK) return s.status;
    RopeFreq fq;
    make_rope_freq(&fq, theta, head_dim);
    launch_rope_rows(dv, dp, rows, num_heads, head_dim, fq, c->stream);
    return s.finish(cudaGetLastError());
}

extern "C" int lc_rope(lc_context* c, float* vec, int pos, int num_heads, int head_dim, float theta) {
    CTX_CHECK(c);
    if (num_heads <= 0 || head_dim <= 0 || (head_dim & 1) || head_dim > 512)
        return fail(LC_ERR_INVALID_ARG, "num_heads=%d head_dim=%d", num_heads, head_dim);
    // The position travels as a one-element array through the same kernel.
    Stager s(c);
    auto* dv = (float*)s.arg(vec, (size_t)num_heads * head_dim * 4, kInOut);
    int32_t hp = pos;
    auto* dp = (const int32_t*)s.arg(&hp, 4, kIn);
    if (s.status != LC_OK) return s.status;
    RopeFreq fq;
    make_rope_freq(&fq, theta, head_dim);
    launch_rope_rows(dv, dp, 1, num_heads, head_dim, fq, c->stream);
    // hp is host memory, so the call is staged and finish() synchronises
    // before this frame (and hp) goes away.
    return s.finish(cudaGetLastError());
}

extern "C" int lc_silu(lc_context* c, float* x, int size) {
    CTX_CHECK(c);
    if (size <= 0) return fail(LC_ERR_INVALID_ARG, "size=%d", size);
    Stager s(c);
    auto* dx = (float*)s.arg(x, (size_t)size * 4, kInOut);
    if (s.status != LC_OK) return s.status;
    launch_silu(dx, size, c->stream);
    return s.finish(cudaGetLastError());
}

extern "C" int lc_swiglu(lc_context* c, float* g, const float* u, int n) {
    CTX_CHECK(c);
    if (n <= 0) return fail(LC_ERR_INVALID_ARG, "n=%d", n);
    Stager s(c);
    auto* dg = (float*)s.arg(g, (size_t)n * 4, kInOut);
    auto* du = (const float*)s.arg(u, (size_t)n * 4, kIn);
    if (s.status != LC_OK) return s.status;
    launch_swiglu(dg, du, n, c->stream);
    return s.finish(cudaGetLastError());
}

extern "C" int lc_softmax_rows(lc_context* c, float* x, int rows, int width) {
    CTX_CHECK(c);
    if (rows <= 0 || width <= 0) return fail(LC_ERR_INVALID_ARG, "rows=%d width=%d", rows, width);
    Stager s(c);
    auto* dx = (float*)s.arg(x, (size_t)rows * width * 4, kInOut);
    if (s.status != LC_OK) return s.status;
    launch_softmax_rows(dx, rows, width, c->stream);
    return s.finish(cudaGetLastError());
}

extern "C" int lc_softmax(lc_context* c, float* x, int size) { return lc_softmax_rows(c, x, 1, size); }

extern "C" int lc_softmax_row(lc_context* c, float* x, int row_offset, int row_size) {
    if (!x || row_offset < 0) return fail(LC_ERR_INVALID_ARG, "x=%p row_offset=%d", (void*)x, row_offset);
    return lc_softmax_rows(c, x + row_offset, 1, row_size);
}

extern "C" int lc_attn_scores(lc_context* c, const float* q, const float* keys, float* scores, int seq_len,
                              int head_dim) {
    CTX_CHECK(c);
    if (seq_len <= 0 || head_dim <= 0) return fail(LC_ERR_INVALID_ARG, "seq_len=%d head_dim=%d", seq_len, head_dim);
    Stager s(c);
    auto* dq = (const float*)s.arg(q, (size_t)head_dim * 4, kIn);
    auto* dk = (const float*)s.arg(keys, (size_t)seq_len * head_dim * 4, kIn);
    auto* ds = (float*)s.arg(scores, (size_t)seq_len * 4, kOut);
    if (s.status != LC_OK) return s.status;
    const float scale = 1.0f / (float)sqrt((double)head_dim);  // Attention.java:33
    launch_attn_scores(dq, dk, ds, seq_len, head_dim, scale, c->stream);
    return s.finish(cudaGetLastError());
}

extern "C" int lc_attn_values(lc_context* c, const float* p, const float* values, float* out, int seq_len,
                              int head_dim) {
    CTX_CHECK(c);
    if (seq_len <= 0 || head_dim <= 0) return fail(LC_ERR_INVALID_ARG, "seq_len=%d head_dim=%d", seq_len, head_dim);
    Stager s(c);
    auto* dp = (const float*)s.arg(p, (size_t)seq_len * 4, kIn);
    auto* dv = (const float*)s.arg(values, (size_t)seq_len * head_dim * 4, kIn);
    auto* dout = (float*)s.arg(out, (size_t)head_dim * 4, kOut);
    if (s.status != LC_OK) return s.status;
    launch_attn_values(dp, dv, dout, seq_len, head_dim, c->stream);
    return s.finish(cudaGetLastError());
}

extern "C" int lc_attention_decode(lc_context* c, const float* q, const float* k, const float* v, float* out,
                                   const int32_t* seq_len, int batch, int n_heads, int n_kv_heads, int head_dim,
                                   int64_t seq_stride, int64_t head_stride, int64_t pos_stride) {
    CTX_CHECK(c);
    if (batch <= 0 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads)
        return fail(LC_ERR_INVALID_ARG, "batch=%d n_heads=%d n_kv_heads=%d", batch, n_heads, n_kv_heads);
    if (head_dim != kAttnHeadDim) return fail(LC_ERR_UNSUPPORTED, "fused attention implements head_dim 64, got %d", head_dim);
    if (n_heads / n_kv_heads > 8) return fail(LC_ERR_UNSUPPORTED, "at most 8 query heads per kv head");
    if ((seq_stride | head_stride | pos_stride) & 3) return fail(LC_ERR_INVALID_ARG, "strides must be multiples of 4 floats");
    // Lengths are needed on the host to size the split plan.
    std::vector<int32_t> lens(batch);
    {
        cudaError_t e = cudaMemcpy(lens.data(), seq_len, (size_t)batch * 4, cudaMemcpyDefault);
        if (e != cudaSuccess) return cuda_fail(e, "read seq_len");
    }
    int max_len = 0;
    for (int b = 0; b < batch; ++b) {
        if (lens[b] < 0) return fail(LC_ERR_INVALID_ARG, "seq_len[%d] = %d", b, lens[b]);
        if (lens[b] > max_len) max_len = lens[b];
    }
    if (max_len < 1) max_len = 1;
    // Extent of the K/V buffers in floats.
    const size_t kv_floats = (size_t)(batch - 1) * seq_stride + (size_t)(n_kv_heads - 1) * head_stride +
                             (size_t)(max_len - 1) * pos_stride + head_dim;
    Stager s(c);
    auto* dq = (const float*)s.arg(q, (size_t)batch * n_heads * head_dim * 4, kIn);
    auto* dk = (const float*)s.arg(k, kv_floats * 4, kIn);
    auto* dv = (const float*)s.arg(v, kv_floats * 4, kIn);
    auto* dout = (float*)s.arg(out, (size_t)batch * n_heads * head_dim * 4, kOut);
    auto* dl = (const int32_t*)s.arg(lens.data(), (size_t)batch * 4, kIn);
    if (s.status != LC_OK) return s.status;
    if (((uintptr_t)dq | (uintptr_t)dk | (uintptr_t)dv) & 15) return fail(LC_ERR_INVALID_ARG, "q/k/v must be 16-byte aligned");
    AttnPlan plan = plan_attention(batch, n_heads, n_kv_heads, head_dim, max_len, c->sms);
    const size_t need = attention_scratch_bytes(plan);
    if (c->attn_scratch_bytes < need) {
        if (c->attn_scratch) cudaFree(c->attn_scratch);
        c->attn_scratch = nullptr;
        c->attn_scratch_bytes = 0;
        CK(cudaMalloc(&c->attn_scratch, need), "attention scratch");
        c->attn_scratch_bytes = need;
    }
    cudaError_t e = launch_attention_decode(plan, dq, dk, dv, dout, dl, seq_stride, head_stride, pos_stride,
                                            c->attn_scratch, c->stream);
    // `lens` is host memory, so the call is staged and finish() synchronises.
    return s.finish(e);
}

extern "C" int lc_attention_decode_maxlen(lc_context* c, const float* q, const float* k, const float* v, float* out,
                                          const int32_t* seq_len, int batch, int n_heads, int n_kv_heads,
                                          int head_dim, int64_t seq_stride, int64_t head_stride, int64_t pos_stride,
                                          int max_len) {
    CTX_CHECK(c);
    if (batch <= 0 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || max_len < 1)
        return fail(LC_ERR_INVALID_ARG, "batch=%d n_heads=%d n_kv_heads=%d max_len=%d", batch, n_heads, n_kv_heads, max_len);
    if (head_dim != kAttnHeadDim) return fail(LC_ERR_UNSUPPORTED, "fused attention implements head_dim 64, got %d", head_dim);
    if (n_heads / n_kv_heads > 8) return fail(LC_ERR_UNSUPPORTED, "at most 8 query heads per kv head");
    if ((seq_stride | head_stride | pos_stride) & 3) return fail(LC_ERR_INVALID_ARG, "strides must be multiples of 4 floats");
    const size_t kv_floats = (size_t)(batch - 1) * seq_stride + (size_t)(n_kv_heads - 1) * head_stride +
                             (size_t)(max_len - 1) * pos_stride + head_dim;
    Stager s(c);
    auto* dq = (const float*)s.arg(q, (size_t)batch * n_heads * head_dim * 4, kIn);
    auto* dk = (const float*)s.arg(k, kv_floats * 4, kIn);
    auto* dv = (const float*)s.arg(v, kv_floats * 4, kIn);
    auto* dout = (float*)s.arg(out, (size_t)batch * n_heads * head_dim * 4, kOut);
    auto* dl = (const int32_t*)s.arg(seq_len, (size_t)batch * 4, kIn);
    if (s.status != LC_OK) return s.status;
    if (((uintptr_t)dq | (uintptr_t)dk | (uintptr_t)dv) & 15) return fail(LC_ERR_INVALID_ARG, "q/k/v must be 16-byte aligned");
    AttnPlan plan = plan_attention(batch, n_heads, n_kv_heads, head_dim, max_len, c->sms);
    const size_t need = attention_scratch_bytes(plan);
    if (c->attn_scratch_bytes < need) {
        if (c->attn_scratch) cudaFree(c->attn_scratch);
        c->attn_scratch = nullptr;
        c->attn_scratch_bytes = 0;
        CK(cudaMalloc(&c->attn_scratch, need), "attention scratch");
        c->attn_scratch_bytes = need;
    }
    return s.finish(launch_attention_decode(plan, dq, dk, dv, dout, dl, seq_stride, head_stride, pos_stride,
                                            c->attn_scratch, c->stream));
}

extern "C" int lc_argmax(lc_context* c, const float* values, int n, int32_t* out_index) {
    CTX_CHECK(c);
    if (n <= 0 || !out_index) return fail(LC_ERR_INVALID_ARG, "n=%d out=%p", n, (void*)out_index);
    Stager s(c);
    auto* dv = (const float*)s.arg(values, (size_t)n * 4, kIn);
    auto* di = (int32_t*)s.arg(out_index, 4, kOut);
    if (s.status != LC_OK) return s.status;
    launch_argmax(dv, n, di, c->stream);
    return s.finish(cudaGetLastError());
}

// -------------------------------------------------------------- model ----

extern "C" void lc_config_llama32_1b(lc_config* o) {
    if (!o) return;
    memset(o, 0, sizeof(*o));
    o->dim = 2048;
    o->hidden = 8192;
    o->n_layers = 16;
    o->n_heads = 32;
    o->n_kv_heads = 8;
    o->head_dim = 64;
    o->vocab = 128256;
    o->max_seq = 2048;
    o->rope_theta = 500000.0f;
    o->rms_eps = 1e-5f;
}

struct LayerStore {
    __half *wqkv, *wo, *wgu, *wdown;
    float *attn_norm, *ffn_norm;
};

struct lc_model {
    lc_context* ctx = nullptr;
    lc_config cfg;
    void* arena = nullptr;  // all weights, one allocation
    size_t arena_bytes = 0;
    __half* tok_emb = nullptr;   // row-major (embedding lookup)
    __half* lm_tiled = nullptr;  // tiled lm_head: output.weight, or tok_emb when tied
    float* out_norm = nullptr;
    void* staging = nullptr;     // device copy of a host matrix before tiling
    size_t staging_bytes = 0;
    std::vector<LayerStore> layers;
    LayerW* d_layers = nullptr;
    std::vector<uint8_t> have;  // received flags
    bool has_output = false;
    bool finalized = false;
    RopeFreq rope;
    float2* d_rope_cs = nullptr;  // [max_seq][head_dim / 2] (sin, cos) of the RoPE angles
    DecodeLaunch launch;
    int l2_prefetch_tiles = -1;   // producer L2 prefetch window (tiles); -1: the default
    // WeightStorageMode.F32: fp32 embedding and projections (row-major), the
    // fused kernel's tiled F16 weights are not kept.
    bool w32 = false;
    float* tok32 = nullptr;       // [vocab][dim]
    float* out32 = nullptr;       // output.weight, own allocation (tied: the embedding)
    std::vector<F32Layer> l32;
    uint32_t* d_sched = nullptr;  // producer tile schedule (decode_build_schedule)
    int* d_sched_n = nullptr;
    int sched_stride = 0;
};

static int validate_config(const lc_config* c) {
    if (!c) return fail(LC_ERR_INVALID_ARG, "config is NULL");
    if (c->dim <= 0 || c->hidden <= 0 || c->n_layers <= 0 || c->n_heads <= 0 || c->n_kv_heads <= 0 ||
        c->head_dim <= 0 || c->vocab <= 1 || c->max_seq <= 0)
        return fail(LC_ERR_INVALID_ARG, "config has a non-positive dimension");
    if (c->n_heads % c->n_kv_heads) return fail(LC_ERR_INVALID_ARG, "n_heads %% n_kv_heads != 0");
    if (c->weight_mode != LC_WEIGHTS_F16 && c->weight_mode != LC_WEIGHTS_F32)
        return fail(LC_ERR_INVALID_ARG, "Unknown weight storage mode %d (F16 = 0, F32 = 1)", c->weight_mode);
    const char* why = nullptr;
    if (c->weight_mode == LC_WEIGHTS_F32 && !f32_supported(c->dim, c->hidden, c->n_heads * c->head_dim, &why))
        return fail(LC_ERR_UNSUPPORTED, "%s", why);
    return LC_OK;
}

// Tensor slots: 0 tok_emb, 1 output, 2 output_norm, then 9 per layer.
enum { kTokEmb = 0, kOutput = 1, kOutNorm = 2, kLayerBase = 3 };
enum { kAttnNorm, kQ, kK, kV, kO, kFfnNorm, kGate, kUp, kDown, kPerLayer };

extern "C" int lc_model_create(lc_context* ctx, const lc_config* cfg, lc_model** out) {
    CTX_CHECK(ctx);
    if (!out) return fail(LC_ERR_INVALID_ARG, "out is NULL");
    int rc = validate_config(cfg);
    if (rc) return rc;
    lc_model* m = new lc_model();
    m->ctx = ctx;
    m->cfg = *cfg;
    const lc_config& c = *cfg;
    const size_t qdim = (size_t)c.n_heads * c.head_dim, kvd = (size_t)c.n_kv_heads * c.head_dim;
    auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
    // Bytes per projection / embedding element: F16, or fp32 in F32 mode.
    const bool w32 = c.weight_mode == LC_WEIGHTS_F32;
    const size_t eb = w32 ? 4 : 2;
    m->w32 = w32;
    size_t per_layer = al((qdim + 2 * kvd) * c.dim * eb) + al((size_t)c.dim * qdim * eb) +
                       al((size_t)2 * c.hidden * c.dim * eb) + al((size_t)c.dim * c.hidden * eb) + 2 * al((size_t)c.dim * 4);
    const size_t vocab8 = ((size_t)c.vocab + 7) / 8 * 8;
    size_t total = al((size_t)c.vocab * c.dim * eb) + (w32 ? 0 : al(vocab8 * c.dim * 2)) + al((size_t)c.dim * 4) +
                   per_layer * c.n_layers;
    cudaError_t e = cudaMalloc(&m->arena, total);
    if (e != cudaSuccess) {
        delete m;
        return cuda_fail(e, "weight arena");
    }
    m->arena_bytes = total;
    uint8_t* p = (uint8_t*)m->arena;
    auto take = [&](size_t b) {
        uint8_t* r = p;
        p += al(b);
        return r;
    };
    m->layers.resize(c.n_layers);
    if (w32) {
        m->tok32 = (float*)take((size_t)c.vocab * c.dim * 4);
        m->out_norm = (float*)take((size_t)c.dim * 4);
        m->l32.resize(c.n_layers);
        for (int l = 0; l < c.n_layers; ++l) {
            LayerStore& L = m->layers[l];
            F32Layer& F = m->l32[l];
            F.wqkv = (float*)take((qdim + 2 * kvd) * c.dim * 4);
            F.wo = (float*)take((size_t)c.dim * qdim * 4);
            F.wgu = (float*)take((size_t)2 * c.hidden * c.dim * 4);
            F.wdown = (float*)take((size_t)c.dim * c.hidden * 4);
            L.wqkv = L.wo = L.wgu = L.wdown = nullptr;
            F.attn_norm = L.attn_norm = (float*)take((size_t)c.dim * 4);
            F.ffn_norm = L.ffn_norm = (float*)take((size_t)c.dim * 4);
        }
    } else {
        m->tok_emb = (__half*)take((size_t)c.vocab * c.dim * 2);
        m->lm_tiled = (__half*)take(vocab8 * c.dim * 2);
        m->out_norm = (float*)take((size_t)c.dim * 4);
        for (int l = 0; l < c.n_layers; ++l) {
            LayerStore& L = m->layers[l];
            L.wqkv = (__half*)take((qdim + 2 * kvd) * c.dim * 2);
            L.wo = (__half*)take((size_t)c.dim * qdim * 2);
            L.wgu = (__half*)take((size_t)2 * c.hidden * c.dim * 2);
            L.wdown = (__half*)take((size_t)c.dim * c.hidden * 2);
            L.attn_norm = (float*)take((size_t)c.dim * 4);
            L.ffn_norm = (float*)take((size_t)c.dim * 4);
        }
    }
    m->have.assign(kLayerBase + kPerLayer * c.n_layers, 0);
    // Padding rows of the tiled lm_head must read as zeros.
    e = w32 ? cudaSuccess : cudaMemset(m->lm_tiled, 0, vocab8 * c.dim * 2);
    if (e != cudaSuccess) {
        lc_model_destroy(m);
        return cuda_fail(e, "weight arena");
    }
    *out = m;
    return LC_OK;
}

extern "C" int lc_model_get_config(const lc_model* m, lc_config* out) {
    if (!m || !out) return fail(LC_ERR_INVALID_ARG, "NULL argument");
    *out = m->cfg;
    return LC_OK;
}

extern "C" int lc_model_destroy(lc_model* m) {
    if (!m) return LC_OK;
    cudaSetDevice(m->ctx->device);
    if (m->arena) cudaFree(m->arena);
    if (m->staging) cudaFree(m->staging);
    if (m->d_layers) cudaFree(m->d_layers);
    if (m->d_sched) cudaFree(m->d_sched);
    if (m->d_sched_n) cudaFree(m->d_sched_n);
    if (m->out32) cudaFree(m->out32);
    if (m->d_rope_cs) cudaFree(m->d_rope_cs);
    delete m;
    return LC_OK;
}

static float f16_bits_to_float(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16, e = ((uint32_t)h >> 10) & 0x1fu, mant = (uint32_t)h & 0x3ffu;
    if (e == 0) {
        float f = (float)mant * 5.9604644775390625e-8f;
        return sign ? -f : f;
    }
    uint32_t bits = (e == 31) ? (sign | 0x7f800000u | (mant << 13)) : (sign | ((e + 112u) << 23) | (mant << 13));
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

// Copies `bytes` from a host or device source into device memory.
static int put(void* dst, const void* src, size_t bytes, cudaStream_t st) {
    CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, st), "tensor upload");
    return LC_OK;
}

// Row-major F16 matrix [rows][cols] from a host or device source into the
// tiled layout of a destination matrix with `cols` columns (lc_internal.h):
// source row r becomes destination row row0 + r * row_step.
static int put_tiled(lc_model* m, __half* dst, const void* data, int rows, int cols, int row0, int row_step) {
    cudaStream_t st = m->ctx->stream;
    const size_t bytes = (size_t)rows * cols * 2;
    cudaPointerAttributes a;
    const __half* src = (const __half*)data;
    const bool on_device = cudaPointerGetAttributes(&a, data) == cudaSuccess && a.type == cudaMemoryTypeDevice &&
                           a.device == m->ctx->device && ((uintptr_t)data & 15) == 0;
    cudaGetLastError();
    if (!on_device) {
        if (m->staging_bytes < bytes) {
            if (m->staging) cudaFree(m->staging);
            m->staging = nullptr;
            m->staging_bytes = 0;
            CK(cudaMalloc(&m->staging, bytes), "weight staging buffer");
            m->staging_bytes = bytes;
        }
        CK(cudaMemcpyAsync(m->staging, data, bytes, cudaMemcpyDefault, st), "tensor upload");
        src = (const __half*)m->staging;
    }
    CK(launch_tile_rows(src, dst, rows, cols, m->cfg.dim, row0, row_step, st), "weight tiling");
    return LC_OK;
}

// F32 storage mode: n elements of a host or device F32 (dtype 0) or F16
// (dtype 1, widened exactly like LlamaModel.mapTensor, H/LlamaModel.java:159-164)
// tensor into dst.
static int put32(lc_model* m, float* dst, const void* data, int64_t n, int dtype) {
    cudaStream_t st = m->ctx->stream;
    if (dtype == 0) {
        CK(cudaMemcpyAsync(dst, data, (size_t)n * 4, cudaMemcpyDefault, st), "tensor upload");
        return LC_OK;
    }
    const size_t bytes = (size_t)n * 2;
    if (m->staging_bytes < bytes) {
        if (m->staging) cudaFree(m->staging);
        m->staging = nullptr;
        m->staging_bytes = 0;
        CK(cudaMalloc(&m->staging, bytes), "weight staging buffer");
        m->staging_bytes = bytes;
    }
    CK(cudaMemcpyAsync(m->staging, data, bytes, cudaMemcpyDefault, st), "tensor upload");
    CK(launch_f16_to_f32((const __half*)m->staging, dst, n, st), "F16 to F32");
    return LC_OK;
}

static int upload_norm(float* dst, const void* data, int64_t n, int dtype, cudaStream_t st) {
    if (dtype == 0) return put(dst, data, (size_t)n * 4, st);
    // F16 norm weights are widened like LlamaModel.mapTensor (H/LlamaModel.java:159-164).
    std::vector<uint16_t> h(n);
    CK(cudaMemcpy(h.data(), data, (size_t)n * 2, cudaMemcpyDefault), "read F16 norm");
    std::vector<float> f(n);
    for (int64_t i = 0; i < n; ++i) f[i] = f16_bits_to_float(h[i]);
    CK(cudaMemcpyAsync(dst, f.data(), (size_t)n * 4, cudaMemcpyHostToDevice, st), "norm upload");
    CK(cudaStreamSynchronize(st), "norm upload");
    return LC_OK;
}

extern "C" int lc_model_upload_tensor(lc_model* m, const char* name, const void* data, int64_t n, int32_t dtype) {
    if (!m || !name || !data) return fail(LC_ERR_INVALID_ARG, "NULL argument");
    CTX_CHECK(m->ctx);
    if (m->finalized) return fail(LC_ERR_STATE, "model already finalized");
    if (dtype != 0 && dtype != 1) return fail(LC_ERR_INVALID_ARG, "unsupported tensor type %d for %s (F32=0, F16=1)", dtype, name);
    const lc_config& c = m->cfg;
    const int64_t qdim = (int64_t)c.n_heads * c.head_dim, kvd = (int64_t)c.n_kv_heads * c.head_dim;
    cudaStream_t st = m->ctx->stream;
    auto expect = [&](int64_t want) -> int {
        if (n != want)
            return fail(LC_ERR_SHAPE, "Shape mismatch: tensor %s has %lld elements, expected %lld", name, (long long)n, (long long)want);
        return LC_OK;
    };
    auto need_f16 = [&]() -> int {
        if (dtype != 1) return fail(LC_ERR_INVALID_ARG, "Expected F16 tensor (type 1), got type %d for tensor: %s", dtype, name);
        return LC_OK;
    };
    int rc;
    if (!strcmp(name, "token_embd.weight") || !strcmp(name, "output.weight")) {
        const bool out_w = name[0] == 'o';
        if (m->w32) {
            if ((rc = expect((int64_t)c.vocab * c.dim))) return rc;
            if (out_w && !m->out32) CK(cudaMalloc(&m->out32, (size_t)n * 4), "output weight");
            if ((rc = put32(m, out_w ? m->out32 : m->tok32, data, n, dtype))) return rc;
            m->have[out_w ? kOutput : kTokEmb] = 1;
            m->has_output |= out_w;
            CK(cudaStreamSynchronize(st), "tensor upload");
            return LC_OK;
        }
        if ((rc = need_f16()) || (rc = expect((int64_t)c.vocab * c.dim))) return rc;
        if (out_w) {
            if ((rc = put_tiled(m, m->lm_tiled, data, c.vocab, c.dim, 0, 1))) return rc;
        } else if ((rc = put(m->tok_emb, data, (size_t)n * 2, st))) {
            return rc;
        }
        m->have[out_w ? kOutput : kTokEmb] = 1;
        m->has_output |= out_w;
    } else if (!strcmp(name, "output_norm.weight")) {
        if ((rc = expect(c.dim)) || (rc = upload_norm(m->out_norm, data, n, dtype, st))) return rc;
        m->have[kOutNorm] = 1;
    } else if (!strncmp(name, "blk.", 4)) {
        char* end = nullptr;
        long l = strtol(name + 4, &end, 10);
        if (end == name + 4 || *end != '.' || l < 0 || l >= c.n_layers)
            return fail(LC_ERR_NOT_FOUND, "Tensor not found: %s", name);
        const char* t = end + 1;
        LayerStore& L = m->layers[l];
        int slot;
        if (!strcmp(t, "attn_norm.weight")) {
            if ((rc = expect(c.dim)) || (rc = upload_norm(L.attn_norm, data, n, dtype, st))) return rc;
            slot = kAttnNorm;
        } else if (!strcmp(t, "ffn_norm.weight")) {
            if ((rc = expect(c.dim)) || (rc = upload_norm(L.ffn_norm, data, n, dtype, st))) return rc;
            slot = kFfnNorm;
        } else if (!strcmp(t, "attn_q.weight") || !strcmp(t, "attn_k.weight") || !strcmp(t, "attn_v.weight")) {
            const int64_t rows = (t[5] == 'q') ? qdim : kvd;
            if ((rc = (m->w32 ? 0 : need_f16())) || (rc = expect(rows * c.dim))) return rc;
            const int64_t row0 = (t[5] == 'q') ? 0 : (t[5] == 'k') ? qdim : qdim + kvd;
            if (m->w32) rc = put32(m, const_cast<float*>(m->l32[l].wqkv) + row0 * c.dim, data, n, dtype);
            else rc = put_tiled(m, L.wqkv, data, (int)rows, c.dim, (int)row0, 1);
            if (rc) return rc;
            slot = (t[5] == 'q') ? kQ : (t[5] == 'k') ? kK : kV;
        } else if (!strcmp(t, "attn_output.weight")) {
            if ((rc = (m->w32 ? 0 : need_f16())) || (rc = expect((int64_t)c.dim * qdim))) return rc;
            if (m->w32) rc = put32(m, const_cast<float*>(m->l32[l].wo), data, n, dtype);
            else rc = put_tiled(m, L.wo, data, c.dim, (int)qdim, 0, 1);
            if (rc) return rc;
            slot = kO;
        } else if (!strcmp(t, "ffn_gate.weight") || !strcmp(t, "ffn_up.weight")) {
            if ((rc = (m->w32 ? 0 : need_f16())) || (rc = expect((int64_t)c.hidden * c.dim))) return rc;
            const bool up = t[4] == 'u';
            // F16: row r of gate -> row 2r of the packed tiled matrix, row r of
            // up -> 2r+1.  F32: gate rows, then up rows.
            if (m->w32) rc = put32(m, const_cast<float*>(m->l32[l].wgu) + (up ? (int64_t)c.hidden * c.dim : 0), data, n, dtype);
            else rc = put_tiled(m, L.wgu, data, c.hidden, c.dim, up ? 1 : 0, 2);
            if (rc) return rc;
            slot = up ? kUp : kGate;
        } else if (!strcmp(t, "ffn_down.weight")) {
            if ((rc = (m->w32 ? 0 : need_f16())) || (rc = expect((int64_t)c.dim * c.hidden))) return rc;
            if (m->w32) rc = put32(m, const_cast<float*>(m->l32[l].wdown), data, n, dtype);
            else rc = put_tiled(m, L.wdown, data, c.dim, c.hidden, 0, 1);
            if (rc) return rc;
            slot = kDown;
        } else {
            return fail(LC_ERR_NOT_FOUND, "Tensor not found: %s", name);
        }
        m->have[kLayerBase + kPerLayer * l + slot] = 1;
    } else {
        return fail(LC_ERR_NOT_FOUND, "Tensor not found: %s", name);
    }
    // Host sources may be freed once the call returns.
    CK(cudaStreamSynchronize(st), "tensor upload");
    return LC_OK;
}

static const char* slot_name(int slot, char* buf) {
    static const char* per[] = {"attn_norm", "attn_q", "attn_k", "attn_v", "attn_output",
                                "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"};
    if (slot == kTokEmb) return "token_embd.weight";
    if (slot == kOutNorm) return "output_norm.weight";
    int l = (slot - kLayerBase) / kPerLayer, k = (slot - kLayerBase) % kPerLayer;
    snprintf(buf, 64, "blk.%d.%s.weight", l, per[k]);
    return buf;
}

static void fill_model_params(const lc_model* m, DecodeParams* p) {
    const lc_config& c = m->cfg;
    memset(p, 0, sizeof(*p));
    p->dim = c.dim;
    p->hidden = c.hidden;
    p->n_layers = c.n_layers;
    p->n_heads = c.n_heads;
    p->n_kv = c.n_kv_heads;
    p->head_dim = c.head_dim;
    p->vocab = c.vocab;
    p->max_seq = c.max_seq;
    p->eps = c.rms_eps;
    p->attn_scale = 1.0f / (float)sqrt((double)c.head_dim);  // Attention.java:33
    p->tok_emb = m->tok_emb;
    p->lm_head = m->lm_tiled;  // output.weight, or the tied embedding (LlamaInference.java:69-72)
    p->out_norm = m->out_norm;
    p->layers = m->d_layers;
    for (int l = 0; l < c.n_layers && l < kMaxDecodeLayers; ++l) {
        p->norm_w[2 * l] = m->layers[l].attn_norm;
        p->norm_w[2 * l + 1] = m->layers[l].ffn_norm;
    }
    p->rope = m->rope;
    p->rope_cs = m->d_rope_cs;
    p->timeout_ns = 2000000000ull;
    p->sched = m->d_sched;
    p->sched_n = m->d_sched_n;
    p->sched_stride = m->sched_stride;
    p->wbase = (const uint8_t*)m->arena;
    p->l2_prefetch_tiles = m->l2_prefetch_tiles;
    p->trace = nullptr;
    p->trace_words = 0;
    p->stream = nullptr;
}

extern "C" int lc_model_finalize(lc_model* m) {
    if (!m) return fail(LC_ERR_INVALID_ARG, "model is NULL");
    CTX_CHECK(m->ctx);
    if (m->finalized) return LC_OK;
    char buf[64];
    for (size_t s = 0; s < m->have.size(); ++s) {
        if (s == kOutput) continue;  // optional: tied embeddings
        if (!m->have[s]) return fail(LC_ERR_NOT_FOUND, "Tensor not found: %s", slot_name((int)s, buf));
    }
    if (m->w32) {
        // Row-major fp32 weights as uploaded; nothing to tile or plan.
        CK(cudaStreamSynchronize(m->ctx->stream), "weight upload");
        if (m->staging) cudaFree(m->staging);
        m->staging = nullptr;
        m->staging_bytes = 0;
        make_rope_freq(&m->rope, m->cfg.rope_theta, m->cfg.head_dim);
        CK(f32_prepare(), "fp32 GEMV setup");
        m->launch.grid = m->ctx->sms;
        m->finalized = true;
        return LC_OK;
    }
    // Tied embeddings: the lm_head is the token embedding (LlamaInference.java:69-72).
    if (!m->has_output) {
        int rc = put_tiled(m, m->lm_tiled, m->tok_emb, m->cfg.vocab, m->cfg.dim, 0, 1);
        if (rc) return rc;
    }
    CK(cudaStreamSynchronize(m->ctx->stream), "weight tiling");
    if (m->staging) cudaFree(m->staging);
    m->staging = nullptr;
    m->staging_bytes = 0;
    make_rope_freq(&m->rope, m->cfg.rope_theta, m->cfg.head_dim);
    {
        // The rotation of pair i at position pos (RoPE.java:42-46): the float
        // angle pos * freq, its sine and cosine in double, rounded to float.
        const int half = m->cfg.head_dim / 2;
        std::vector<float2> cs((size_t)m->cfg.max_seq * half);
        for (int pos = 0; pos < m->cfg.max_seq; ++pos)
            for (int i = 0; i < half; ++i) {
                const float val = (float)pos * m->rope.f[i];
                cs[(size_t)pos * half + i] = make_float2((float)sin((double)val), (float)cos((double)val));
            }
        CK(cudaMalloc(&m->d_rope_cs, cs.size() * sizeof(float2)), "rope table");
        CK(cudaMemcpy(m->d_rope_cs, cs.data(), cs.size() * sizeof(float2), cudaMemcpyHostToDevice), "rope table");
    }
    if (const char* e = getenv("LLAMACUDA_L2_PREFETCH_TILES")) m->l2_prefetch_tiles = atoi(e);
    if (m->l2_prefetch_tiles < 0) {
        // Default window: 8 tiles ahead of the copies (1B decode: 598 -> 589
        // us per forward; 16 tiles 619, 32 tiles 977), capped so the windows
        // of all CTAs hold at most 40 MB of the 126 MB L2.
        const size_t tile = (size_t)8 * m->cfg.dim * 2, cap = (size_t)40 << 20;
        const size_t per = tile * (size_t)(m->ctx->sms > 0 ? m->ctx->sms : 148);
        m->l2_prefetch_tiles = (int)std::min<size_t>(8, cap / per);
    }
    std::vector<LayerW> lw(m->cfg.n_layers);
    for (int l = 0; l < m->cfg.n_layers; ++l) {
        const LayerStore& L = m->layers[l];
        lw[l] = {L.wqkv, L.wo, L.wgu, L.wdown, L.attn_norm, L.ffn_norm};
    }
    CK(cudaMalloc(&m->d_layers, lw.size() * sizeof(LayerW)), "layer table");
    CK(cudaMemcpy(m->d_layers, lw.data(), lw.size() * sizeof(LayerW), cudaMemcpyHostToDevice), "layer table");
    DecodeParams p;
    fill_model_params(m, &p);
    const char* why = nullptr;
    if (!decode_plan(p, m->ctx->sms, &m->launch, &why)) return fail(LC_ERR_UNSUPPORTED, "%s", why);
    {
        std::vector<uint32_t> sched;
        std::vector<int> counts;
        decode_build_schedule(p, lw.data(), m->launch.grid, &sched, &counts, &m->sched_stride);
        CK(cudaMalloc(&m->d_sched, sched.size() * 4), "tile schedule");
        CK(cudaMalloc(&m->d_sched_n, counts.size() * 4), "tile schedule");
        CK(cudaMemcpy(m->d_sched, sched.data(), sched.size() * 4, cudaMemcpyHostToDevice), "tile schedule");
        CK(cudaMemcpy(m->d_sched_n, counts.data(), counts.size() * 4, cudaMemcpyHostToDevice), "tile schedule");
    }
    CK(decode_prepare(m->launch), "decode kernel setup");
    CK(decode_prepare_traced(m->launch), "decode kernel setup");
    m->finalized = true;
    return LC_OK;
}

// ------------------------------------------------------------ session ----

struct lc_session {
    lc_model* m = nullptr;
    void* mem = nullptr;
    size_t tagged_bytes = 0;  // the tagged exchange words at the start of mem
    uint64_t *xa, *xb, *q, *kv, *att, *part, *amax;
    float* h;
    uint32_t epoch = 0;       // launch counter: tags of launch e are e << 20 | exchange
    uint32_t* flags;
    float *kcache, *vcache, *logits;
    int *err, *n_done;
    int32_t* tokens;
    int attn_max_splits = 0;
    int32_t* pinned = nullptr;  // host staging for small transfers
    int32_t* stream_host = nullptr;  // mapped token stream: [0] = count, [1 + i] = token i
    int32_t* stream_dev = nullptr;   // its device address
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    float last_ms = 0.0f;
    unsigned long long* trace = nullptr;  // phase trace buffer (debug), grid x trace_words
    int trace_words = 0;
    void* f32mem = nullptr;  // F32 storage mode: the per-launch scratch of F32Step
    F32Step f32;
};

// F32 storage mode: the session's F32Step (its caches, logits and tokens,
// plus the fp32 path's scratch, position / length tables and attention
// scratch sized for max_seq positions).
static cudaError_t f32_session_setup(lc_session* s) {
    lc_model* m = s->m;
    const lc_config& c = m->cfg;
    const size_t qd = (size_t)c.n_heads * c.head_dim, kvd = (size_t)c.n_kv_heads * c.head_dim;
    // Splits hold at least 64 positions, so ceil(max_seq / 64) bounds every plan.
    AttnPlan bound = plan_attention(1, c.n_heads, c.n_kv_heads, c.head_dim, c.max_seq, m->ctx->sms);
    bound.max_splits = (c.max_seq + 63) / 64;
    const size_t att_bytes = attention_scratch_bytes(bound);
    auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
    const size_t sizes[] = {(size_t)c.dim * 4, (size_t)c.dim * 4, (qd + 2 * kvd) * 4, qd * 4, (size_t)c.hidden * 8,
                            (size_t)c.max_seq * 4, (size_t)c.max_seq * 4, att_bytes};
    size_t total = 0;
    for (size_t x : sizes) total += al(x);
    cudaError_t e = cudaMalloc(&s->f32mem, total);
    if (e != cudaSuccess) return e;
    uint8_t* p = (uint8_t*)s->f32mem;
    void* ptr[8];
    for (int i = 0; i < 8; ++i) {
        ptr[i] = p;
        p += al(sizes[i]);
    }
    std::vector<int32_t> pv(c.max_seq), lv(c.max_seq);
    for (int i = 0; i < c.max_seq; ++i) {
        pv[i] = i;
        lv[i] = i + 1;
    }
    if ((e = cudaMemcpy(ptr[5], pv.data(), pv.size() * 4, cudaMemcpyHostToDevice)) != cudaSuccess) return e;
    if ((e = cudaMemcpy(ptr[6], lv.data(), lv.size() * 4, cudaMemcpyHostToDevice)) != cudaSuccess) return e;
    F32Step& f = s->f32;
    f.dim = c.dim;
    f.hidden = c.hidden;
    f.n_layers = c.n_layers;
    f.n_heads = c.n_heads;
    f.n_kv = c.n_kv_heads;
    f.head_dim = c.head_dim;
    f.vocab = c.vocab;
    f.max_seq = c.max_seq;
    f.num_sms = m->ctx->sms;
    f.eps = c.rms_eps;
    f.tok_emb = m->tok32;
    f.lm = m->has_output ? m->out32 : m->tok32;  // tied embeddings, LlamaInference.java:69-72
    f.out_norm = m->out_norm;
    f.layers = m->l32.data();
    f.rope = m->rope;
    f.kcache = s->kcache;
    f.vcache = s->vcache;
    f.logits = s->logits;
    f.tokens = s->tokens;
    f.err = s->err;
    f.x = (float*)ptr[0];
    f.xb = (float*)ptr[1];
    f.qkv = (float*)ptr[2];
    f.att = (float*)ptr[3];
    f.gu = (float*)ptr[4];
    f.posv = (const int32_t*)ptr[5];
    f.lenv = (const int32_t*)ptr[6];
    f.attn_scratch = ptr[7];
    f.attn_scratch_bytes = att_bytes;
    return cudaSuccess;
}

extern "C" int lc_session_create(lc_model* m, lc_session** out) {
    if (!m || !out) return fail(LC_ERR_INVALID_ARG, "NULL argument");
    CTX_CHECK(m->ctx);
    if (!m->finalized) return fail(LC_ERR_STATE, "model not finalized");
    const lc_config& c = m->cfg;
    lc_session* s = new lc_session();
    s->m = m;
    const int kv_mul = c.n_heads / c.n_kv_heads;
    s->attn_max_splits = decode_attn_max_splits(c.max_seq, m->launch.grid, c.n_kv_heads);
    const size_t G = (size_t)m->launch.grid;
    auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
    const size_t qd = (size_t)c.n_heads * c.head_dim, kvd = (size_t)c.n_kv_heads * c.head_dim;
    const size_t kv = (size_t)c.n_layers * c.n_kv_heads * c.max_seq * c.head_dim * 4;
    // Tagged exchange words (8 bytes each) first, then plain buffers.
    const size_t sizes[] = {(size_t)c.dim * 8,
                            (size_t)c.dim * 8,
                            qd * 8,
                            2 * kvd * 8,
                            qd * 8,
                            (size_t)c.n_kv_heads * s->attn_max_splits * kv_mul * kDecodePartStride * 8,
                            G * 2 * 8,
                            (size_t)c.hidden * 4,
                            G * 4,
                            kv,
                            kv,
                            (size_t)c.vocab * 4,
                            4,
                            4,
                            (size_t)(c.max_seq + 1) * 4};
    constexpr int kN = sizeof(sizes) / sizeof(sizes[0]);
    size_t total = 0;
    for (size_t b : sizes) total += al(b);
    cudaError_t e = cudaMalloc(&s->mem, total);
    if (e != cudaSuccess) {
        delete s;
        return cuda_fail(e, "session buffers");
    }
    void* ptr[kN];
    uint8_t* p = (uint8_t*)s->mem;
    for (int i = 0; i < kN; ++i) {
        ptr[i] = p;
        p += al(sizes[i]);
    }
    s->xa = (uint64_t*)ptr[0];
    s->xb = (uint64_t*)ptr[1];
    s->q = (uint64_t*)ptr[2];
    s->kv = (uint64_t*)ptr[3];
    s->att = (uint64_t*)ptr[4];
    s->part = (uint64_t*)ptr[5];
    s->amax = (uint64_t*)ptr[6];
    s->tagged_bytes = (size_t)((uint8_t*)ptr[7] - (uint8_t*)ptr[0]);
    s->h = (float*)ptr[7];
    s->flags = (uint32_t*)ptr[8];
    s->kcache = (float*)ptr[9];
    s->vcache = (float*)ptr[10];
    s->logits = (float*)ptr[11];
    s->err = (int*)ptr[12];
    s->n_done = (int*)ptr[13];
    s->tokens = (int32_t*)ptr[14];
    e = cudaMemset(s->mem, 0, total);
    if (e == cudaSuccess) e = cudaMallocHost((void**)&s->pinned, (size_t)(c.max_seq + 8) * 4);
    if (e == cudaSuccess) e = cudaHostAlloc((void**)&s->stream_host, (size_t)(c.max_seq + 2) * 4, cudaHostAllocMapped);
    if (e == cudaSuccess) e = cudaHostGetDevicePointer((void**)&s->stream_dev, s->stream_host, 0);
    if (e == cudaSuccess) e = cudaEventCreate(&s->ev0);
    if (e == cudaSuccess) e = cudaEventCreate(&s->ev1);
    if (e == cudaSuccess && m->w32) e = f32_session_setup(s);
    if (e != cudaSuccess) {
        lc_session_destroy(s);
        return cuda_fail(e, "session setup");
    }
    *out = s;
    return LC_OK;
}

extern "C" int lc_session_destroy(lc_session* s) {
    if (!s) return LC_OK;
    cudaSetDevice(s->m->ctx->device);
    cudaStreamSynchronize(s->m->ctx->stream);
    if (s->mem) cudaFree(s->mem);
    if (s->pinned) cudaFreeHost(s->pinned);
    if (s->stream_host) cudaFreeHost(s->stream_host);
    if (s->ev0) cudaEventDestroy(s->ev0);
    if (s->ev1) cudaEventDestroy(s->ev1);
    if (s->trace) cudaFree(s->trace);
    if (s->f32mem) cudaFree(s->f32mem);
    delete s;
    return LC_OK;
}

// Host end of the token stream: the callback and its argument.
struct TokenSink {
    lc_token_callback cb;
    void* user;
};

// Launches the fused kernel for positions pos0..pos0+nsteps-1 and waits.  With
// a sink, the kernel publishes each generated token to the session's mapped
// stream buffer and this thread hands them to the callback while it waits.
// F32 storage mode: the same contract as the fused launch below, one
// enqueued forward per position.  Position pos feeds tokens[pos] (the prompt,
// or the greedy token the previous position stored); logits are computed when
// needed (not for prompt positions under skip_prefill_logits) and the argmax
// goes to tokens[pos + 1] from the last prompt position on.  With stop tokens
// or a sink the generated token is read back after each position.
static int run_steps_f32(lc_session* s, int pos0, int nsteps, int n_prompt, int skip_prefill_logits,
                         const int32_t* stop, int n_stop, int* n_done, const TokenSink* sink) {
    lc_model* m = s->m;
    cudaStream_t st = m->ctx->stream;
    CK(cudaMemsetAsync(s->err, 0, sizeof(int), st), "clear error word");
    CK(cudaEventRecord(s->ev0, st), "event");
    int done = 0;
    for (int k = 0; k < nsteps; ++k) {
        const int pos = pos0 + k;
        const bool lm = !(skip_prefill_logits && pos + 1 < n_prompt);
        const bool store = lm && pos + 1 >= n_prompt;
        CK(f32_forward(s->f32, pos, lm, store, st), "fp32-weight forward");
        done = k + 1;
        if (store && (n_stop > 0 || sink)) {
            CK(cudaMemcpyAsync(s->pinned + 3, s->tokens + pos + 1, 4, cudaMemcpyDeviceToHost, st), "token read");
            CK(cudaStreamSynchronize(st), "fp32-weight forward");
            const int tok = s->pinned[3];
            if (sink) sink->cb(tok, pos + 1 - n_prompt, sink->user);
            bool stop_now = false;
            for (int j = 0; j < n_stop; ++j) stop_now |= stop[j] == tok;
            if (stop_now) break;
        }
    }
    CK(cudaEventRecord(s->ev1, st), "event");
    CK(cudaMemcpyAsync(s->pinned, s->err, 4, cudaMemcpyDeviceToHost, st), "read error word");
    CK(cudaStreamSynchronize(st), "fp32-weight forward");
    cudaEventElapsedTime(&s->last_ms, s->ev0, s->ev1);
    if (s->pinned[0] != 0) {
        if (s->pinned[0] == kDevBadToken) return fail(LC_ERR_INVALID_ARG, "token id outside [0, %d)", m->cfg.vocab);
        return fail(LC_ERR_TIMEOUT, "fp32-weight forward: device error code %d", s->pinned[0]);
    }
    *n_done = done;
    return LC_OK;
}

static int run_steps(lc_session* s, int pos0, int nsteps, int n_prompt, int skip_prefill_logits,
                     const int32_t* stop, int n_stop, int* n_done, const TokenSink* sink = nullptr) {
    if (s->m->w32) return run_steps_f32(s, pos0, nsteps, n_prompt, skip_prefill_logits, stop, n_stop, n_done, sink);
    lc_model* m = s->m;
    cudaStream_t st = m->ctx->stream;
    DecodeParams p;
    fill_model_params(m, &p);
    p.kcache = s->kcache;
    p.vcache = s->vcache;
    p.logits = s->logits;
    p.tokens = s->tokens;
    p.err = s->err;
    p.n_done = s->n_done;
    p.xa = s->xa;
    p.xb = s->xb;
    p.q = s->q;
    p.kv = s->kv;
    p.att = s->att;
    p.part = s->part;
    p.h = s->h;
    p.amax = s->amax;
    p.flags = s->flags;
    // Exchange indices of one launch must fit the 20 low bits of a tag.
    if ((int64_t)nsteps * (5 * m->cfg.n_layers + 1) >= (int64_t)(1 << 20) - 1)
        return fail(LC_ERR_UNSUPPORTED, "%d steps in one launch exceed the exchange-tag range", nsteps);
    // Tags are epoch << 20 | exchange + 1: words left by earlier launches never
    // match.  When the 12-bit epoch wraps, the words are cleared.  The flags
    // restart from 0 every launch.
    if (++s->epoch >= 4096u) {
        CK(cudaMemsetAsync(s->mem, 0, s->tagged_bytes, st), "clear exchange words");
        s->epoch = 1;
    }
    CK(cudaMemsetAsync(s->flags, 0, (size_t)m->launch.grid * 4, st), "clear exchange flags");
    p.tag_base = s->epoch << 20;
    p.pos0 = pos0;
    p.nsteps = nsteps;
    p.n_prompt = n_prompt;
    p.skip_prefill_logits = skip_prefill_logits;
    p.n_stop = n_stop;
    for (int i = 0; i < n_stop; ++i) p.stop[i] = stop[i];
    p.attn_max_splits = s->attn_max_splits;
    p.trace = s->trace;
    p.trace_words = s->trace_words;
    if (sink) {
        s->stream_host[0] = 0;  // host memory: written before the launch is enqueued
        p.stream = s->stream_dev;
    }
    if (s->trace)
        CK(cudaMemsetAsync(s->trace, 0, (size_t)m->launch.grid * s->trace_words * 8, st), "clear trace");
    CK(cudaMemsetAsync(s->err, 0, sizeof(int), st), "clear error word");
    CK(cudaEventRecord(s->ev0, st), "event");
    CK(s->trace ? launch_decode_traced(p, m->launch, st) : launch_decode(p, m->launch, st), "decode kernel launch");
    CK(cudaEventRecord(s->ev1, st), "event");
    CK(cudaMemcpyAsync(s->pinned, s->err, 4, cudaMemcpyDeviceToHost, st), "read error word");
    CK(cudaMemcpyAsync(s->pinned + 1, s->n_done, 4, cudaMemcpyDeviceToHost, st), "read step count");
    if (sink) {
        // Poll the published count; after the stream reports completion one
        // more pass delivers what the last check had not seen.
        const volatile int32_t* hs = s->stream_host;
        const int limit = m->cfg.max_seq;
        int delivered = 0;
        for (;;) {
            const cudaError_t q = cudaStreamQuery(st);
            if (q != cudaSuccess && q != cudaErrorNotReady) CK(q, "decode kernel");
            int avail = hs[0];
            std::atomic_thread_fence(std::memory_order_acquire);
            if (avail > limit) avail = limit;
            for (; delivered < avail; ++delivered) sink->cb(hs[1 + delivered], delivered, sink->user);
            if (q == cudaSuccess) break;
            std::this_thread::sleep_for(std::chrono::microseconds(20));
        }
    }
    CK(cudaStreamSynchronize(st), "decode kernel");
    cudaEventElapsedTime(&s->last_ms, s->ev0, s->ev1);
    const int err = s->pinned[0];
    if (err != 0) {
        if (err == kDevBadToken) return fail(LC_ERR_INVALID_ARG, "token id outside [0, %d)", m->cfg.vocab);
        return fail(LC_ERR_TIMEOUT, "decode kernel: bounded device wait gave up (code %d)", err);
    }
    *n_done = s->pinned[1];
    return LC_OK;
}

extern "C" int lc_forward(lc_session* s, int32_t token, int32_t pos, float* logits, int32_t* argmax_out) {
    if (!s) return fail(LC_ERR_INVALID_ARG, "session is NULL");
    CTX_CHECK(s->m->ctx);
    const lc_config& c = s->m->cfg;
    if (token < 0 || token >= c.vocab) return fail(LC_ERR_INVALID_ARG, "token %d outside [0, %d)", token, c.vocab);
    if (pos < 0 || pos >= c.max_seq) return fail(LC_ERR_INVALID_ARG, "pos %d outside [0, %d)", pos, c.max_seq);
    cudaStream_t st = s->m->ctx->stream;
    s->pinned[2] = token;
    CK(cudaMemcpyAsync(s->tokens + pos, s->pinned + 2, 4, cudaMemcpyHostToDevice, st), "token upload");
    int done = 0;
    int rc = run_steps(s, pos, 1, 0, 0, nullptr, 0, &done);
    if (rc) return rc;
    if (logits) CK(cudaMemcpyAsync(logits, s->logits, (size_t)c.vocab * 4, cudaMemcpyDefault, st), "logits copy");
    if (argmax_out) CK(cudaMemcpyAsync(argmax_out, s->tokens + pos + 1, 4, cudaMemcpyDefault, st), "argmax copy");
    CK(cudaStreamSynchronize(st), "forward");
    return LC_OK;
}

static int generate_impl(lc_session* s, const int32_t* prompt, int32_t n_prompt, int32_t max_new, const int32_t* stop,
                         int32_t n_stop, int32_t* out_tokens, int32_t* n_out, const TokenSink* sink) {
    if (!s || !prompt || !out_tokens || !n_out) return fail(LC_ERR_INVALID_ARG, "NULL argument");
    CTX_CHECK(s->m->ctx);
    const lc_config& c = s->m->cfg;
    if (n_prompt <= 0) return fail(LC_ERR_INVALID_ARG, "empty prompt");
    if (max_new <= 0) return fail(LC_ERR_INVALID_ARG, "max_new must be positive");
    if ((int64_t)n_prompt + max_new - 1 > c.max_seq)
        return fail(LC_ERR_INVALID_ARG, "prompt %d + %d new tokens exceed max_seq %d", n_prompt, max_new, c.max_seq);
    if (n_stop < 0 || n_stop > kMaxStop || (n_stop > 0 && !stop))
        return fail(LC_ERR_UNSUPPORTED, "n_stop=%d (at most %d stop tokens)", n_stop, kMaxStop);
    cudaStream_t st = s->m->ctx->stream;
    int32_t hstop[kMaxStop];
    if (n_stop) CK(cudaMemcpy(hstop, stop, (size_t)n_stop * 4, cudaMemcpyDefault), "stop tokens");
    CK(cudaMemcpyAsync(s->tokens, prompt, (size_t)n_prompt * 4, cudaMemcpyDefault, st), "prompt upload");
    int done = 0;
    int rc = run_steps(s, 0, n_prompt + max_new - 1, n_prompt, 1, hstop, n_stop, &done, sink);
    if (rc) return rc;
    const int n_gen = done - (n_prompt - 1);
    if (n_gen > 0)
        CK(cudaMemcpyAsync(out_tokens, s->tokens + n_prompt, (size_t)n_gen * 4, cudaMemcpyDefault, st), "tokens copy");
    CK(cudaStreamSynchronize(st), "generate");
    *n_out = n_gen > 0 ? n_gen : 0;
    return LC_OK;
}

extern "C" int lc_generate(lc_session* s, const int32_t* prompt, int32_t n_prompt, int32_t max_new,
                           const int32_t* stop, int32_t n_stop, int32_t* out_tokens, int32_t* n_out) {
    return generate_impl(s, prompt, n_prompt, max_new, stop, n_stop, out_tokens, n_out, nullptr);
}

extern "C" int lc_generate_stream(lc_session* s, const int32_t* prompt, int32_t n_prompt, int32_t max_new,
                                  const int32_t* stop, int32_t n_stop, lc_token_callback on_token, void* user,
                                  int32_t* out_tokens, int32_t* n_out) {
    if (!on_token) return fail(LC_ERR_INVALID_ARG, "NULL callback");
    const TokenSink sink{on_token, user};
    return generate_impl(s, prompt, n_prompt, max_new, stop, n_stop, out_tokens, n_out, &sink);
}

extern "C" int lc_decode(lc_session* s, int32_t token, int32_t start_pos, int32_t n_steps, int32_t* out_tokens) {
    if (!s || !out_tokens) return fail(LC_ERR_INVALID_ARG, "NULL argument");
    CTX_CHECK(s->m->ctx);
    const lc_config& c = s->m->cfg;
    if (token < 0 || token >= c.vocab) return fail(LC_ERR_INVALID_ARG, "token %d outside [0, %d)", token, c.vocab);
    if (n_steps <= 0 || start_pos < 0 || (int64_t)start_pos + n_steps > c.max_seq)
        return fail(LC_ERR_INVALID_ARG, "start_pos=%d n_steps=%d max_seq=%d", start_pos, n_steps, c.max_seq);
    cudaStream_t st = s->m->ctx->stream;
    s->pinned[2] = token;
    CK(cudaMemcpyAsync(s->tokens + start_pos, s->pinned + 2, 4, cudaMemcpyHostToDevice, st), "token upload");
    int done = 0;
    int rc = run_steps(s, start_pos, n_steps, 0, 0, nullptr, 0, &done);
    if (rc) return rc;
    CK(cudaMemcpyAsync(out_tokens, s->tokens + start_pos + 1, (size_t)n_steps * 4, cudaMemcpyDefault, st), "tokens copy");
    CK(cudaStreamSynchronize(st), "decode");
    return LC_OK;
}

extern "C" int lc_session_enable_trace(lc_session* s, int32_t words_per_cta) {
    if (!s || words_per_cta < 0) return fail(LC_ERR_INVALID_ARG, "bad argument");
    CTX_CHECK(s->m->ctx);
    if (s->m->w32) return fail(LC_ERR_UNSUPPORTED, "the phase trace belongs to the fused F16 decode kernel");
    CK(cudaStreamSynchronize(s->m->ctx->stream), "synchronize");
    if (s->trace) cudaFree(s->trace);
    s->trace = nullptr;
    s->trace_words = 0;
    if (words_per_cta == 0) return LC_OK;
    CK(cudaMalloc(&s->trace, (size_t)s->m->launch.grid * words_per_cta * 8), "trace buffer");
    s->trace_words = words_per_cta;
    return LC_OK;
}

extern "C" int lc_session_read_trace(lc_session* s, uint64_t* out, int64_t n_words, int32_t* grid,
                                     int32_t* words_per_cta) {
    if (!s) return fail(LC_ERR_INVALID_ARG, "session is NULL");
    CTX_CHECK(s->m->ctx);
    if (grid) *grid = s->m->launch.grid;
    if (words_per_cta) *words_per_cta = s->trace_words;
    if (!out || !s->trace) return LC_OK;
    const int64_t total = (int64_t)s->m->launch.grid * s->trace_words;
    CK(cudaMemcpy(out, s->trace, (size_t)(n_words < total ? n_words : total) * 8, cudaMemcpyDeviceToHost),
       "trace copy");
    return LC_OK;
}

extern "C" int lc_session_last_ms(lc_session* s, float* ms) {
    if (!s || !ms) return fail(LC_ERR_INVALID_ARG, "NULL argument");
    *ms = s->last_ms;
    return LC_OK;
}

// ------------------------------------------------------------ batch ----

struct lc_batch {
    lc_model* m = nullptr;
    BatchEngine* e = nullptr;
};

extern "C" int lc_batch_create(lc_model* m, int32_t max_batch, lc_batch** out) {
    if (!m || !out) return fail(LC_ERR_INVALID_ARG, "NULL argument");
    CTX_CHECK(m->ctx);
    if (!m->finalized) return fail(LC_ERR_STATE, "model not finalized");
    if (m->w32) return fail(LC_ERR_UNSUPPORTED, "multi-sequence batches run on F16 weights (LC_WEIGHTS_F16)");
    if (max_batch < 1 || max_batch > kGemmMaxB) return fail(LC_ERR_INVALID_ARG, "max_batch %d not in 1..%d", max_batch, kGemmMaxB);
    BatchModel bm;
    const lc_config& c = m->cfg;
    bm.dim = c.dim;
    bm.hidden = c.hidden;
    bm.n_layers = c.n_layers;
    bm.n_heads = c.n_heads;
    bm.n_kv = c.n_kv_heads;
    bm.head_dim = c.head_dim;
    bm.vocab = c.vocab;
    bm.max_seq = c.max_seq;
    bm.eps = c.rms_eps;
    bm.tok_emb = m->tok_emb;
    bm.lm_head = m->lm_tiled;
    bm.out_norm = m->out_norm;
    for (const LayerStore& L : m->layers) bm.layers.push_back({L.wqkv, L.wo, L.wgu, L.wdown, L.attn_norm, L.ffn_norm});
    bm.rope = m->rope;
    const char* why = nullptr;
    if (!batch_supported(bm, &why)) return fail(LC_ERR_UNSUPPORTED, "%s", why);
    cudaError_t ce;
    BatchEngine* e = batch_create(bm, max_batch, m->ctx->sms, m->ctx->stream, m->ctx->d_err, &ce);
    if (!e) return cuda_fail(ce, "batch buffers");
    lc_batch* b = new lc_batch();
    b->m = m;
    b->e = e;
    *out = b;
    return LC_OK;
}

extern "C" int lc_batch_destroy(lc_batch* b) {
    if (!b) return LC_OK;
    cudaSetDevice(b->m->ctx->device);
    batch_destroy(b->e);
    delete b;
    return LC_OK;
}

extern "C" int lc_batch_generate(lc_batch* b, int32_t n, const int32_t* prompts, const int32_t* lens,
                                 int32_t max_new, const int32_t* stop, int32_t n_stop, int32_t* out) {
    if (!b || !prompts || !lens || !out) return fail(LC_ERR_INVALID_ARG, "NULL argument");
    CTX_CHECK(b->m->ctx);
    const lc_config& c = b->m->cfg;
    if (n < 1 || n > batch_max(b->e)) return fail(LC_ERR_INVALID_ARG, "n_seqs %d not in 1..%d", n, batch_max(b->e));
    if (max_new < 1) return fail(LC_ERR_INVALID_ARG, "max_new %d", max_new);
    if (n_stop < 0 || n_stop > kMaxStop || (n_stop > 0 && !stop)) return fail(LC_ERR_INVALID_ARG, "n_stop %d", n_stop);
    const int ts = batch_tok_stride(b->e);
    std::vector<int32_t> tok((size_t)n * ts, 0), L(lens, lens + n);
    size_t off = 0;
    for (int s = 0; s < n; ++s) {
        if (L[s] < 1 || L[s] + max_new - 1 > c.max_seq)
            return fail(LC_ERR_INVALID_ARG, "sequence %d: prompt length %d + max_new %d exceeds max_seq %d", s, L[s], max_new, c.max_seq);
        for (int i = 0; i < L[s]; ++i) {
            const int32_t t = prompts[off + i];
            if (t < 0 || t >= c.vocab) return fail(LC_ERR_INVALID_ARG, "sequence %d: token %d out of range", s, t);
            tok[(size_t)s * ts + i] = t;
        }
        off += L[s];
    }
    std::vector<int32_t> res;
    cudaError_t ce = batch_run(b->e, n, tok, L, max_new, &res);
    if (ce != cudaSuccess) return cuda_fail(ce, "batch generate");
    int rc = check_device_error(b->m->ctx);
    if (rc) return rc;
    for (int s = 0; s < n; ++s) {
        bool stopped = false;
        for (int i = 0; i < max_new; ++i) {
            int32_t t = stopped ? -1 : res[(size_t)s * ts + L[s] + i];
            out[(size_t)s * max_new + i] = t;
            for (int k = 0; k < n_stop && !stopped; ++k) stopped = (t == stop[k]);
        }
    }
    return LC_OK;
}

extern "C" int lc_batch_last_ms(lc_batch* b, float* total_ms, float* decode_ms, int32_t* steps) {
    if (!b || !total_ms || !decode_ms) return fail(LC_ERR_INVALID_ARG, "NULL argument");
    int st = 0;
    batch_times(b->e, total_ms, decode_ms, &st);
    if (steps) *steps = st;
    return LC_OK;
}

extern "C" int lc_batch_logits(lc_batch* b, int32_t seq, float* out) {
    if (!b || !out) return fail(LC_ERR_INVALID_ARG, "NULL argument");
    CTX_CHECK(b->m->ctx);
    if (seq < 0 || seq >= batch_max(b->e)) return fail(LC_ERR_INVALID_ARG, "seq %d", seq);
    CK(batch_logits(b->e, seq, out), "read logits");
    return LC_OK;
}

// Error hook for lc_gguf.cpp (not part of the public ABI).
extern "C" __attribute__((visibility("hidden"))) int lc_gguf_set_error(int code, const char* msg) {
    return fail(code, "%s", msg);
}

// Accessors for lc_attention_static.cu (not part of the public ABI).
extern "C" __attribute__((visibility("hidden"))) int lc_internal_set_error(int code, const char* msg) {
    return fail(code, "%s", msg);
}

extern "C" __attribute__((visibility("hidden"))) int lc_internal_context_device(const lc_context* c) {
    return c ? c->device : -1;
}

// ------------------------------------------------ peer key exchange ----

struct lc_keyx {
    lc_context* ctx = nullptr;
    int world = 0, rank = 0, max_batch = 0;
    uint8_t* mbox = nullptr;                   // this rank's mailbox (cudaMalloc)
    void* peer[LC_KEYX_MAX_WORLD] = {};        // the other ranks' mailboxes, mapped through IPC
    uint32_t epoch = 0;
    bool open = false;
};

static_assert(sizeof(cudaIpcMemHandle_t) == LC_KEYX_HANDLE_BYTES, "IPC handle size");
static_assert(LC_KEYX_MAX_WORLD == kKeyxMaxWorld, "world bound");

extern "C" int lc_keyx_create(lc_context* c, int32_t world, int32_t rank, int32_t max_batch, lc_keyx** out,
                              void* handle_out) {
    if (!c || !out || !handle_out) return fail(LC_ERR_INVALID_ARG, "NULL argument");
    if (world < 1 || world > LC_KEYX_MAX_WORLD || rank < 0 || rank >= world)
        return fail(LC_ERR_INVALID_ARG, "world %d rank %d (world 1..%d)", world, rank, LC_KEYX_MAX_WORLD);
    if (max_batch < 1 || max_batch > 4096) return fail(LC_ERR_INVALID_ARG, "max_batch %d (1..4096)", max_batch);
    CTX_CHECK(c);
    lc_keyx* x = new lc_keyx();
    x->ctx = c;
    x->world = world;
    x->rank = rank;
    x->max_batch = max_batch;
    const size_t bytes = keyx_mailbox_bytes(world, max_batch);
    cudaError_t e = cudaMalloc(&x->mbox, bytes);
    if (e == cudaSuccess) e = cudaMemset(x->mbox, 0, bytes);
    cudaIpcMemHandle_t h;
    memset(&h, 0, sizeof(h));
    if (e == cudaSuccess && world > 1) e = cudaIpcGetMemHandle(&h, x->mbox);
    if (e != cudaSuccess) {
        if (x->mbox) cudaFree(x->mbox);
        delete x;
        return cuda_fail(e, "key-exchange mailbox");
    }
    memcpy(handle_out, &h, sizeof(h));
    *out = x;
    return LC_OK;
}

extern "C" int lc_keyx_open(lc_keyx* x, const void* handles) {
    if (!x || !handles) return fail(LC_ERR_INVALID_ARG, "NULL argument");
    if (x->open) return fail(LC_ERR_STATE, "key exchange already open");
    CTX_CHECK(x->ctx);
    const uint8_t* hs = (const uint8_t*)handles;
    for (int p = 0; p < x->world; ++p) {
        if (p == x->rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, hs + (size_t)p * LC_KEYX_HANDLE_BYTES, sizeof(h));
        cudaError_t e = cudaIpcOpenMemHandle(&x->peer[p], h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < p; ++q)
                if (x->peer[q]) cudaIpcCloseMemHandle(x->peer[q]);
            for (int q = 0; q < LC_KEYX_MAX_WORLD; ++q) x->peer[q] = nullptr;
            return cuda_fail(e, "mapping a peer mailbox");
        }
    }
    x->open = true;
    return LC_OK;
}

extern "C" int lc_keyx_allreduce(lc_keyx* x, uint64_t* keys, int32_t batch) {
    if (!x || !keys) return fail(LC_ERR_INVALID_ARG, "NULL argument");
    if (!x->open) return fail(LC_ERR_STATE, "key exchange not open (lc_keyx_open)");
    if (batch < 1 || batch > x->max_batch) return fail(LC_ERR_INVALID_ARG, "batch %d (1..%d)", batch, x->max_batch);
    if ((uintptr_t)keys & 7) return fail(LC_ERR_INVALID_ARG, "keys must be 8-byte aligned device memory");
    CTX_CHECK(x->ctx);
    KeyxArgs a;
    memset(&a, 0, sizeof(a));
    const size_t foff = keyx_flags_offset(x->world, x->max_batch);
    for (int p = 0; p < x->world; ++p) {
        uint8_t* base = p == x->rank ? x->mbox : (uint8_t*)x->peer[p];
        a.keys_mbox[p] = (uint64_t*)base;
        a.flags_mbox[p] = (uint32_t*)(base + foff);
    }
    a.keys = keys;
    a.world = x->world;
    a.rank = x->rank;
    a.batch = batch;
    a.max_batch = x->max_batch;
    a.epoch = ++x->epoch;
    a.err = x->ctx->d_err;
    a.timeout_ns = 2000000000ull;
    CK(launch_keyx(a, x->ctx->stream, true), "key exchange launch");
    return LC_OK;
}

extern "C" int lc_keyx_destroy(lc_keyx* x) {
    if (!x) return LC_OK;
    cudaSetDevice(x->ctx->device);
    cudaStreamSynchronize(x->ctx->stream);
    for (int p = 0; p < LC_KEYX_MAX_WORLD; ++p)
        if (x->peer[p]) cudaIpcCloseMemHandle(x->peer[p]);
    if (x->mbox) cudaFree(x->mbox);
    delete x;
    return LC_OK;
}
