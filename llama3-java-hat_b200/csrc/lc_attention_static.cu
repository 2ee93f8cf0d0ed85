// lc_attention_static.cu -- GQA decode attention that allocates no device
// memory: lc_attention_decode_static().
//
// Who needs it: hosts that cannot call cudaMalloc when they run attention --
// a host whose device memory is owned by its own pooling allocator (a JVM or
// framework that reserved the GPU's memory at start-up, so a driver
// allocation would fail or bypass its accounting), a latency-critical decode
// loop where cudaFree's device-wide synchronisation is not acceptable, or a
// deployment that must keep the library's device footprint fixed after
// load.  lc_attention_decode() grows a per-context scratch buffer with
// cudaMalloc and stages host buffers through allocated device memory; this
// entry point does neither.
//
// Its scratch (split partials, completion counters, a copy of host-side
// sequence lengths) is the file-scope device array below: kStaticScratchBytes
// (8 MiB) on every GPU that loads the library, held until the process exits.
// Requests whose plan needs more are rejected with LC_ERR_INVALID_ARG.
//
// Set-up: the array's device address is resolved once per device, with that
// device current, by cudaGetSymbolAddress (host code must not pass the
// array's name itself to a kernel: on the host it is only a stand-in for the
// device symbol).  The first call on each device performs this set-up, so
// make that first call before any stream capture.
//
// Sharing: every call on a device uses the same array and leaves its contents
// behind; the completion counters that must start at zero are cleared on the
// stream by each call.  Calls that overlap on the GPU (different streams or
// contexts on one device, without ordering between them) race on the array.
#include <mutex>

#include "../../include/llamacuda.h"
#include "lc_attention.cuh"
#include "lc_internal.h"

extern "C" int lc_internal_set_error(int code, const char* msg);
extern "C" int lc_internal_context_device(const lc_context* c);

namespace {

constexpr size_t kStaticScratchBytes = 8u << 20;  // per device
constexpr int kStaticMaxBatch = 1024;             // sequences per call
constexpr int kMaxDevices = 64;

__device__ __align__(256) uint8_t g_attn_scratch[kStaticScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_addr[kMaxDevices];  // resolved device address per device

// Returns the device address of g_attn_scratch on `device` (current), or
// nullptr with the error recorded.
void* scratch_address(int device) {
    if (device < 0 || device >= kMaxDevices) {
        lc_internal_set_error(LC_ERR_UNSUPPORTED, "device index beyond the static scratch table");
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_addr[device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (e != cudaSuccess || !p) {
            lc_internal_set_error(LC_ERR_CUDA, "cudaGetSymbolAddress of the static attention scratch failed");
            return nullptr;
        }
        g_scratch_addr[device] = p;
    }
    return g_scratch_addr[device];
}

// Where a buffer lives, as this entry point sees it.
enum class Where { kHost, kThisDevice, kElsewhere };

Where where_is(const void* p, int device) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return Where::kHost;  // not known to CUDA: plain host memory
    }
    switch (a.type) {
        case cudaMemoryTypeUnregistered:
        case cudaMemoryTypeHost: return Where::kHost;
        case cudaMemoryTypeManaged: return Where::kThisDevice;
        default: return a.device == device ? Where::kThisDevice : Where::kElsewhere;
    }
}

bool on_device(const void* p, int device) { return where_is(p, device) == Where::kThisDevice; }

}  // namespace

extern "C" int lc_attention_decode_static(lc_context* ctx, const float* q, const float* k, const float* v,
                                          float* out, const int32_t* seq_len, int batch, int n_heads,
                                          int n_kv_heads, int head_dim, int64_t seq_stride, int64_t head_stride,
                                          int64_t pos_stride) {
    using namespace lc;
    if (!ctx) return lc_internal_set_error(LC_ERR_INVALID_ARG, "context is NULL");
    const int device = lc_internal_context_device(ctx);
    if (cudaSetDevice(device) != cudaSuccess) return lc_internal_set_error(LC_ERR_CUDA, "cudaSetDevice failed");
    if (!q || !k || !v || !out || !seq_len) return lc_internal_set_error(LC_ERR_INVALID_ARG, "NULL buffer");
    if (batch <= 0 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads)
        return lc_internal_set_error(LC_ERR_INVALID_ARG, "bad batch / head counts");
    if (batch > kStaticMaxBatch)
        return lc_internal_set_error(LC_ERR_INVALID_ARG,
                                     "batch exceeds the static-scratch limit of 1024 sequences per call");
    if (head_dim != kAttnHeadDim) return lc_internal_set_error(LC_ERR_UNSUPPORTED, "head_dim must be 64");
    if (n_heads / n_kv_heads > 8) return lc_internal_set_error(LC_ERR_UNSUPPORTED, "at most 8 query heads per kv head");
    if ((seq_stride | head_stride | pos_stride) & 3)
        return lc_internal_set_error(LC_ERR_INVALID_ARG, "strides must be multiples of 4 floats");
    if (!on_device(q, device) || !on_device(k, device) || !on_device(v, device) || !on_device(out, device))
        return lc_internal_set_error(LC_ERR_INVALID_ARG,
                                     "lc_attention_decode_static needs q, k, v and out in device memory of the "
                                     "context's device (it stages nothing)");
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) & 15)
        return lc_internal_set_error(LC_ERR_INVALID_ARG, "q/k/v must be 16-byte aligned");

    void* scratch = scratch_address(device);
    if (!scratch) return LC_ERR_CUDA;
    cudaStream_t st = (cudaStream_t)lc_context_stream(ctx);

    // Sequence lengths: read on the host for the split plan (fixed-size stack
    // buffer, no allocation); a host array is also copied into the scratch.
    // Lengths in device memory are read on the context stream and waited
    // for, so values written by work queued there before this call are the
    // ones planned with.
    int32_t hl[kStaticMaxBatch];
    const Where lw = where_is(seq_len, device);
    if (lw == Where::kElsewhere)
        return lc_internal_set_error(LC_ERR_INVALID_ARG,
                                     "seq_len is device memory of another GPU (host memory or the context's "
                                     "device only)");
    const bool lens_on_device = lw == Where::kThisDevice;
    if (lens_on_device) {
        if (cudaMemcpyAsync(hl, seq_len, (size_t)batch * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaStreamSynchronize(st) != cudaSuccess)
            return lc_internal_set_error(LC_ERR_CUDA, "reading seq_len failed");
    } else {
        for (int b = 0; b < batch; ++b) hl[b] = seq_len[b];
    }
    int max_len = 0;
    for (int b = 0; b < batch; ++b) {
        if (hl[b] < 0) return lc_internal_set_error(LC_ERR_INVALID_ARG, "negative seq_len");
        if (hl[b] > max_len) max_len = hl[b];
    }
    if (max_len < 1) max_len = 1;

    AttnPlan plan = plan_attention(batch, n_heads, n_kv_heads, head_dim, max_len, lc_context_sm_count(ctx));
    const size_t need = attention_scratch_bytes(plan);
    const size_t lens_off = (need + 255) / 256 * 256;
    if (lens_off + (size_t)batch * 4 > kStaticScratchBytes)
        return lc_internal_set_error(LC_ERR_INVALID_ARG,
                                     "attention plan needs more than the 8 MiB static scratch (fewer sequences "
                                     "or shorter contexts per call)");
    const int32_t* dlens = seq_len;
    if (!lens_on_device) {
        int32_t* slot = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(scratch) + lens_off);
        if (cudaMemcpyAsync(slot, hl, (size_t)batch * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
            return lc_internal_set_error(LC_ERR_CUDA, "copying seq_len failed");
        dlens = slot;
    }
    cudaError_t e = launch_attention_decode(plan, q, k, v, out, dlens, seq_stride, head_stride, pos_stride, scratch,
                                            st);
    if (e != cudaSuccess) return lc_internal_set_error(LC_ERR_CUDA, cudaGetErrorString(e));
    // The host lengths were copied out of `hl` before cudaMemcpyAsync
    // returned (pageable source), so nothing here waits for the attention.
    return LC_OK;
}
