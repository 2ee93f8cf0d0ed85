// lc_keyx.cu -- all-reduce (max) of packed argmax keys over NVLink peer memory.
//
// The lm_head row shard (H/LlamaInference.java:151-156 split by rows over N
// GPUs, one process per GPU) leaves every rank with one packed 64-bit argmax
// key per sequence (value bits above the inverted index: the maximum key is
// LlamaInference.argmax, :252-262).  The exchange is N * B * 8 bytes, so it
// is pure latency: instead of a library collective, one CTA per rank stores
// its keys straight into every rank's mailbox (peer memory mapped through
// CUDA IPC, plain NVLink stores, no multicast), raises one release flag per
// mailbox, waits (bounded) for the other ranks' flags in its own mailbox and
// takes the maximum.
//
// Mailbox of a rank: keys [2][world][max_batch] (slot parity = epoch & 1),
// then flags [world] (the latest epoch rank p has published there).  A rank
// can run at most one call ahead of another -- call e + 2 waits for the
// other's flag e + 1, which that rank raises only after its call e has read
// its mailbox -- so two parities keep every slot intact until it is read.
#include "lc_internal.h"

namespace lc {
namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(256) keyx_kernel(const __grid_constant__ KeyxArgs a) {
    __shared__ int fail;
    griddep_wait();  // the keys come from the predecessor (the lm_head product)
    const int tid = threadIdx.x, W = a.world, B = a.batch;
    const size_t par = a.epoch & 1u;
    // 1. this rank's keys into slot [par][rank] of every mailbox (its own too)
    for (int i = tid; i < W * B; i += blockDim.x) {
        const int p = i / B, b = i - p * B;
        a.keys_mbox[p][(par * W + a.rank) * a.max_batch + b] = a.keys[b];
    }
    if (tid == 0) fail = 0;
    __syncthreads();
    // 2. one release per mailbox (cumulative over the CTA's stores above)
    if (tid < W) {
        __threadfence_system();
        st_release_sys(a.flags_mbox[tid] + a.rank, a.epoch);
    }
    // 3. every other rank's flag in this rank's mailbox, bounded
    if (tid < W && tid != a.rank) {
        const uint32_t* f = a.flags_mbox[a.rank] + tid;
        const uint64_t deadline = globaltimer_ns() + a.timeout_ns;
        for (uint32_t it = 0; (int32_t)(ld_acquire_sys(f) - a.epoch) < 0; ++it) {
            if ((it & 15u) == 15u &&
                (*reinterpret_cast<volatile int*>(a.err) != 0 || globaltimer_ns() > deadline)) {
                atomicCAS(a.err, 0, (int)kDevTimeoutGrid);
                fail = 1;
                break;
            }
            __nanosleep(32);
        }
    }
    __syncthreads();
    if (fail) return;
    // 4. maximum over the ranks' slots (order-free: the result is exact)
    const uint64_t* mine = a.keys_mbox[a.rank] + par * W * a.max_batch;
    for (int b = tid; b < B; b += blockDim.x) {
        unsigned long long k = 0ull;
        for (int p = 0; p < W; ++p) {
            const unsigned long long v = __ldcg(reinterpret_cast<const unsigned long long*>(mine) + (size_t)p * a.max_batch + b);
            k = v > k ? v : k;
        }
        a.keys[b] = k;
    }
}

}  // namespace

size_t keyx_mailbox_bytes(int world, int max_batch) {
    return keyx_flags_offset(world, max_batch) + (size_t)world * sizeof(uint32_t);
}

cudaError_t launch_keyx(const KeyxArgs& a, cudaStream_t st, bool pdl) {
    if (a.world < 1 || a.world > kKeyxMaxWorld || a.rank < 0 || a.rank >= a.world || a.batch < 1 ||
        a.batch > a.max_batch)
        return cudaErrorInvalidValue;
    return launch_ex(keyx_kernel, dim3(1), dim3(256), 0, st, pdl, a);
}

}  // namespace lc
