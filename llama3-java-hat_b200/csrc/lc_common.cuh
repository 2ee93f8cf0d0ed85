// lc_common.cuh -- device helpers shared by the llamacuda kernels (sm_100a).
//
// PTX wrappers for mbarriers, 1-D bulk async copies (cp.async.bulk, no tensor
// map, no multicast), L2 cache policies, gpu-scope acquire/release, and the
// bounded-wait helpers every spin loop in this library goes through: a wait
// that runs past its deadline sets the device error word and returns false
// instead of spinning forever.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define LC_DEV __device__ __forceinline__

namespace lc {

// Device error codes written to the error word (host maps them to LC_ERR_*).
enum DevError : int {
    kDevOk = 0,
    kDevTimeoutFull = 1,     // consumer waited too long for a weight stage
    kDevTimeoutEmpty = 2,    // producer waited too long for a free stage
    kDevTimeoutGrid = 3,     // grid barrier did not complete in time
    kDevTimeoutDrain = 4,    // in-flight copies did not land at exit
    kDevBadToken = 5,        // token id outside [0, vocab)
    kDevBadPos = 6,          // position outside [0, max_seq)
};

LC_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

LC_DEV uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- mbarrier --

LC_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

LC_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

LC_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}

LC_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

LC_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and records `code` in the
// error word) when the deadline passes or another thread already failed.
LC_DEV bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, volatile int* err, uint64_t deadline_ns, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 0u) {
            if (*err != 0) return false;
            if (globaltimer_ns() > deadline_ns) {
                atomicCAS(const_cast<int*>(err), 0, code);
                return false;
            }
        }
    }
}

// ------------------------------------------------------------ bulk copies --

// L2 policy for weights: they are streamed once per decode step and must not
// push activations and the KV cache out of L2.
LC_DEV uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// L2 policy for data every CTA reads again (batched activations).
LC_DEV uint64_t l2_policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// 1-D bulk copy global -> this CTA's shared memory, completion signalled as
// transaction bytes on `bar`.  dst, src and bytes must be multiples of 16.
LC_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Starts pulling [src, src+bytes) from HBM into L2 without waiting for it
// (no shared-memory destination, no completion tracking).  bytes % 16 == 0.
LC_DEV void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ------------------------------------------- programmatic dependent launch --
//
// A kernel launched with programmatic stream serialisation may start while
// its predecessor in the stream is still running.  griddep_wait() blocks
// until the predecessor grid has completed and its memory operations are
// visible; it returns at once when the kernel was launched normally.
// griddep_launch() lets the dependent kernel be scheduled before this one
// finishes (each dependent still waits for this grid's completion).
LC_DEV void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
LC_DEV void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------ named CTA barriers --

LC_DEV void named_bar_sync(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------ gpu-scope ordering --

LC_DEV uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

LC_DEV void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

LC_DEV void red_release_gpu_add(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// --------------------------------------------------------- small numerics --

LC_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

LC_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// (float)Math.exp((double)x) -- the reference widens to double before exp.
LC_DEV float exp_via_double(float x) { return static_cast<float>(exp(static_cast<double>(x))); }

// x / (1.0f + (float)Math.exp(-x))  (SiLU.java:36-39), no contraction.
LC_DEV float silu_ref(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, exp_via_double(-x))); }

// Out-of-line copies for the fused kernel: one body each instead of one per
// call site keeps its instruction footprint small.
static __device__ __noinline__ float exp_via_double_nl(float x) { return exp_via_double(x); }
static __device__ __noinline__ float silu_ref_nl(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, exp_via_double(-x))); }
// (float)Math.cos / Math.sin of (double)val (RoPE.java:45-46).
static __device__ __noinline__ float2 sincos_ref_nl(float val) {
    double s, c;
    sincos((double)val, &s, &c);
    return make_float2((float)s, (float)c);
}

// 8 packed halves -> 8 floats.
LC_DEV void unpack_h8(const uint4& w, float f[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&w);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float2 t = __half22float2(h[j]);
        f[2 * j] = t.x;
        f[2 * j + 1] = t.y;
    }
}

// Argmax candidate merge with LlamaInference.argmax semantics
// (LlamaInference.java:252-262): larger value wins, equal values keep the
// lower index; idx < 0 marks "no non-NaN value seen".
LC_DEV void argmax_merge(float& bv, int& bi, float v, int i) {
    if (i < 0) return;
    if (bi < 0 || v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}

}  // namespace lc


namespace lc {

// ------------------------------------------------- tagged exchange words --
//
// Exchanged activations travel as 64-bit words: the float's bits in the low
// half, the tag of the exchange that produced them in the high half.  An
// aligned 64-bit store is single-copy atomic, so a reader that sees the tag
// it waits for also sees the value stored with it, without a fence on
// either side.

LC_DEV uint64_t tag_word(float v, uint32_t tag) { return ((uint64_t)tag << 32) | (uint64_t)__float_as_uint(v); }

// Two tagged words, 16 bytes, p 16-byte aligned.
LC_DEV void st_tag2(uint64_t* p, float a, float b, uint32_t tag) {
    asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(tag_word(a, tag)), "l"(tag_word(b, tag))
                 : "memory");
}
LC_DEV void st_tag1(uint64_t* p, float a, uint32_t tag) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(tag_word(a, tag)) : "memory");
}
LC_DEV void ld_word2(const uint64_t* p, uint64_t& a, uint64_t& b) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
// Four tagged words at p (16-byte aligned) -> v; true when all carry `want`.
LC_DEV bool ld_tag4(const uint64_t* p, uint32_t want, float4& v) {
    uint64_t a, b, c, d;
    ld_word2(p, a, b);
    ld_word2(p + 2, c, d);
    v = make_float4(__uint_as_float((uint32_t)a), __uint_as_float((uint32_t)b), __uint_as_float((uint32_t)c),
                    __uint_as_float((uint32_t)d));
    return (uint32_t)(a >> 32) == want && (uint32_t)(b >> 32) == want && (uint32_t)(c >> 32) == want &&
           (uint32_t)(d >> 32) == want;
}
LC_DEV bool ld_tag2(const uint64_t* p, uint32_t want, float2& v) {
    uint64_t a, b;
    ld_word2(p, a, b);
    v = make_float2(__uint_as_float((uint32_t)a), __uint_as_float((uint32_t)b));
    return (uint32_t)(a >> 32) == want && (uint32_t)(b >> 32) == want;
}

// ------------------------------------------------------ exchange flags --
LC_DEV void st_flag(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
LC_DEV uint32_t ld_flag(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// CTA-uniform OR of a predicate over the threads of named barrier `id`.
LC_DEV bool bar_red_or(uint32_t id, uint32_t nthreads, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
        : "memory");
    return r != 0;
}

}  // namespace lc
