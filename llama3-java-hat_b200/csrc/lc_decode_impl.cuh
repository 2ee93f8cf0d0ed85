// lc_decode.cu -- the fused decode step: LlamaInference.forward
// (LlamaInference.java:117-164) with all TransformerBlock.forward calls
// (TransformerBlock.java:130-217), the final RMSNorm, the lm_head GEMV and the
// greedy argmax, for `nsteps` consecutive positions, in ONE cooperative
// persistent launch (one CTA per SM).
//
// Jobs of one position, in order, each ending with an exchange:
//   QKV  rmsnorm(x, attn_norm) -> [Wq;Wk;Wv] GEMV -> RoPE(q,k) -> q, KV cache
//   ATT  GQA attention units (kv head x split of positions) -> att / partials
//   O    (combine partials) -> Wo GEMV + residual -> x
//   GU   rmsnorm(x, ffn_norm) -> [gate|up] GEMV -> silu(gate)*up -> h
//   DN   Wdown GEMV + residual -> x
//   LM   rmsnorm(x, out_norm) -> lm_head GEMV -> logits, per-CTA argmax;
//        every CTA then merges the candidates into the next token.
//
// Weight bytes are >99.8% of the traffic.  One producer thread per CTA walks
// the CTA's whole multi-step tile schedule and moves 8-row weight tiles
// (layout in lc_internal.h) into a ring of shared-memory stages with 1-D bulk
// copies; it never waits for activations, so HBM keeps streaming while the
// consumer warps exchange data with the other CTAs.  A mover thread copies
// each landed tile into a ring of tensor-memory slots (tcgen05.cp), which
// frees the stage and adds the 256 KB of TMEM to the data in flight per SM.
// Eight consumer warps each read a fixed share of every tile with
// tcgen05.ld: 64 weights of one row against 64 fp32 inputs held in registers
// for the whole job, exact fp32 products on the FMA pipe.  Per-warp partial
// sums meet in shared memory and the job epilogue adds them in a fixed
// order.
//
// Exchanges: x (after O and DN), q, this position's k and v, the attention
// outputs and partials and the argmax candidates travel as 64-bit words
// {fp32 bits, tag}, the tag unique per (launch, position, exchange); readers
// poll the words themselves until every one carries the wanted tag, so one
// L2 round trip brings data and completion together.  h (the gate/up output,
// the widest vector) stays plain fp32: writers fence, then raise a per-CTA
// flag word to the tag, and readers wait for all flags with acquire.  The end
// of a position is a fenced flag exchange, which orders the plain KV-cache
// stores before every later position.  Every wait is bounded: a timeout
// records an error code in p.err, every later wait returns at once, all CTAs
// leave at the next step boundary, the producer drains its in-flight copies,
// and the host reports LC_ERR_TIMEOUT.
#pragma once
// Included by lc_decode.cu (LC_DECODE_TRACE 0) and lc_decode_trace.cu
// (LC_DECODE_TRACE 1, the phase-trace build of the same kernel).
#include "lc_attention.cuh"
#include "lc_internal.h"
#include "lc_stream.cuh"
#include "lc_tcgen05.cuh"

#ifndef LC_DECODE_TRACE
#error "define LC_DECODE_TRACE before including lc_decode_impl.cuh"
#endif

namespace lc {

namespace {

constexpr int kCW = 8;                // consumer warps
constexpr int kCT = kCW * 32;         // consumer threads
constexpr int kThreads = kCT + 128;   // + one warpgroup: producer (warp kCW), mover (warp kCW + 1), idle warps
// Register split (setmaxnreg, per warpgroup): the launch gives every thread
// 65536 / kThreads -> 168 registers; the producer warpgroup gives most of its
// share to the consumer warpgroups.  The sum must stay within the launch
// total or setmaxnreg.inc would wait forever.
constexpr int kRegLaunch = 168, kRegConsumer = 224, kRegProducer = 56;
static_assert(kCT * kRegConsumer + 128 * kRegProducer <= kThreads * kRegLaunch, "register split exceeds the pool");
constexpr uint32_t kBarC = 1;         // named barrier of the consumer threads
constexpr uint32_t kBarEnd = 6;       // consumers + the mover warp, before the TMEM is freed (2..5: attention pairs)
constexpr int kBatchTiles = 8;        // tiles per epilogue batch
constexpr int kBatchTilesWide = 16;   // ... of a job with one column block (partials past 8 tiles in act)
constexpr int kMaxStages = 24;
// Five 32 KB stages at dim 2048: the plan then fits the 196 KB shared-memory
// carveout and leaves 60 KB of L1 for the attention and activation loads
// (measured: 668 us per 1B forward against 674 us with six stages and a
// 28 KB L1, 689 us with four).
constexpr int kRingBytes = 160 * 1024;
constexpr int kAttnTmin = 64;         // positions per attention unit, at least
constexpr int kAttnTmax = 384;        // ... and at most
constexpr int kVChunk = 64;           // V positions staged in shared memory at a time
// Tensor memory: the whole 512 columns as a ring of weight tiles.  A tile of
// 8 rows x dim columns (dim = 128 KS) takes 4 KS columns of all 128 lanes.
constexpr int kTmemCols = 512;
constexpr int kTSlotsMax = 16;
__host__ __device__ constexpr int tmem_slots(int KS) {
    return kTmemCols / (4 * KS) < kTSlotsMax ? kTmemCols / (4 * KS) : kTSlotsMax;
}

enum Kind : int { kQKV = 0, kO = 1, kGU = 2, kDN = 3, kLM = 4 };

__host__ __device__ inline bool lm_needed(const DecodeParams& p, int pos) {
    return !(p.skip_prefill_logits && pos + 1 < p.n_prompt);
}

// Positions per attention unit at sequence length `seq`: one unit per kv head
// up to kAttnTmin positions (the exact single-split path), else about one
// unit per CTA.
__host__ __device__ inline int attn_split_len(int seq, int G, int n_kv) {
    if (seq <= kAttnTmin) return seq;
    int per = G / n_kv;
    if (per < 1) per = 1;
    int T = (seq + per - 1) / per;
    if (T < kAttnTmin) T = kAttnTmin;
    if (T > kAttnTmax) T = kAttnTmax;
    return T;
}

// Attention scratch in the act region: a K chunk and a V chunk (q and the
// probabilities sit in the ys region, see attn_unit).
__host__ __device__ inline int attn_scratch_floats(int /*kv_mul*/) { return 2 * kVChunk * kAttnHeadDim; }

struct Shared {
    int stop;       // consumers -> producer and mover: leave
    int next;       // argmax broadcast
    uint32_t tmem;  // TMEM base address (tcgen05.alloc)
    int pad;
    float red[kCW];
    float rmax[kCW];
    float bv[kCW];
    int bi[kCW];
};

// Shared-memory layout for dim = 128 * KS (offsets in bytes from the
// 1024-aligned base), all compile-time constants: act holds the largest GEMV
// input (h, up to kActFloats floats) or the attention scratch.
constexpr int kActFloats = 8192;
static_assert(2048 + (kBatchTilesWide - kBatchTiles) * 8 * kCW <= kActFloats,
              "the wide batches' partials must fit in act beside an input of dim <= 2048 floats");
struct Layout {
    int tile_bytes, stages;
    int off_bar, off_sh, off_act, off_ys, total;
};

__host__ __device__ constexpr Layout make_layout(int dim) {
    return Layout{16 * dim,
                  kRingBytes / (16 * dim) < kMaxStages ? kRingBytes / (16 * dim) : kMaxStages,
                  (kRingBytes / (16 * dim) < kMaxStages ? kRingBytes / (16 * dim) : kMaxStages) * 16 * dim,
                  0, 0, 0, 0};
}

// Barriers: full[kMaxStages], empty[kMaxStages] (smem stages), tfull,
// tempty[kTSlotsMax] (TMEM slots), mdone.
constexpr int kNumBars = 2 * kMaxStages + 2 * kTSlotsMax + 1;

__host__ __device__ constexpr Layout finish_layout(Layout L) {
    L.off_sh = (L.off_bar + kNumBars * 8 + 15) / 16 * 16;  // act and ys take float4 accesses
    L.off_act = L.off_sh + (int)((sizeof(Shared) + 15) / 16 * 16);
    L.off_ys = L.off_act + kActFloats * 4;
    L.total = L.off_ys + kBatchTiles * 8 * kCW * 4;
    return L;
}

template <int KS>
struct LayoutOf {
    static constexpr Layout L = finish_layout(make_layout(128 * KS));
    static_assert((L.off_act & 15) == 0 && (L.off_ys & 15) == 0, "act and ys take float4 accesses");
};

struct Smem {
    uint8_t* ring;
    uint64_t* full;    // smem stage landed (TMA transaction bytes)
    uint64_t* empty;   // smem stage copied to TMEM (mover's commit)
    uint64_t* tfull;   // TMEM slot written (mover's commit)
    uint64_t* tempty;  // TMEM slot read by every consumer warp
    uint64_t* mdone;   // the mover's last copies finished
    Shared* sh;
    float* act;   // GEMV input (normalised x, att, h) in fp32; attention scratch
    float* ys;    // [tile][row][warp] partial dot products of one batch
    int stages, tile_bytes;
};

// ------------------------------------------------------------- schedule --

struct JobGeo {
    const __half* W;
    int groups;  // row groups of 8
    int ncb;     // column blocks of dim columns
};

// Geometry of job `kind` of layer l (W from the layer table `layers`).
__host__ __device__ __forceinline__ JobGeo job_geo(const DecodeParams& p, const LayerW* layers, int kind, int l) {
    const int qdim = p.n_heads * p.head_dim, kvd = p.n_kv * p.head_dim;
    if (kind == kLM) return {p.lm_head, (p.vocab + 7) / 8, 1};
    const LayerW& L = layers[l];
    switch (kind) {
        case kQKV: return {L.wqkv, (qdim + 2 * kvd) / 8, 1};
        case kO: return {L.wo, p.dim / 8, qdim / p.dim};
        case kGU: return {L.wgu, 2 * p.hidden / 8, 1};
        default: return {L.wdown, p.dim / 8, p.hidden / p.dim};
    }
}

// Groups of a batch: at most kBatchTiles tiles, column-block-major inside;
// jobs of one column block take kBatchTilesWide (their input fills only dim
// floats of act, and the partials of the tiles past kBatchTiles go there).
// With one column block the tile order does not depend on the batch size.
__host__ __device__ __forceinline__ int batch_groups(int ncb) {
    if (ncb == 1) return kBatchTilesWide;
    const int b = kBatchTiles / ncb;
    return b < 1 ? 1 : b;
}

// ------------------------------------------------------------- producer --

// The producer warp walks the CTA's tile list of one position (built on the
// host, same order as the consumers' jobs) once per position.  The 32 lanes
// hold the next 32 entries (and prefetch the 32 after); lane 0 waits for a
// free stage and issues the copy.
__device__ __forceinline__ void run_producer(const DecodeParams& p, const Smem& sm) {
    const int lane = threadIdx.x & 31, cta = blockIdx.x;
    volatile int* err = p.err;
    volatile int* stop = &sm.sh->stop;
    const uint64_t policy = l2_policy_evict_first();
    const uint32_t tb = (uint32_t)sm.tile_bytes;
    const uint32_t nst = (uint32_t)sm.stages;
    const uint32_t* row = p.sched + (size_t)cta * p.sched_stride;
    const int nlay = p.sched_n[2 * cta], ntot = nlay + p.sched_n[2 * cta + 1];
    uint32_t it = 0, slot = 0, par = 1;
    bool ok = true;
    // L2 prefetch window (lane 0): cursor (ps, pi) at absolute tile Q runs up
    // to D tiles ahead of the copies, also while the copy waits for a free
    // stage, so HBM keeps streaming while the consumers wait for an exchange.
    // The table entry of the next prefetch is loaded one call ahead.
    const int D = p.l2_prefetch_tiles;
    int ps = 0, pi = 0;
    uint32_t Q = 0, pend = 0;
    bool have = false;
    auto pf_advance = [&]() {
        ++Q;
        if (++pi >= (lm_needed(p, p.pos0 + ps) ? ntot : nlay)) {
            pi = 0;
            ++ps;
        }
    };
    auto pf_step = [&](uint32_t copied) {
        if (D == 0) return;
        while (Q < copied && ps < p.nsteps) {
            pf_advance();
            have = false;
        }
        if (ps >= p.nsteps || Q >= copied + (uint32_t)D) return;
        if (!have) {
            pend = __ldg(row + pi);
            have = true;
            return;
        }
        prefetch_l2(p.wbase + ((size_t)pend << 8), tb);
        have = false;
        pf_advance();
    };
    for (int s = 0; s < p.nsteps && ok; ++s) {
        const int n = lm_needed(p, p.pos0 + s) ? ntot : nlay;
        uint32_t cur = lane < ntot ? __ldg(row + lane) : 0u;
        uint32_t nxt = 32 + lane < ntot ? __ldg(row + 32 + lane) : 0u;
        for (int i = 0; i < n; ++i) {
            if ((i & 31) == 0 && i > 0) {
                cur = nxt;
                nxt = i + 32 + lane < ntot ? __ldg(row + i + 32 + lane) : 0u;
            }
            const uint32_t e = __shfl_sync(0xffffffffu, cur, i & 31);
            int fail = 0;
            if (lane == 0) {
                if (!mbar_try_wait(&sm.empty[slot], par)) {
                    const uint64_t deadline = globaltimer_ns() + p.timeout_ns;
                    for (uint32_t k = 1;; ++k) {
                        pf_step(it);
                        if (mbar_try_wait(&sm.empty[slot], par)) break;
                        if ((k & 63u) == 0u) {
                            if (*stop != 0 || *err != 0) {
                                fail = 1;
                                break;
                            }
                            if (globaltimer_ns() > deadline) {
                                atomicCAS(const_cast<int*>(err), 0, (int)kDevTimeoutEmpty);
                                fail = 1;
                                break;
                            }
                        }
                    }
                }
                if (!fail) {
                    mbar_arrive_expect_tx(&sm.full[slot], tb);
                    bulk_g2s(sm.ring + (size_t)slot * tb, p.wbase + ((size_t)e << 8), tb, &sm.full[slot], policy);
                    pf_step(it + 1);
                }
            }
            if (__shfl_sync(0xffffffffu, fail, 0)) {
                ok = false;
                break;
            }
            ++it;
            if (++slot == nst) {
                slot = 0;
                par ^= 1u;
            }
        }
    }
    // Every issued copy must land before the CTA may exit.
    if (lane == 0) {
        const uint32_t first = it > nst ? it - nst : 0u;
        for (uint32_t k = first; k < it; ++k) {
            const uint64_t deadline = globaltimer_ns() + 200000000ull;
            while (!mbar_try_wait(&sm.full[k % nst], (k / nst) & 1u)) {
                if (globaltimer_ns() > deadline) {
                    atomicCAS(const_cast<int*>(err), 0, (int)kDevTimeoutDrain);
                    break;
                }
            }
        }
    }
}

// --------------------------------------------------------------- mover --

// The mover thread takes the CTA's tiles in the producer's order: once a
// tile has landed in its shared-memory stage and the next TMEM slot has been
// read by every consumer warp, it copies the tile into the slot with
// tcgen05.cp (kCopies pieces of 128 lanes x 256 bits) and commits twice, so
// the slot turns full for the consumers and the stage free for the producer
// when the copies are done.  With the stages and the slots together, up to
// stages + slots tiles are in flight or resident per SM while the consumers
// wait for an exchange.  Bounded waits, as the producer's.
template <int KS>
__device__ __forceinline__ void run_mover(const DecodeParams& p, const Smem& sm) {
    constexpr uint32_t kSlotCols = 4 * KS, kSlots = tmem_slots(KS), kCopies = KS / 2;
    const int cta = blockIdx.x;
    volatile int* err = p.err;
    volatile int* stop = &sm.sh->stop;
    const int nlay = p.sched_n[2 * cta], ntot = nlay + p.sched_n[2 * cta + 1];
    const uint32_t nst = (uint32_t)sm.stages, tb = (uint32_t)sm.tile_bytes;
    const uint32_t ring = smem_u32(sm.ring), tmem = sm.sh->tmem;
    auto wait = [&](uint64_t* bar, uint32_t par, int code) -> bool {
        if (mbar_try_wait(bar, par)) return true;
        const uint64_t deadline = globaltimer_ns() + p.timeout_ns;
        for (uint32_t k = 1;; ++k) {
            if (mbar_try_wait(bar, par)) return true;
            if ((k & 63u) == 0u) {
                if (*stop != 0 || *err != 0) return false;
                if (globaltimer_ns() > deadline) {
                    atomicCAS(const_cast<int*>(err), 0, code);
                    return false;
                }
            }
        }
    };
    uint32_t it = 0;
    bool ok = true;
    for (int s = 0; s < p.nsteps && ok; ++s) {
        const int n = lm_needed(p, p.pos0 + s) ? ntot : nlay;
        for (int i = 0; i < n; ++i, ++it) {
            const uint32_t stage = it % nst, spar = (it / nst) & 1u;
            const uint32_t slot = it % kSlots, tpar = ((it / kSlots) & 1u) ^ 1u;
            if (!wait(&sm.full[stage], spar, kDevTimeoutFull) || !wait(&sm.tempty[slot], tpar, kDevTimeoutEmpty)) {
                ok = false;
                break;
            }
            tc_fence_after();
#pragma unroll
            for (uint32_t j = 0; j < kCopies; ++j)
                tc_cp_128x256b(tmem + slot * kSlotCols + 8u * j, tc_desc_kmajor(ring + stage * tb + 4096u * j, 128, 256));
            tc_commit(&sm.tfull[slot]);
            tc_commit(&sm.empty[stage]);
        }
    }
    // Every issued copy must be done before the TMEM is freed.
    tc_commit(sm.mdone);
    const uint64_t deadline = globaltimer_ns() + 200000000ull;
    while (!mbar_try_wait(sm.mdone, 0)) {
        if (globaltimer_ns() > deadline) {
            atomicCAS(const_cast<int*>(err), 0, (int)kDevTimeoutDrain);
            break;
        }
    }
}

// ------------------------------------------------------- consumer helpers --

// The staged GEMV input in act, fp32: the thread's values v[k] are the
// float4 at index idx[k] of the vector (idx < 0: none).  Ends with a barrier
// that also makes `ok` (the thread's status so far) CTA-uniform.
template <int NV>
__device__ __forceinline__ bool stage_store(const Smem& sm, const float4 (&v)[NV], const int (&idx)[NV], bool ok) {
#pragma unroll
    for (int k = 0; k < NV; ++k)
        if (idx[k] >= 0) reinterpret_cast<float4*>(sm.act)[idx[k]] = v[k];
    return !bar_red_or(kBarC, kCT, !ok);
}

// Weight tiles in tensor memory.  tcgen05.cp.128x256b of a tile's bytes
// [4096 j, 4096 j + 4096) (column octets 32 j .. 32 j + 31 of the 8 rows,
// tiled layout of lc_internal.h) under a K-major no-swizzle descriptor with
// leading byte offset 128 and stride byte offset 256 puts row r, columns
// 256 j + 16 m + 2 cc and +1 into TMEM lane 8 m + r, column 8 j + cc of the
// tile's slot (m < 16, cc < 8).  Consumer warp w reads the lanes of its
// quarter q = w % 4 (m = 4 q + lane / 8, row r = lane % 8) and the slot's
// columns [2 KS h, 2 KS (h + 1)), h = w / 4: 2 KS words = 4 KS halves of one
// row, whose input columns are fixed per thread (xs_col; dot_share reads them
// from the staged vector).

// Input column of half e (0, 1) of word k of the thread's share of a tile.
template <int KS>
__device__ __forceinline__ int xs_col(int k, int e) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m = 4 * (warp & 3) + (lane >> 3), c = 2 * KS * (warp >> 2) + k;
    return 256 * (c >> 3) + 16 * m + 2 * (c & 7) + e;
}

// 2 KS consecutive 32-bit TMEM columns of the warp's 32 lanes (thread i:
// lane base + i), waited for.
template <int KS>
__device__ __forceinline__ void tmem_ld_share(uint32_t taddr, uint32_t (&v)[2 * KS]) {
    if constexpr (KS == 16) {
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
              "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]),
              "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),
              "=r"(v[30]), "=r"(v[31])
            : "r"(taddr));
    } else if constexpr (KS == 8) {
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
            : "r"(taddr));
    } else if constexpr (KS == 4) {
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                     : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                     : "r"(taddr));
    } else {
        static_assert(KS == 2, "dim 256, 512, 1024 or 2048");
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                     : "r"(taddr));
    }
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// d0 = fma(a0, b0, d0) and d1 = fma(a1, b1, d1), each an IEEE fma.rn, issued
// as one packed instruction (fma.rn.f32x2, sm_100a).
__device__ __forceinline__ void fma_pair(float& d0, float& d1, float a0, float a1, float b0, float b1) {
    asm("{\n\t.reg .b64 pa, pb, pc;\n\tmov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\tmov.b64 pc, {%0, %1};\n\t"
        "fma.rn.f32x2 pc, pa, pb, pc;\n\tmov.b64 {%0, %1}, pc;\n\t}"
        : "+f"(d0), "+f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// The thread's partial dot product over its share of one tile: exact
// products of the F16 weights with the fp32 inputs, four fp32 chains (word k
// of the share feeds chains 0, 1 when k is even and 2, 3 when k is odd), two
// of them advanced per packed FMA.  The inputs are read from the staged
// vector in shared memory (xrow: act at the column block's first column), a
// float4 per pair of words: the eight lanes of a row quarter read the same
// four floats, so a warp's load is four broadcast addresses.  Holding the
// 4 KS inputs in registers instead cost spills, and with them most of the
// consumers' time per tile.
template <int KS>
__device__ __forceinline__ float dot_share(const uint32_t (&v)[2 * KS], const float* xrow) {
    float a[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < 2 * KS; k += 2) {
        const float4 x = *reinterpret_cast<const float4*>(xrow + xs_col<KS>(k, 0));
        const float2 w0 = __half22float2(*reinterpret_cast<const __half2*>(&v[k]));
        const float2 w1 = __half22float2(*reinterpret_cast<const __half2*>(&v[k + 1]));
        fma_pair(a[0], a[1], w0.x, w0.y, x.x, x.y);
        fma_pair(a[2], a[3], w1.x, w1.y, x.z, x.w);
    }
    return (a[0] + a[1]) + (a[2] + a[3]);
}

// Tag of exchange k (0..5L) of step s: QKV, ATT, O, GU, DN of layer l are
// 5l+0..5l+4, the lm_head candidates 5L.
__device__ __forceinline__ uint32_t xtag(const DecodeParams& p, int s, int k) {
    return p.tag_base + (uint32_t)(s * (5 * p.n_layers + 1) + k) + 1u;
}

// After an exchange's stores (all consumer threads have issued theirs),
// thread 0 raises the CTA's flag.  The flag is a hint for when to look: the
// data words carry their own tags, so no fence is needed -- except at the
// end of a position (`fenced`), which orders the plain stores of the step
// (KV-cache rows, logits) before every CTA's next position.
__device__ __forceinline__ void publish(const DecodeParams& p, uint32_t tag, bool fenced = false) {
    named_bar_sync(kBarC, kCT);
    if (threadIdx.x == 0) {
        if (fenced) fence_acq_rel_gpu();
        st_flag(p.flags + blockIdx.x, tag);
    }
}

// The thread's float4 chunks idx[k] (< 0: none) of a tagged vector: all
// loads in flight together, stale chunks re-read.  Per-thread result.
template <int NV>
__device__ __forceinline__ bool gather_tagged(const DecodeParams& p, const uint64_t* src, const int (&idx)[NV],
                                              uint32_t want, float4 (&v)[NV]) {
    // All loads first (one round trip), then the tag checks.
    uint64_t w[NV][4];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        if (idx[k] >= 0) {
            ld_word2(src + 4 * (size_t)idx[k], w[k][0], w[k][1]);
            ld_word2(src + 4 * (size_t)idx[k] + 2, w[k][2], w[k][3]);
        }
    }
    bool fresh[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        fresh[k] = true;
        if (idx[k] >= 0) {
            v[k] = make_float4(__uint_as_float((uint32_t)w[k][0]), __uint_as_float((uint32_t)w[k][1]),
                               __uint_as_float((uint32_t)w[k][2]), __uint_as_float((uint32_t)w[k][3]));
#pragma unroll
            for (int j = 0; j < 4; ++j) fresh[k] = fresh[k] && (uint32_t)(w[k][j] >> 32) == want;
        }
    }
    // Slow path (chunks not yet written): re-read every stale chunk each
    // round, all loads of a round in flight together; bounded.
    bool stale = false;
#pragma unroll
    for (int k = 0; k < NV; ++k) stale = stale || !fresh[k];
    if (!stale) return true;
    // No sleep between rounds: each round is one L2 round trip already
    // (measured 3.5 us per 1B forward faster than a 128 ns back-off).
    const uint64_t deadline = globaltimer_ns() + p.timeout_ns;
    for (uint32_t it = 1;; ++it) {
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            if (!fresh[k]) {
                ld_word2(src + 4 * (size_t)idx[k], w[k][0], w[k][1]);
                ld_word2(src + 4 * (size_t)idx[k] + 2, w[k][2], w[k][3]);
            }
        }
        stale = false;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            if (!fresh[k]) {
                bool f = true;
#pragma unroll
                for (int j = 0; j < 4; ++j) f = f && (uint32_t)(w[k][j] >> 32) == want;
                if (f) {
                    v[k] = make_float4(__uint_as_float((uint32_t)w[k][0]), __uint_as_float((uint32_t)w[k][1]),
                                       __uint_as_float((uint32_t)w[k][2]), __uint_as_float((uint32_t)w[k][3]));
                    fresh[k] = true;
                } else {
                    stale = true;
                }
            }
        }
        if (!stale) return true;
        if ((it & 15u) == 0u && (*reinterpret_cast<volatile int*>(p.err) != 0 || globaltimer_ns() > deadline)) {
            atomicCAS(p.err, 0, (int)kDevTimeoutGrid);
            return false;
        }
    }
}

// A set of CTAs whose exchange flags a reader waits for: with units > 0,
// CTA i * G / units for i < units (all CTAs when units == G); otherwise the
// CTAs of ranks [ra[k], rb[k]) under rotation `shift` (rank = (cta + shift)
// % G), k < 3.
struct FlagSet {
    int units;
    int shift;
    int ra[3], rb[3];
};

__device__ __forceinline__ FlagSet all_ctas() {
    FlagSet f;
    f.units = gridDim.x;
    f.shift = 0;
    for (int k = 0; k < 3; ++k) f.ra[k] = f.rb[k] = 0;
    return f;
}

// Warp 0 polls the flags of the set until all reached `want` (bounded); the
// barrier (and with `acquire` a fence) orders the CTA's later loads after the
// flags.  Each lane polls at most kPollPerLane flags, all loads of a round in
// flight together.  Returns false (CTA-uniform) on timeout or a reported
// error.
constexpr int kPollPerLane = 8;  // grids up to 256 CTAs
__device__ __forceinline__ bool wait_flags(const DecodeParams& p, uint32_t want, FlagSet f, bool acquire = false) {
    bool ok = true;
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x, G = gridDim.x;
        int n = f.units;
        if (n == 0)
            for (int k = 0; k < 3; ++k) n += f.rb[k] - f.ra[k];
        // CTA index of each flag this lane polls (all CTAs: lane + 32 k).
        const bool all = f.units == G;
        int c[kPollPerLane];
#pragma unroll
        for (int k = 0; k < kPollPerLane; ++k) {
            const int i = lane + 32 * k;
            c[k] = 0;
            if (!all && i < n) {
                if (f.units > 0) {
                    c[k] = i * G / f.units;
                } else {
                    int j = i, q = 0;
                    while (q < 2 && j >= f.rb[q] - f.ra[q]) j -= f.rb[q] - f.ra[q++];
                    c[k] = (f.ra[q] + j - f.shift + G) % G;
                }
            }
        }
        const uint64_t deadline = globaltimer_ns() + p.timeout_ns;
        for (uint32_t it = 0;; ++it) {
            uint32_t v[kPollPerLane];
#pragma unroll
            for (int k = 0; k < kPollPerLane; ++k)
                v[k] = lane + 32 * k < n ? ld_flag(p.flags + (all ? lane + 32 * k : c[k])) : want;
            bool mine = true;
#pragma unroll
            for (int k = 0; k < kPollPerLane; ++k) mine &= (v[k] - want) < 0x80000000u;
            if (__all_sync(0xffffffffu, mine)) break;
            if ((it & 15u) == 15u) {
                if (*reinterpret_cast<volatile int*>(p.err) != 0) {
                    ok = false;
                    break;
                }
                if (globaltimer_ns() > deadline) {
                    if (lane == 0) atomicCAS(p.err, 0, (int)kDevTimeoutGrid);
                    ok = false;
                    break;
                }
            }
        }
        if (acquire) fence_acq_rel_gpu();
    }
    return !bar_red_or(kBarC, kCT, !ok);
}

// Phase-trace writer (consumer thread 0): one stamp per mark().
#if LC_DECODE_TRACE
struct Tracer {
    unsigned long long* base = nullptr;
    int n = 0, cap = 0;
    __device__ __forceinline__ void mark() { put(globaltimer_ns()); }
    __device__ __forceinline__ void put(unsigned long long v) {
        if (base) {
            if (n < cap) base[n] = v;
            ++n;
        }
    }
};
#else
// Untraced build: every trace call compiles away.
struct Tracer {
    static constexpr unsigned long long* base = nullptr;
    int n = 0, cap = 0;
    __device__ __forceinline__ void mark() {}
    __device__ __forceinline__ void put(unsigned long long) {}
};
#endif

// x*invRms*w (RMSNorm.java:43,48) of a vector -> act.  The weights
// are loaded before the exchange wait so their latency overlaps it.  src is
// an exchange buffer (fp32, after waiting for `want`) or, when null, the
// embedding row emb (f16).
__device__ __forceinline__ bool stage_norm(const DecodeParams& p, const Smem& sm, const uint64_t* src,
                                           const __half* emb, const float* __restrict__ w, uint32_t want,
                                           Tracer& tr) {
    const int tid = threadIdx.x, warp = tid >> 5, n4 = p.dim / 4;
    float4 wv[2], xv[2];
    int idx[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int i = tid + k * kCT;
        idx[k] = i < n4 ? i : -1;
        if (i < n4) wv[k] = __ldg(reinterpret_cast<const float4*>(w) + i);
    }
    bool ok = true;
    if (src) {
        // The tagged words are polled directly: no flag round trip.
        tr.mark();
        ok = gather_tagged<2>(p, src, idx, want, xv);
        tr.mark();
    } else {
        tr.mark();
        tr.mark();
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            if (idx[k] >= 0) {
                const uint2 u = __ldg(reinterpret_cast<const uint2*>(emb) + idx[k]);
                const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
                const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
                xv[k] = make_float4(a.x, a.y, b.x, b.y);
            }
        }
    }
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int i = tid + k * kCT;
        if (i < n4) {
            ss = fmaf(xv[k].x, xv[k].x, ss);
            ss = fmaf(xv[k].y, xv[k].y, ss);
            ss = fmaf(xv[k].z, xv[k].z, ss);
            ss = fmaf(xv[k].w, xv[k].w, ss);
        }
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) sm.sh->red[warp] = ss;
    named_bar_sync(kBarC, kCT);
    float tot = 0.0f;
#pragma unroll
    for (int k = 0; k < kCW; ++k) tot += sm.sh->red[k];
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)p.dim), p.eps)));
    float4 o[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        if (idx[k] >= 0) {
            o[k].x = __fmul_rn(__fmul_rn(xv[k].x, inv), wv[k].x);
            o[k].y = __fmul_rn(__fmul_rn(xv[k].y, inv), wv[k].y);
            o[k].z = __fmul_rn(__fmul_rn(xv[k].z, inv), wv[k].z);
            o[k].w = __fmul_rn(__fmul_rn(xv[k].w, inv), wv[k].w);
        }
    }
    return stage_store<2>(sm, o, idx, ok);
}

// Attention output of all heads -> act.  One split: copy; several: merge the
// partials (flash-decoding combine), one (head, 8 dims) per thread.  A
// partial record is [m, l, 0, 0, o[64]] in tagged words.
__device__ __forceinline__ bool stage_att(const DecodeParams& p, const Smem& sm, int nsplit, uint32_t want,
                                          Tracer& tr) {
    constexpr int HD = kAttnHeadDim;
    bool ok = true;  // tagged words, polled directly
    tr.mark();
    const int tid = threadIdx.x, qdim = p.n_heads * HD;
    float4 v[2];
    int idx[2] = {-1, -1};
    if (nsplit == 1) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int i = tid + k * kCT;
            if (i < qdim / 4) idx[k] = i;
        }
        ok = gather_tagged<2>(p, p.att, idx, want, v) && ok;
    } else if (tid < p.n_heads * (HD / 8)) {
        const int kv_mul = p.n_heads / p.n_kv;
        const int H = tid / (HD / 8), d0 = (tid % (HD / 8)) * 8;
        const uint64_t* base =
            p.part + ((size_t)(H / kv_mul) * p.attn_max_splits * kv_mul + H % kv_mul) * kDecodePartStride;
        const size_t sstride = (size_t)kv_mul * kDecodePartStride;
        float M = -INFINITY, L = 0.0f, O[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) O[j] = 0.0f;
        for (int sp = 0; sp < nsplit; ++sp) {
            // (m, l, -, -), o[d0..d0+3], o[d0+4..d0+7] of split sp
            const int widx[3] = {0, (4 + d0) / 4, (8 + d0) / 4};
            float4 w[3];
            ok = gather_tagged<3>(p, base + (size_t)sp * sstride, widx, want, w) && ok;
            const float Mn = fmaxf(M, w[0].x);
            const float wo = (M == -INFINITY) ? 0.0f : exp_via_double(__fsub_rn(M, Mn));
            const float wn = exp_via_double(__fsub_rn(w[0].x, Mn));
            L = fmaf(L, wo, w[0].y * wn);
            const float o8[8] = {w[1].x, w[1].y, w[1].z, w[1].w, w[2].x, w[2].y, w[2].z, w[2].w};
#pragma unroll
            for (int c = 0; c < 8; ++c) O[c] = fmaf(O[c], wo, o8[c] * wn);
            M = Mn;
        }
        const float inv = __fdiv_rn(1.0f, L);
        v[0] = make_float4(__fmul_rn(O[0], inv), __fmul_rn(O[1], inv), __fmul_rn(O[2], inv), __fmul_rn(O[3], inv));
        v[1] = make_float4(__fmul_rn(O[4], inv), __fmul_rn(O[5], inv), __fmul_rn(O[6], inv), __fmul_rn(O[7], inv));
        idx[0] = (H * HD + d0) / 4;
        idx[1] = idx[0] + 1;
    }
    tr.mark();
    return stage_store<2>(sm, v, idx, ok);
}

// Partials of tile t of a batch: [8 rows][kCW warps] floats.  Tiles past
// kBatchTiles (wide batches of one-column-block jobs, whose input takes the
// first dim floats of act) use act after the input.
__device__ __forceinline__ float* ys_tile(const Smem& sm, int dim, int t) {
    return t < kBatchTiles ? sm.ys + t * 8 * kCW : sm.act + dim + (t - kBatchTiles) * 8 * kCW;
}

// Sum over column blocks and warps of row r (0..7) of group gg of a batch of
// ng groups, fixed order.
__device__ __forceinline__ float row_sum(const Smem& sm, int dim, int ng, int ncb, int gg, int r) {
    float y = 0.0f;
    for (int cb = 0; cb < ncb; ++cb) {
        const float4* v = reinterpret_cast<const float4*>(ys_tile(sm, dim, cb * ng + gg) + r * kCW);
        const float4 a = v[0], b = v[1];
        y += ((a.x + a.y) + (a.z + a.w)) + ((b.x + b.y) + (b.z + b.w));
    }
    return y;
}

// x / (1 + exp(-x)) (SiLU.java:36-39) with the single-precision exponential:
// within two ulp of the reference's double-precision one.
__device__ __forceinline__ float silu_f(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }

// RoPE of one interleaved pair (RoPE.java:42-49); sc = (sin, cos) of the
// pair's angle at this position, from the model's table.
__device__ __forceinline__ void rope_pair(float& v0, float& v1, float2 sc) {
    const float a = v0, b = v1;
    v0 = __fsub_rn(__fmul_rn(a, sc.y), __fmul_rn(b, sc.x));
    v1 = __fadd_rn(__fmul_rn(a, sc.x), __fmul_rn(b, sc.y));
}

struct LmState {
    float bv;
    int bi;
    bool nan0;  // logits[0] is NaN (owner of row 0 only)
};

// Epilogue of one batch: groups [b0, b1) of job `kind`, ys complete; results
// go out as tagged words with tag `tg`.  For O and DN, `res` is this thread's
// residual x[b0 * 8 + tid] (tid < rows).
__device__ __forceinline__ void epilogue(const DecodeParams& p, const Smem& sm, int kind, int l, int pos, int b0,
                                         int b1, int ncb, float res, uint32_t tg, LmState& lm) {
    constexpr int HD = kAttnHeadDim;  // decode_plan: head_dim == 64
    const int tid = threadIdx.x, ng = b1 - b0, nrows = ng * 8;
    const int qdim = p.n_heads * HD, kvd = p.n_kv * HD;
    if (kind == kQKV) {
        for (int pi = tid; pi < nrows / 2; pi += kCT) {
            const int gg = pi >> 2, r = (pi & 3) * 2, R = (b0 + gg) * 8 + r;
            float y0 = row_sum(sm, p.dim, ng, 1, gg, r), y1 = row_sum(sm, p.dim, ng, 1, gg, r + 1);
            // q rows, then k rows, then v rows; k and q are rotated.
            const int kv = R < qdim ? -1 : (R < qdim + kvd ? 0 : 1);
            const int rr = R - (kv < 0 ? 0 : qdim + kv * kvd), i = rr & (HD - 1);
            if (kv <= 0) rope_pair(y0, y1, __ldg(p.rope_cs + (size_t)pos * (HD / 2) + (i >> 1)));
            if (kv < 0) {
                st_tag2(p.q + R, y0, y1, tg);
            } else {
                // the KV cache (plain, read at later positions) and this
                // position's k / v for the attention units (tagged)
                float* dst = (kv == 0 ? p.kcache : p.vcache) + (((size_t)l * p.n_kv + rr / HD) * p.max_seq + pos) * HD + i;
                *reinterpret_cast<float2*>(dst) = make_float2(y0, y1);
                st_tag2(p.kv + kv * kvd + rr, y0, y1, tg);
            }
        }
    } else if (kind == kGU) {
        // rows 4m..4m+3 = (gate, up) of h[2m], h[2m+1] (TransformerBlock.java:205-209)
        for (int pi = tid; pi < nrows / 4; pi += kCT) {
            const int gg = pi >> 1, r = (pi & 1) * 4, R = (b0 + gg) * 8 + r;
            const float h0 = __fmul_rn(silu_f(row_sum(sm, p.dim, ng, 1, gg, r)), row_sum(sm, p.dim, ng, 1, gg, r + 1));
            const float h1 =
                __fmul_rn(silu_f(row_sum(sm, p.dim, ng, 1, gg, r + 2)), row_sum(sm, p.dim, ng, 1, gg, r + 3));
            *reinterpret_cast<float2*>(p.h + (R >> 1)) = make_float2(h0, h1);
        }
    } else if (kind == kLM) {
        for (int k = tid; k < nrows; k += kCT) {
            const int R = b0 * 8 + k;
            if (R < p.vocab) {
                const float v = row_sum(sm, p.dim, ng, 1, k >> 3, k & 7);
                p.logits[R] = v;
                if (R == 0 && v != v) lm.nan0 = true;
                if (v == v && (lm.bi < 0 || v > lm.bv)) {
                    lm.bv = v;
                    lm.bi = R;
                }
            }
        }
    } else if (tid < nrows) {  // O, DN: residual add (TransformerBlock.java:195-198, 211-216)
        uint64_t* out = (kind == kO) ? p.xa : p.xb;
        st_tag1(out + b0 * 8 + tid, __fadd_rn(res, row_sum(sm, p.dim, ng, ncb, tid >> 3, tid & 7)), tg);
    }
}

LC_DEV uint64_t ld_word(const uint64_t* p) {
    uint64_t w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

// Value of tagged word w loaded from src; re-read until it carries `want`
// (bounded).  For residuals, which the prologue already saw complete.
__device__ __forceinline__ bool resolve_tagged1(const DecodeParams& p, const uint64_t* src, uint64_t w, uint32_t want,
                                                float* v) {
    const uint64_t deadline = globaltimer_ns() + p.timeout_ns;
    for (uint32_t it = 0; (uint32_t)(w >> 32) != want; ++it) {
        if ((it & 15u) == 15u && (*reinterpret_cast<volatile int*>(p.err) != 0 || globaltimer_ns() > deadline)) {
            atomicCAS(p.err, 0, (int)kDevTimeoutGrid);
            return false;
        }
        __nanosleep(64);
        w = ld_word(src);
    }
    *v = __uint_as_float((uint32_t)w);
    return true;
}

// Shared-memory view from the dynamic shared-memory base and the
// compile-time layout (no registers needed for it).
template <int KS>
__device__ __forceinline__ Smem smem_view() {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    constexpr Layout L = LayoutOf<KS>::L;
    Smem sm;
    sm.ring = smem_raw;
    sm.full = reinterpret_cast<uint64_t*>(smem_raw + L.off_bar);
    sm.empty = sm.full + kMaxStages;
    sm.tfull = sm.empty + kMaxStages;
    sm.tempty = sm.tfull + kTSlotsMax;
    sm.mdone = sm.tempty + kTSlotsMax;
    sm.sh = reinterpret_cast<Shared*>(smem_raw + L.off_sh);
    sm.act = reinterpret_cast<float*>(smem_raw + L.off_act);
    sm.ys = reinterpret_cast<float*>(smem_raw + L.off_ys);
    sm.stages = L.stages;
    sm.tile_bytes = L.tile_bytes;
    return sm;
}

struct RingPos {
    uint32_t slot, par;         // next TMEM slot and its phase parity
    int ok;                     // every slot so far was seen written
    unsigned long long waited;  // trace only: thread 0's ns waiting for slots
};

// The tiles of one batch (column blocks 0..ncb-1, groups [b0, b1)) into ys:
// per tile, the warp waits for its TMEM slot, loads its share, releases the
// slot at once (the mover may refill it while the products run), and lanes
// r < 8 write the warp's partial sum of row r.
template <int KS>
__device__ __forceinline__ RingPos consume_batch(const DecodeParams& p, RingPos r, int b0, int b1, int ncb, bool timing) {
    constexpr uint32_t kSlotCols = 4 * KS, kSlots = tmem_slots(KS);
    const Smem sm = smem_view<KS>();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, ng = b1 - b0;
    const uint32_t tbase = sm.sh->tmem + ((uint32_t)(32 * (warp & 3)) << 16) + 2u * KS * (uint32_t)(warp >> 2);
    for (int cb = 0; cb < ncb; ++cb) {
        const float* xrow = sm.act + cb * p.dim;
#pragma unroll 1
        for (int g = b0; g < b1; ++g) {
            const unsigned long long t0 = timing ? globaltimer_ns() : 0ull;
            bool got = r.ok && (mbar_try_wait(&sm.tfull[r.slot], r.par) ||
                                mbar_wait_bounded(&sm.tfull[r.slot], r.par, p.err, globaltimer_ns() + p.timeout_ns,
                                                  kDevTimeoutFull));
            // tcgen05.ld is warp-collective: the whole warp takes the same
            // branch.  A slot that was not seen written is never released
            // (the mover then stops on the error word).
            got = __all_sync(0xffffffffu, got);
            if (timing) r.waited += globaltimer_ns() - t0;
            float y = 0.0f;
            if (got) {
                uint32_t v[2 * KS];
                tc_fence_after();
                tmem_ld_share<KS>(tbase + r.slot * kSlotCols, v);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.tempty[r.slot]);
                y = dot_share<KS>(v, xrow);
            } else {
                r.ok = 0;
            }
            y += __shfl_xor_sync(0xffffffffu, y, 8);
            y += __shfl_xor_sync(0xffffffffu, y, 16);
            if (lane < 8) ys_tile(sm, p.dim, cb * ng + (g - b0))[lane * kCW + warp] = y;
            if (++r.slot == kSlots) {
                r.slot = 0;
                r.par ^= 1u;
            }
        }
    }
    return r;
}

// The CTA's groups [g0, g1) of one job: batches of tiles through the ring,
// epilogue per batch.  The only place tiles are consumed.
template <int KS>
__device__ __forceinline__ bool consume_job(const DecodeParams& p, const Smem& sm, RingPos& ring, int kind, int l,
                                            int pos, int g0, int g1, int ncb, const uint64_t* res_src,
                                            uint32_t res_tag, const __half* res_emb, uint32_t out_tag, LmState& lm,
                                            Tracer& tr) {
    const int tid = threadIdx.x;
    const int bg = batch_groups(ncb);
    bool ok = true;
    for (int b0 = g0; b0 < g1; b0 += bg) {
        const int b1 = min(g1, b0 + bg), ng = b1 - b0;
        // Residual of the thread's row (O, DN): requested now, used in the epilogue.
        const bool has_res = (kind == kO || kind == kDN) && tid < ng * 8;
        uint64_t resw = 0;
        float res = 0.0f;
        if (has_res) {
            if (res_src) resw = ld_word(res_src + b0 * 8 + tid);
            else res = __half2float(res_emb[b0 * 8 + tid]);
        }
        if (b0 == g0) tr.mark();
        ring.waited = 0;
        ring = consume_batch<KS>(p, ring, b0, b1, ncb, tr.base != nullptr);
        named_bar_sync(kBarC, kCT);
        if (b0 == g0) {
            tr.mark();
            tr.put(ring.waited);
        }
        if (has_res && res_src) ok = resolve_tagged1(p, res_src + b0 * 8 + tid, resw, res_tag, &res) && ok;
        epilogue(p, sm, kind, l, pos, b0, b1, ncb, res, out_tag, lm);
        named_bar_sync(kBarC, kCT);
        if (b0 == g0) tr.mark();
    }
    if (g0 >= g1) {
        tr.mark();
        tr.mark();
        tr.put(0);
        tr.mark();
    }
    return ok && ring.ok;
}

// ------------------------------------------------------------- consumer --

// One attention unit: positions [t0, t1) of kv head kvh for its kv_mul query
// heads at position pos (TransformerBlock.java:153-192 with
// Attention.java:32-61 and Softmax.java:28-51), written for latency.  The
// positions go through an online softmax in chunks of kVChunk.  With
// kv_mul <= 4 two warps serve each query head: warp (h, dp) scores positions
// [32 dp, 32 dp + 32) of the chunk, one per lane, the pair exchanges its
// chunk maximum and sum through a 64-thread named barrier, and each warp
// then produces dims [32 dp, 32 dp + 32) from the chunk's probabilities in
// shared memory.  With kv_mul > 4 one warp serves a head (two positions and
// two dims per lane, probabilities by shuffle).  Scores use four independent
// FMA chains over a K chunk held swizzled in shared memory (conflict-free
// row reads); values use eight.  K and V rows of earlier positions (plain
// fp32 cache, written at earlier positions) are requested into registers
// before the wait for this position's q, k and v (tagged words), and the
// next chunk's rows while the current one is computed.  One split writes the
// normalised output; several write (max, sum, unnormalised output) partials
// for the merge in stage_att.
__device__ __forceinline__ bool attn_unit(const DecodeParams& p, int s, int l, int pos, int kvh, int t0, int t1,
                                          int nsplit, int sp, const Smem& smv, Tracer& tr) {
    constexpr int HD = kAttnHeadDim, C = kVChunk;
    constexpr int NF4 = C * (HD / 4) / kCT;  // float4 of a K (and of a V) chunk per thread
    static_assert(NF4 * kCT == C * (HD / 4), "chunk must divide over the consumer threads");
    static_assert(C == 64 && HD == 64, "two lanes' worth of positions and dims per warp");
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int kv_mul = p.n_heads / p.n_kv, T = t1 - t0, pr = pos - t0;  // pr: row of pos in the unit
    const int kvd = p.n_kv * HD;
    const bool pair = kv_mul <= kCW / 2;  // two warps per query head
    const int h = pair ? warp >> 1 : warp, dp = pair ? warp & 1 : 0;
    const bool active = h < kv_mul;
    const uint32_t in_tag = xtag(p, s, 5 * l + 0), out_tag = xtag(p, s, 5 * l + 1);
    const size_t kvbase = (((size_t)l * p.n_kv + kvh) * p.max_seq + t0) * HD;
    const float4* K4 = reinterpret_cast<const float4*>(p.kcache + kvbase);
    const float4* V4 = reinterpret_cast<const float4*>(p.vcache + kvbase);
    float4* Ks4 = reinterpret_cast<float4*>(smv.act);  // [C][16] float4, slot j ^ (row & 15)
    float4* Vs4 = Ks4 + C * (HD / 4);                   // [C][16] float4
    const float* Vs = reinterpret_cast<const float*>(Vs4);
    float* qs = smv.ys;                                 // [kv_mul][HD]
    float* ps = smv.ys + (kCW / 2) * HD;                // [kv_mul][C] probabilities (pair mode)
    float4 kr[NF4], vr[NF4];
    // Cache rows [c0, c0 + C) of the unit into registers (row pos excluded).
    auto fetch = [&](int c0) {
        const int n4 = min(C, T - c0) * (HD / 4);
#pragma unroll
        for (int k = 0; k < NF4; ++k) {
            const int f = tid + k * kCT;
            if (f < n4 && c0 + (f >> 4) != pr) {
                kr[k] = __ldcg(K4 + (size_t)c0 * (HD / 4) + f);
                vr[k] = __ldcg(V4 + (size_t)c0 * (HD / 4) + f);
            }
        }
    };
    fetch(0);
    bool ok = true;
    tr.mark();
    // q of the kv head's query heads and this position's k, v: one float4
    // of tagged words per thread; q goes to shared memory, k and v stay in
    // the gathering threads' registers until their chunk is staged.
    const int nq = kv_mul * (HD / 4), cj = tid - nq;  // cj in [0, 32): k (< 16) or v chunk j of row pos
    float4 g = make_float4(0.f, 0.f, 0.f, 0.f);
    {
        const uint64_t* src = nullptr;
        if (tid < nq) src = p.q + ((size_t)kvh * kv_mul * HD + 4 * tid);
        else if (cj < HD / 2) src = p.kv + (size_t)(cj >> 4) * kvd + kvh * HD + (cj & 15) * 4;
        if (src) {
            const int one[1] = {0};
            float4 v[1];
            ok = gather_tagged<1>(p, src, one, in_tag, v) && ok;
            g = v[0];
        }
        if (tid < nq) reinterpret_cast<float4*>(qs)[tid] = g;
    }
    float m = -INFINITY, lsum = 0.0f;
    float acc[2][8];  // [dim of the lane][chain]
#pragma unroll
    for (int d = 0; d < 2; ++d)
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[d][c] = 0.0f;
    const float4* q4 = reinterpret_cast<const float4*>(qs + h * HD);
    const int i0 = pair ? dp * 32 + lane : lane;  // the lane's dim (one warp per head: also i0 + 32)
    const uint32_t pbar = 2u + (uint32_t)h;       // named barrier of the head's warp pair
    for (int c0 = 0; c0 < T; c0 += C) {
        const int n = min(C, T - c0);
        if (c0 > 0) named_bar_sync(kBarC, kCT);  // the previous chunk's reads are done
#pragma unroll
        for (int k = 0; k < NF4; ++k) {
            const int f = tid + k * kCT, row = f >> 4, j = f & 15;
            if (row < n && c0 + row != pr) {
                Ks4[row * 16 + (j ^ (row & 15))] = kr[k];
                Vs4[f] = vr[k];
            }
        }
        if (cj >= 0 && cj < HD / 2 && pr >= c0 && pr < c0 + C) {
            const int row = pr - c0, j = cj & 15;
            if (cj < 16) Ks4[row * 16 + (j ^ (row & 15))] = g;
            else Vs4[row * 16 + j] = g;
        }
        if (c0 == 0) {
            ok = !bar_red_or(kBarC, kCT, !ok);
            tr.mark();
        } else {
            named_bar_sync(kBarC, kCT);
        }
        if (c0 + C < T) fetch(c0 + C);
        if (active && ok) {
            // Scores of the lane's positions.
            float sc[2] = {-INFINITY, -INFINITY};
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                if (pair && k == 1) break;
                const int t = pair ? dp * 32 + lane : lane + 32 * k;
                if (t < n) {
                    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
                    for (int j = 0; j < HD / 4; ++j) {
                        const float4 kk = Ks4[t * 16 + (j ^ (t & 15))], qq = q4[j];
                        a0 = fmaf(qq.x, kk.x, a0);
                        a1 = fmaf(qq.y, kk.y, a1);
                        a2 = fmaf(qq.z, kk.z, a2);
                        a3 = fmaf(qq.w, kk.w, a3);
                    }
                    sc[k] = ((a0 + a1) + (a2 + a3)) * p.attn_scale;
                }
            }
            float mc = warp_max(fmaxf(sc[0], sc[1]));
            if (pair) {
                if (lane == 0) smv.sh->rmax[warp] = mc;
                named_bar_sync(pbar, 64);
                mc = fmaxf(smv.sh->rmax[warp & ~1], smv.sh->rmax[warp | 1]);
            }
            const float mn = fmaxf(m, mc);
            const float rs = (m == -INFINITY) ? 0.0f : expf(m - mn);
            const float e0 = sc[0] == -INFINITY ? 0.0f : expf(sc[0] - mn);
            const float e1 = sc[1] == -INFINITY ? 0.0f : expf(sc[1] - mn);
            float es = warp_sum(e0 + e1);
            if (pair) {
                ps[h * C + dp * 32 + lane] = e0;
                if (lane == 0) smv.sh->red[warp] = es;
                named_bar_sync(pbar, 64);
                es = smv.sh->red[warp & ~1] + smv.sh->red[warp | 1];
            }
            lsum = fmaf(lsum, rs, es);
            m = mn;
#pragma unroll
            for (int d = 0; d < 2; ++d)
#pragma unroll
                for (int c = 0; c < 8; ++c) acc[d][c] *= rs;
            // Weighted values.
            if (pair) {
                const float* prow = ps + h * C;
                const float* vcol = Vs + i0;
                for (int t8 = 0; t8 < n; t8 += 8) {
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const int t = t8 + c;
                        const float vv = t < n ? vcol[t * HD] : 0.0f;
                        acc[0][c] = fmaf(prow[t], vv, acc[0][c]);  // prow[t] is 0 past n
                    }
                }
            } else {
#pragma unroll
                for (int k = 0; k < 2; ++k) {
                    const float ek = k == 0 ? e0 : e1;
                    for (int t8 = 32 * k; t8 < min(n, 32 * k + 32); t8 += 8) {
#pragma unroll
                        for (int c = 0; c < 8; ++c) {
                            const int t = t8 + c;
                            const float pt = __shfl_sync(0xffffffffu, ek, t & 31);
                            const float v0 = t < n ? Vs[t * HD + i0] : 0.0f;
                            const float v1 = t < n ? Vs[t * HD + i0 + 32] : 0.0f;
                            acc[0][c] = fmaf(pt, v0, acc[0][c]);
                            acc[1][c] = fmaf(pt, v1, acc[1][c]);
                        }
                    }
                }
            }
        }
    }
    tr.mark();
    if (active && ok) {
        const float inv = __fdiv_rn(1.0f, lsum);
#pragma unroll
        for (int d = 0; d < 2; ++d) {
            if (d == 1 && pair) break;
            const int i = i0 + 32 * d;
            const float o = ((acc[d][0] + acc[d][1]) + (acc[d][2] + acc[d][3])) +
                            ((acc[d][4] + acc[d][5]) + (acc[d][6] + acc[d][7]));
            if (nsplit == 1) {
                st_tag1(p.att + ((size_t)kvh * kv_mul + h) * HD + i, __fmul_rn(o, inv), out_tag);
            } else {
                uint64_t* pp = p.part + (((size_t)kvh * p.attn_max_splits + sp) * kv_mul + h) * kDecodePartStride;
                st_tag1(pp + 4 + i, o, out_tag);
                if (i == 0) {
                    st_tag2(pp, m, lsum, out_tag);
                    st_tag2(pp + 2, 0.0f, 0.0f, out_tag);
                }
            }
        }
    }
    return ok;
}

// Attention units of layer l at position pos: unit u = (kv head, split) runs
// on CTA u * G / units.
__device__ __forceinline__ bool run_attention(const DecodeParams& p, const Smem& sm, int s, int l, int pos,
                                              Tracer& tr) {
    const int G = gridDim.x, cta = blockIdx.x, seq = pos + 1;
    const int T = attn_split_len(seq, G, p.n_kv), nsplit = (seq + T - 1) / T, units = p.n_kv * nsplit;
    bool ok = true;
    const int trace_n = tr.n;
    // units * G < 2^31 (units <= n_kv * max splits)
    for (int u = (cta * units + G - 1) / G; u < units && (u * G) / units == cta; ++u) {
        const int kvh = u / nsplit, sp = u % nsplit;
        const int t0 = sp * T, t1 = min(seq, t0 + T);
        ok &= attn_unit(p, s, l, pos, kvh, t0, t1, nsplit, sp, sm, tr);
        named_bar_sync(kBarC, kCT);
        tr.mark();
    }
    // Fixed trace layout: four stamps per layer (first unit), with or without
    // units.  (Only thread 0 records; the loop is bounded for every thread.)
    for (int k = tr.n - trace_n; k < 4; ++k) tr.mark();
    if (tr.base) tr.n = trace_n + 4;
    return ok;
}

// h (all hidden floats) -> act, after the gate/up exchange.
__device__ __forceinline__ bool stage_h(const DecodeParams& p, const Smem& sm, uint32_t want, Tracer& tr) {
    // h is plain fp32 (half the bytes of tagged words): the gate/up
    // epilogues publish it with a fence, the flags are read with acquire.
    // (Tagged h measured slower: 639 against 598 us per 1B forward, and 666
    // with the flags polled first; the fence costs about 1.5 us per layer.)
    constexpr int NV = 8;  // float4 per thread: hidden <= 8 * 4 * kCT (decode_plan)
    const bool ok = wait_flags(p, want, all_ctas(), true);
    tr.mark();
    float4 v[NV];
    int idx[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int i = threadIdx.x + k * kCT;
        idx[k] = i < p.hidden / 4 ? i : -1;
        if (idx[k] >= 0) v[k] = __ldcg(reinterpret_cast<const float4*>(p.h) + i);
    }
    tr.mark();
    return stage_store<NV>(sm, v, idx, ok);
}

// lm_head epilogue: the CTA's argmax candidate (LlamaInference.argmax
// semantics, :252-262) goes out, then every CTA merges all candidates.
__device__ __forceinline__ bool argmax_exchange(const DecodeParams& p, const Smem& sm, int s, const LmState& lm,
                                                int* next) {
    const int G = gridDim.x, cta = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t tag = xtag(p, s, 5 * p.n_layers);
    float bv = lm.bv;
    int bi = lm.bi;
    for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_merge(bv, bi, v2, i2);
    }
    const bool nan0 = bar_red_or(kBarC, kCT, lm.nan0);
    if (lane == 0) {
        sm.sh->bv[warp] = bv;
        sm.sh->bi[warp] = bi;
    }
    named_bar_sync(kBarC, kCT);
    if (tid == 0) {
        float B = sm.sh->bv[0];
        int I = sm.sh->bi[0];
        for (int w = 1; w < kCW; ++w) argmax_merge(B, I, sm.sh->bv[w], sm.sh->bi[w]);
        // NaN in logits[0] makes the Java argmax return 0 (nothing is '>'
        // NaN): the owner of row 0 offers (+inf, 0), which wins.
        if (nan0) {
            B = INFINITY;
            I = 0;
        }
        st_tag2(p.amax + 2 * cta, B, __int_as_float(I), tag);
    }
    // The end of a position: fenced, so the step's plain stores (KV-cache
    // rows, h) are visible to every CTA's next position.
    publish(p, tag, true);
    bool ok = wait_flags(p, tag, all_ctas(), true);
    if (warp == 0) {
        float B = -INFINITY;
        int I = -1;
        float2 v[kPollPerLane];
        bool got[kPollPerLane];
#pragma unroll
        for (int k = 0; k < kPollPerLane; ++k)
            got[k] = lane + 32 * k < G && ld_tag2(p.amax + 2 * (lane + 32 * k), tag, v[k]);
#pragma unroll
        for (int k = 0; k < kPollPerLane; ++k) {
            if (lane + 32 * k < G) {
                // cannot fail after the fenced exchange
                if (!got[k]) ok = false;
                else argmax_merge(B, I, v[k].x, __float_as_int(v[k].y));
            }
        }
        for (int o = 16; o > 0; o >>= 1) {
            const float v2 = __shfl_xor_sync(0xffffffffu, B, o);
            const int i2 = __shfl_xor_sync(0xffffffffu, I, o);
            argmax_merge(B, I, v2, i2);
        }
        if (lane == 0) sm.sh->next = I < 0 ? 0 : I;
    }
    ok = !bar_red_or(kBarC, kCT, !ok);
    *next = *reinterpret_cast<volatile int*>(&sm.sh->next);
    return ok;
}

// One position = jobs j = 0 .. 4L-1 (layer j/4, kind j%4) and, when logits
// are needed, the lm_head job j = 4L.  Every job is: prologue (exchange
// wait + staging), consume_job, publish, then the attention units after QKV
// and the argmax exchange after LM.  Each piece appears once in the code.
template <int KS>
__device__ __forceinline__ void run_consumer(const DecodeParams& p, const Smem& sm) {
    const int G = gridDim.x, cta = blockIdx.x, tid = threadIdx.x, NL = p.n_layers;
    Tracer tr;
#if LC_DECODE_TRACE
    if (p.trace && tid == 0) {
        tr.base = p.trace + (size_t)cta * p.trace_words;
        tr.cap = p.trace_words;
    }
#endif
    Rotation rot;
    RingPos ring;
    ring.slot = 0;
    ring.par = 0;
    ring.ok = 1;
    ring.waited = 0;
    int next = 0, steps_done = 0;
    bool ok = true;
    LmState lm;
    lm.bv = -INFINITY;
    lm.bi = -1;
    lm.nan0 = false;

    for (int s = 0; s < p.nsteps; ++s) {
        const int pos = p.pos0 + s;
        const int token = (s == 0 || pos < p.n_prompt) ? __ldcg(p.tokens + pos) : next;
        if (token < 0 || token >= p.vocab) {
            if (cta == 0 && tid == 0) atomicCAS(p.err, 0, (int)kDevBadToken);
            ok = false;
        }
        // Leave on a CTA-uniform decision only.
        if (bar_red_or(kBarC, kCT, !ok || *reinterpret_cast<volatile int*>(p.err) != 0)) break;
        const __half* emb = p.tok_emb + (size_t)token * (size_t)p.dim;
        rot = Rotation();  // every position deals rows alike (the producer's tile list)
        const int seq = pos + 1;
        const int nsplit = (seq + attn_split_len(seq, G, p.n_kv) - 1) / attn_split_len(seq, G, p.n_kv);
        const int njobs = 4 * NL + (lm_needed(p, pos) ? 1 : 0);

#pragma unroll 1
        for (int j = 0; j < njobs; ++j) {
            const int kind = (j == 4 * NL) ? (int)kLM : (j & 3), l = (j == 4 * NL) ? NL - 1 : (j >> 2);
            // Exchange this job waits for: the previous job's output.
            const uint32_t want = xtag(p, s, 5 * l + (kind == kQKV ? -1 : kind == kO ? 1 : kind == kGU ? 2 : kind == kDN ? 3 : 4));
            tr.mark();
            const JobGeo jg = job_geo(p, p.layers, kind, l);
            int g0, g1;
            job_range(jg.groups, 1, G, rot.rank(cta, G), &g0, &g1);
            rot.advance(jg.groups, 1, G);
            if (kind == kO) {
                ok &= stage_att(p, sm, nsplit, want, tr);
            } else if (kind == kDN) {
                ok &= stage_h(p, sm, want, tr);
            } else {
                const bool first = (kind == kQKV && l == 0);
                const float* w = (kind == kQKV) ? p.norm_w[2 * l] : (kind == kGU) ? p.norm_w[2 * l + 1] : p.out_norm;
                // x after O for GU, after DN (previous layer) for QKV and LM
                ok &= stage_norm(p, sm, first ? nullptr : (kind == kGU ? p.xa : p.xb), emb, w, want, tr);
            }
            if (kind == kLM) {
                lm.bv = -INFINITY;
                lm.bi = -1;
                lm.nan0 = false;
            }
            tr.mark();
            // residual of O: x of the block input (embedding in layer 0); of DN: x after O
            const uint64_t* res_src = (kind == kDN) ? p.xa : (l == 0 ? nullptr : p.xb);
            const uint32_t res_tag = (kind == kDN) ? xtag(p, s, 5 * l + 2) : xtag(p, s, 5 * l - 1);
            // kinds QKV, O, GU, DN publish exchanges 5l + 0, 2, 3, 4
            const uint32_t out_tag = xtag(p, s, 5 * l + (kind == kQKV ? 0 : kind + 1));
            ok &= consume_job<KS>(p, sm, ring, kind, l, pos, g0, g1, jg.ncb, res_src, res_tag, emb, out_tag, lm, tr);
            if (kind == kLM) {
                ok &= argmax_exchange(p, sm, s, lm, &next);
            } else {
                publish(p, out_tag, kind == kGU);  // h is plain fp32: fenced
                if (kind == kQKV) {
                    tr.mark();
                    ok &= run_attention(p, sm, s, l, pos, tr);
                    publish(p, xtag(p, s, 5 * l + 1));
                }
            }
            tr.mark();
        }

        if (!lm_needed(p, pos)) {
            // End of a position without logits: the same fenced exchange.
            publish(p, xtag(p, s, 5 * NL), true);
            ok &= wait_flags(p, xtag(p, s, 5 * NL), all_ctas(), true);
        }
        bool stop_now = false;
        if (lm_needed(p, pos) && pos + 1 >= p.n_prompt) {
            if (cta == 0 && tid == 0) {
                p.tokens[pos + 1] = next;
                if (p.stream) {
                    volatile int32_t* hs = p.stream;
                    const int i = pos + 1 - p.n_prompt;
                    hs[1 + i] = next;
                    __threadfence_system();
                    hs[0] = i + 1;
                }
            }
            for (int k = 0; k < p.n_stop; ++k) stop_now |= (p.stop[k] == next);
        }
        if (ok) steps_done = s + 1;
        if (stop_now) break;
    }
    if (tid == 0) {
        sm.sh->stop = 1;
        if (cta == 0) *p.n_done = steps_done;
    }
}

template <int KS>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ DecodeParams p) {
    constexpr Layout L = LayoutOf<KS>::L;
    const Smem sm = smem_view<KS>();
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        for (int s = 0; s < L.stages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);
        }
        for (int t = 0; t < tmem_slots(KS); ++t) {
            mbar_init(&sm.tfull[t], 1);
            mbar_init(&sm.tempty[t], kCW);
        }
        mbar_init(sm.mdone, 1);
        sm.sh->stop = 0;
        sm.sh->next = 0;
        fence_mbar_init();
    }
    // One CTA per SM (all shared memory taken): the whole TMEM is free.
    if (warp == kCW + 1) {
        tmem_alloc(&sm.sh->tmem, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x >= kCT) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegProducer));
        if (warp == kCW) {
            run_producer(p, sm);
        } else if (warp == kCW + 1) {
            if ((threadIdx.x & 31) == 0) run_mover<KS>(p, sm);
            __syncwarp();
            named_bar_sync(kBarEnd, kCT + 32);
            tc_fence_after();
            tmem_dealloc(sm.sh->tmem, kTmemCols);
        }
        return;
    }
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegConsumer));
    run_consumer<KS>(p, sm);
    tc_fence_before();
    named_bar_sync(kBarEnd, kCT + 32);
}

template <int KS>
cudaError_t launch_ks(const DecodeParams& p, const DecodeLaunch& l, cudaStream_t st) {
    void* args[] = {const_cast<DecodeParams*>(&p)};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(l.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = l.smem_bytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, (const void*)decode_kernel<KS>, args);
}

// Sets the shared-memory attribute and checks the register count the
// setmaxnreg split is built on: with fewer registers per thread at launch the
// pool could not serve the consumers' increase.
template <int KS>
cudaError_t set_smem(int bytes) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, decode_kernel<KS>);
    if (e != cudaSuccess) return e;
    if (fa.numRegs != kRegLaunch) return cudaErrorInvalidKernelImage;
    return cudaFuncSetAttribute(decode_kernel<KS>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

cudaError_t impl_prepare(const DecodeLaunch& l) {
    switch (l.ks) {
        case 2: return set_smem<2>(l.smem_bytes);
        case 4: return set_smem<4>(l.smem_bytes);
        case 8: return set_smem<8>(l.smem_bytes);
        default: return set_smem<16>(l.smem_bytes);
    }
}

cudaError_t impl_launch(const DecodeParams& p, const DecodeLaunch& l, cudaStream_t st) {
    switch (l.ks) {
        case 2: return launch_ks<2>(p, l, st);
        case 4: return launch_ks<4>(p, l, st);
        case 8: return launch_ks<8>(p, l, st);
        default: return launch_ks<16>(p, l, st);
    }
}

}  // namespace
}  // namespace lc
