// lc_decode.cu -- host side of the fused decode step (planning, tile
// schedule, weight tiling) and the untraced build of its kernel
// (lc_decode_impl.cuh).
#define LC_DECODE_TRACE 0
#include "lc_decode_impl.cuh"

namespace lc {

int decode_attn_max_splits(int max_seq, int grid, int n_kv) {
    int best = 1;
    // nsplit(seq) is not monotone in seq; take the maximum over the range.
    for (int seq = kAttnTmin + 1; seq <= max_seq; ++seq) {
        const int T = attn_split_len(seq, grid, n_kv);
        const int n = (seq + T - 1) / T;
        if (n > best) best = n;
    }
    return best;
}

void decode_build_schedule(const DecodeParams& p, const LayerW* layers, int G, std::vector<uint32_t>* sched,
                           std::vector<int>* counts, int* stride) {
    std::vector<std::vector<uint32_t>> rows(G);
    counts->assign(2 * (size_t)G, 0);
    const size_t tile_halves = (size_t)8 * p.dim;
    size_t longest = 0;
    for (int c = 0; c < G; ++c) {
        Rotation rot;
        auto emit = [&](int kind, int l) {
            const JobGeo jg = job_geo(p, layers, kind, l);
            int g0, g1;
            job_range(jg.groups, 1, G, rot.rank(c, G), &g0, &g1);
            rot.advance(jg.groups, 1, G);
            const int bg = batch_groups(jg.ncb);
            for (int b0 = g0; b0 < g1; b0 += bg) {
                const int b1 = b0 + bg < g1 ? b0 + bg : g1;
                for (int cb = 0; cb < jg.ncb; ++cb)
                    for (int g = b0; g < b1; ++g) {
                        const __half* t = jg.W + ((size_t)g * jg.ncb + cb) * tile_halves;
                        rows[c].push_back((uint32_t)(((const uint8_t*)t - p.wbase) >> 8));
                    }
            }
        };
        for (int l = 0; l < p.n_layers; ++l)
            for (int kind = kQKV; kind <= kDN; ++kind) emit(kind, l);
        (*counts)[2 * c] = (int)rows[c].size();
        emit(kLM, 0);
        (*counts)[2 * c + 1] = (int)rows[c].size() - (*counts)[2 * c];
        if (rows[c].size() > longest) longest = rows[c].size();
    }
    *stride = (int)((longest + 31) / 32 * 32);
    sched->assign((size_t)G * *stride, 0u);
    for (int c = 0; c < G; ++c)
        for (size_t i = 0; i < rows[c].size(); ++i) (*sched)[(size_t)c * *stride + i] = rows[c][i];
}

bool decode_plan(const DecodeParams& p, int num_sms, DecodeLaunch* out, const char** why) {
    const int qdim = p.n_heads * p.head_dim, kv_mul = p.n_heads / p.n_kv;
    if (p.head_dim != kAttnHeadDim) return *why = "fused decode implements head_dim 64", false;
    if (p.n_layers > kMaxDecodeLayers) return *why = "fused decode implements at most 64 layers", false;
    if (p.dim != 256 && p.dim != 512 && p.dim != 1024 && p.dim != 2048)
        return *why = "fused decode implements dim 256, 512, 1024 or 2048", false;
    if (qdim != p.dim) return *why = "fused decode needs n_heads * head_dim == dim", false;
    if (p.hidden % p.dim) return *why = "fused decode needs hidden to be a multiple of dim", false;
    if (p.n_heads % p.n_kv || kv_mul < 1 || kv_mul > 8)
        return *why = "fused decode implements n_heads / n_kv_heads in 1..8", false;
    if (p.n_heads * (kAttnHeadDim / 8) > kCT) return *why = "fused decode implements at most 32 heads", false;
    if (p.hidden / p.dim > kBatchTiles) return *why = "fused decode needs hidden <= 8 * dim", false;
    if (p.hidden > 8 * 4 * kCT) return *why = "fused decode implements hidden <= 8192", false;
    if (attn_scratch_floats(kv_mul) > kActFloats) return *why = "fused decode attention scratch exceeds its region", false;
    if (kv_mul * kAttnHeadDim > kBatchTiles * 8 * kCW) return *why = "fused decode q staging exceeds its region", false;
    const Layout L = finish_layout(make_layout(p.dim));
    if (L.total > 227 * 1024) return *why = "fused decode shared-memory plan exceeds 227 KB", false;
    out->grid = num_sms;
    out->smem_bytes = L.total;
    out->ks = p.dim / 128;
    out->stages = L.stages;
    return true;
}

cudaError_t decode_prepare(const DecodeLaunch& l) { return impl_prepare(l); }

cudaError_t launch_decode(const DecodeParams& p, const DecodeLaunch& l, cudaStream_t st) { return impl_launch(p, l, st); }

// ------------------------------------------------------- weight tiling --

__global__ void tile_rows_kernel(const uint4* __restrict__ src, __half* __restrict__ dst, int rows, int cols, int cb,
                                 int row0, int row_step) {
    const int per_row = cols / 8;
    const long long n = (long long)rows * per_row;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / per_row), c = (int)(i % per_row) * 8;
        const int64_t R = row0 + (int64_t)r * row_step;
        *reinterpret_cast<uint4*>(dst + tiled_offset(R, c, cols, cb)) = src[i];
    }
}

cudaError_t launch_tile_rows(const __half* src, __half* dst, int rows, int cols, int cb, int row0, int row_step,
                             cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    const long long n = (long long)rows * (cols / 8);
    const long long blocks = (n + 255) / 256;
    tile_rows_kernel<<<(int)(blocks < 4096 ? blocks : 4096), 256, 0, st>>>(reinterpret_cast<const uint4*>(src), dst,
                                                                           rows, cols, cb, row0, row_step);
    return cudaGetLastError();
}

}  // namespace lc
