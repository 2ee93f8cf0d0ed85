// lc_decode_trace.cu -- the phase-trace build of the fused decode kernel
// (lc_decode_impl.cuh): consumer thread 0 of each CTA stamps %globaltimer at
// fixed points of every job (lc_session_enable_trace).
#define LC_DECODE_TRACE 1
#include "lc_decode_impl.cuh"

namespace lc {

cudaError_t decode_prepare_traced(const DecodeLaunch& l) { return impl_prepare(l); }

cudaError_t launch_decode_traced(const DecodeParams& p, const DecodeLaunch& l, cudaStream_t st) {
    return impl_launch(p, l, st);
}

}  // namespace lc
