// ple_backward_f16.cu - backward kernel instantiations (histogram and sorted) for compute type
// __half with gradients in __half.
#include "ple_backward_hist.cuh"

namespace ple {

int launch_bwd_f16(const BwdArgs& a, int vec, cudaStream_t st) { return launch_backward_dtype<__half, __half>(a, vec, st); }

}  // namespace ple
