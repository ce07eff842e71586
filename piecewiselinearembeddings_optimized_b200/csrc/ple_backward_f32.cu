// ple_backward_f32.cu - backward kernel instantiations (histogram and sorted) for compute type
// float with gradients in float.
#include "ple_backward_hist.cuh"

namespace ple {

int launch_bwd_f32(const BwdArgs& a, int vec, cudaStream_t st) { return launch_backward_dtype<float, float>(a, vec, st); }

}  // namespace ple
