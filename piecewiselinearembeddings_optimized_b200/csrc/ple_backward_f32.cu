// ple_backward_f32.cu - backward kernel instantiations for compute type
// float with gradients in float.
#include "ple_backward_impl.cuh"

namespace ple {

int launch_bwd_f32(const BwdArgs& a, int vec, cudaStream_t st) { return launch_bwd_dtype<float, float>(a, vec, st); }

}  // namespace ple
