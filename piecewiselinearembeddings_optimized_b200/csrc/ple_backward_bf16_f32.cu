// ple_backward_bf16_f32.cu - backward kernel instantiations (histogram and sorted) for compute type
// __nv_bfloat16 with gradients in float.
#include "ple_backward_hist.cuh"

namespace ple {

int launch_bwd_bf16_f32(const BwdArgs& a, int vec, cudaStream_t st) { return launch_backward_dtype<__nv_bfloat16, float>(a, vec, st); }

}  // namespace ple
