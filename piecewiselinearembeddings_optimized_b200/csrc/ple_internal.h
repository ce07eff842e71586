// ple_internal.h - launch arguments and host helpers shared by the .cu files.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/ple_capi.h"

namespace ple {

enum { kEpiNone = PLE_EPILOGUE_NONE, kEpiA = PLE_EPILOGUE_A, kEpiB = PLE_EPILOGUE_B };

// backward tuning: 16 warps, one persistent CTA per SM
constexpr int kBwdThreads = 512;

// forward tuning
constexpr int kFwdMaxThreads = 512;
constexpr size_t kFwdTableBudget = 64 * 1024;
constexpr size_t kFwdTableBudgetF32 = 128 * 1024;  // fp32 outputs with D <= 16 (see launch_forward)
constexpr int kFwdPairsPerTile = 2048;  // measured: 2048 beats 512 and 1024 on the c4 and c5 forwards

struct FwdArgs {
  const float* x;
  const float* edges;
  const float* inv_w;
  const int32_t* n_bins;
  const float* W;
  const float* bias;
  const float* w0;
  const float* b0;
  void* out;
  void* bin_idx;
  int bin_idx_bytes;
  int64_t N;
  int F, B, D;
  int epi, relu;
  // filled by the launcher
  int lgFc, n_chunks, S_t, lgk, ldK, x_vec4;
  // slots of `group` CTAs over the same samples, member j on chunk g * group + j of chunk group g
  int group, n_groups;
};

struct BwdArgs {
  const void* g;
  const void* bin_idx;  // optional forward bins (U8 / I16 / I32)
  int bin_idx_bytes;
  const float* x;
  const float* edges;
  const float* inv_w;
  const int32_t* n_bins;
  const float* W;
  const float* bias;
  const float* w0;
  const float* b0;
  float* grad_x;
  float* grad_W;
  float* grad_bias;
  float* grad_w0;
  float* grad_b0;
  float* ws;          // partials: [n_parts][F][B + 3][D] floats
  size_t ws_bytes;
  int64_t N;
  int F, B, D;
  int epi, relu;
  // filled by the launcher: Fc = 1 << lgFc features per chunk, 1 << lgWf warps per feature, tiles of
  // 1 << lgSt samples, 2^lgk - 1 >= B - 1 interior-edge search keys; `group` CTAs (one chunk each) share
  // the sample ranges of a group of chunks; g_wide: 32-byte gradient chunks may be read at once
  int lgFc, lgWf, lgSt, n_chunks, max_segs, Fc;
  int lgk;
  int group, n_groups, g_wide;
  int g_prefetch;  // the gradient tensor map is valid (per-tile L2 prefetch)
  int gx_vec4;     // grad_x rows may be stored 16 bytes at a time (16-byte aligned, F % 4 == 0)
  int hist_St;     // histogram kernel: samples per tile (a multiple of 32 x warps per feature)
};

struct EncArgs {
  const float* x;
  const float* edges;
  const float* inv_w;
  const int32_t* n_bins;
  const int64_t* col_off;  // [F + 1] column offsets (ragged layout)
  const void* g;           // backward: grad of the encoding
  void* out;               // forward: the encoding
  float* grad_x;           // backward
  int64_t N, total_cols;
  int F, B, layout;
};

// embeddings forward fused into a consumer Linear (ple_linear.cu)
struct LinearCall {
  const float* x;
  const float* edges;
  const float* inv_w;
  const int32_t* n_bins;
  const float* W;
  const float* bias;
  const float* w0;
  const float* b0;
  const void* W1;  // bf16 [H, F * D]
  const float* b1;  // [H] or null
  void* z;          // [N, H]
  void* ws;
  size_t ws_bytes;
  int64_t N, H;
  int F, B, D;
  int epi, relu, compute_dtype, out_dtype;
};

// error plumbing (ple_capi.cu)
int set_error(int code, const char* msg);
int set_cuda_error(cudaError_t e, const char* what);

// cached properties of the current device (ple_capi.cu)
int device_sm_count();
size_t device_max_smem_optin();

int launch_forward(FwdArgs a, int compute_dtype, int output_dtype, int vec, cudaStream_t st);
// max_n_bins above 256 (bare x_ple ops only): global-memory kernels in ple_wide.cu
constexpr int64_t kWideMaxBins = (int64_t)1 << 20;
int launch_forward_wide(const FwdArgs& a, int compute_dtype, int output_dtype, cudaStream_t st);
int launch_backward_wide(const BwdArgs& a, int compute_dtype, int grad_dtype, cudaStream_t st);
size_t wide_workspace_bytes(int64_t F, int64_t B, int64_t D);
int launch_backward(BwdArgs a, int compute_dtype, int grad_dtype, int vec, cudaStream_t st);
int backward_vec(int64_t D, int grad_bytes);
size_t backward_workspace_bytes(int64_t N, int64_t F, int64_t B, int64_t D);
bool backward_uses_hist(int64_t F, int64_t B, int64_t D);
int launch_linear(const LinearCall& c, cudaStream_t st);
size_t linear_workspace_bytes(int64_t F, int64_t B, int64_t D, int64_t H, int compute_dtype);
int linear_status();
int launch_encoding_forward(const EncArgs& a, int output_dtype, cudaStream_t st);
int launch_encoding_backward(const EncArgs& a, int grad_dtype, cudaStream_t st);
int launch_bins(const float* sorted, int64_t N, int64_t F, int n_q, float* edges, float* inv_w, int32_t* n_bins,
                int ld_e, cudaStream_t st);

}  // namespace ple
