/*
 * ple_capi.h - C ABI of the B200-native piecewise-linear embedding (PLE) path.
 *
 * Every entry point takes plain device pointers, int64 sizes, dtype codes and
 * a CUDA stream (cudaStream_t passed as void*; NULL = legacy default stream),
 * enqueues its kernels on that stream and returns a ple_status (0 = success).
 * Nothing here allocates device memory: outputs and the backward workspace
 * are provided by the caller.  Work is asynchronous; launch failures are
 * reported through the return value, execution faults surface on the stream.
 *
 * Shapes (N = batch, F = n_features, B = max_n_bins, D = d_embedding):
 *   x               [N, F]     float32, row-major contiguous
 *   bin_edges       [F, B + 1] float32, feature i's n_i + 1 edges then +inf
 *   inv_bin_widths  [F, B]     float32, 1 / (e[j+1] - e[j]) then 0
 *   n_bins          [F]        int32, 1 <= n_i <= B
 *   weight          [F, B, D]  float32, logical bin j < n_i - 1 at row j and
 *                              the last real bin at row B - 1
 *   bias            [F, D]     float32 (epilogue A)
 *   w0, b0          [F, D]     float32 (epilogue B: linear0(x) = x * w0 + b0)
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   ple_forward           csrc/ops.cpp:35-44 -> csrc/forward_cuda.cu:687-860
 *   ple_backward          csrc/ops.cpp:46-58 -> csrc/backward_cuda.cu:1528-1725
 *   ple_embeddings_*      src/rtdl_num_embeddings_cuda/module.py:207-248 (forward
 *                         composition) and its autograd (_autograd.py:42-96 plus
 *                         the PyTorch epilogue), fused into single kernels.
 */
#ifndef PLE_CAPI_H
#define PLE_CAPI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PLE_ABI_VERSION 7

/* Element types (codes shared by every entry point). */
enum {
  PLE_DTYPE_F32 = 0,
  PLE_DTYPE_F16 = 1,
  PLE_DTYPE_BF16 = 2,
  PLE_DTYPE_U8 = 3,
  PLE_DTYPE_I16 = 4,
  PLE_DTYPE_I32 = 5
};

/* Epilogue fused after x_ple (module.py:230-248). */
enum {
  PLE_EPILOGUE_NONE = 0, /* x_ple only (the reference op)                    */
  PLE_EPILOGUE_A = 1,    /* act(x_ple + bias)                                */
  PLE_EPILOGUE_B = 2     /* (x * w0 + b0) + act(x_ple)                       */
};

/* Layouts of the standalone encoding (ple_encoding_forward). */
enum {
  PLE_ENC_RAGGED = 0, /* [N, sum_i n_i]: feature-major, logical bin order, no padding       */
  PLE_ENC_PADDED = 1  /* [N, F, B]: the weights' physical layout, zero padding columns   */
};

/* Status codes. */
enum {
  PLE_OK = 0,
  PLE_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad enum value            */
  PLE_ERR_SHAPE = 2,            /* non-positive or inconsistent sizes      */
  PLE_ERR_OVERFLOW = 3,         /* a size overflows the index types        */
  PLE_ERR_UNSUPPORTED = 4,      /* dtype / size combination not provided   */
  PLE_ERR_WORKSPACE = 5,        /* workspace missing, small or misaligned  */
  PLE_ERR_CUDA = 6,             /* a CUDA runtime call failed              */
  PLE_ERR_ALIGNMENT = 7         /* a pointer is not 16-byte aligned        */
};

/* ABI version of the loaded library (PLE_ABI_VERSION at build time). */
int ple_abi_version(void);

/* Static description of a status code. */
const char* ple_status_string(int status);

/*
 * Backward kernels.  ple_backward and ple_embeddings_backward (and the
 * no-allocation variant) run one of two fused kernels up to 256 bins
 * (ple_backward_kernel_kind tells which): the histogram kernel (samples in
 * natural order, per-warp bin sums in shared memory updated in sample order;
 * d_embedding 8, 16 or 24) or the sorted kernel (per tile of samples a
 * counting sort of each feature's samples by bin, then a segmented walk over
 * the sorted lists that keeps each run's gradient sums in registers).  Either
 * way the parameter gradients are summed per partition in the workspace and
 * reduced in a fixed order, so every result is bitwise deterministic for a
 * given shape and device.  Above 256 bins the bare x_ple backward sums
 * grad_weight with atomics (not bitwise reproducible).
 */

/* Detail message of the last failing call on the calling host thread. */
const char* ple_last_error_message(void);

/*
 * x_ple forward (reference op rtdl_num_embeddings_cuda::forward).
 *   output[N, F, D] in output_dtype (F32 / F16 / BF16):
 *     x_ple[b,i,:] = sum_{j<k} q(W[i,j,:]) + q(t) * q(W[i,phys(k),:])
 *   with k the right-sided clamped bin of x[b,i], t = (x - e_k) * r_k and q()
 *   rounding through output_dtype (autocast emulation, fp32 accumulation).
 *   bin_indices[N, F] (optional, may be NULL) receives k as U8 / I16 / I32
 *   according to bin_index_dtype.
 *   max_n_bins up to 2^20: above 256 (the reference's int16 / int32 bin-index
 *   range) the op and ple_backward run plain global-memory kernels, correct at
 *   any bin count but not tuned; the epilogue entry points stay at <= 256
 *   (PLE_ERR_UNSUPPORTED above).
 */
int ple_forward(const float* x, const float* bin_edges, const float* inv_bin_widths,
                const int32_t* n_bins, const float* weight, int64_t batch,
                int64_t n_features, int64_t max_n_bins, int64_t d_embedding,
                int output_dtype, void* output, int bin_index_dtype, void* bin_indices,
                void* stream);

/*
 * Workspace bytes ple_backward / ple_embeddings_backward need for these sizes
 * (per-partition partial sums of the parameter gradients; 0 never returned).
 */
size_t ple_backward_workspace_size(int64_t batch, int64_t n_features, int64_t max_n_bins,
                                   int64_t d_embedding);

/*
 * Which kernel ple_backward / ple_embeddings_backward run for these sizes on
 * the current device: PLE_BACKWARD_HISTOGRAM (natural sample order, per-warp
 * bin sums in shared memory; d_embedding 8, 16 or 24, at most 256 bins),
 * PLE_BACKWARD_SORTED (per-tile counting sort and segmented walk; the other
 * shapes up to 256 bins, or every shape when the environment variable
 * PLE_BACKWARD_KERNEL=sorted is set when the library first plans a backward),
 * PLE_BACKWARD_WIDE (more than 256 bins), or minus the PLE_ERR_* status of
 * sizes the backward refuses.  Both fused kernels give bitwise-deterministic results.
 */
#define PLE_BACKWARD_SORTED 0
#define PLE_BACKWARD_HISTOGRAM 1
#define PLE_BACKWARD_WIDE 2
int ple_backward_kernel_kind(int64_t n_features, int64_t max_n_bins, int64_t d_embedding);

/*
 * x_ple backward (reference op rtdl_num_embeddings_cuda::backward).
 *   grad_output[N, F, D] in grad_dtype (F32 / F16 / BF16).
 *   grad_x[N, F] (may be NULL):
 *     r_k <g, q(W[phys k])> + [k > 0 and x == e_k] r_{k-1} <g, q(W[k-1])>
 *   grad_weight[F, B, D] (may be NULL; padding rows are written as zero):
 *     grad_W[i, phys(j)] = sum_{k_b = j} q(t_b) g_b + sum_{k_b > j} g_b
 *   bin_indices (optional, may be NULL) are the forward's bins; when NULL they
 *   are recomputed from x.  Values are clamped to [0, n_i - 1].  The result is
 *   bitwise deterministic.
 */
int ple_backward(const void* grad_output, int grad_dtype, const float* x,
                 const float* bin_edges, const float* inv_bin_widths, const int32_t* n_bins,
                 const float* weight, const void* bin_indices, int bin_index_dtype,
                 int64_t batch, int64_t n_features, int64_t max_n_bins, int64_t d_embedding,
                 float* grad_x, float* grad_weight, void* workspace, size_t workspace_bytes,
                 void* stream);

/*
 * Fused embeddings forward (the whole module forward in one kernel):
 *   epilogue A: y = act(x_ple + bias); epilogue B: y = (x * w0 + b0) + act(x_ple)
 *   act = ReLU when activation != 0.  x_ple is computed as in ple_forward with
 *   rounding through compute_dtype (F32 = plain fp32; BF16 / F16 = autocast);
 *   the epilogue runs in fp32 and the result is stored as output_dtype.  With
 *   epilogue B and a 16-bit output_dtype, x_ple is rounded once, at the store.
 *   bin_indices[N, F] (optional, may be NULL) receives the bins as in
 *   ple_forward, for reuse by the backward.
 */
int ple_embeddings_forward(const float* x, const float* bin_edges, const float* inv_bin_widths,
                           const int32_t* n_bins, const float* weight, const float* bias,
                           const float* w0, const float* b0, int epilogue, int activation,
                           int compute_dtype, int64_t batch, int64_t n_features,
                           int64_t max_n_bins, int64_t d_embedding, int output_dtype,
                           void* output, int bin_index_dtype, void* bin_indices, void* stream);

/*
 * Fused embeddings backward: every gradient of ple_embeddings_forward from the
 * upstream gradient in one pass over grad_output.  Gradient pointers may be
 * NULL when not needed; grad_bias is used with epilogue A, grad_w0 / grad_b0
 * with epilogue B.  bin_indices (optional) are the forward's bins, as in
 * ple_backward.  Parameter gradients are written (not accumulated) and are
 * bitwise deterministic.
 */
int ple_embeddings_backward(const void* grad_output, int grad_dtype, const float* x,
                            const float* bin_edges, const float* inv_bin_widths,
                            const int32_t* n_bins, const float* weight, const float* bias,
                            const float* w0, const float* b0, int epilogue, int activation,
                            int compute_dtype, int64_t batch, int64_t n_features,
                            int64_t max_n_bins, int64_t d_embedding, const void* bin_indices,
                            int bin_index_dtype, float* grad_x, float* grad_weight,
                            float* grad_bias, float* grad_w0, float* grad_b0, void* workspace,
                            size_t workspace_bytes, void* stream);

/*
 * ple_embeddings_backward_noalloc: ple_embeddings_backward with its workspace
 * taken from scratch memory built into the library instead of from the caller.
 * No counterpart in the reference (its backward allocates through torch).
 *
 * For callers that cannot hand over device memory of their own: a host binding
 * over plain C FFI (Go, Java, a ctypes script) that holds only its input and
 * output buffers and has no device allocator to draw a workspace from, and a
 * serving process that reserves its whole memory budget at start-up and may
 * not allocate afterwards.  This entry point itself allocates nothing on any
 * call: the scratch is a static device array of PLE_NOALLOC_SCRATCH_BYTES
 * (16 MiB) per device, placed when the library's module is loaded.
 *
 *   - Same arguments, results, size limits and status codes as
 *     ple_embeddings_backward, without workspace / workspace_bytes (more
 *     than 256 bins only for the bare x_ple case: no epilogue, no
 *     activation).
 *   - Sizes whose workspace (ple_backward_workspace_size) exceeds
 *     PLE_NOALLOC_SCRATCH_BYTES are rejected with PLE_ERR_WORKSPACE before
 *     anything is launched; use ple_embeddings_backward for those.
 *   - The scratch does not need to start at zero: every slot that the
 *     finalize step reads is written earlier in the same call (the
 *     wide-bin path clears what it accumulates into with cudaMemsetAsync).
 *   - The first call on each device looks up the scratch address
 *     (cudaGetSymbolAddress, with that device current) and caches it; a
 *     lookup that fails is not cached and the next call tries again.  Make
 *     the first call before any stream capture on the device.
 *   - One scratch per device, shared by all calls: two calls whose kernels
 *     can overlap on the same device (different streams, or host threads
 *     without ordering) race on it and corrupt each other's results.  Order
 *     such calls on one stream.
 */
#define PLE_NOALLOC_SCRATCH_BYTES ((size_t)16 << 20)

int ple_embeddings_backward_noalloc(const void* grad_output, int grad_dtype, const float* x,
                                    const float* bin_edges, const float* inv_bin_widths,
                                    const int32_t* n_bins, const float* weight, const float* bias,
                                    const float* w0, const float* b0, int epilogue, int activation,
                                    int compute_dtype, int64_t batch, int64_t n_features,
                                    int64_t max_n_bins, int64_t d_embedding,
                                    const void* bin_indices, int bin_index_dtype, float* grad_x,
                                    float* grad_weight, float* grad_bias, float* grad_w0,
                                    float* grad_b0, void* stream);

/*
 * Standalone piecewise-linear encoding (upstream
 * rtdl_num_embeddings.PiecewiseLinearEncoding; the reference has no CUDA path
 * for it, only the x_ple op of which it is the inner factor).
 *   column j of feature i (logical bin j < n_i):
 *     t_j = (x - e_j) * r_j, clamped to <= 1 (j = 0), [0, 1] (middle bins),
 *     >= 0 (j = n_i - 1); a single-bin feature is unclamped; NaN propagates.
 *   layout PLE_ENC_RAGGED: output [N, total_cols], total_cols = sum_i n_i,
 *     col_offsets[F + 1] (int64, device) = exclusive prefix of n_bins;
 *   layout PLE_ENC_PADDED: output [N, F, B] (total_cols = F * B), the bins in
 *     the weights' physical layout (last real bin at column B - 1), padding
 *     columns 0; col_offsets may be NULL.
 *   output_dtype F32 / F16 / BF16 (values computed in fp32, rounded once).
 * Columns whose offsets disagree with n_bins are written as 0 (never read or
 * written out of bounds).
 */
int ple_encoding_forward(const float* x, const float* bin_edges, const float* inv_bin_widths,
                         const int32_t* n_bins, const int64_t* col_offsets, int layout,
                         int64_t batch, int64_t n_features, int64_t max_n_bins, int64_t total_cols,
                         int output_dtype, void* output, void* stream);

/*
 * Gradient of ple_encoding_forward with respect to x:
 *   grad_x[b, i] = sum_j g[b, col(i, j)] * r_j * [lo_j <= t_j <= hi_j]
 * (the clamp passes the gradient at its bounds, as torch.clamp's backward;
 * no gradient where t_j is NaN).  grad_output has the forward's layout, in
 * grad_dtype F32 / F16 / BF16; grad_x[N, F] fp32.
 */
int ple_encoding_backward(const void* grad_output, int grad_dtype, const float* x,
                          const float* bin_edges, const float* inv_bin_widths,
                          const int32_t* n_bins, const int64_t* col_offsets, int layout,
                          int64_t batch, int64_t n_features, int64_t max_n_bins,
                          int64_t total_cols, float* grad_x, void* stream);

/*
 * Quantile bin edges on the device (upstream rtdl_num_embeddings.compute_bins
 * without a tree; the reference builds its tables on the host,
 * module.py:58-109).  sorted_columns[F][n_rows]: each feature's training
 * column sorted ascending (n_rows >= 2, finite).  For every feature the
 * quantiles at j / n_bins (j = 0..n_bins), linearly interpolated between order
 * statistics, with repeated values removed, are written as
 *   bin_edges[F][n_bins + 1]   (+inf after the n_i + 1 distinct edges),
 *   inv_bin_widths[F][n_bins]  (1 / (e_{j+1} - e_j), 0 padding),
 *   n_bins_out[F]              (n_i = distinct edges - 1; 0 for a constant column).
 * 1 <= n_bins <= 1023.
 */
int ple_compute_bins(const float* sorted_columns, int64_t n_rows, int64_t n_features, int n_bins,
                     float* bin_edges, float* inv_bin_widths, int32_t* n_bins_out, void* stream);

/*
 * Embeddings forward fused into the first Linear layer of its consumer
 * (flatten + nn.Linear(F * D, H), the layer that follows the module in an
 * MLP); the reference ends at the module output (module.py:207-248) and has
 * no counterpart.
 *   z[N, H] = flatten(y)[N, F * D] @ linear_weight[H, F * D]^T + linear_bias
 * where y is ple_embeddings_forward's result in compute_dtype (BF16 = the
 * autocast module output, rounded to bf16; F32 = the fp32 module output,
 * rounded to bf16 for the product).  The product runs on the tensor cores
 * with bf16 operands and fp32 accumulation, as an autocast nn.Linear does;
 * y is never written to memory.
 *   linear_weight  [H, F * D] BF16 (linear_weight_dtype = PLE_DTYPE_BF16)
 *   linear_bias    [H] f32, may be NULL
 *   output         [N, H] F32 or BF16, 16-byte aligned
 *   d_embedding a multiple of 8; compute_dtype F32 or BF16.
 * The workspace (256-byte aligned, ple_embeddings_linear_workspace_size bytes)
 * receives per-call images of the tables and of linear_weight.
 */
size_t ple_embeddings_linear_workspace_size(int64_t n_features, int64_t max_n_bins, int64_t d_embedding,
                                            int64_t out_features, int compute_dtype); /* 0: unsupported */

int ple_embeddings_linear_forward(const float* x, const float* bin_edges, const float* inv_bin_widths,
                                  const int32_t* n_bins, const float* weight, const float* bias,
                                  const float* w0, const float* b0, int epilogue, int activation,
                                  int compute_dtype, int64_t batch, int64_t n_features,
                                  int64_t max_n_bins, int64_t d_embedding, const void* linear_weight,
                                  int linear_weight_dtype, const float* linear_bias,
                                  int64_t out_features, int output_dtype, void* output,
                                  void* workspace, size_t workspace_bytes, void* stream);

/*
 * Status word of ple_embeddings_linear_forward on the current device: 1 if a
 * wait of the kernel ran past its iteration limit since the last call (that
 * launch's output is incomplete), 0 if not, -1 if unreadable.  Reading clears
 * it.  Synchronous (a device-to-host copy).
 */
int ple_linear_status(void);

#ifdef __cplusplus
}
#endif

#endif /* PLE_CAPI_H */
