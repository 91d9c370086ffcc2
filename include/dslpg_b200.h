/*
 * dslpg_b200.h — C ABI of the B200 (sm_100a) row-wise reduction backend.
 *
 * One entry point per ViperBench kernel of the row-reduction family. Each takes
 * plain device pointers, sizes and a dtype code, launches on the given stream
 * and returns 0 on success, a positive cudaError_t when a CUDA call failed, or
 * a negative DSLPG_ERR_* code when the arguments were rejected before any
 * launch. No entry point allocates memory, synchronises, or keeps state other
 * than a per-device cache of SM counts and occupancy figures (lock-protected),
 * the per-thread kernel-shape selection below, and the per-device copy streams
 * of the host-buffer entry points.
 *
 * Layout: every row-wise operand is a dense row-major [M, N] matrix (the
 * reference flattens x[..., D] to [M, D] the same way). The caller owns every
 * buffer; inputs are never written.
 *
 * Reference interfaces (paths inside tingxi-li/DSLPerfGap):
 *   layer_norm      ViperBench/layer_norm/pytorch_impl.py:5-12
 *   rms_norm        ViperBench/rms_norm/pytorch_impl.py:3-10
 *   softmax         ViperBench/softmax/pytorch_impl.py:4-6
 *   log_softmax     ViperBench/log_softmax/pytorch_impl.py:4-8
 *   logsumexp       ViperBench/logsumexp/pytorch_impl.py:3-5
 *   cross_entropy   ViperBench/cross_entropy/pytorch_impl.py:4-90 and the
 *                   kernel layout of ViperBench/cross_entropy/triton_impl.py:13-75,123-140
 */
#ifndef DSLPG_B200_H
#define DSLPG_B200_H

#include <stdint.h>
#include <cuda_runtime_api.h>

#if defined(__GNUC__)
#define DSLPG_API __attribute__((visibility("default")))
#else
#define DSLPG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element type codes (storage types; arithmetic is always fp32). */
enum {
  DSLPG_F32 = 0,
  DSLPG_F16 = 1,
  DSLPG_BF16 = 2,
  DSLPG_I32 = 3, /* labels only */
  DSLPG_I64 = 4  /* labels only */
};

/* Argument errors (returned before anything is launched). */
enum {
  DSLPG_OK = 0,
  DSLPG_ERR_NULL_POINTER = -1,
  DSLPG_ERR_BAD_SHAPE = -2,
  DSLPG_ERR_BAD_DTYPE = -3,
  DSLPG_ERR_BAD_EPS = -4,
  DSLPG_ERR_BAD_ARGUMENT = -5,
  DSLPG_ERR_TOO_LARGE = -6 /* dslpg_kernel_ff_static: the problem does not fit its static scratch */
};

/* Kernel-shape selection (normally DSLPG_PATH_AUTO; the others exist so tests
 * and benchmarks can exercise one implementation on purpose). */
enum {
  DSLPG_PATH_AUTO = 0,     /* pick per shape */
  DSLPG_PATH_RESIDENT = 1, /* rows read straight into registers; kernel_ff: one CTA per 128x128 tile */
  DSLPG_PATH_TMA = 2,      /* rows / row chunks staged by TMA bulk copies */
  DSLPG_PATH_STREAM = 3,   /* two-pass streaming (any length or alignment); kernel_ff: the weight-streaming
                              kernel for M <= 8 (chosen by default for M <= 3) */
  DSLPG_PATH_CLUSTER = 4   /* a row split over a thread-block cluster (DSMEM exchange);
                              kernel_ff: CTA pairs (tcgen05 cta_group::2) on 256x128 tiles */
};

/* Select the kernel shape for the calling host thread's subsequent calls
 * (a per-thread setting: other threads keep their own, DSLPG_PATH_AUTO unless
 * they set one). A path that cannot handle a given shape falls back to one
 * that can. Returns 0 or DSLPG_ERR_BAD_ARGUMENT. No reference counterpart: a
 * testing aid. */
DSLPG_API int dslpg_set_kernel_path(int path);

/* The calling thread's kernel-shape selection. No reference counterpart. */
DSLPG_API int dslpg_get_kernel_path(void);

/* Number of bounded device-side waits (TMA pipeline barriers) that ran out of
 * time since the last call, and reset the count. Synchronises the device.
 * A non-zero value means some outputs of the affected launches were not
 * written. No reference counterpart. */
DSLPG_API unsigned int dslpg_take_wait_timeouts(void);

/* Library version, (major << 16) | minor. */
DSLPG_API int dslpg_version(void);

/* Human-readable text for a return code (negative: ours; positive: CUDA's). */
DSLPG_API const char* dslpg_error_string(int code);

/*
 * LayerNorm forward over the last dimension:
 *   y = (x - mean) / sqrt(var + eps) * weight + bias      (var biased)
 * x, y: [M, N] of x_dtype; weight, bias: [N] of w_dtype (bias may be NULL).
 * Replaces layer_norm(x, weight, bias, eps) of
 * ViperBench/layer_norm/pytorch_impl.py:5-12 (F.layer_norm). The eps == 1e-5
 * restriction of that file is enforced by the Python wrapper, not here.
 */
DSLPG_API int dslpg_layer_norm_fwd(const void* x, const void* weight, const void* bias, void* y,
                         int64_t M, int64_t N, int x_dtype, int w_dtype, float eps,
                         cudaStream_t stream);

/*
 * RMSNorm forward over the trailing N elements of each row:
 *   y = (x / sqrt(mean(x^2) + eps) * weight)  computed in fp32, stored as x_dtype
 * Replaces rms_norm(x, normalized_shape, weight, eps) of
 * ViperBench/rms_norm/pytorch_impl.py:3-10.
 */
DSLPG_API int dslpg_rms_norm_fwd(const void* x, const void* weight, void* y, int64_t M, int64_t N,
                       int x_dtype, int w_dtype, float eps, cudaStream_t stream);

/*
 * Softmax along the last dimension: y = exp(x - max) / sum(exp(x - max)).
 * Replaces softmax(x) of ViperBench/softmax/pytorch_impl.py:4-6.
 */
DSLPG_API int dslpg_softmax_fwd(const void* x, void* y, int64_t M, int64_t N, int dtype,
                      cudaStream_t stream);

/*
 * Log-softmax over the middle axis of a dense [M, N, K] tensor
 * (K == 1 is the last-dimension case): y = x - max - log(sum(exp(x - max))).
 * x is in_dtype, y is out_dtype; when they differ, x is first rounded to
 * out_dtype, as F.log_softmax(x, dim, dtype=out_dtype) does.
 * Replaces log_softmax(x, dim, dtype) of ViperBench/log_softmax/pytorch_impl.py:4-8.
 */
DSLPG_API int dslpg_log_softmax_fwd(const void* x, void* y, int64_t M, int64_t N, int64_t K,
                          int in_dtype, int out_dtype, cudaStream_t stream);

/*
 * logsumexp along the last dimension, with torch.logsumexp's treatment of
 * infinite maxima (a +inf entry gives +inf, an all -inf row gives -inf):
 * y[M] of dtype.  Replaces logsumexp(x) of ViperBench/logsumexp/pytorch_impl.py:3-5.
 */
DSLPG_API int dslpg_logsumexp_fwd(const void* x, void* y, int64_t M, int64_t N, int dtype,
                        cudaStream_t stream);

/*
 * Blockwise cross-entropy forward. For every row r and column block
 * cb < ceil(n_cols / block_size) it writes, at flat index cb * n_rows + r of
 * the three fp32 outputs, the block's log-sum-exp of logits * logit_scale, the
 * loss term and the z-loss term, exactly as
 * ViperBench/cross_entropy/pytorch_impl.py:4-90 (and the Triton kernel at
 * ViperBench/cross_entropy/triton_impl.py:13-75) define them. Flat entries at or
 * beyond ceil(n_cols / block_size) * n_rows are not written. Under split != 0
 * the z-loss entries are written as 0.
 * logits: [n_rows, n_cols] rows `logits_row_stride` elements apart;
 * labels: [n_rows] of labels_dtype (DSLPG_I32 or DSLPG_I64).
 * Replaces cross_entropy_fwd(...) of ViperBench/cross_entropy/pytorch_impl.py:4-90.
 */
DSLPG_API int dslpg_cross_entropy_fwd(const void* logits, const void* labels, float* loss, float* lse,
                            float* z_loss, int64_t n_rows, int64_t n_cols,
                            int64_t logits_row_stride, int logits_dtype, int labels_dtype,
                            float smoothing, float logit_scale, float lse_square_scale,
                            int64_t ignored_index, float total_classes, int64_t class_start_idx,
                            int64_t block_size, int has_smoothing, int split,
                            cudaStream_t stream);

/*
 * Blockwise cross-entropy backward: for every row r and column c < n_cols,
 *   p = exp(logits[r,c] * logit_scale - lse[r]);  p += 2 * lse_square_scale * lse[r] * p;
 *   p -= (has_smoothing ? 1 - smoothing : 1) at c == labels[r] - class_start_idx;
 *   p -= smoothing / total_classes                  (has_smoothing only);
 *   dlogits[r,c] = (dloss[r] * logit_scale) * p, with dloss[r] = 0 where
 *   labels[r] == ignored_index,
 * stored in logits_dtype. lse holds one fp32 value per row (the forward's lse
 * for a single column block); dloss[r] is read at r * dloss_stride.
 * Replaces cross_entropy_bwd(...) of ViperBench/cross_entropy/pytorch_impl.py:93-141
 * (kernel: ViperBench/cross_entropy/triton_impl.py:79-120, wrapper :143-158).
 */
DSLPG_API int dslpg_cross_entropy_bwd(const void* dloss, int dloss_dtype, int64_t dloss_stride,
                            const void* logits, const float* lse, const void* labels, void* dlogits,
                            int64_t n_rows, int64_t n_cols, int64_t logits_row_stride,
                            int64_t dlogits_row_stride, int logits_dtype, int labels_dtype,
                            float smoothing, float logit_scale, float lse_square_scale,
                            int64_t ignored_index, float total_classes, int64_t class_start_idx,
                            int has_smoothing, cudaStream_t stream);

/*
 * Cross-entropy forward and backward in one pass over the logits, for one
 * column block per row (the reference's BLOCK_SIZE >= n_cols) without SPLIT,
 * when dloss is known before the forward (the gradient of a mean or sum of
 * the per-row losses). loss / lse / z_loss: [n_rows] fp32, the values
 * dslpg_cross_entropy_fwd stores at flat index r; dlogits as
 * dslpg_cross_entropy_bwd computes them from that lse. The logits are read
 * from HBM once (the second pass over a row hits L2) instead of twice.
 * Serves cross_entropy_fwd followed by cross_entropy_bwd of
 * ViperBench/cross_entropy/triton_impl.py:123-140 and :79-120
 * (pytorch_impl.py:4-90 and :93-141).
 */
DSLPG_API int dslpg_cross_entropy_fwd_bwd(const void* logits, const void* labels, const void* dloss, int dloss_dtype,
                                          int64_t dloss_stride, float* loss, float* lse, float* z_loss, void* dlogits,
                                          int64_t n_rows, int64_t n_cols, int64_t logits_row_stride,
                                          int64_t dlogits_row_stride, int logits_dtype, int labels_dtype,
                                          float smoothing, float logit_scale, float lse_square_scale,
                                          int64_t ignored_index, float total_classes, int64_t class_start_idx,
                                          int has_smoothing, cudaStream_t stream);

/*
 * Reductions over the middle axis of a dense [M, N, K] tensor (a reduced run
 * of adjacent axes is one N; K == 1 reduces rows). Index outputs are int64 and
 * follow torch: the first NaN is the maximum; equal maxima give the smallest
 * index.
 *
 * mean: y[M*K] of out_dtype = sum / N, accumulated in fp32 after converting x
 * to out_dtype (torch.mean(x, dim, dtype=out_dtype)).
 * Replaces mean_reduction(input_tensor, dim, keepdim, dtype) of
 * ViperBench/mean_reduction/pytorch_impl.py:4-8.
 */
DSLPG_API int dslpg_mean_reduction(const void* x, void* y, int64_t M, int64_t N, int64_t K, int in_dtype,
                                   int out_dtype, cudaStream_t stream);

/* values[M*K] (x's dtype) and indices[M*K] of the maximum along N.
 * Replaces max_reduction(input, dim, keepdim) of ViperBench/max_reduction/pytorch_impl.py:4-11. */
DSLPG_API int dslpg_max_reduction(const void* x, void* values, int64_t* indices, int64_t M, int64_t N,
                                  int64_t K, int dtype, cudaStream_t stream);

/* indices[M*K] of the maximum along N.
 * Replaces argmax(input_tensor, dim, keepdim) of ViperBench/argmax/pytorch_impl.py:4-8. */
DSLPG_API int dslpg_argmax(const void* x, int64_t* indices, int64_t M, int64_t N, int64_t K, int dtype,
                           cudaStream_t stream);

/*
 * dslpg_rms_norm_fwd on HOST buffers: x_host [M, N] (x_dtype) in, y_host
 * [M, N] out; weight is a device pointer. The rows stream through the GPU in
 * chunks of about 16 MiB, the upload of one chunk, the kernel on the previous
 * one and the download of the one before overlapping (two copy streams of
 * this library plus `stream`; one cudaMemcpyAsync per chunk and direction).
 * With pinned host memory the copies run asynchronously in both directions at
 * once; pageable memory works but the copies do not overlap. `workspace`
 * (device, 256-byte aligned) holds the chunk buffers: at least
 * dslpg_rms_norm_fwd_host_workspace_bytes(M, N, x_dtype) bytes. The call
 * returns once the work is enqueued; everything is ordered on `stream`, so
 * synchronise it before reading y_host. Calls on one device are serialised by
 * a lock while they enqueue. Same result as dslpg_rms_norm_fwd row by row.
 * Serves the reference's rms_norm (ViperBench/rms_norm/pytorch_impl.py:3-10)
 * for inputs that live in host memory.
 */
DSLPG_API int dslpg_rms_norm_fwd_host_workspace_bytes(int64_t M, int64_t N, int x_dtype, int64_t* bytes);
DSLPG_API int dslpg_rms_norm_fwd_host(const void* x_host, const void* weight, void* y_host, int64_t M, int64_t N,
                                      int x_dtype, int w_dtype, float eps, void* workspace, int64_t workspace_bytes,
                                      cudaStream_t stream);

/*
 * dslpg_layer_norm_fwd on HOST buffers, with the same chunked pipeline,
 * workspace rule and ordering as dslpg_rms_norm_fwd_host above; weight and
 * bias (bias may be NULL) are device pointers. Same result as
 * dslpg_layer_norm_fwd row by row. Serves the reference's layer_norm
 * (ViperBench/layer_norm/pytorch_impl.py:5-12) for inputs that live in host
 * memory, e.g. one row block per GPU of a batch held by the host.
 */
DSLPG_API int dslpg_layer_norm_fwd_host_workspace_bytes(int64_t M, int64_t N, int x_dtype, int64_t* bytes);
DSLPG_API int dslpg_layer_norm_fwd_host(const void* x_host, const void* weight, const void* bias, void* y_host,
                                        int64_t M, int64_t N, int x_dtype, int w_dtype, float eps, void* workspace,
                                        int64_t workspace_bytes, cudaStream_t stream);

/*
 * Llama feed-forward with the RMSNorm fused around a dual GEMM (tcgen05 tensor
 * cores; for M <= 3 rows a kernel that streams the weight rows instead):
 *   a_norm[m] = rsqrt(sum_k x[m,k]^2 / K + 1e-6);  xs = x * rms_w (fp16);
 *   out[m,n] = silu(a_norm[m] * (xs @ w1^T)[m,n]) * (a_norm[m] * (xs @ w3^T)[m,n])   (fp16)
 * x [M, K], w1 and w3 [N, K], rms_w [K], out [M, N]: all fp16, row-major,
 * 16-byte aligned; K % 8 == 0. `workspace` (256-byte aligned) holds xs and
 * a_norm: at least dslpg_kernel_ff_workspace_bytes(M, K) bytes.
 * Replaces kernel_ff(x, w1, w3, rms_w) of ViperBench/linear_activation/pytorch_impl.py:5-54.
 */
DSLPG_API int dslpg_kernel_ff_workspace_bytes(int64_t M, int64_t K, int64_t* bytes);
DSLPG_API int dslpg_kernel_ff(const void* x, const void* w1, const void* w3, const void* rms_w, void* out,
                              int64_t M, int64_t N, int64_t K, void* workspace, int64_t workspace_bytes,
                              cudaStream_t stream);

/*
 * dslpg_kernel_ff without a caller-provided workspace and without any device
 * allocation: xs and a_norm live in a file-scope static __device__ scratch of
 * DSLPG_KERNEL_FF_STATIC_SCRATCH_BYTES (16 MiB + 64 KiB), enough for
 * M * K <= 8,388,608 fp16 elements (e.g. 2048 x 4096) as measured by
 * dslpg_kernel_ff_workspace_bytes; larger problems return DSLPG_ERR_TOO_LARGE
 * before anything is launched. It is meant for callers that cannot allocate
 * device memory per call: a C / FFI host that owns no device allocator (the
 * memory belongs to another framework's pool), or a loop where the device-wide
 * synchronisation of cudaMalloc / cudaFree is not acceptable.
 * Set-up: the first call on each device (the device current at the call) looks
 * up the scratch address with cudaGetSymbolAddress, which may load this
 * library's device code; make that first call before any stream capture. The
 * address is kept per device together with the id of the CUDA context it
 * belongs to, so after a cudaDeviceReset (or any replacement of the device's
 * context) the next call repeats the set-up instead of using a stale address.
 * The scratch is part of this library's device code: once any kernel_ff entry
 * point has loaded that code on a device, its 16 MiB + 64 KiB stay allocated
 * there until the context ends, also for callers that only use dslpg_kernel_ff.
 * No part of the scratch has to start at zero (every call writes all of xs and
 * a_norm before reading them). There is ONE scratch per device: calls that
 * overlap on the same device (different streams, or different host threads
 * without ordering) race on it and give wrong results; order them on one stream.
 * No reference counterpart: the reference's kernel_ff always allocates its
 * temporaries through torch.
 */
#define DSLPG_KERNEL_FF_STATIC_SCRATCH_BYTES ((int64_t)(16 * 1024 * 1024 + 64 * 1024))
DSLPG_API int dslpg_kernel_ff_static(const void* x, const void* w1, const void* w3, const void* rms_w, void* out,
                                     int64_t M, int64_t N, int64_t K, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* DSLPG_B200_H */
