// xent_bwd.cu — blockwise cross-entropy backward (sm_100a).
//
// The gradient of each row (xent_grad.cuh) from the forward's lse: there is no
// reduction, each row is streamed once (read logits, write dlogits) by one CTA
// with 16-byte loads. Column blocks only tile the computation in the
// reference (ViperBench/cross_entropy/triton_impl.py:79-120), so the result
// does not depend on BLOCK_SIZE.
#include "xent_grad.cuh"

namespace dslpg {

struct BwdArgs {
  const void* dloss;
  int dloss_dt;
  int64_t dloss_stride;
  const void* x;
  const float* lse;
  const void* labels;
  int label64;
  void* dx;
  int64_t M, N, ld, ldo;
  int nvec;
  float smoothing, scale, lse_sq, total_classes;
  int64_t ignored, class_start;
  int has_smoothing;
};

template <typename T, int V>
__global__ void __launch_bounds__(256) xent_bwd_kernel(const BwdArgs a) {
  const bool smooth = a.has_smoothing != 0;
  for (int64_t r = blockIdx.x; r < a.M; r += gridDim.x) {
    const int64_t label = a.label64 ? static_cast<const int64_t*>(a.labels)[r]
                                    : static_cast<int64_t>(static_cast<const int32_t*>(a.labels)[r]);
    const float dl = (label != a.ignored) ? load_any(a.dloss, r * a.dloss_stride, a.dloss_dt) : 0.f;
    const GradRow b = grad_row_consts(dl, a.scale, a.lse[r], a.lse_sq, smooth, a.smoothing, a.total_classes, label,
                                      a.class_start);
    grad_row<T, V>(static_cast<const T*>(a.x) + r * a.ld, static_cast<T*>(a.dx) + r * a.ldo, a.nvec, a.N, b, a.scale,
                   smooth, threadIdx.x, blockDim.x);
  }
}

namespace {
template <typename T>
cudaError_t launch_bwd(BwdArgs a, cudaStream_t st) {
  constexpr int E = Elt<T>::kPerVec;
  const bool vec = aligned(a.x, 16) && aligned(a.dx, 16) && (a.N % E == 0) && (a.ld % E == 0) &&
                   (a.ldo % E == 0) && a.N / E <= 0x7fffffff;
  const int block = 256;
  if (vec) {
    a.nvec = static_cast<int>(a.N / E);
    const void* fn = reinterpret_cast<const void*>(&xent_bwd_kernel<T, E>);
    const int grid = persistent_grid(fn, block, 0, a.M);
    xent_bwd_kernel<T, E><<<grid, block, 0, st>>>(a);
  } else {
    a.nvec = 0;
    const void* fn = reinterpret_cast<const void*>(&xent_bwd_kernel<T, 1>);
    const int grid = persistent_grid(fn, block, 0, a.M);
    xent_bwd_kernel<T, 1><<<grid, block, 0, st>>>(a);
  }
  return cudaGetLastError();
}
}  // namespace
}  // namespace dslpg

using namespace dslpg;

extern "C" int dslpg_cross_entropy_bwd(const void* dloss, int dloss_dtype, int64_t dloss_stride,
                                       const void* logits, const float* lse, const void* labels,
                                       void* dlogits, int64_t n_rows, int64_t n_cols,
                                       int64_t logits_row_stride, int64_t dlogits_row_stride,
                                       int logits_dtype, int labels_dtype, float smoothing,
                                       float logit_scale, float lse_square_scale,
                                       int64_t ignored_index, float total_classes,
                                       int64_t class_start_idx, int has_smoothing,
                                       cudaStream_t stream) {
  if (!dloss || !logits || !lse || !labels || !dlogits) return DSLPG_ERR_NULL_POINTER;
  if (n_rows < 0 || n_cols < 0 || logits_row_stride < n_cols || dlogits_row_stride < n_cols ||
      dloss_stride < 0)
    return DSLPG_ERR_BAD_SHAPE;
  if (!is_float_dtype(logits_dtype) || !is_float_dtype(dloss_dtype)) return DSLPG_ERR_BAD_DTYPE;
  if (labels_dtype != DSLPG_I32 && labels_dtype != DSLPG_I64) return DSLPG_ERR_BAD_DTYPE;
  if (n_rows == 0 || n_cols == 0) return DSLPG_OK;
  BwdArgs a{};
  a.dloss = dloss;
  a.dloss_dt = dloss_dtype;
  a.dloss_stride = dloss_stride;
  a.x = logits;
  a.lse = lse;
  a.labels = labels;
  a.label64 = labels_dtype == DSLPG_I64 ? 1 : 0;
  a.dx = dlogits;
  a.M = n_rows;
  a.N = n_cols;
  a.ld = logits_row_stride;
  a.ldo = dlogits_row_stride;
  a.smoothing = smoothing;
  a.scale = logit_scale;
  a.lse_sq = lse_square_scale;
  a.total_classes = total_classes;
  a.ignored = ignored_index;
  a.class_start = class_start_idx;
  a.has_smoothing = has_smoothing ? 1 : 0;
  cudaError_t e;
  switch (logits_dtype) {
    case DSLPG_F32: e = launch_bwd<float>(a, stream); break;
    case DSLPG_F16: e = launch_bwd<__half>(a, stream); break;
    default: e = launch_bwd<__nv_bfloat16>(a, stream); break;
  }
  return static_cast<int>(e);
}
