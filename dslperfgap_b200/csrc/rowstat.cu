// rowstat.cu — reductions of a row (or row segment) to a few scalars:
// logsumexp and the blockwise cross-entropy forward (sm_100a).
//
// One kernel, rowstat_kernel, streams each work item (a row for logsumexp, a
// (row, column block) pair for cross-entropy) exactly once from HBM with
// 16-byte loads, U vectors in flight per thread, and keeps an online
// (max, sum of exp) pair per thread in the log2 domain:
//     t = x * scale * log2(e);  m = max t;  s = sum 2^(t - m)
// so each element costs one multiply, one max, one subtract, one SFU ex2 and
// one add. Per-thread pairs are merged with warp shuffles and a shared-memory
// step, and lse = (m + log2 s) * ln 2.
//
// Work item i maps to row r = i / nseg, block cb = i % nseg, so consecutive
// work items touch consecutive memory. Cross-entropy outputs land at flat
// index cb * n_rows + r, the layout of
// ViperBench/cross_entropy/triton_impl.py:46,75-76.
#include "common.cuh"

namespace dslpg {

enum StatKind : int { kLse = 0, kXent = 1 };

struct StatArgs {
  const void* x;
  int64_t M;      // rows
  int64_t N;      // columns
  int64_t ld;     // row stride in elements
  int64_t seg;    // segment (column block) length
  int64_t nseg;   // segments per row
  int tpr;        // threads per work item
  int rpc;        // work items per CTA
  float c;        // scale * log2(e)
  void* out;      // logsumexp: [M] of x's dtype
  // cross-entropy
  const void* labels;
  int label64;
  float* loss;
  float* lse;
  float* zloss;
  float smoothing, scale, lse_sq, total_classes;
  int64_t ignored, class_start;
  int split;
};

constexpr float kNaN = __builtin_nanf("");

// Fold a chunk of n log2-domain values into the running (m, s).
template <int n>
DSLPG_DEV void fold_chunk(float& m, float& s, const float* t) {
  float cm = t[0];
#pragma unroll
  for (int i = 1; i < n; ++i) cm = max_nan(cm, t[i]);
  const float nm = max_nan(m, cm);
  if (nm == kNegInf) return;  // nothing but -inf so far
  float acc = (m == nm) ? s : s * ex2(m - nm);
#pragma unroll
  for (int i = 0; i < n; ++i) acc += ex2(t[i] - nm);
  s = acc;
  m = nm;
}

template <int KIND, typename T, int V, bool SMOOTH>
__global__ void __launch_bounds__(1024) rowstat_kernel(const StatArgs a) {
  constexpr int U = (V == 1) ? 8 : 4;  // loads in flight per thread per iteration
  __shared__ float red[2][32];
  const int g = threadIdx.x / a.tpr;
  const int t = threadIdx.x - g * a.tpr;
  const int nw = a.tpr >> 5;
  const int first_warp = g * nw;
  int buf = 0;
  const int64_t items = a.M * a.nseg;
  const int64_t step = static_cast<int64_t>(gridDim.x) * a.rpc;

  for (int64_t base = static_cast<int64_t>(blockIdx.x) * a.rpc; base < items; base += step) {
    const int64_t item = base + g;
    const bool iv = item < items;
    const int64_t r = iv ? item / a.nseg : 0;
    const int64_t cb = iv ? item - r * a.nseg : 0;
    const int64_t col0 = cb * a.seg;
    const int64_t len = iv ? ((a.N - col0) < a.seg ? (a.N - col0) : a.seg) : 0;
    const T* xs = static_cast<const T*>(a.x) + r * a.ld + col0;

    float m = kNegInf, s = 0.f, sum = 0.f;
    int64_t done = 0;
    if constexpr (V > 1) {
      const int64_t nv = len / V;
      for (int64_t j0 = t; j0 < nv; j0 += static_cast<int64_t>(U) * a.tpr) {
        Vec16 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t j = j0 + static_cast<int64_t>(u) * a.tpr;
          v[u] = Vec16{{0u, 0u, 0u, 0u}};
          if (j < nv) v[u] = ld_stream(xs + j * V);
        }
        float tv[U * V];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t j = j0 + static_cast<int64_t>(u) * a.tpr;
          float f[V];
          unpack<T>(v[u], f);
#pragma unroll
          for (int i = 0; i < V; ++i) {
            if constexpr (SMOOTH) sum += f[i];  // masked vectors read as 0
            tv[u * V + i] = (j < nv) ? f[i] * a.c : kNegInf;
          }
        }
        fold_chunk<U * V>(m, s, tv);
      }
      done = nv * V;
    }
    // Scalar remainder (the whole item on the scalar path).
    for (int64_t j0 = done + t; j0 < len; j0 += static_cast<int64_t>(U) * a.tpr) {
      float tv[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t j = j0 + static_cast<int64_t>(u) * a.tpr;
        float f = 0.f;
        if (j < len) f = to_f(xs[j]);
        if constexpr (SMOOTH) sum += f;
        tv[u] = (j < len) ? f * a.c : kNegInf;
      }
      fold_chunk<U>(m, s, tv);
    }

    // Merge the group's (m, s) pairs.
    const float gm = group_reduce<MaxOp>(m, red[buf], nw, first_warp);
    buf ^= 1;
    const float sc = (m == gm) ? s : s * ex2(m - gm);
    const float gs = group_reduce<SumOp>(sc, red[buf], nw, first_warp);
    buf ^= 1;
    float gsum = 0.f;
    if constexpr (SMOOTH) {
      gsum = group_reduce<SumOp>(sum, red[buf], nw, first_warp);
      buf ^= 1;
    }

    if (t == 0 && iv) {
      const float lse_fin = (gm + log2f(gs)) * kLn2;
      if constexpr (KIND == kLse) {
        // torch.logsumexp shifts by the max only when it is finite.
        float v = lse_fin;
        if (gm == kPosInf) v = kPosInf;
        else if (gm == kNegInf) v = kNegInf;
        static_cast<T*>(a.out)[r] = from_f<T>(v);
      } else {
        const float lse = (fabsf(gm) < kPosInf) ? lse_fin : kNaN;
        const int64_t oi = cb * a.M + r;
        a.lse[oi] = lse;
        const int64_t label = a.label64 ? static_cast<const int64_t*>(a.labels)[r]
                                        : static_cast<int64_t>(static_cast<const int32_t*>(a.labels)[r]);
        float loss = 0.f, z = 0.f;
        if (label != a.ignored) {
          const int64_t adj = label - a.class_start;
          const float lse_term = a.split ? 0.f : lse;
          const float sum_logits = gsum * a.scale;
          const int64_t hi = (cb + 1) * a.seg < a.N ? (cb + 1) * a.seg : a.N;
          if (adj >= col0 && adj < hi) {
            const float xl = to_f(static_cast<const T*>(a.x)[r * a.ld + adj]) * a.scale;
            if constexpr (SMOOTH)
              loss = lse_term - a.smoothing * sum_logits / a.total_classes - (1.f - a.smoothing) * xl;
            else
              loss = lse_term - xl;
          } else if constexpr (SMOOTH) {
            loss = a.smoothing * (lse_term - sum_logits / a.total_classes);
          }
          if (!a.split) {
            z = a.lse_sq * lse * lse;
            loss += z;
          }
        }
        a.loss[oi] = loss;
        a.zloss[oi] = z;
      }
    }
  }
}

namespace {

inline int round_up32(int v) { return (v + 31) & ~31; }

template <int KIND, typename T, int V, bool SMOOTH>
cudaError_t launch_stat(StatArgs a, cudaStream_t st) {
  // Threads per work item: about 16 vectors (or 64 scalars) per thread per item.
  const int64_t units = (V > 1) ? a.seg / V : a.seg;
  const int64_t per_thread = (V > 1) ? 16 : 64;
  int64_t want = (units + per_thread - 1) / per_thread;
  int tpr = static_cast<int>(want > 256 ? 256 : want);
  tpr = round_up32(tpr < 32 ? 32 : tpr);
  a.tpr = tpr;
  a.rpc = tpr >= 256 ? 1 : 256 / tpr;
  const int block = a.tpr * a.rpc;
  const void* fn = reinterpret_cast<const void*>(&rowstat_kernel<KIND, T, V, SMOOTH>);
  const int64_t items = a.M * a.nseg;
  const int grid = persistent_grid(fn, block, 0, (items + a.rpc - 1) / a.rpc);
  rowstat_kernel<KIND, T, V, SMOOTH><<<grid, block, 0, st>>>(a);
  return cudaGetLastError();
}

template <int KIND, typename T, bool SMOOTH>
cudaError_t dispatch_vec(StatArgs a, cudaStream_t st) {
  constexpr int E = Elt<T>::kPerVec;
  const bool vec = aligned(a.x, 16) && (a.ld % E == 0) && (a.seg % E == 0);
  if (vec) return launch_stat<KIND, T, E, SMOOTH>(a, st);
  return launch_stat<KIND, T, 1, SMOOTH>(a, st);
}

template <int KIND, bool SMOOTH>
cudaError_t dispatch_dtype(StatArgs a, int dt, cudaStream_t st) {
  switch (dt) {
    case DSLPG_F32: return dispatch_vec<KIND, float, SMOOTH>(a, st);
    case DSLPG_F16: return dispatch_vec<KIND, __half, SMOOTH>(a, st);
    default: return dispatch_vec<KIND, __nv_bfloat16, SMOOTH>(a, st);
  }
}

}  // namespace
}  // namespace dslpg

using namespace dslpg;

extern "C" int dslpg_logsumexp_fwd(const void* x, void* y, int64_t M, int64_t N, int dtype,
                                   cudaStream_t stream) {
  if (x == nullptr || y == nullptr) return DSLPG_ERR_NULL_POINTER;
  if (M < 0 || N < 0) return DSLPG_ERR_BAD_SHAPE;
  if (!is_float_dtype(dtype)) return DSLPG_ERR_BAD_DTYPE;
  if (M == 0) return DSLPG_OK;
  if (N == 0) return DSLPG_ERR_BAD_SHAPE;  // torch.logsumexp of an empty row is -inf; callers handle it
  StatArgs a{};
  a.x = x;
  a.M = M;
  a.N = N;
  a.ld = N;
  a.seg = N;
  a.nseg = 1;
  a.c = kLog2e;
  a.out = y;
  return static_cast<int>(dispatch_dtype<kLse, false>(a, dtype, stream));
}

extern "C" int dslpg_cross_entropy_fwd(const void* logits, const void* labels, float* loss,
                                       float* lse, float* z_loss, int64_t n_rows, int64_t n_cols,
                                       int64_t logits_row_stride, int logits_dtype,
                                       int labels_dtype, float smoothing, float logit_scale,
                                       float lse_square_scale, int64_t ignored_index,
                                       float total_classes, int64_t class_start_idx,
                                       int64_t block_size, int has_smoothing, int split,
                                       cudaStream_t stream) {
  if (!logits || !labels || !loss || !lse || !z_loss) return DSLPG_ERR_NULL_POINTER;
  if (n_rows < 0 || n_cols < 0 || block_size <= 0 || logits_row_stride < n_cols)
    return DSLPG_ERR_BAD_SHAPE;
  if (!is_float_dtype(logits_dtype)) return DSLPG_ERR_BAD_DTYPE;
  if (labels_dtype != DSLPG_I32 && labels_dtype != DSLPG_I64) return DSLPG_ERR_BAD_DTYPE;
  if (n_rows == 0 || n_cols == 0) return DSLPG_OK;
  StatArgs a{};
  a.x = logits;
  a.M = n_rows;
  a.N = n_cols;
  a.ld = logits_row_stride;
  // One segment per column block; a block wider than the row is the whole row.
  a.seg = block_size < n_cols ? block_size : n_cols;
  a.nseg = (n_cols + block_size - 1) / block_size;
  a.c = logit_scale * kLog2e;
  a.labels = labels;
  a.label64 = labels_dtype == DSLPG_I64 ? 1 : 0;
  a.loss = loss;
  a.lse = lse;
  a.zloss = z_loss;
  a.smoothing = smoothing;
  a.scale = logit_scale;
  a.lse_sq = lse_square_scale;
  a.total_classes = total_classes;
  a.ignored = ignored_index;
  a.class_start = class_start_idx;
  a.split = split ? 1 : 0;
  cudaError_t e = has_smoothing ? dispatch_dtype<kXent, true>(a, logits_dtype, stream)
                                : dispatch_dtype<kXent, false>(a, logits_dtype, stream);
  return static_cast<int>(e);
}
