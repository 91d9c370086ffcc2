/*
 * oracle.c — CPU restatement of the reference's row-reduction family.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity checker for the CUDA
 * backend (and the timed CPU baseline of bench.py); no product code path
 * calls it.
 *
 * Each function restates the algorithm of the reference's PyTorch backend,
 * which the reference uses as its own correctness oracle (tingxi-li/DSLPerfGap,
 * paths inside that project):
 *   layer_norm     ViperBench/layer_norm/pytorch_impl.py:5-12  (F.layer_norm)
 *   rms_norm       ViperBench/rms_norm/pytorch_impl.py:3-10
 *   softmax        ViperBench/softmax/pytorch_impl.py:4-6      (F.softmax, dim -1)
 *   log_softmax    ViperBench/log_softmax/pytorch_impl.py:4-8  (F.log_softmax)
 *   logsumexp      ViperBench/logsumexp/pytorch_impl.py:3-5    (torch.logsumexp)
 *   cross_entropy  ViperBench/cross_entropy/pytorch_impl.py:4-90
 * The reference computes these with torch's fp32 CPU/GPU kernels; here every
 * row is accumulated in double and the result is rounded to fp32 and then to
 * the output dtype (round to nearest even), i.e. "computed in fp32, stored in
 * the output dtype" with the fp32 error removed. NaN/Inf handling follows the
 * torch operators (a NaN max poisons softmax rows; logsumexp shifts by the
 * max only when it is finite).
 *
 * Storage dtype codes match include/dslpg_b200.h: 0 f32, 1 f16, 2 bf16,
 * 3 i32, 4 i64. Rows are split over host threads (pthreads, static chunks).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <pthread.h>
#include <stdlib.h>
#include <unistd.h>

enum { F32 = 0, F16 = 1, BF16 = 2, I32 = 3, I64 = 4 };

/* ---------------------------------------------------------------- dtypes */
static inline float bits_f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* IEEE binary16 -> binary32 (exact). */
static float half_to_float(uint16_t h) {
  uint32_t s = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  if (e == 0) {
    float v = ldexpf((float)m, -24); /* zero or subnormal */
    return s ? -v : v;
  }
  if (e == 31) return bits_f(s | 0x7f800000u | (m << 13));
  return bits_f(s | ((e + 112u) << 23) | (m << 13));
}

/* binary32 -> binary16, round to nearest even. */
static uint16_t float_to_half(float f) {
  uint32_t x = f_bits(f);
  uint16_t s = (uint16_t)((x >> 16) & 0x8000u);
  uint32_t ax = x & 0x7fffffffu;
  if (ax > 0x7f800000u) return s | 0x7e00u;           /* NaN */
  if (ax >= 0x477ff000u) return s | 0x7c00u;          /* >= 65520 rounds to inf */
  if (ax >= 0x38800000u) {                            /* normal half */
    uint32_t e = (ax >> 23) - 112u, mant = ax & 0x7fffffu;
    uint32_t h = (e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return s | (uint16_t)h;
  }
  /* subnormal half: multiples of 2^-24; the product is exact in double */
  double v = nearbyint((double)bits_f(ax) * 16777216.0);
  return s | (uint16_t)v;
}

/* binary32 -> bfloat16, round to nearest even. */
static uint16_t float_to_bf16(float f) {
  uint32_t x = f_bits(f);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u); /* quiet NaN */
  x += 0x7fffu + ((x >> 16) & 1u);
  return (uint16_t)(x >> 16);
}

static inline double load(const void* p, int64_t i, int dt) {
  switch (dt) {
    case F32: return (double)((const float*)p)[i];
    case F16: return (double)half_to_float(((const uint16_t*)p)[i]);
    default: return (double)bits_f((uint32_t)((const uint16_t*)p)[i] << 16);
  }
}

/* Round a double to fp32, then to dtype dt, and store it. */
static inline void store(void* p, int64_t i, int dt, double v) {
  float f = (float)v;
  switch (dt) {
    case F32: ((float*)p)[i] = f; break;
    case F16: ((uint16_t*)p)[i] = float_to_half(f); break;
    default: ((uint16_t*)p)[i] = float_to_bf16(f); break;
  }
}

/* v rounded to fp32 and then to dtype dt (x.to(dtype) in the reference). */
static inline double round_to(double v, int dt) {
  float f = (float)v;
  if (dt == F16) return (double)half_to_float(float_to_half(f));
  if (dt == BF16) return (double)bits_f((uint32_t)float_to_bf16(f) << 16);
  return (double)f;
}

/* torch.max / amax semantics: NaN wins. */
static inline double max_nan(double a, double b) {
  if (isnan(a) || isnan(b)) return NAN;
  return a > b ? a : b;
}

/* ------------------------------------------------------- parallel for */
static int g_threads = 0; /* 0: one per online CPU */

void oracle_set_threads(int n) { g_threads = n > 0 ? n : 0; }
int oracle_max_threads(void) {
  if (g_threads > 0) return g_threads;
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

typedef void (*range_fn)(const void* ctx, int64_t i0, int64_t i1);
typedef struct { range_fn fn; const void* ctx; int64_t i0, i1; } task_t;

static void* run_task(void* p) {
  task_t* t = (task_t*)p;
  if (t->i1 > t->i0) t->fn(t->ctx, t->i0, t->i1);
  return NULL;
}

/* Run fn over [0, n) split into equal contiguous chunks, one per thread. */
static void parallel_for(int64_t n, range_fn fn, const void* ctx) {
  int nt = oracle_max_threads();
  if (nt > 256) nt = 256;
  if (n < nt) nt = n > 0 ? (int)n : 1;
  if (nt <= 1) { if (n > 0) fn(ctx, 0, n); return; }
  pthread_t th[256];
  task_t tk[256];
  int started[256];
  for (int i = 0; i < nt; ++i) {
    tk[i].fn = fn;
    tk[i].ctx = ctx;
    tk[i].i0 = n * i / nt;
    tk[i].i1 = n * (i + 1) / nt;
    started[i] = i > 0 && pthread_create(&th[i], NULL, run_task, &tk[i]) == 0;
  }
  run_task(&tk[0]);
  for (int i = 1; i < nt; ++i) {
    if (started[i]) pthread_join(th[i], NULL);
    else run_task(&tk[i]); /* could not start a thread: run the chunk here */
  }
}

/* ------------------------------------------------------------ operators */
typedef struct {
  const void *x, *w, *b, *labels;
  void* y;
  float *loss, *lse, *zl;
  int64_t M, N, K, BS, nb, ignored, class_start;
  int xdt, wdt, odt, lbdt, has_smoothing, split;
  double eps, smoothing, scale, lse_sq, total_classes;
} args_t;

/* F.layer_norm over the last N elements: biased variance. */
static void layer_norm_rows(const void* ctx, int64_t r0, int64_t r1) {
  const args_t* a = (const args_t*)ctx;
  const int64_t N = a->N;
  for (int64_t r = r0; r < r1; ++r) {
    const int64_t o = r * N;
    double s = 0.0;
    for (int64_t j = 0; j < N; ++j) s += load(a->x, o + j, a->xdt);
    const double mean = s / (double)N;
    double q = 0.0;
    for (int64_t j = 0; j < N; ++j) {
      const double d = load(a->x, o + j, a->xdt) - mean;
      q += d * d;
    }
    const double rstd = 1.0 / sqrt(q / (double)N + a->eps);
    for (int64_t j = 0; j < N; ++j) {
      double v = (load(a->x, o + j, a->xdt) - mean) * rstd * load(a->w, j, a->wdt);
      if (a->b) v += load(a->b, j, a->wdt);
      store(a->y, o + j, a->xdt, v);
    }
  }
}

void oracle_layer_norm(const void* x, const void* w, const void* b, void* y, int64_t M, int64_t N,
                       int xdt, int wdt, double eps) {
  args_t a = {0};
  a.x = x; a.w = w; a.b = b; a.y = y; a.M = M; a.N = N; a.xdt = xdt; a.wdt = wdt; a.eps = eps;
  parallel_for(M, layer_norm_rows, &a);
}

/* rms = sqrt(mean(x.float()**2) + eps); y = (x.float() / rms * w.float()).to(x.dtype) */
static void rms_norm_rows(const void* ctx, int64_t r0, int64_t r1) {
  const args_t* a = (const args_t*)ctx;
  const int64_t N = a->N;
  for (int64_t r = r0; r < r1; ++r) {
    const int64_t o = r * N;
    double ss = 0.0;
    for (int64_t j = 0; j < N; ++j) {
      const double v = load(a->x, o + j, a->xdt);
      ss += v * v;
    }
    const double rms = sqrt(ss / (double)N + a->eps);
    for (int64_t j = 0; j < N; ++j)
      store(a->y, o + j, a->xdt, load(a->x, o + j, a->xdt) / rms * load(a->w, j, a->wdt));
  }
}

void oracle_rms_norm(const void* x, const void* w, void* y, int64_t M, int64_t N, int xdt, int wdt,
                     double eps) {
  args_t a = {0};
  a.x = x; a.w = w; a.y = y; a.M = M; a.N = N; a.xdt = xdt; a.wdt = wdt; a.eps = eps;
  parallel_for(M, rms_norm_rows, &a);
}

/* F.softmax(x, -1): exp(x - max) / sum; a NaN or infinite max gives a NaN row. */
static void softmax_rows(const void* ctx, int64_t r0, int64_t r1) {
  const args_t* a = (const args_t*)ctx;
  const int64_t N = a->N;
  for (int64_t r = r0; r < r1; ++r) {
    const int64_t o = r * N;
    double m = -INFINITY;
    for (int64_t j = 0; j < N; ++j) m = max_nan(m, load(a->x, o + j, a->xdt));
    double s = 0.0;
    for (int64_t j = 0; j < N; ++j) s += exp(load(a->x, o + j, a->xdt) - m);
    for (int64_t j = 0; j < N; ++j) store(a->y, o + j, a->xdt, exp(load(a->x, o + j, a->xdt) - m) / s);
  }
}

void oracle_softmax(const void* x, void* y, int64_t M, int64_t N, int dt) {
  args_t a = {0};
  a.x = x; a.y = y; a.M = M; a.N = N; a.xdt = dt;
  parallel_for(M, softmax_rows, &a);
}

/* F.log_softmax(x, dim, dtype) over the middle axis of [M, N, K]: x is first
 * converted to the output dtype, then y = (x - max) - log(sum(exp(x - max))). */
static void log_softmax_cols(const void* ctx, int64_t c0, int64_t c1) {
  const args_t* a = (const args_t*)ctx;
  const int64_t N = a->N, K = a->K;
  for (int64_t c = c0; c < c1; ++c) {
    const int64_t mi = c / K, k = c % K;
    const int64_t o = mi * N * K + k;
    double m = -INFINITY;
    for (int64_t n = 0; n < N; ++n) m = max_nan(m, round_to(load(a->x, o + n * K, a->xdt), a->odt));
    double s = 0.0;
    for (int64_t n = 0; n < N; ++n) s += exp(round_to(load(a->x, o + n * K, a->xdt), a->odt) - m);
    const double ls = log(s);
    for (int64_t n = 0; n < N; ++n)
      store(a->y, o + n * K, a->odt, (round_to(load(a->x, o + n * K, a->xdt), a->odt) - m) - ls);
  }
}

void oracle_log_softmax(const void* x, void* y, int64_t M, int64_t N, int64_t K, int idt, int odt) {
  args_t a = {0};
  a.x = x; a.y = y; a.M = M; a.N = N; a.K = K; a.xdt = idt; a.odt = odt;
  parallel_for(M * K, log_softmax_cols, &a);
}

/* torch.logsumexp(x, -1): shift by the max only when it is finite. */
static void logsumexp_rows(const void* ctx, int64_t r0, int64_t r1) {
  const args_t* a = (const args_t*)ctx;
  const int64_t N = a->N;
  for (int64_t r = r0; r < r1; ++r) {
    const int64_t o = r * N;
    double m = -INFINITY;
    for (int64_t j = 0; j < N; ++j) m = max_nan(m, load(a->x, o + j, a->xdt));
    const double shift = isinf(m) ? 0.0 : m;
    double s = 0.0;
    for (int64_t j = 0; j < N; ++j) s += exp(load(a->x, o + j, a->xdt) - shift);
    store(a->y, r, a->xdt, log(s) + shift);
  }
}

void oracle_logsumexp(const void* x, void* y, int64_t M, int64_t N, int dt) {
  args_t a = {0};
  a.x = x; a.y = y; a.M = M; a.N = N; a.xdt = dt;
  parallel_for(M, logsumexp_rows, &a);
}

/*
 * cross_entropy_fwd of ViperBench/cross_entropy/pytorch_impl.py:4-90.
 * Per (row r, column block cb): L = logits * scale over the block (columns
 * beyond n_cols are -inf, pytorch_impl.py:29-31); lse = log(sum(exp(L - max)))
 * + max (:34-35); the loss terms of :52-70; ignored rows get loss = z = 0 but
 * keep their lse (:74-76). Results go to flat index cb * R + r of [R, C]
 * outputs and every other entry is 0 (:80-88).
 */
static void cross_entropy_items(const void* ctx, int64_t i0, int64_t i1) {
  const args_t* a = (const args_t*)ctx;
  const int64_t R = a->M, C = a->N, BS = a->BS;
  for (int64_t it = i0; it < i1; ++it) {
    const int64_t r = it / a->nb, cb = it % a->nb;
    const int64_t c0 = cb * BS, c1 = (cb + 1) * BS < C ? (cb + 1) * BS : C;
    const int64_t o = r * C;
    /* The -inf padding of a short last block neither raises the max nor adds
     * to the sum; an all -inf block gives NaN through exp(-inf - -inf). */
    double m = -INFINITY, sum_logits = 0.0;
    for (int64_t j = c0; j < c1; ++j) {
      const double v = (double)(float)(load(a->x, o + j, a->xdt) * a->scale);
      m = max_nan(m, v);
      sum_logits += v;
    }
    double s = 0.0;
    for (int64_t j = c0; j < c1; ++j) s += exp((double)(float)(load(a->x, o + j, a->xdt) * a->scale) - m);
    const double l = log(s) + m;
    const int64_t label = a->lbdt == I64 ? ((const int64_t*)a->labels)[r]
                                         : (int64_t)((const int32_t*)a->labels)[r];
    const int64_t adj = label - a->class_start;
    const int64_t fi = cb * R + r;
    double ls = 0.0, z = 0.0;
    if (label != a->ignored) {
      const double lt = a->split ? 0.0 : l;
      if (adj >= c0 && adj < c1) {
        const double xl = (double)(float)(load(a->x, o + adj, a->xdt) * a->scale);
        ls = a->has_smoothing
                 ? lt - a->smoothing * sum_logits / a->total_classes - (1.0 - a->smoothing) * xl
                 : lt - xl;
      } else {
        ls = a->has_smoothing ? a->smoothing * (lt - sum_logits / a->total_classes) : 0.0;
      }
      if (!a->split) {
        z = a->lse_sq * l * l;
        ls += z;
      }
    }
    a->lse[fi] = (float)l;
    a->loss[fi] = (float)ls;
    a->zl[fi] = (float)z;
  }
}

void oracle_cross_entropy_fwd(const void* logits, const void* labels, float* loss, float* lse,
                              float* zl, int64_t R, int64_t C, int ldt, int lbdt, double smoothing,
                              double scale, double lse_sq, int64_t ignored, double total_classes,
                              int64_t class_start, int64_t BS, int has_smoothing, int split,
                              int64_t out_len) {
  /* Outputs hold out_len floats: R * C for the reference layout, or just the
   * nb * R valid entries. Entries past the valid prefix are zero. */
  const int64_t nvalid = R * ((C + BS - 1) / BS);
  if (out_len > nvalid) {
    const size_t tail = sizeof(float) * (size_t)(out_len - nvalid);
    memset(loss + nvalid, 0, tail);
    memset(lse + nvalid, 0, tail);
    memset(zl + nvalid, 0, tail);
  }
  args_t a = {0};
  a.x = logits; a.labels = labels; a.loss = loss; a.lse = lse; a.zl = zl;
  a.M = R; a.N = C; a.BS = BS; a.nb = (C + BS - 1) / BS;
  a.xdt = ldt; a.lbdt = lbdt; a.smoothing = smoothing; a.scale = scale; a.lse_sq = lse_sq;
  a.ignored = ignored; a.total_classes = total_classes; a.class_start = class_start;
  a.has_smoothing = has_smoothing; a.split = split;
  parallel_for(R * a.nb, cross_entropy_items, &a);
}

/*
 * cross_entropy_bwd of ViperBench/cross_entropy/pytorch_impl.py:93-141 (the
 * Triton kernel's arithmetic, triton_impl.py:98-120): for every column,
 * probs = exp(logits * scale - lse[r]); probs += 2 * lse_sq * lse[r] * probs;
 * the label column loses (1 - smoothing) (or 1); with smoothing every column
 * loses smoothing / total_classes; dlogits = (dloss[r] * scale) * probs, with
 * dloss = 0 on ignored rows. lse[r] and dloss[r] are read at flat index r.
 */
typedef struct {
  const void *dloss, *x, *labels;
  const float* lse;
  void* dx;
  int64_t R, C, ignored, class_start;
  int ddt, xdt, lbdt, has_smoothing;
  double smoothing, scale, lse_sq, total_classes;
} bwd_t;

static void cross_entropy_bwd_rows(const void* ctx, int64_t r0, int64_t r1) {
  const bwd_t* a = (const bwd_t*)ctx;
  for (int64_t r = r0; r < r1; ++r) {
    const int64_t label = a->lbdt == I64 ? ((const int64_t*)a->labels)[r] : (int64_t)((const int32_t*)a->labels)[r];
    const double dl = label != a->ignored ? load(a->dloss, r, a->ddt) : 0.0;
    const double lse = (double)a->lse[r];
    const int64_t adj = label - a->class_start;
    for (int64_t c = 0; c < a->C; ++c) {
      double p = exp((double)(float)(load(a->x, r * a->C + c, a->xdt) * a->scale) - lse);
      p += 2.0 * a->lse_sq * lse * p;
      if (c == adj) p -= a->has_smoothing ? (1.0 - a->smoothing) : 1.0;
      if (a->has_smoothing) p -= a->smoothing / a->total_classes;
      store(a->dx, r * a->C + c, a->xdt, (dl * a->scale) * p);
    }
  }
}

void oracle_cross_entropy_bwd(const void* dloss, int ddt, const void* logits, const float* lse, const void* labels,
                              void* dlogits, int64_t R, int64_t C, int xdt, int lbdt, double smoothing,
                              double scale, double lse_sq, int64_t ignored, double total_classes,
                              int64_t class_start, int has_smoothing) {
  bwd_t a;
  memset(&a, 0, sizeof(a));
  a.dloss = dloss; a.ddt = ddt; a.x = logits; a.lse = lse; a.labels = labels; a.dx = dlogits;
  a.R = R; a.C = C; a.xdt = xdt; a.lbdt = lbdt; a.smoothing = smoothing; a.scale = scale;
  a.lse_sq = lse_sq; a.ignored = ignored; a.total_classes = total_classes; a.class_start = class_start;
  a.has_smoothing = has_smoothing;
  parallel_for(R, cross_entropy_bwd_rows, &a);
}

/*
 * Reductions over the middle axis of [M, N, K]:
 *   mean   torch.mean(x, dim, dtype=odt)  (ViperBench/mean_reduction/pytorch_impl.py:4-8):
 *          x converted to odt, summed (double here), divided by N;
 *   max    torch.max(x, dim)               (ViperBench/max_reduction/pytorch_impl.py:4-11)
 *   argmax torch.argmax(x, dim)            (ViperBench/argmax/pytorch_impl.py:4-8):
 *          the first NaN is the maximum; equal maxima give the first index.
 */
typedef struct {
  const void* x;
  void* y;
  int64_t* idx;
  int64_t M, N, K;
  int idt, odt, want_vals;
} red_t;

static void mean_cols(const void* ctx, int64_t c0, int64_t c1) {
  const red_t* a = (const red_t*)ctx;
  for (int64_t c = c0; c < c1; ++c) {
    const int64_t mi = c / a->K, k = c % a->K, o = mi * a->N * a->K + k;
    double s = 0.0;
    for (int64_t n = 0; n < a->N; ++n) s += round_to(load(a->x, o + n * a->K, a->idt), a->odt);
    store(a->y, c, a->odt, s / (double)a->N);
  }
}

static void max_cols(const void* ctx, int64_t c0, int64_t c1) {
  const red_t* a = (const red_t*)ctx;
  for (int64_t c = c0; c < c1; ++c) {
    const int64_t mi = c / a->K, k = c % a->K, o = mi * a->N * a->K + k;
    double best = load(a->x, o, a->idt);
    int64_t bi = 0;
    for (int64_t n = 1; n < a->N && !isnan(best); ++n) {
      const double v = load(a->x, o + n * a->K, a->idt);
      if (isnan(v) || v > best) { best = v; bi = n; }
    }
    if (a->want_vals) store(a->y, c, a->idt, best);
    a->idx[c] = bi;
  }
}

void oracle_mean_reduction(const void* x, void* y, int64_t M, int64_t N, int64_t K, int idt, int odt) {
  red_t a;
  memset(&a, 0, sizeof(a));
  a.x = x; a.y = y; a.M = M; a.N = N; a.K = K; a.idt = idt; a.odt = odt;
  parallel_for(M * K, mean_cols, &a);
}

void oracle_max_reduction(const void* x, void* values, int64_t* indices, int64_t M, int64_t N, int64_t K,
                          int dt) {
  red_t a;
  memset(&a, 0, sizeof(a));
  a.x = x; a.y = values; a.idx = indices; a.M = M; a.N = N; a.K = K; a.idt = dt; a.want_vals = values != 0;
  parallel_for(M * K, max_cols, &a);
}

/*
 * kernel_ff of ViperBench/linear_activation/pytorch_impl.py:5-54 (fp16 in/out):
 * a_norm = 1/sqrt(sum(x^2)/K + 1e-6); xs = fp16(x * rms_w); acc1 = xs @ w1^T,
 * acc3 = xs @ w3^T (double here); out = fp16((acc1 * a) * sigmoid(acc1 * a) * (acc3 * a)).
 */
typedef struct {
  const uint16_t *x, *w1, *w3, *rw;
  uint16_t* out;
  int64_t M, N, K;
} ff_t;

static void ff_rows(const void* ctx, int64_t m0, int64_t m1) {
  const ff_t* a = (const ff_t*)ctx;
  const int64_t K = a->K;
  double* xs = (double*)malloc(sizeof(double) * (size_t)K);
  if (!xs) return;
  for (int64_t m = m0; m < m1; ++m) {
    double ss = 0.0;
    for (int64_t k = 0; k < K; ++k) {
      const double v = half_to_float(a->x[m * K + k]);
      ss += v * v;
      xs[k] = half_to_float(float_to_half((float)(v * half_to_float(a->rw[k]))));
    }
    const double an = 1.0 / sqrt(ss / (double)K + 1e-6);
    for (int64_t n = 0; n < a->N; ++n) {
      double acc1 = 0.0, acc3 = 0.0;
      for (int64_t k = 0; k < K; ++k) {
        acc1 += xs[k] * half_to_float(a->w1[n * K + k]);
        acc3 += xs[k] * half_to_float(a->w3[n * K + k]);
      }
      const double g = acc1 * an, u = acc3 * an;
      a->out[m * a->N + n] = float_to_half((float)(g / (1.0 + exp(-g)) * u));
    }
  }
  free(xs);
}

void oracle_kernel_ff(const uint16_t* x, const uint16_t* w1, const uint16_t* w3, const uint16_t* rms_w,
                      uint16_t* out, int64_t M, int64_t N, int64_t K) {
  ff_t a = {x, w1, w3, rms_w, out, M, N, K};
  parallel_for(M, ff_rows, &a);
}

/* Bit-level conversions, exported so tests can check them. */
float oracle_half_to_float(uint16_t h) { return half_to_float(h); }
uint16_t oracle_float_to_half(float f) { return float_to_half(f); }
uint16_t oracle_float_to_bf16(float f) { return float_to_bf16(f); }
