// host_pipe.cu — row ops (RMSNorm, LayerNorm) on HOST buffers: the rows stream through the GPU in
// chunks, with the upload of chunk i+1, the kernel on chunk i and the download
// of chunk i-1 in flight together (PCIe is full duplex, so with pinned host
// memory the two copy directions overlap).
//
// Per device this file keeps two non-blocking copy streams (upload, download)
// and a set of events, created on first use. The kernels run on the caller's
// stream. Slot k of the caller-provided device workspace holds one input
// chunk and one output chunk; the dependencies between the streams are:
//   upload i    waits  kernel i-S      (slot k's input buffer is free)
//   kernel i    waits  upload i, download i-S (slot k's output buffer is free)
//   download i  waits  kernel i
// and the caller's stream finally waits for every download, so the call is
// ordered on `stream` like any other launch: the host reads y after
// synchronising that stream. Copies are one cudaMemcpyAsync each.
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace dslpg {
namespace {

constexpr int kSlots = 4;
#ifndef DSLPG_HOST_CHUNK_BYTES
#define DSLPG_HOST_CHUNK_BYTES (16 << 20)  // measured best of 1, 4, 16, 64 MiB on the RMSNorm headline
#endif
constexpr int64_t kChunkBytes = DSLPG_HOST_CHUNK_BYTES;  // input bytes per chunk (at least one row)
constexpr int kMaxDevices = 64;

struct HostPipe {
  bool ready = false;
  cudaStream_t up = nullptr, down = nullptr;
  cudaEvent_t entry = nullptr;
  cudaEvent_t uploaded[kSlots] = {}, computed[kSlots] = {}, downloaded[kSlots] = {};
};

HostPipe g_pipes[kMaxDevices];
std::mutex g_pipe_mu;

cudaError_t pipe_for_current_device(HostPipe** out) {
  int dev = 0;
  if (cudaError_t e = cudaGetDevice(&dev)) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  HostPipe& p = g_pipes[dev];
  if (!p.ready) {
    if (cudaError_t e = cudaStreamCreateWithFlags(&p.up, cudaStreamNonBlocking)) return e;
    if (cudaError_t e = cudaStreamCreateWithFlags(&p.down, cudaStreamNonBlocking)) return e;
    if (cudaError_t e = cudaEventCreateWithFlags(&p.entry, cudaEventDisableTiming)) return e;
    for (int k = 0; k < kSlots; ++k) {
      if (cudaError_t e = cudaEventCreateWithFlags(&p.uploaded[k], cudaEventDisableTiming)) return e;
      if (cudaError_t e = cudaEventCreateWithFlags(&p.computed[k], cudaEventDisableTiming)) return e;
      if (cudaError_t e = cudaEventCreateWithFlags(&p.downloaded[k], cudaEventDisableTiming)) return e;
    }
    p.ready = true;
  }
  *out = &p;
  return cudaSuccess;
}

int64_t chunk_rows(int64_t M, int64_t in_row_bytes) {
  const int64_t r = kChunkBytes / (in_row_bytes > 0 ? in_row_bytes : 1);
  return std::max<int64_t>(1, std::min<int64_t>(r, M));
}

int64_t align256(int64_t b) { return (b + 255) / 256 * 256; }

int64_t pipe_workspace_bytes(int64_t M, int64_t in_row_bytes, int64_t out_row_bytes) {
  const int64_t rows = chunk_rows(M, in_row_bytes);
  return kSlots * (align256(rows * in_row_bytes) + align256(rows * out_row_bytes));
}

// Run launch(in_dev, out_dev, rows, stream) over all M rows in chunks.
template <class Launch>
int host_rows_pipeline(const void* x_host, void* y_host, int64_t M, int64_t in_row_bytes, int64_t out_row_bytes,
                       void* workspace, int64_t workspace_bytes, cudaStream_t stream, Launch launch) {
  if (workspace_bytes < pipe_workspace_bytes(M, in_row_bytes, out_row_bytes)) return DSLPG_ERR_BAD_ARGUMENT;
  if (!aligned(workspace, 256)) return DSLPG_ERR_BAD_ARGUMENT;
  const int64_t rows = chunk_rows(M, in_row_bytes);
  const int64_t in_slot = align256(rows * in_row_bytes), out_slot = align256(rows * out_row_bytes);
  char* ws = static_cast<char*>(workspace);
  std::lock_guard<std::mutex> lock(g_pipe_mu);  // the per-device streams and events are shared
  HostPipe* p = nullptr;
  if (cudaError_t e = pipe_for_current_device(&p)) return static_cast<int>(e);
  // nothing of this call starts before the caller's earlier work on `stream`
  if (cudaError_t e = cudaEventRecord(p->entry, stream)) return static_cast<int>(e);
  if (cudaError_t e = cudaStreamWaitEvent(p->up, p->entry, 0)) return static_cast<int>(e);
  if (cudaError_t e = cudaStreamWaitEvent(p->down, p->entry, 0)) return static_cast<int>(e);
  const int64_t chunks = (M + rows - 1) / rows;
  for (int64_t i = 0; i < chunks; ++i) {
    const int k = static_cast<int>(i % kSlots);
    const int64_t r0 = i * rows, n = std::min(rows, M - r0);
    char* in = ws + k * (in_slot + out_slot);
    char* out = in + in_slot;
    if (i >= kSlots)
      if (cudaError_t e = cudaStreamWaitEvent(p->up, p->computed[k], 0)) return static_cast<int>(e);
    if (cudaError_t e = cudaMemcpyAsync(in, static_cast<const char*>(x_host) + r0 * in_row_bytes, n * in_row_bytes,
                                        cudaMemcpyHostToDevice, p->up))
      return static_cast<int>(e);
    if (cudaError_t e = cudaEventRecord(p->uploaded[k], p->up)) return static_cast<int>(e);
    if (cudaError_t e = cudaStreamWaitEvent(stream, p->uploaded[k], 0)) return static_cast<int>(e);
    if (i >= kSlots)
      if (cudaError_t e = cudaStreamWaitEvent(stream, p->downloaded[k], 0)) return static_cast<int>(e);
    if (int rc = launch(in, out, n, stream)) return rc;
    if (cudaError_t e = cudaEventRecord(p->computed[k], stream)) return static_cast<int>(e);
    if (cudaError_t e = cudaStreamWaitEvent(p->down, p->computed[k], 0)) return static_cast<int>(e);
    if (cudaError_t e = cudaMemcpyAsync(static_cast<char*>(y_host) + r0 * out_row_bytes, out, n * out_row_bytes,
                                        cudaMemcpyDeviceToHost, p->down))
      return static_cast<int>(e);
    if (cudaError_t e = cudaEventRecord(p->downloaded[k], p->down)) return static_cast<int>(e);
  }
  // the last download is recorded after all earlier ones on the same stream
  const int last = static_cast<int>((chunks - 1) % kSlots);
  if (cudaError_t e = cudaStreamWaitEvent(stream, p->downloaded[last], 0)) return static_cast<int>(e);
  return DSLPG_OK;
}

}  // namespace
}  // namespace dslpg

using namespace dslpg;

extern "C" int dslpg_rms_norm_fwd_host_workspace_bytes(int64_t M, int64_t N, int x_dtype, int64_t* bytes) {
  if (bytes == nullptr) return DSLPG_ERR_NULL_POINTER;
  if (M < 0 || N < 0) return DSLPG_ERR_BAD_SHAPE;
  if (!is_float_dtype(x_dtype)) return DSLPG_ERR_BAD_DTYPE;
  const int64_t rb = N * dtype_size(x_dtype);
  *bytes = (M == 0 || N == 0) ? 0 : pipe_workspace_bytes(M, rb, rb);
  return DSLPG_OK;
}

extern "C" int dslpg_rms_norm_fwd_host(const void* x_host, const void* weight, void* y_host, int64_t M, int64_t N,
                                       int x_dtype, int w_dtype, float eps, void* workspace, int64_t workspace_bytes,
                                       cudaStream_t stream) {
  if (!x_host || !weight || !y_host) return DSLPG_ERR_NULL_POINTER;
  if (M < 0 || N < 0) return DSLPG_ERR_BAD_SHAPE;
  if (!is_float_dtype(x_dtype) || !is_float_dtype(w_dtype)) return DSLPG_ERR_BAD_DTYPE;
  if (!(eps >= 0.f) || !(eps < kPosInf)) return DSLPG_ERR_BAD_EPS;
  if (M == 0 || N == 0) return DSLPG_OK;
  if (!workspace) return DSLPG_ERR_NULL_POINTER;
  const int64_t rb = N * dtype_size(x_dtype);
  return host_rows_pipeline(x_host, y_host, M, rb, rb, workspace, workspace_bytes, stream,
                            [&](void* in, void* out, int64_t rows, cudaStream_t st) {
                              return dslpg_rms_norm_fwd(in, weight, out, rows, N, x_dtype, w_dtype, eps, st);
                            });
}

extern "C" int dslpg_layer_norm_fwd_host_workspace_bytes(int64_t M, int64_t N, int x_dtype, int64_t* bytes) {
  return dslpg_rms_norm_fwd_host_workspace_bytes(M, N, x_dtype, bytes);
}

extern "C" int dslpg_layer_norm_fwd_host(const void* x_host, const void* weight, const void* bias, void* y_host,
                                         int64_t M, int64_t N, int x_dtype, int w_dtype, float eps, void* workspace,
                                         int64_t workspace_bytes, cudaStream_t stream) {
  if (!x_host || !weight || !y_host) return DSLPG_ERR_NULL_POINTER;
  if (M < 0 || N < 0) return DSLPG_ERR_BAD_SHAPE;
  if (!is_float_dtype(x_dtype) || !is_float_dtype(w_dtype)) return DSLPG_ERR_BAD_DTYPE;
  if (!(eps >= 0.f) || !(eps < kPosInf)) return DSLPG_ERR_BAD_EPS;
  if (M == 0 || N == 0) return DSLPG_OK;
  if (!workspace) return DSLPG_ERR_NULL_POINTER;
  const int64_t rb = N * dtype_size(x_dtype);
  return host_rows_pipeline(x_host, y_host, M, rb, rb, workspace, workspace_bytes, stream,
                            [&](void* in, void* out, int64_t rows, cudaStream_t st) {
                              return dslpg_layer_norm_fwd(in, weight, bias, out, rows, N, x_dtype, w_dtype, eps, st);
                            });
}
