// Kernel 5: pinned-host ping-pong for row-sparse AdamW on offloaded state.
//
// Reference: the two reusable device windows + pinned host staging of
// streamtrain/engine.py:60-163 (Slot, h2d/d2h streams, loaded/done/copied
// events; slot reuse waits for the previous DMA, engine.py:111-112) and
// streamtrain/disk.py:287-359, applied to the conditional update of
// streamtrain/sparse_disk.py:122-138 (DiskState.update on the touched rows).
//
// The optimizer state of a [rows, cols] table lives in pinned host memory as
// three FP32 planes w, m, v. One step updates the sorted row list idx[0..k):
//   for window j (rows idx[j*W .. j*W + n)):
//     h2d stream:     wait until window j%2 is free (its previous scatter done);
//                     k_rows_gather pulls the n rows of w, m, v over PCIe
//                     (zero-copy reads of the mapped pinned planes) into the
//                     device window [3][W][cols];
//     compute stream: wait for the gather; kernel 1 updates the window (dense,
//                     3 segments of n*cols) with gradient rows j*W .. j*W + n;
//     d2h stream:     wait for the update; k_rows_scatter writes the rows back
//                     (zero-copy writes).
// Gathers, updates and scatters of different windows run concurrently: PCIe
// carries reads and writes at the same time and the update is HBM-bound and
// short. At the end the compute stream waits for the last scatters, so a
// caller that synchronises the compute stream sees the host state final.
// The events are per device and reused: calls on one device must be issued
// in order from one thread.
#include <chrono>
#include <mutex>
#include <thread>
#include <vector>

#include "mb_common.cuh"

namespace mb {
namespace {

constexpr int kCopyBlocks = 96;  // CTAs per transfer kernel: enough requests in flight for PCIe

// Copy the listed rows of three host planes into the window, or back.
template <bool kToWindow>
__global__ void __launch_bounds__(kThreads) k_rows_copy(float* hw, float* hm, float* hv, int64_t rows, int64_t cols,
                                                         const int64_t* __restrict__ idx, int64_t n, float* win,
                                                         int64_t win_rows, int32_t* err) {
  const bool vec = (cols % 4) == 0 && aligned(hw, 16) && aligned(hm, 16) && aligned(hv, 16) && aligned(win, 16);
  for (int64_t r = blockIdx.x; r < n; r += gridDim.x) {
    const int64_t row = __ldg(&idx[r]);
    if (row < 0 || row >= rows) {
      if (threadIdx.x == 0 && err) atomicExch(err, 1);
      continue;
    }
    float* planes[3] = {hw + row * cols, hm + row * cols, hv + row * cols};
#pragma unroll
    for (int p = 0; p < 3; ++p) {
      float* h = planes[p];
      float* d = win + ((int64_t)p * win_rows + r) * cols;
      if (vec) {
        for (int64_t e = (int64_t)threadIdx.x * 4; e < cols; e += kThreads * 4) {
          if (kToWindow) *reinterpret_cast<float4*>(d + e) = __ldcs(reinterpret_cast<const float4*>(h + e));
          else __stcs(reinterpret_cast<float4*>(h + e), *reinterpret_cast<const float4*>(d + e));
        }
      } else {
        for (int64_t e = threadIdx.x; e < cols; e += kThreads) {
          if (kToWindow) d[e] = h[e];
          else h[e] = d[e];
        }
      }
    }
  }
}

struct Events {
  cudaEvent_t start, gathered[2], updated[2], scattered[2];
  bool ok = false;
};

// One event set per device (created on first use, reused; events are not memory).
Events* events_for_device() {
  static std::mutex mu;
  static std::vector<Events> per_dev(64);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  Events& e = per_dev[dev];
  if (!e.ok) {
    if (cudaEventCreateWithFlags(&e.start, cudaEventDisableTiming) != cudaSuccess) return nullptr;
    for (int b = 0; b < 2; ++b) {
      if (cudaEventCreateWithFlags(&e.gathered[b], cudaEventDisableTiming) != cudaSuccess ||
          cudaEventCreateWithFlags(&e.updated[b], cudaEventDisableTiming) != cudaSuccess ||
          cudaEventCreateWithFlags(&e.scattered[b], cudaEventDisableTiming) != cudaSuccess)
        return nullptr;
    }
    e.ok = true;
  }
  return &e;
}

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" {

MB_API int mb_offload_rows_step(float* host_w, float* host_m, float* host_v, int64_t rows, int64_t cols,
                                const int64_t* idx, int64_t k, const void* grads, int32_t grad_dtype,
                                const mb_host_scalars* s, float* window0, float* window1, int64_t window_rows,
                                mb_stream_t compute, mb_stream_t h2d, mb_stream_t d2h, int32_t* err_flag) {
  if (!host_w || !host_m || !host_v || !s || !window0 || !window1 || rows < 0 || cols <= 0 || k < 0)
    return MB_ERR_ARG;
  if (window_rows <= 0 || (k > 0 && (!idx || !grads))) return MB_ERR_ARG;
  if (grad_dtype < MB_F32 || grad_dtype > MB_BF16) return MB_ERR_ARG;
  if (k == 0) return MB_OK;
  // Device addresses of the mapped pinned planes.
  float *dw = nullptr, *dm = nullptr, *dv = nullptr;
  if (cudaHostGetDevicePointer((void**)&dw, host_w, 0) != cudaSuccess ||
      cudaHostGetDevicePointer((void**)&dm, host_m, 0) != cudaSuccess ||
      cudaHostGetDevicePointer((void**)&dv, host_v, 0) != cudaSuccess)
    return MB_ERR_ARG;  // not pinned, mapped host memory
  Events* ev = events_for_device();
  if (!ev) return MB_ERR_CUDA;
  cudaStream_t sc = (cudaStream_t)compute, sh = (cudaStream_t)h2d, sd = (cudaStream_t)d2h;
  // Nothing may read the grads or indices before the caller's compute-stream
  // work (which also orders this call after the previous call's scatters).
  if (cudaEventRecord(ev->start, sc) != cudaSuccess) return MB_ERR_CUDA;
  if (cudaStreamWaitEvent(sh, ev->start, 0) != cudaSuccess) return MB_ERR_CUDA;
  const int64_t nwin = (k + window_rows - 1) / window_rows;
  const size_t elem = grad_dtype == MB_F32 ? 4 : 2;
  for (int64_t j = 0; j < nwin; ++j) {
    const int b = (int)(j & 1);
    float* win = b ? window1 : window0;
    const int64_t r0 = j * window_rows;
    const int64_t n = k - r0 < window_rows ? k - r0 : window_rows;
    if (j >= 2 && cudaStreamWaitEvent(sh, ev->scattered[b], 0) != cudaSuccess) return MB_ERR_CUDA;
    int blocks = (int)(n < kCopyBlocks ? n : kCopyBlocks);
    k_rows_copy<true><<<blocks, kThreads, 0, sh>>>(dw, dm, dv, rows, cols, idx + r0, n, win, window_rows, err_flag);
    if (cudaGetLastError() != cudaSuccess) return MB_ERR_CUDA;
    if (cudaEventRecord(ev->gathered[b], sh) != cudaSuccess) return MB_ERR_CUDA;
    if (cudaStreamWaitEvent(sc, ev->gathered[b], 0) != cudaSuccess) return MB_ERR_CUDA;
    const int64_t nel = n * cols;
    const char* g = static_cast<const char*>(grads) + (size_t)r0 * cols * elem;
    int rc = mb_adamw_update(win, win + window_rows * cols, win + 2 * window_rows * cols, g, grad_dtype, nullptr,
                             MB_NONE, nel, s, compute);
    if (rc) return rc;
    if (cudaEventRecord(ev->updated[b], sc) != cudaSuccess) return MB_ERR_CUDA;
    if (cudaStreamWaitEvent(sd, ev->updated[b], 0) != cudaSuccess) return MB_ERR_CUDA;
    k_rows_copy<false><<<blocks, kThreads, 0, sd>>>(dw, dm, dv, rows, cols, idx + r0, n, win, window_rows, err_flag);
    if (cudaGetLastError() != cudaSuccess) return MB_ERR_CUDA;
    if (cudaEventRecord(ev->scattered[b], sd) != cudaSuccess) return MB_ERR_CUDA;
  }
  for (int b = 0; b < 2 && b < nwin; ++b)
    if (cudaStreamWaitEvent(sc, ev->scattered[b], 0) != cudaSuccess) return MB_ERR_CUDA;
  return MB_OK;
}

MB_API int mb_stream_wait(mb_stream_t stream, int64_t timeout_us) {
  if (timeout_us < 0) return MB_ERR_ARG;
  const auto t0 = std::chrono::steady_clock::now();
  int64_t pause_us = 1;
  while (true) {
    const cudaError_t q = cudaStreamQuery((cudaStream_t)stream);
    if (q == cudaSuccess) return MB_OK;
    if (q != cudaErrorNotReady) return MB_ERR_CUDA;
    const int64_t waited =
        std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - t0).count();
    if (waited >= timeout_us) return MB_ERR_TIMEOUT;
    std::this_thread::sleep_for(std::chrono::microseconds(pause_us));
    if (pause_us < 200) pause_us *= 2;  // poll densely at first, then every 0.2 ms
  }
}

}  // extern "C"
