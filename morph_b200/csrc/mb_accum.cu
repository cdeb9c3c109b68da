// Device-side microbatch gradient accumulation with the loss-scale division,
// optionally fused with the FP64 norm statistics of the accumulated result.
//
// Reference: streamtrain/sparse_disk.py:82-110 zeroes one FP32 gradient window
// per stage and, for each microbatch, adds value = g.detach().float() /
// loss_scale into it (destination.add_(value)); the norm pass then sums
// piece.double().square() over the accumulated gradient
// (sparse_disk.py:119-120, disk.py:466-468). Here one pass per microbatch does
//   acc = acc + f32(g) / loss_scale        (first microbatch: 0 + f32(g) / loss_scale)
// with IEEE division (a power-of-two scale uses its exact reciprocal, which is
// the same value), and, when a record is given, adds {sum of acc^2 in FP64,
// nonfinite} of the new acc values to it. The statistics reduce through
// per-CTA partials in a fixed order (deterministic), and the last CTA adds the
// call's total into the record.
#include "mb_common.cuh"

namespace mb {
namespace {

constexpr int kAccBlocks = 1024;  // most CTAs (and partials) per call

template <int GDT, bool FIRST, bool STATS>
__global__ void __launch_bounds__(kThreads) k_accumulate(float* __restrict__ acc, const void* __restrict__ g,
                                                          int64_t n, float scale, bool vec, double* partials,
                                                          unsigned int* ticket, double* record) {
  const GradPrep prep = make_prep(scale, 1.0f);
  double ss = 0.0;
  const int64_t stride = (int64_t)gridDim.x * kThreads * kQuad;
  for (int64_t e = ((int64_t)blockIdx.x * kThreads + threadIdx.x) * kQuad; e < n; e += stride) {
    if (vec && e + kQuad <= n) {
      float x[4];
      load4<GDT>(g, e, x);
      float4 a = FIRST ? make_float4(0.f, 0.f, 0.f, 0.f) : *reinterpret_cast<const float4*>(acc + e);
      float r[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        r[j] = __fadd_rn(r[j], prep(x[j]));
        if (STATS) ss = __fma_rn((double)r[j], (double)r[j], ss);
      }
      *reinterpret_cast<float4*>(acc + e) = make_float4(r[0], r[1], r[2], r[3]);
    } else {
      const int64_t end = e + kQuad < n ? e + kQuad : n;
      for (int64_t j = e; j < end; ++j) {
        const float r = __fadd_rn(FIRST ? 0.0f : acc[j], prep(load1<GDT>(g, j)));
        acc[j] = r;
        if (STATS) ss = __fma_rn((double)r, (double)r, ss);
      }
    }
  }
  if constexpr (STATS) {
    __shared__ double red[kThreads / 32];
    __shared__ bool last;
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_down_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      double b = 0.0;
      for (int i = 0; i < kThreads / 32; ++i) b += red[i];
      partials[blockIdx.x] = b;
      __threadfence();
      last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
      __threadfence();
      double t = 0.0;
      for (unsigned i = 0; i < gridDim.x; ++i) t += __ldcg(&partials[i]);
      // squares are >= 0, so the sum is finite exactly when every element is
      record[0] += t;
      record[1] += isfinite(t) ? 0.0 : 1.0;
      *ticket = 0u;
    }
  }
}

template <int GDT>
int launch(float* acc, const void* g, int64_t n, float scale, bool first, double* record, char* ws,
           cudaStream_t s) {
  const bool vec = aligned(acc, 16) && aligned(g, GDT == MB_F32 ? 16 : 8);
  int64_t blocks = (n + (int64_t)kThreads * kQuad * 4 - 1) / ((int64_t)kThreads * kQuad * 4);
  blocks = blocks < 1 ? 1 : (blocks > kAccBlocks ? kAccBlocks : blocks);
  double* partials = reinterpret_cast<double*>(ws);
  unsigned int* ticket = reinterpret_cast<unsigned int*>(ws + sizeof(double) * kAccBlocks);
  const int grid = (int)blocks;
  if (record) {
    if (first) k_accumulate<GDT, true, true><<<grid, kThreads, 0, s>>>(acc, g, n, scale, vec, partials, ticket, record);
    else k_accumulate<GDT, false, true><<<grid, kThreads, 0, s>>>(acc, g, n, scale, vec, partials, ticket, record);
  } else {
    if (first) k_accumulate<GDT, true, false><<<grid, kThreads, 0, s>>>(acc, g, n, scale, vec, nullptr, nullptr, nullptr);
    else k_accumulate<GDT, false, false><<<grid, kThreads, 0, s>>>(acc, g, n, scale, vec, nullptr, nullptr, nullptr);
  }
  return cudaGetLastError() == cudaSuccess ? MB_OK : MB_ERR_CUDA;
}

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" {

MB_API size_t mb_accumulate_workspace_bytes(void) { return sizeof(double) * kAccBlocks + 256; }

MB_API int mb_grad_accumulate(float* acc, const void* g, int32_t grad_dtype, int64_t n, float loss_scale,
                              int32_t first, double* record, void* workspace, mb_stream_t stream) {
  if (!acc || n < 0 || (n > 0 && !g)) return MB_ERR_ARG;
  if (!(loss_scale > 0.0f) || isinf(loss_scale)) return MB_ERR_ARG;
  if (record && !workspace) return MB_ERR_ARG;
  if (workspace && !aligned(workspace, 16)) return MB_ERR_ALIGN;
  if (n == 0) return MB_OK;
  char* ws = static_cast<char*>(workspace);
  cudaStream_t s = (cudaStream_t)stream;
  switch (grad_dtype) {
    case MB_F32: return launch<MB_F32>(acc, g, n, loss_scale, first != 0, record, ws, s);
    case MB_F16: return launch<MB_F16>(acc, g, n, loss_scale, first != 0, record, ws, s);
    case MB_BF16: return launch<MB_BF16>(acc, g, n, loss_scale, first != 0, record, ws, s);
    default: return MB_ERR_ARG;
  }
}

}  // extern "C"
