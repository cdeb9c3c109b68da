// FP16 export cast with the representability check, written straight into
// pinned host memory (the device side of streamtrain/export.py:30-35).
//
// The reference walks each FP32 master in chunks of chunk_elements, raises
// ValueError('weights cannot be represented by finite FP16') on the first chunk
// holding a nonfinite value or |x| > 65504 (after writing the chunks before
// it), and writes value.astype('<f2') (round to nearest even, subnormals kept).
// k_export_f16 converts one staging chunk, storing the FP16 values through the
// device mapping of a pinned host buffer (or into device memory), and lowers
// *first_bad (device memory) to the index of the first offending element, so
// the host can write exactly the reference's good prefix before raising.
#include "mb_common.cuh"

namespace mb {
namespace {

__global__ void __launch_bounds__(kThreads) k_export_f16(const float* __restrict__ src, int64_t n,
                                                          __half* __restrict__ dst, bool vec,
                                                          unsigned long long* first_bad) {
  unsigned long long bad = ~0ull;
  const int64_t stride = (int64_t)gridDim.x * kThreads * kQuad;
  for (int64_t e = ((int64_t)blockIdx.x * kThreads + threadIdx.x) * kQuad; e < n; e += stride) {
    if (vec && e + kQuad <= n) {
      float4 q = __ldcs(reinterpret_cast<const float4*>(src + e));
      float x[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int j = 3; j >= 0; --j)
        if (!(fabsf(x[j]) <= 65504.0f)) bad = (unsigned long long)(e + j);
      __half2 lo = __halves2half2(__float2half_rn(x[0]), __float2half_rn(x[1]));
      __half2 hi = __halves2half2(__float2half_rn(x[2]), __float2half_rn(x[3]));
      uint2 pk = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
      *reinterpret_cast<uint2*>(dst + e) = pk;
    } else {
      const int64_t end = e + kQuad < n ? e + kQuad : n;
      for (int64_t j = end - 1; j >= e; --j) {
        const float x = src[j];
        if (!(fabsf(x) <= 65504.0f)) bad = (unsigned long long)j;
        dst[j] = __float2half_rn(x);
      }
    }
    if (bad != ~0ull) break;  // later elements of this thread cannot be earlier
  }
  // block minimum, then one atomic per block that saw a bad value
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long other = __shfl_down_sync(0xffffffffu, bad, o);
    bad = other < bad ? other : bad;
  }
  __shared__ unsigned long long red[kThreads / 32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = bad;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = red[0];
    for (int i = 1; i < kThreads / 32; ++i) b = red[i] < b ? red[i] : b;
    if (b != ~0ull) atomicMin(first_bad, b);
  }
}

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" {

MB_API int mb_export_f16(const float* src, int64_t n, void* dst, uint64_t* first_bad, mb_stream_t stream) {
  if (!src || !dst || !first_bad || n < 0) return MB_ERR_ARG;
  if (n == 0) return MB_OK;
  // A pinned host buffer is written through its device mapping.
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, dst) != cudaSuccess) return MB_ERR_ARG;
  void* ddst = dst;
  if (attr.type == cudaMemoryTypeHost) {
    if (!attr.devicePointer) return MB_ERR_ARG;
    ddst = attr.devicePointer;
  } else if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) {
    return MB_ERR_ARG;  // pageable host memory cannot be written by the device
  }
  cudaPointerAttributes fattr;
  if (cudaPointerGetAttributes(&fattr, first_bad) != cudaSuccess || fattr.type != cudaMemoryTypeDevice)
    return MB_ERR_ARG;
  const bool vec = aligned(src, 16) && aligned(ddst, 8);
  int64_t blocks = (n + (int64_t)kThreads * kQuad * 4 - 1) / ((int64_t)kThreads * kQuad * 4);
  int grid = grid_for((const void*)&k_export_f16, blocks);
  k_export_f16<<<grid, kThreads, 0, (cudaStream_t)stream>>>(src, n, static_cast<__half*>(ddst), vec,
                                                             reinterpret_cast<unsigned long long*>(first_bad));
  return cudaGetLastError() == cudaSuccess ? MB_OK : MB_ERR_CUDA;
}

}  // extern "C"
