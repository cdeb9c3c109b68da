// Block-scaled FP8 (E4M3FN) transport: pack and unpack.
//
// Reference: streamtrain/precision.py:24-37, used for the temporary H2D weight
// transport at streamtrain/disk.py:336-349. Per block of 256 elements:
//   scale = max(amax(|x|) / 448, 1e-30)   (FP32 divide, clamp_min)
//   code  = e4m3fn(clamp(x / scale, -448, 448))   (FP32 divide, round to nearest even)
//   value = float(code) * scale, then rounded to the compute dtype.
// A NaN in a block propagates to its scale and every code of the block, as
// torch's amax, clamp and division propagate it. The final partial block is
// padded with zeros, which are not written.
//
// Layout: one warp per 256-element block, 8 consecutive elements per lane
// (two 16-byte loads, one 8-byte store of codes); grid-stride over blocks.
#include <cuda_fp8.h>

#include "mb_common.cuh"

namespace mb {
namespace {

constexpr int kBlock = 256;

__global__ void __launch_bounds__(kThreads) k_fp8_pack(const float* __restrict__ x, int64_t n,
                                                        uint8_t* __restrict__ codes, float* __restrict__ scales,
                                                        bool vec) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (kThreads / 32);
  const int64_t nblocks = (n + kBlock - 1) / kBlock;
  for (int64_t b = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); b < nblocks; b += warps) {
    const int64_t e0 = b * kBlock + lane * 8;
    float v[8];
    if (vec && e0 + 8 <= n) {
      float4 p = __ldcs(reinterpret_cast<const float4*>(x + e0));
      float4 q = __ldcs(reinterpret_cast<const float4*>(x + e0 + 4));
      v[0] = p.x; v[1] = p.y; v[2] = p.z; v[3] = p.w; v[4] = q.x; v[5] = q.y; v[6] = q.z; v[7] = q.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = e0 + j < n ? x[e0 + j] : 0.0f;
    }
    float amax = 0.0f;
    bool nan = false;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      nan |= v[j] != v[j];
      amax = fmaxf(amax, fabsf(v[j]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      nan |= __shfl_xor_sync(0xffffffffu, (int)nan, o) != 0;
    }
    float scale = nan ? __int_as_float(0x7fc00000) : __fdiv_rn(amax, 448.0f);
    if (scale < 1e-30f) scale = 1e-30f;  // clamp_min(1e-30); NaN compares false and stays NaN
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float q = __fdiv_rn(v[j], scale);
      if (q == q) q = fminf(fmaxf(q, -448.0f), 448.0f);
      uint32_t c = (uint32_t)__nv_cvt_float_to_fp8(q, __NV_SATFINITE, __NV_E4M3);
      if (j < 4) lo |= c << (8 * j);
      else hi |= c << (8 * (j - 4));
    }
    if (vec && e0 + 8 <= n) {
      *reinterpret_cast<uint2*>(codes + e0) = make_uint2(lo, hi);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (e0 + j < n) codes[e0 + j] = (uint8_t)((j < 4 ? lo >> (8 * j) : hi >> (8 * (j - 4))) & 0xffu);
    }
    if (lane == 0) scales[b] = scale;
  }
}

template <int DT>
__global__ void __launch_bounds__(kThreads) k_fp8_unpack(const uint8_t* __restrict__ codes,
                                                          const float* __restrict__ scales, int64_t n, void* out) {
  for (int64_t e = (int64_t)blockIdx.x * kThreads + threadIdx.x; e < n; e += (int64_t)gridDim.x * kThreads) {
    __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)codes[e], __NV_E4M3);
    float v = __fmul_rn(__half2float(__half(h)), scales[e / kBlock]);
    store1<DT>(out, e, v);
  }
}

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" {

MB_API int mb_fp8_pack(const float* src, int64_t n, uint8_t* codes, float* scales, mb_stream_t stream) {
  if (n < 0 || (n > 0 && (!src || !codes || !scales))) return MB_ERR_ARG;
  if (n == 0) return MB_OK;
  const bool vec = aligned(src, 16) && aligned(codes, 8);
  const int64_t nblocks = (n + kBlock - 1) / kBlock;
  int64_t grid = (nblocks + kThreads / 32 - 1) / (kThreads / 32);
  int cap = grid_for(reinterpret_cast<const void*>(&k_fp8_pack), grid);
  k_fp8_pack<<<cap, kThreads, 0, (cudaStream_t)stream>>>(src, n, codes, scales, vec);
  return cudaGetLastError() == cudaSuccess ? MB_OK : MB_ERR_CUDA;
}

MB_API int mb_fp8_unpack(const uint8_t* codes, const float* scales, int64_t n, void* out, int32_t out_dtype,
                         mb_stream_t stream) {
  if (n < 0 || (n > 0 && (!codes || !scales || !out))) return MB_ERR_ARG;
  if (n == 0) return MB_OK;
  const void* fn;
  switch (out_dtype) {
    case MB_F32: fn = (const void*)&k_fp8_unpack<MB_F32>; break;
    case MB_F16: fn = (const void*)&k_fp8_unpack<MB_F16>; break;
    case MB_BF16: fn = (const void*)&k_fp8_unpack<MB_BF16>; break;
    default: return MB_ERR_ARG;
  }
  int grid = grid_for(fn, (n + kThreads - 1) / kThreads);
  cudaStream_t s = (cudaStream_t)stream;
  if (out_dtype == MB_F32) k_fp8_unpack<MB_F32><<<grid, kThreads, 0, s>>>(codes, scales, n, out);
  else if (out_dtype == MB_F16) k_fp8_unpack<MB_F16><<<grid, kThreads, 0, s>>>(codes, scales, n, out);
  else k_fp8_unpack<MB_BF16><<<grid, kThreads, 0, s>>>(codes, scales, n, out);
  return cudaGetLastError() == cudaSuccess ? MB_OK : MB_ERR_CUDA;
}

}  // extern "C"
