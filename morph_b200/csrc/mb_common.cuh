// Shared device helpers for the morph_b200 kernels (sm_100a).
//
// Every arithmetic step of the reference-ordered expressions uses an explicit
// IEEE intrinsic (__fmul_rn, __fadd_rn, __fdiv_rn, __fsqrt_rn, __fmaf_rn) so
// that nvcc never contracts or reassociates them: the kernels reproduce the
// reference's float32 rounding sequence operation by operation.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/morph_b200.h"

namespace mb {

constexpr int kThreads = 256;          // threads per CTA of the streaming kernels
constexpr int kQuad = 4;               // elements per vector access (one float4)
constexpr int kHalf = kThreads * kQuad;// 1024 elements: one coalesced sweep of a CTA
constexpr int kTile = 2 * kHalf;       // 2048 elements per tile (two sweeps)
constexpr int kMaxStatsBlocks = 4096;  // capacity of the per-block partials

// Workspace layout (device): [partials: kMaxStatsBlocks x double2][ticket:
// 16 B][segment scalars: n_segs x float2], each region 256-byte aligned.
constexpr size_t kPartialsBytes = sizeof(double2) * kMaxStatsBlocks;
constexpr size_t kTicketOffset = kPartialsBytes;
constexpr size_t kSegScalOffset = kPartialsBytes + 256;

inline size_t workspace_bytes(int n_segs) {
  size_t seg = sizeof(float2) * (size_t)(n_segs > 0 ? n_segs : 1);
  return kSegScalOffset + ((seg + 255) / 256) * 256;
}

// ------------------------------------------------------------ conversions --
template <int DT> struct Elem;
template <> struct Elem<MB_F32> { using T = float; };
template <> struct Elem<MB_F16> { using T = __half; };
template <> struct Elem<MB_BF16> { using T = __nv_bfloat16; };

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

template <int DT> __device__ __forceinline__ typename Elem<DT>::T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<MB_F32>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<MB_F16>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<MB_BF16>(float x) {
  return __float2bfloat16_rn(x);
}

// Load 4 consecutive gradient elements starting at element e as floats.
template <int DT> __device__ __forceinline__ void load4(const void* p, int64_t e, float (&x)[4]);
template <> __device__ __forceinline__ void load4<MB_F32>(const void* p, int64_t e, float (&x)[4]) {
  float4 q = __ldcs(reinterpret_cast<const float4*>(static_cast<const float*>(p) + e));
  x[0] = q.x; x[1] = q.y; x[2] = q.z; x[3] = q.w;
}
template <> __device__ __forceinline__ void load4<MB_F16>(const void* p, int64_t e, float (&x)[4]) {
  uint2 q = __ldcs(reinterpret_cast<const uint2*>(static_cast<const __half*>(p) + e));
  __half2 a = *reinterpret_cast<__half2*>(&q.x), b = *reinterpret_cast<__half2*>(&q.y);
  float2 fa = __half22float2(a), fb = __half22float2(b);
  x[0] = fa.x; x[1] = fa.y; x[2] = fb.x; x[3] = fb.y;
}
template <> __device__ __forceinline__ void load4<MB_BF16>(const void* p, int64_t e, float (&x)[4]) {
  uint2 q = __ldcs(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(p) + e));
  x[0] = __uint_as_float(q.x << 16); x[1] = __uint_as_float(q.x & 0xffff0000u);
  x[2] = __uint_as_float(q.y << 16); x[3] = __uint_as_float(q.y & 0xffff0000u);
}

// The same 4 elements from any address space (plain loads; for shared memory,
// which the global-only streaming loads above cannot address).
template <int DT> __device__ __forceinline__ void load4_any(const void* p, int64_t e, float (&x)[4]);
template <> __device__ __forceinline__ void load4_any<MB_F32>(const void* p, int64_t e, float (&x)[4]) {
  float4 q = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + e);
  x[0] = q.x; x[1] = q.y; x[2] = q.z; x[3] = q.w;
}
template <> __device__ __forceinline__ void load4_any<MB_F16>(const void* p, int64_t e, float (&x)[4]) {
  uint2 q = *reinterpret_cast<const uint2*>(static_cast<const __half*>(p) + e);
  __half2 a = *reinterpret_cast<__half2*>(&q.x), b = *reinterpret_cast<__half2*>(&q.y);
  float2 fa = __half22float2(a), fb = __half22float2(b);
  x[0] = fa.x; x[1] = fa.y; x[2] = fb.x; x[3] = fb.y;
}
template <> __device__ __forceinline__ void load4_any<MB_BF16>(const void* p, int64_t e, float (&x)[4]) {
  uint2 q = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(p) + e);
  x[0] = __uint_as_float(q.x << 16); x[1] = __uint_as_float(q.x & 0xffff0000u);
  x[2] = __uint_as_float(q.y << 16); x[3] = __uint_as_float(q.y & 0xffff0000u);
}

template <int DT> __device__ __forceinline__ float load1(const void* p, int64_t e) {
  return to_f32(static_cast<const typename Elem<DT>::T*>(p)[e]);
}

// Store 4 consecutive floats at element e, converted to DT.
template <int DT> __device__ __forceinline__ void store4(void* p, int64_t e, const float (&x)[4]);
template <> __device__ __forceinline__ void store4<MB_F32>(void* p, int64_t e, const float (&x)[4]) {
  __stcs(reinterpret_cast<float4*>(static_cast<float*>(p) + e), make_float4(x[0], x[1], x[2], x[3]));
}
template <> __device__ __forceinline__ void store4<MB_F16>(void* p, int64_t e, const float (&x)[4]) {
  __half2 a = __floats2half2_rn(x[0], x[1]), b = __floats2half2_rn(x[2], x[3]);
  uint2 q;
  q.x = *reinterpret_cast<uint32_t*>(&a);
  q.y = *reinterpret_cast<uint32_t*>(&b);
  __stcs(reinterpret_cast<uint2*>(static_cast<__half*>(p) + e), q);
}
template <> __device__ __forceinline__ void store4<MB_BF16>(void* p, int64_t e, const float (&x)[4]) {
  __nv_bfloat162 a = __floats2bfloat162_rn(x[0], x[1]), b = __floats2bfloat162_rn(x[2], x[3]);
  uint2 q;
  q.x = *reinterpret_cast<uint32_t*>(&a);
  q.y = *reinterpret_cast<uint32_t*>(&b);
  __stcs(reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p) + e), q);
}

template <int DT> __device__ __forceinline__ void store1(void* p, int64_t e, float x) {
  static_cast<typename Elem<DT>::T*>(p)[e] = from_f32<DT>(x);
}

// Compile-time tuning knobs for the streaming state accesses of kernels 1 and 3:
// MB_LD_MODE 0 = ld.global.cs (evict-first), 1 = ld.global.nc (read-only
// path), 2 = plain ld; MB_ST_MODE 0 = st.global.cs, 1 = plain st.
#ifndef MB_LD_MODE
#define MB_LD_MODE 0
#endif
#ifndef MB_ST_MODE
#define MB_ST_MODE 0
#endif

__device__ __forceinline__ float4 ld4f(const float* p) {
#if MB_LD_MODE == 0
  return __ldcs(reinterpret_cast<const float4*>(p));
#elif MB_LD_MODE == 1
  return __ldg(reinterpret_cast<const float4*>(p));
#else
  return *reinterpret_cast<const float4*>(p);
#endif
}
__device__ __forceinline__ void st4f(float* p, float4 v) {
#if MB_ST_MODE == 0
  __stcs(reinterpret_cast<float4*>(p), v);
#else
  *reinterpret_cast<float4*>(p) = v;
#endif
}

// ------------------------------------------------------------- arithmetic --

// Scalars of one AdamW step (see mb_group / mb_host_scalars).
struct StepScalars {
  float cwd, lw, b2, omb2, bc2s, eps, nss;
  bool small;  // |omb1| < 0.5: lerp base is the start value
};

// Gradient preparation: g' = (g / scale) * coef. When scale is a power of two,
// the quotient equals the product with its exact reciprocal, so `inv` is used.
struct GradPrep {
  float scale, inv, coef;
  bool div, pow2, mul;
  __device__ __forceinline__ float operator()(float x) const {
    if (div) x = pow2 ? __fmul_rn(x, inv) : __fdiv_rn(x, scale);
    if (mul) x = __fmul_rn(x, coef);
    return x;
  }
};

__device__ __forceinline__ GradPrep make_prep(float scale, float coef) {
  GradPrep p;
  p.scale = scale;
  p.coef = coef;
  p.div = scale != 1.0f;
  p.mul = coef != 1.0f;
  // A normal power of two has a zero mantissa; its reciprocal 2^-k is exact
  // when the mirrored exponent field stays normal.
  uint32_t bits = __float_as_uint(scale);
  uint32_t ebits = (bits >> 23) & 0xffu;
  p.pow2 = (bits >> 31) == 0 && (bits & 0x7fffffu) == 0 && ebits >= 1 && ebits <= 253;
  p.inv = p.pow2 ? __uint_as_float((254u - ebits) << 23) : 1.0f;
  return p;
}

// torch AdamW element update (decoupled weight decay), ATen CPU op order:
//   w *= cwd; m = lerp(m, g, omb1) as fma(coeff, g - m, base);
//   v = fma(omb2 * g, g, v * b2); d = sqrt(v) / bc2s + eps; w += (nss * m) / d
__device__ __forceinline__ void adam_elem(float& w, float& m, float& v, float g, const StepScalars& s) {
  float wi = __fmul_rn(w, s.cwd);
  float mi = __fmaf_rn(s.lw, __fsub_rn(g, m), s.small ? m : g);
  float vi = __fmaf_rn(__fmul_rn(s.omb2, g), g, __fmul_rn(v, s.b2));
  float d = __fadd_rn(__fdiv_rn(__fsqrt_rn(vi), s.bc2s), s.eps);
  w = __fadd_rn(wi, __fdiv_rn(__fmul_rn(s.nss, mi), d));
  m = mi;
  v = vi;
}

__device__ __forceinline__ bool is_finite(float x) { return (__float_as_uint(x) & 0x7f800000u) != 0x7f800000u; }

__host__ __device__ __forceinline__ bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

// Segment lookup: largest s with segs[s].tile_begin <= tile (segments sorted).
__device__ __forceinline__ int find_segment(const mb_segment* segs, int n, int64_t tile) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (__ldg(&segs[mid].tile_begin) <= tile) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Matrices one batched Muon / GEMM launch covers (pointer tables travel as
// kernel parameters).
constexpr int kMaxBatch = 64;

// One (possibly batched) launch of kernel 4's tcgen05 GEMM:
//   out[b] = alpha * A[b] . B[b]^T + beta * C[b] + diag * I   for b < batch,
// A[b] at a + b*sa, etc. (element strides); see mb_gemm.cu.
struct GemmCall {
  int dtype;  // MB_BF16 or MB_F16 operands and 16-bit outputs
  const void* a;
  int64_t lda, sa;
  const void* b;
  int64_t ldb, sb;
  int64_t M, N, K;
  int batch;
  float alpha, beta, diag;
  const void* c;
  int64_t ldc, sc;
  void* d;
  int64_t ldd, sd;
  void* dt;
  int64_t lddt, sdt;
  float* df;
  int64_t lddf, sdf;
  bool sym;
  float* const* upd_w;  // fused Muon update: host array of `batch` w pointers (or null)
  void* const* upd_out; // host array of `batch` copy pointers (or null)
  int upd_odt;
  bool upd_tall;
  int64_t upd_m, upd_n, upd_cols;
  float upd_scale, upd_cwd, upd_neglr;
  int32_t* err;
  const int32_t* skip;  // optional device flag: nonzero = the launch returns at once
  int max_sms = 0;      // 0: persistent grid over every SM; else at most this many SMs
};
int gemm16(const GemmCall& call, cudaStream_t stream);

// Test-only fault injection (mb_debug_arm_fault): the next launch of the named
// kernel in this process takes the armed plan; every other launch gets
// {unit -1, the default wait bound}.
enum { kFaultApply = 1, kFaultStats = 2, kFaultGemm = 4 };
void take_fault(int kernel, int64_t* unit, uint64_t* limit_ns);

// Host-side validation of a fused AdamW plan and of finalize options (MB_OK or
// the status the entry points return).
int check_plan(const mb_adamw_plan* p);
int check_fin(const mb_finalize_opts* f);

// Number of CTAs a persistent streaming kernel launches on the current device.
int persistent_blocks(const void* kernel, int threads, size_t smem);
// Persistent grid for `fn` (kThreads threads), capped at n_tiles; cached per device.
int grid_for(const void* fn, int64_t n_tiles);

}  // namespace mb
