// Kernel 3: lazy row-sparse AdamW, and the FP32 -> F16/BF16 cast/export kernel.
//
// Row update semantics: streamtrain/sparse_disk.py:122-138 updates only the
// parameters that received a gradient, each with DiskState.update
// (streamtrain/disk.py:207-215). At row granularity the touched rows of one
// table take that update with the table's clock; untouched rows are neither
// read nor written (no moment decay, no weight decay).
//
// Layout: w, m, v are [rows, cols] FP32 planes; grads is [k, cols] with
// gradient row r belonging to table row idx[r]. One CTA updates one touched
// row per iteration, sweeping it in coalesced passes of 1024 elements, up to
// three passes' loads issued together; the grid is persistent and strides
// over the k touched rows.
#include "mb_common.cuh"

namespace mb {
namespace {

constexpr int kRowPasses = 3;  // 1024-element sweeps of a row loaded together

template <int GDT>
__global__ void __launch_bounds__(kThreads) k_sparse_rows(float* __restrict__ w, float* __restrict__ m,
                                                           float* __restrict__ v, int64_t rows, int64_t cols,
                                                           const int64_t* __restrict__ idx, int64_t k,
                                                           const void* __restrict__ grads, mb_host_scalars hs,
                                                           int32_t* err_flag) {
  StepScalars s;
  s.small = fabsf(hs.omb1) < 0.5f;
  s.lw = s.small ? hs.omb1 : __fsub_rn(hs.omb1, 1.0f);
  s.cwd = hs.cwd; s.b2 = hs.beta2; s.omb2 = hs.omb2; s.eps = hs.eps; s.nss = hs.nss; s.bc2s = hs.bc2s;
  GradPrep prep = make_prep(hs.scale, hs.coef);
  const bool vec = (cols % kQuad) == 0 && aligned(w, 16) && aligned(m, 16) && aligned(v, 16) &&
                   aligned(grads, GDT == MB_F32 ? 16 : 8);
  for (int64_t r = blockIdx.x; r < k; r += gridDim.x) {
    int64_t row = __ldg(&idx[r]);
    if (row < 0 || row >= rows) {
      if (threadIdx.x == 0 && err_flag) atomicExch(err_flag, 1);
      continue;
    }
    float* wr = w + row * cols;
    float* mr = m + row * cols;
    float* vr = v + row * cols;
    int64_t gbase = r * cols;
    if (vec) {
      // up to kRowPasses sweeps of 1024 elements: every load of the batch is issued
      // before any arithmetic (a 3072-wide row is one batch)
      for (int64_t e0 = (int64_t)threadIdx.x * kQuad; e0 < cols; e0 += kRowPasses * kHalf) {
        float4 a[kRowPasses], b[kRowPasses], c[kRowPasses];
        float g[kRowPasses][4];
#pragma unroll
        for (int u = 0; u < kRowPasses; ++u) {
          const int64_t e = e0 + u * kHalf;
          if (e < cols) {  // cols % 4 == 0: a quad is all in or all out
            load4<GDT>(grads, gbase + e, g[u]);
            a[u] = ld4f(wr + e);
            b[u] = ld4f(mr + e);
            c[u] = ld4f(vr + e);
          }
        }
#pragma unroll
        for (int u = 0; u < kRowPasses; ++u) {
          const int64_t e = e0 + u * kHalf;
          if (e >= cols) continue;
          float ww[4] = {a[u].x, a[u].y, a[u].z, a[u].w}, mm[4] = {b[u].x, b[u].y, b[u].z, b[u].w};
          float vv[4] = {c[u].x, c[u].y, c[u].z, c[u].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) adam_elem(ww[j], mm[j], vv[j], prep(g[u][j]), s);
          st4f(wr + e, make_float4(ww[0], ww[1], ww[2], ww[3]));
          st4f(mr + e, make_float4(mm[0], mm[1], mm[2], mm[3]));
          st4f(vr + e, make_float4(vv[0], vv[1], vv[2], vv[3]));
        }
      }
      continue;
    }
    for (int64_t e = (int64_t)threadIdx.x * kQuad; e < cols; e += kHalf) {
      const int64_t end = e + kQuad < cols ? e + kQuad : cols;
      for (int64_t j = e; j < end; ++j) {
        float ww = wr[j], mm = mr[j], vv = vr[j];
        adam_elem(ww, mm, vv, prep(load1<GDT>(grads, gbase + j)), s);
        wr[j] = ww;
        mr[j] = mm;
        vr[j] = vv;
      }
    }
  }
}

// FP32 -> DT cast, round to nearest even; with CHECK, nonfinite or |x| > 65504
// raises *err (export.py:33). The cast is written either way.
template <int DT, bool CHECK>
__global__ void __launch_bounds__(kThreads) k_cast(const float* __restrict__ src, void* __restrict__ dst,
                                                    int64_t n, bool vec, int32_t* err) {
  bool bad = false;
  int64_t stride = (int64_t)gridDim.x * kHalf;
  for (int64_t e = ((int64_t)blockIdx.x * kThreads + threadIdx.x) * kQuad; e < n; e += stride) {
    if (vec && e + kQuad <= n) {
      float4 q = ld4f(src + e);
      float x[4] = {q.x, q.y, q.z, q.w};
      if (CHECK) {
#pragma unroll
        for (int j = 0; j < 4; ++j) bad |= !(fabsf(x[j]) <= 65504.0f);
      }
      store4<DT>(dst, e, x);
    } else {
      int64_t end = e + kQuad < n ? e + kQuad : n;
      for (int64_t j = e; j < end; ++j) {
        float x = src[j];
        if (CHECK) bad |= !(fabsf(x) <= 65504.0f);
        store1<DT>(dst, j, x);
      }
    }
  }
  if (CHECK && __syncthreads_or(bad) && threadIdx.x == 0) atomicExch(err, 1);
}

using RowsFn = void (*)(float*, float*, float*, int64_t, int64_t, const int64_t*, int64_t, const void*,
                        mb_host_scalars, int32_t*);

RowsFn pick_rows(int gdt) {
  switch (gdt) {
    case MB_F32: return &k_sparse_rows<MB_F32>;
    case MB_F16: return &k_sparse_rows<MB_F16>;
    case MB_BF16: return &k_sparse_rows<MB_BF16>;
    default: return nullptr;
  }
}

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" {

MB_API int mb_sparse_rows_update(float* w, float* m, float* v, int64_t rows, int64_t cols,
                                 const int64_t* idx, int64_t k, const void* grads, int32_t gdt,
                                 const mb_host_scalars* s, int32_t* err_flag, mb_stream_t stream) {
  if (!w || !m || !v || !s || rows < 0 || cols <= 0 || k < 0) return MB_ERR_ARG;
  if (k > 0 && (!idx || !grads)) return MB_ERR_ARG;
  RowsFn fn = pick_rows(gdt);
  if (!fn) return MB_ERR_ARG;
  if (k == 0) return MB_OK;
  int grid = grid_for(reinterpret_cast<const void*>(fn), k);
  fn<<<grid, kThreads, 0, (cudaStream_t)stream>>>(w, m, v, rows, cols, idx, k, grads, *s, err_flag);
  return cudaGetLastError() == cudaSuccess ? MB_OK : MB_ERR_CUDA;
}

MB_API int mb_cast_f32(const float* src, void* dst, int32_t dtype, int64_t n, int32_t check,
                       int32_t* err_flag, mb_stream_t stream) {
  if (!src || !dst || n < 0) return MB_ERR_ARG;
  if (check && (dtype != MB_F16 || !err_flag)) return MB_ERR_ARG;
  if (n == 0) return MB_OK;
  bool vec = aligned(src, 16) && aligned(dst, 8);
  const void* fn;
  if (dtype == MB_F16) fn = check ? (const void*)&k_cast<MB_F16, true> : (const void*)&k_cast<MB_F16, false>;
  else if (dtype == MB_BF16) fn = (const void*)&k_cast<MB_BF16, false>;
  else return MB_ERR_ARG;
  int64_t tiles = (n + kHalf - 1) / kHalf;
  int grid = grid_for(fn, tiles);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == MB_F16 && check) k_cast<MB_F16, true><<<grid, kThreads, 0, st>>>(src, dst, n, vec, err_flag);
  else if (dtype == MB_F16) k_cast<MB_F16, false><<<grid, kThreads, 0, st>>>(src, dst, n, vec, err_flag);
  else k_cast<MB_BF16, false><<<grid, kThreads, 0, st>>>(src, dst, n, vec, err_flag);
  return cudaGetLastError() == cudaSuccess ? MB_OK : MB_ERR_CUDA;
}

}  // extern "C"
