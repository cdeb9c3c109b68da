// Kernel 4: Muon — momentum, Nesterov blend, Frobenius normalisation,
// Newton-Schulz on the tcgen05 GEMM, and the decoupled-weight-decay update.
//
// Reference (streamtrain/optimizer.py):
//   52-61  momentum.lerp_(g, .05); u = g.lerp(momentum, .95);
//          o = orthogonalize(u); o *= max(1, rows/cols) ** .5;
//          p.mul_(1 - lr*wd).add_(o, alpha=-lr)
//   13-22  orthogonalize: x = u.float(); transpose if rows > cols;
//          x /= (x.norm() + 1e-7); 5 x { A = x x^T; x = a x + (b A + c A A) x }
// The reference runs Newton-Schulz in FP32; here the operands are BF16 with
// FP32 tensor-core accumulation (the published Muon formulation), compared
// against the FP32 reference by relative Frobenius error.
//
// Pipeline for one matrix w [rows, cols], m = min(rows, cols), n = max:
//   k_muon_sumsq     momentum update in place, u = Nesterov blend, FP64 sum
//                    of u^2 (last CTA writes the norm divisor);
//   k_ns_normalize   x = u / (||u|| + 1e-7) in BF16 as X [mp, np] and its
//                    transpose XT [np, mp] (mp, np = m, n rounded up to 256,
//                    zero padding written explicitly), through 32x32 tiles;
//   15 GEMMs         per iteration: A = X X^T; M = a I + b A + c A A (one
//                    FP32 epilogue, rounded once); X' = M X (reads XT, writes
//                    X' and X'^T; the last iteration writes FP32);
//   k_muon_apply     w = fma(o * shape_scale, -lr, w * (1 - lr*wd)) from the
//                    FP32 result, transposing back through a 32x32 tile, with
//                    an optional BF16/FP16 copy of w.
#include "mb_common.cuh"

namespace mb {

int gemm16_nt(int dtype, const void* a, int64_t lda, const void* b, int64_t ldb, int64_t M, int64_t N, int64_t K,
              float alpha, float beta, float diag, const void* c, int64_t ldc, void* d, int64_t ldd, void* dt,
              int64_t lddt, float* df, int64_t lddf, int32_t* err, cudaStream_t stream, bool sym);

namespace {

constexpr int kPad = 256;
constexpr int kStatBlocks = 1024;

inline int64_t pad_to(int64_t x) { return (x + kPad - 1) / kPad * kPad; }
inline size_t up256(size_t x) { return (x + 255) / 256 * 256; }

struct Layout {
  int64_t mp, np;
  size_t stats, x0, x1, t0, t1, a, b, o, total;
};

// Workspace: [FP64 partials + ticket + divisor][X0][X1][XT0][XT1][A][B][O f32].
Layout layout_for(int64_t rows, int64_t cols) {
  Layout L;
  int64_t m = rows < cols ? rows : cols, n = rows < cols ? cols : rows;
  L.mp = pad_to(m);
  L.np = pad_to(n);
  size_t off = 0;
  L.stats = off; off += up256(sizeof(double2) * kStatBlocks + 64);
  L.x0 = off;    off += up256((size_t)L.mp * L.np * 2);
  L.x1 = off;    off += up256((size_t)L.mp * L.np * 2);
  L.t0 = off;    off += up256((size_t)L.mp * L.np * 2);
  L.t1 = off;    off += up256((size_t)L.mp * L.np * 2);
  L.a = off;     off += up256((size_t)L.mp * L.mp * 2);
  L.b = off;     off += up256((size_t)L.mp * L.mp * 2);
  L.o = off;     off += up256((size_t)L.mp * L.np * 4);
  L.total = off;
  return L;
}

struct MuonIn {
  float* mom;          // momentum, updated in place (null: u is read from `u32`)
  const void* g;       // gradient (MB_F32 / MB_F16 / MB_BF16)
  int gdt;
  const float* u32;    // FP32 input when mom == null
  float beta_lerp;     // .05
  float nesterov;      // .95
};

// Nesterov input of element e (also writes the updated momentum when `write`).
template <int GDT>
__device__ __forceinline__ float muon_u(const MuonIn& in, int64_t e, bool write) {
  if (in.mom == nullptr) return in.u32[e];
  float g = load1<GDT>(in.g, e);
  float mo = in.mom[e];
  if (write) {
    // momentum.lerp_(g, .05): small weight, fma(w, g - m, m)
    mo = __fmaf_rn(in.beta_lerp, __fsub_rn(g, mo), mo);
    in.mom[e] = mo;
  }
  // g.lerp(momentum, .95): large weight, fma(w - 1, m - g, m)
  return __fmaf_rn(__fsub_rn(in.nesterov, 1.0f), __fsub_rn(mo, g), mo);
}

template <int GDT>
__global__ void __launch_bounds__(kThreads) k_muon_sumsq(MuonIn in, int64_t total, double2* partials,
                                                          unsigned int* ticket, float* divisor) {
  double acc = 0.0;
  for (int64_t e = (int64_t)blockIdx.x * kThreads + threadIdx.x; e < total; e += (int64_t)gridDim.x * kThreads) {
    float u = muon_u<GDT>(in, e, true);
    acc = __fma_rn((double)u, (double)u, acc);
  }
  // block reduce
  __shared__ double red[kThreads / 32];
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  __shared__ unsigned int s_last;
  if (threadIdx.x == 0) {
    double b = 0.0;
    for (int i = 0; i < kThreads / 32; ++i) b += red[i];
    partials[blockIdx.x] = make_double2(b, 0.0);
    __threadfence();
    s_last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    __threadfence();
    double t = 0.0;
    for (unsigned i = 0; i < gridDim.x; ++i) t += __ldcg(&partials[i]).x;
    // x.norm() + 1e-7 in float (optimizer.py:18)
    *divisor = __fadd_rn(__double2float_rn(sqrt(t)), 1e-7f);
    *ticket = 0u;
  }
}

// Writes X [mp, np] and XT [np, mp] (16-bit, type OUT) from prescale * u /
// divisor, zero outside the valid m x n block. The grid covers the padded X in
// 32x32 tiles. `prescale` is a power of two (exact); it lifts the first
// iterate's elements (RMS 1/sqrt(m n)) toward their converged size
// (1/sqrt(n)) so FP16 operands stay out of the subnormal range, and the first
// iteration's GEMMs divide it back out exactly.
template <int GDT, int OUT>
__global__ void __launch_bounds__(1024) k_ns_normalize(MuonIn in, int64_t rows, int64_t cols, bool tall,
                                                       int64_t mp, int64_t np, const float* divisor, float prescale,
                                                       void* Xv, void* XTv) {
  using T = typename Elem<OUT>::T;
  T* X = static_cast<T*>(Xv);
  T* XT = static_cast<T*>(XTv);
  __shared__ float tile[32][33];
  const float d = *divisor;
  const int64_t m = tall ? cols : rows, n = tall ? rows : cols;
  const int64_t xi0 = (int64_t)blockIdx.y * 32, xj0 = (int64_t)blockIdx.x * 32;  // X tile origin
  const int tx = threadIdx.x, ty = threadIdx.y;
  // X[i][j] = x(u) where u index is (i, j) for wide and (j, i) for tall.
  float val = 0.0f;
  {
    const int64_t i = xi0 + ty, j = xj0 + tx;
    if (i < m && j < n) {
      int64_t e = tall ? j * cols + i : i * cols + j;
      val = __fmul_rn(__fdiv_rn(muon_u<GDT>(in, e, false), d), prescale);
    }
  }
  X[(xi0 + ty) * np + xj0 + tx] = from_f32<OUT>(val);
  tile[ty][tx] = val;
  __syncthreads();
  // XT[j][i] = X[i][j]: thread (ty, tx) writes XT[xj0 + ty][xi0 + tx]
  XT[(xj0 + ty) * mp + xi0 + tx] = from_f32<OUT>(tile[tx][ty]);
}

struct ApplyIn {
  float* w;
  void* out;
  int odt;
  const float* O;  // [mp, np] FP32
  int64_t rows, cols, np;
  bool tall;
  float shape_scale, cwd, neg_lr;
};

// w[r][c] = fma(o * shape_scale, -lr, w * cwd), o = O[r][c] (wide) or O[c][r] (tall).
__global__ void __launch_bounds__(1024) k_muon_apply(ApplyIn a) {
  __shared__ float tile[32][33];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;  // w tile origin
  float o;
  if (a.tall) {
    // O tile rows are w columns: load O[c0 + ty][r0 + tx] coalesced, read transposed.
    const int64_t oc = c0 + ty, orr = r0 + tx;
    tile[ty][tx] = (oc < a.cols && orr < a.rows) ? a.O[oc * a.np + orr] : 0.0f;
    __syncthreads();
    o = tile[tx][ty];
  } else {
    const int64_t r = r0 + ty, c = c0 + tx;
    o = (r < a.rows && c < a.cols) ? a.O[r * a.np + c] : 0.0f;
  }
  const int64_t r = r0 + ty, c = c0 + tx;
  if (r < a.rows && c < a.cols) {
    const int64_t e = r * a.cols + c;
    float u = __fmul_rn(o, a.shape_scale);
    float w = __fmaf_rn(u, a.neg_lr, __fmul_rn(a.w[e], a.cwd));
    a.w[e] = w;
    if (a.odt == MB_BF16) static_cast<__nv_bfloat16*>(a.out)[e] = __float2bfloat16_rn(w);
    else if (a.odt == MB_F16) static_cast<__half*>(a.out)[e] = __float2half_rn(w);
  }
}

// FP32 result in the input's orientation (orthogonalize's return value).
__global__ void __launch_bounds__(1024) k_ns_output(const float* O, float* out, int64_t rows, int64_t cols,
                                                    int64_t np, bool tall) {
  __shared__ float tile[32][33];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
  float o;
  if (tall) {
    const int64_t oc = c0 + ty, orr = r0 + tx;
    tile[ty][tx] = (oc < cols && orr < rows) ? O[oc * np + orr] : 0.0f;
    __syncthreads();
    o = tile[tx][ty];
  } else {
    const int64_t r = r0 + ty, c = c0 + tx;
    o = (r < rows && c < cols) ? O[r * np + c] : 0.0f;
  }
  const int64_t r = r0 + ty, c = c0 + tx;
  if (r < rows && c < cols) out[r * cols + c] = o;
}

template <typename K>
void launch_sumsq(K kern, const MuonIn& in, int64_t total, char* ws, const Layout& L, cudaStream_t s, int* grid) {
  int64_t blocks = (total + kThreads - 1) / kThreads;
  if (blocks > kStatBlocks) blocks = kStatBlocks;
  if (blocks < 1) blocks = 1;
  *grid = (int)blocks;
  double2* partials = reinterpret_cast<double2*>(ws + L.stats);
  unsigned int* ticket = reinterpret_cast<unsigned int*>(ws + L.stats + sizeof(double2) * kStatBlocks);
  float* divisor = reinterpret_cast<float*>(ws + L.stats + sizeof(double2) * kStatBlocks + 16);
  kern<<<(int)blocks, kThreads, 0, s>>>(in, total, partials, ticket, divisor);
}

// Power of two nearest below sqrt(m): the first iterate's prescale.
float prescale_for(int64_t m) {
  int k = 0;
  while ((int64_t)1 << (2 * (k + 1)) <= m) ++k;
  return (float)(1 << k);
}

template <int GDT, int OUT>
void launch_normalize(const MuonIn& in, int64_t rows, int64_t cols, const Layout& L, const float* divisor,
                      float prescale, void* X, void* XT, cudaStream_t s) {
  dim3 blk(32, 32), grd((unsigned)(L.np / 32), (unsigned)(L.mp / 32));
  k_ns_normalize<GDT, OUT><<<grd, blk, 0, s>>>(in, rows, cols, rows > cols, L.mp, L.np, divisor, prescale, X, XT);
}

template <int GDT>
void launch_normalize_any(int out, const MuonIn& in, int64_t rows, int64_t cols, const Layout& L, const float* d,
                          float ps, void* X, void* XT, cudaStream_t s) {
  if (out == MB_F16) launch_normalize<GDT, MB_F16>(in, rows, cols, L, d, ps, X, XT, s);
  else launch_normalize<GDT, MB_BF16>(in, rows, cols, L, d, ps, X, XT, s);
}

// Normalise + Newton-Schulz iterations on `dtype` (MB_BF16 or MB_F16)
// operands; leaves the FP32 result in O.
int ns_core(const MuonIn& in, int64_t rows, int64_t cols, int steps, const float* coeffs, int dtype, char* ws,
            const Layout& L, int32_t* err, cudaStream_t s) {
  if (dtype != MB_BF16 && dtype != MB_F16) return MB_ERR_ARG;
  if (steps <= 0) return MB_ERR_ARG;
  const int64_t total = rows * cols;
  int grid = 0;
  switch (in.gdt) {
    case MB_F32: launch_sumsq(k_muon_sumsq<MB_F32>, in, total, ws, L, s, &grid); break;
    case MB_F16: launch_sumsq(k_muon_sumsq<MB_F16>, in, total, ws, L, s, &grid); break;
    case MB_BF16: launch_sumsq(k_muon_sumsq<MB_BF16>, in, total, ws, L, s, &grid); break;
    default: return MB_ERR_ARG;
  }
  if (cudaGetLastError() != cudaSuccess) return MB_ERR_CUDA;
  const float* divisor = reinterpret_cast<const float*>(ws + L.stats + sizeof(double2) * kStatBlocks + 16);
  void* X0 = ws + L.x0;
  void* X1 = ws + L.x1;
  void* T0 = ws + L.t0;
  void* T1 = ws + L.t1;
  void* A = ws + L.a;
  void* B = ws + L.b;
  float* O = reinterpret_cast<float*>(ws + L.o);
  const int64_t m = rows < cols ? rows : cols;
  const float ps = prescale_for(m);
  switch (in.gdt) {
    case MB_F32: launch_normalize_any<MB_F32>(dtype, in, rows, cols, L, divisor, ps, X0, T0, s); break;
    case MB_F16: launch_normalize_any<MB_F16>(dtype, in, rows, cols, L, divisor, ps, X0, T0, s); break;
    default: launch_normalize_any<MB_BF16>(dtype, in, rows, cols, L, divisor, ps, X0, T0, s); break;
  }
  if (cudaGetLastError() != cudaSuccess) return MB_ERR_CUDA;
  const float a = coeffs[0], b = coeffs[1], c = coeffs[2];
  void *X = X0, *XT = T0, *Xn = X1, *XTn = T1;
  for (int it = 0; it < steps; ++it) {
    const bool last = it == steps - 1;
    // the first iterate carries the prescale: undo it exactly in the FP32 epilogues
    const float s1 = it == 0 ? 1.0f / ps : 1.0f;
    // A = X X^T (symmetric: upper tiles only, lower triangle by transposition)
    int rc = gemm16_nt(dtype, X, L.np, X, L.np, L.mp, L.mp, L.np, s1 * s1, 0.0f, 0.0f, nullptr, 0, A, L.mp, A,
                       L.mp, nullptr, 0, err, s, true);
    if (rc) return rc;
    // M = a I + b A + c A A, formed in FP32 and rounded once: the reference's
    // a X + (b A + c A A) X would add two nearly cancelling products.
    rc = gemm16_nt(dtype, A, L.mp, A, L.mp, L.mp, L.mp, L.mp, c, b, a, A, L.mp, B, L.mp, B, L.mp, nullptr, 0, err,
                   s, true);
    if (rc) return rc;
    // X' = M X (reads X^T as the K-major operand; writes X' and X'^T, or FP32 at the end)
    rc = gemm16_nt(dtype, B, L.mp, XT, L.mp, L.mp, L.np, L.mp, s1, 0.0f, 0.0f, nullptr, 0, last ? nullptr : Xn, L.np,
                   last ? nullptr : XTn, L.mp, last ? O : nullptr, L.np, err, s, false);
    if (rc) return rc;
    void* t = X; X = Xn; Xn = t;
    t = XT; XT = XTn; XTn = t;
  }
  return MB_OK;
}

int check_dims(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return MB_ERR_ARG;
  int64_t m = rows < cols ? rows : cols, n = rows < cols ? cols : rows;
  if (pad_to(m) > (1 << 16) || pad_to(n) > (1 << 20)) return MB_ERR_ARG;
  return MB_OK;
}

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" {

MB_API size_t mb_muon_workspace_bytes(int64_t rows, int64_t cols) {
  if (check_dims(rows, cols)) return 0;
  return layout_for(rows, cols).total;
}

MB_API int mb_newton_schulz(const float* x, int64_t rows, int64_t cols, int32_t steps, const float* coeffs,
                            int32_t ns_dtype, float* out, void* workspace, size_t workspace_bytes,
                            int32_t* err_flag, mb_stream_t stream) {
  if (!x || !out || !coeffs || !workspace || steps <= 0) return MB_ERR_ARG;
  int rc = check_dims(rows, cols);
  if (rc) return rc;
  Layout L = layout_for(rows, cols);
  if (workspace_bytes < L.total) return MB_ERR_ARG;
  if (!aligned(workspace, 256)) return MB_ERR_ALIGN;
  cudaStream_t s = (cudaStream_t)stream;
  char* ws = static_cast<char*>(workspace);
  if (cudaMemsetAsync(ws + L.stats, 0, up256(sizeof(double2) * kStatBlocks + 64), s) != cudaSuccess) return MB_ERR_CUDA;
  MuonIn in{nullptr, nullptr, MB_F32, x, 0.0f, 0.0f};
  rc = ns_core(in, rows, cols, steps, coeffs, ns_dtype, ws, L, err_flag, s);
  if (rc) return rc;
  dim3 blk(32, 32), grd((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32));
  k_ns_output<<<grd, blk, 0, s>>>(reinterpret_cast<const float*>(ws + L.o), out, rows, cols, L.np, rows > cols);
  return cudaGetLastError() == cudaSuccess ? MB_OK : MB_ERR_CUDA;
}

MB_API int mb_muon_step(float* w, float* momentum, const void* g, int32_t grad_dtype, void* out, int32_t out_dtype,
                        int64_t rows, int64_t cols, const mb_muon_args* args, void* workspace,
                        size_t workspace_bytes, int32_t* err_flag, mb_stream_t stream) {
  if (!w || !momentum || !g || !args || !workspace) return MB_ERR_ARG;
  if (grad_dtype < MB_F32 || grad_dtype > MB_BF16) return MB_ERR_ARG;
  if (out_dtype != MB_NONE && out_dtype != MB_F16 && out_dtype != MB_BF16) return MB_ERR_ARG;
  if (out_dtype != MB_NONE && !out) return MB_ERR_ARG;
  if (args->ns_steps <= 0) return MB_ERR_ARG;
  int rc = check_dims(rows, cols);
  if (rc) return rc;
  Layout L = layout_for(rows, cols);
  if (workspace_bytes < L.total) return MB_ERR_ARG;
  if (!aligned(workspace, 256)) return MB_ERR_ALIGN;
  cudaStream_t s = (cudaStream_t)stream;
  char* ws = static_cast<char*>(workspace);
  if (cudaMemsetAsync(ws + L.stats, 0, up256(sizeof(double2) * kStatBlocks + 64), s) != cudaSuccess) return MB_ERR_CUDA;
  MuonIn in{momentum, g, grad_dtype, nullptr, args->beta_lerp, args->nesterov};
  const float coeffs[3] = {args->ns_a, args->ns_b, args->ns_c};
  rc = ns_core(in, rows, cols, args->ns_steps, coeffs, args->ns_dtype, ws, L, err_flag, s);
  if (rc) return rc;
  ApplyIn ap{w, out, out_dtype, reinterpret_cast<const float*>(ws + L.o), rows, cols, L.np, rows > cols,
             args->shape_scale, args->cwd, args->neg_lr};
  dim3 blk(32, 32), grd((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32));
  k_muon_apply<<<grd, blk, 0, s>>>(ap);
  return cudaGetLastError() == cudaSuccess ? MB_OK : MB_ERR_CUDA;
}

}  // extern "C"
