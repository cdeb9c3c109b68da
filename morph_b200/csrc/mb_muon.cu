// Kernel 4: Muon — momentum, Nesterov blend, Frobenius normalisation,
// Newton-Schulz on the tcgen05 GEMM, and the decoupled-weight-decay update.
//
// Reference (streamtrain/optimizer.py):
//   52-61  momentum.lerp_(g, .05); u = g.lerp(momentum, .95);
//          o = orthogonalize(u); o *= max(1, rows/cols) ** .5;
//          p.mul_(1 - lr*wd).add_(o, alpha=-lr)
//   13-22  orthogonalize: x = u.float(); transpose if rows > cols;
//          x /= (x.norm() + 1e-7); 5 x { A = x x^T; x = a x + (b A + c A A) x }
// The reference runs Newton-Schulz in FP32; here the operands are BF16 (or
// FP16) with FP32 tensor-core accumulation (the published Muon formulation),
// compared against the FP32 reference by relative Frobenius error.
//
// One call covers a batch of up to kMaxBatch matrices of one shape [rows,
// cols] (m = min, n = max; every launch below handles the whole batch):
//   k_muon_sumsq     momentum update in place, u = Nesterov blend, FP64 sum
//                    of u^2 per matrix (the last CTA of a matrix writes its
//                    norm divisor);
//   k_ns_normalize   x = u / (||u|| + 1e-7) as X [mp, np] and its transpose
//                    XT [np, mp] (mp, np = m, n rounded up to 256, zero
//                    padding written explicitly) through 32x64 tiles with
//                    vector loads and stores, both orientations coalesced;
//   15 GEMMs         per iteration: A = X X^T; M = a I + b A + c A A (one
//                    FP32 epilogue, rounded once); X' = M X (reads XT, writes
//                    X' and X'^T). The last X' = M X applies the update
//                    w = fma(o * shape_scale, -lr, w * (1 - lr*wd)) in its
//                    epilogue straight from the FP32 accumulators (and writes
//                    the optional BF16/FP16 copy of w), so the orthogonalised
//                    matrix never goes to memory.
#include "mb_common.cuh"

namespace mb {
namespace {

constexpr int kPad = 256;
constexpr int kStatBlocks = 1024;  // per matrix

inline int64_t pad_to(int64_t x) { return (x + kPad - 1) / kPad * kPad; }
inline size_t up256(size_t x) { return (x + 255) / 256 * 256; }

struct Layout {
  int batch;
  int64_t mp, np;
  size_t partials, tickets, divisors, x, t0, t1, a, b, o, total;
};

// Workspace: [FP64 partials][tickets][divisors][X][XT0][XT1][A][B][O f32 (optional)],
// each region `batch` matrices back to back.
Layout layout_for(int batch, int64_t rows, int64_t cols, bool with_o) {
  Layout L;
  L.batch = batch;
  int64_t m = rows < cols ? rows : cols, n = rows < cols ? cols : rows;
  L.mp = pad_to(m);
  L.np = pad_to(n);
  const size_t xb = (size_t)L.mp * L.np * 2, ab = (size_t)L.mp * L.mp * 2;
  size_t off = 0;
  L.partials = off; off += up256(sizeof(double) * kStatBlocks * batch);
  L.tickets = off;  off += up256(sizeof(unsigned) * batch);
  L.divisors = off; off += up256(sizeof(float) * batch);
  L.x = off;        off += xb * batch;
  L.t0 = off;       off += xb * batch;
  L.t1 = off;       off += xb * batch;
  L.a = off;        off += ab * batch;
  L.b = off;        off += ab * batch;
  L.o = off;        off += with_o ? (size_t)L.mp * L.np * 4 * batch : 0;
  L.total = off;
  return L;
}

// Per-matrix inputs. mom[b] == nullptr: src[b] is the FP32 matrix u itself
// (orthogonalize of a given matrix); otherwise src[b] is the gradient.
struct MuonSrc {
  float* mom[kMaxBatch];
  const void* src[kMaxBatch];
};

struct MuonParams {
  float beta_lerp;  // .05
  float nesterov;   // .95
  const int32_t* skip = nullptr;  // device flag: nonzero = the step changes nothing
  int max_sms = 0;                // the GEMMs' SM cap (0: every SM)
};

// Nesterov input of one element (also writes the updated momentum when `write`).
template <int GDT>
__device__ __forceinline__ float muon_u(float* mom, const void* src, const MuonParams& p, int64_t e, bool write) {
  if (mom == nullptr) return static_cast<const float*>(src)[e];
  float g = load1<GDT>(src, e);
  float mo = mom[e];
  if (write) {
    // momentum.lerp_(g, .05): small weight, fma(w, g - m, m)
    mo = __fmaf_rn(p.beta_lerp, __fsub_rn(g, mo), mo);
    mom[e] = mo;
  }
  // g.lerp(momentum, .95): large weight, fma(w - 1, m - g, m)
  return __fmaf_rn(__fsub_rn(p.nesterov, 1.0f), __fsub_rn(mo, g), mo);
}

// Four consecutive elements e..e+3 (16-byte aligned momentum / FP32 source).
template <int GDT>
__device__ __forceinline__ void muon_u4(float* mom, const void* src, const MuonParams& p, int64_t e, float (&u)[4]) {
  if (mom == nullptr) {
    load4<MB_F32>(src, e, u);
    return;
  }
  float g[4];
  load4<GDT>(src, e, g);
  float4 m4 = *reinterpret_cast<const float4*>(mom + e);
  float mo[4] = {m4.x, m4.y, m4.z, m4.w};
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    mo[h] = __fmaf_rn(p.beta_lerp, __fsub_rn(g[h], mo[h]), mo[h]);
    u[h] = __fmaf_rn(__fsub_rn(p.nesterov, 1.0f), __fsub_rn(mo[h], g[h]), mo[h]);
  }
  *reinterpret_cast<float4*>(mom + e) = make_float4(mo[0], mo[1], mo[2], mo[3]);
}

// grid (blocks per matrix, batch). `vec`: total % 4 == 0 and every pointer of
// the batch 16-byte aligned (8 for 16-bit gradients).
template <int GDT>
__global__ void __launch_bounds__(kThreads) k_muon_sumsq(MuonSrc t, MuonParams p, int64_t total, bool vec,
                                                          double* partials, unsigned int* tickets, float* divisors) {
  if (p.skip != nullptr && *p.skip != 0) return;  // a refused step: momentum untouched
  const int b = blockIdx.y;
  float* mom = t.mom[b];
  const void* src = t.src[b];
  double acc = 0.0;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  if (vec) {
    const int64_t quads = total >> 2;
    int64_t q = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    for (; q + stride < quads; q += 2 * stride) {  // two quads in flight per thread
      float u0[4], u1[4];
      muon_u4<GDT>(mom, src, p, q * 4, u0);
      muon_u4<GDT>(mom, src, p, (q + stride) * 4, u1);
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        acc = __fma_rn((double)u0[h], (double)u0[h], acc);
        acc = __fma_rn((double)u1[h], (double)u1[h], acc);
      }
    }
    if (q < quads) {
      float u0[4];
      muon_u4<GDT>(mom, src, p, q * 4, u0);
#pragma unroll
      for (int h = 0; h < 4; ++h) acc = __fma_rn((double)u0[h], (double)u0[h], acc);
    }
  } else {
    for (int64_t e = (int64_t)blockIdx.x * kThreads + threadIdx.x; e < total; e += stride) {
      float u = muon_u<GDT>(mom, src, p, e, true);
      acc = __fma_rn((double)u, (double)u, acc);
    }
  }
  __shared__ double red[kThreads / 32];
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  __shared__ unsigned int s_last;
  double* part = partials + (size_t)b * kStatBlocks;
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int i = 0; i < kThreads / 32; ++i) s += red[i];
    part[blockIdx.x] = s;
    __threadfence();
    s_last = atomicAdd(&tickets[b], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    __threadfence();
    double s = 0.0;
    for (unsigned i = 0; i < gridDim.x; ++i) s += __ldcg(&part[i]);
    // x.norm() + 1e-7 in float (optimizer.py:18)
    divisors[b] = __fadd_rn(__double2float_rn(sqrt(s)), 1e-7f);
    tickets[b] = 0u;
  }
}

// Read-only Nesterov blend of four consecutive elements (the momentum already
// holds this step's value): u = fma(w - 1, m - g, m), or the FP32 source itself.
template <int GDT>
__device__ __forceinline__ void muon_u4_read(const float* mom, const void* src, const MuonParams& p, int64_t e,
                                             float (&u)[4]) {
  if (mom == nullptr) {
    load4<MB_F32>(src, e, u);
    return;
  }
  float g[4];
  load4<GDT>(src, e, g);
  const float4 m4 = *reinterpret_cast<const float4*>(mom + e);
  const float mo[4] = {m4.x, m4.y, m4.z, m4.w};
#pragma unroll
  for (int h = 0; h < 4; ++h) u[h] = __fmaf_rn(__fsub_rn(p.nesterov, 1.0f), __fsub_rn(mo[h], g[h]), mo[h]);
}

// grid (cols_p / 64, rows_p / 32, batch), 256 threads: one 32 x 64 tile of u
// (the matrix in its stored orientation, padded to rows_p x cols_p) per CTA.
// Thread (ty, tx) of a 16 x 16 grid reads rows ty and ty + 16, columns 4tx..4tx+3
// (16-byte momentum / 8-byte gradient loads when `vec`), writes them to D
// [rows_p, cols_p] as 8-byte vectors, and after a shared-memory transpose
// writes 8 consecutive elements of one row of T [cols_p, rows_p]. Wide
// matrices: D is X and T is XT; tall: D is XT and T is X. Values are
// prescale * u / divisor, zero in the padding. `prescale` is a power of two
// (exact); it lifts the first iterate's elements (RMS 1/sqrt(m n)) toward their
// converged size (1/sqrt(n)) so FP16 operands stay out of the subnormal range,
// and the first iteration's GEMMs divide it back out exactly.
template <int GDT, int OUT>
__global__ void __launch_bounds__(256) k_ns_normalize(MuonSrc t, MuonParams p, int64_t rows, int64_t cols,
                                                      int64_t ld_d, int64_t ld_t, size_t stride, const float* divisors,
                                                      float prescale, void* Dv, void* Tv, bool vec) {
  if (p.skip != nullptr && *p.skip != 0) return;
  using T = typename Elem<OUT>::T;
  const int b = blockIdx.z;
  T* D = static_cast<T*>(Dv) + stride * b;
  T* Tt = static_cast<T*>(Tv) + stride * b;
  const float* mom = t.mom[b];
  const void* src = t.src[b];
  __shared__ float tile[32][65];
  const float d = divisors[b];
  const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 64;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int lr = ty + 16 * h, lc = 4 * tx;
    const int64_t r = r0 + lr, c = c0 + lc;
    float val[4];
    if (vec && r < rows && c + 4 <= cols) {
      float u[4];
      muon_u4_read<GDT>(mom, src, p, r * cols + c, u);
#pragma unroll
      for (int j = 0; j < 4; ++j) val[j] = __fmul_rn(__fdiv_rn(u[j], d), prescale);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        val[j] = 0.0f;
        if (r < rows && c + j < cols)
          val[j] = __fmul_rn(__fdiv_rn(muon_u<GDT>(const_cast<float*>(mom), src, p, r * cols + c + j, false), d),
                             prescale);
      }
    }
    store4<OUT>(D, r * ld_d + c, val);
#pragma unroll
    for (int j = 0; j < 4; ++j) tile[lr][lc + j] = val[j];
  }
  __syncthreads();
  const int tc = tid >> 2, tr0 = (tid & 3) * 8;
  float lo[4], hi[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    lo[i] = tile[tr0 + i][tc];
    hi[i] = tile[tr0 + 4 + i][tc];
  }
  store4<OUT>(Tt, (c0 + tc) * ld_t + r0 + tr0, lo);
  store4<OUT>(Tt, (c0 + tc) * ld_t + r0 + tr0 + 4, hi);
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

// Power of two nearest below sqrt(m): the first iterate's prescale.
float prescale_for(int64_t m) {
  int k = 0;
  while ((int64_t)1 << (2 * (k + 1)) <= m) ++k;
  return (float)(1 << k);
}

template <int GDT>
int launch_sumsq(const MuonSrc& t, const MuonParams& p, int batch, int64_t total, bool vec, char* ws,
                 const Layout& L, cudaStream_t s) {
  int64_t blocks = (total / 4 + (int64_t)kThreads * 8 - 1) / ((int64_t)kThreads * 8);
  if (blocks > kStatBlocks) blocks = kStatBlocks;
  if (blocks < 1) blocks = 1;
  k_muon_sumsq<GDT><<<dim3((unsigned)blocks, (unsigned)batch), kThreads, 0, s>>>(
      t, p, total, vec, reinterpret_cast<double*>(ws + L.partials), reinterpret_cast<unsigned*>(ws + L.tickets),
      reinterpret_cast<float*>(ws + L.divisors));
  return cudaGetLastError() == cudaSuccess ? MB_OK : MB_ERR_CUDA;
}

template <int GDT, int OUT>
int launch_normalize(const MuonSrc& t, const MuonParams& p, int batch, int64_t rows, int64_t cols, const Layout& L,
                     char* ws, float ps, bool vec, cudaStream_t s) {
  const bool tall = rows > cols;
  // the stored orientation of u, padded: wide [mp, np], tall [np, mp]
  const int64_t rp = tall ? L.np : L.mp, cp = tall ? L.mp : L.np;
  void* D = ws + (tall ? L.t0 : L.x);
  void* T = ws + (tall ? L.x : L.t0);
  dim3 grd((unsigned)(cp / 64), (unsigned)(rp / 32), (unsigned)batch);
  k_ns_normalize<GDT, OUT><<<grd, 256, 0, s>>>(t, p, rows, cols, cp, rp, (size_t)L.mp * L.np,
                                               reinterpret_cast<const float*>(ws + L.divisors), ps, D, T, vec);
  return cudaGetLastError() == cudaSuccess ? MB_OK : MB_ERR_CUDA;
}

template <int GDT>
int launch_normalize_any(int out, const MuonSrc& t, const MuonParams& p, int batch, int64_t rows, int64_t cols,
                         const Layout& L, char* ws, float ps, bool vec, cudaStream_t s) {
  if (out == MB_F16) return launch_normalize<GDT, MB_F16>(t, p, batch, rows, cols, L, ws, ps, vec, s);
  return launch_normalize<GDT, MB_BF16>(t, p, batch, rows, cols, L, ws, ps, vec, s);
}

// The final update of a batch (null for orthogonalize, which keeps O).
struct Update {
  float* const* w;
  void* const* out;  // null: no copy
  int odt;
  float shape_scale, cwd, neg_lr;
};

// Normalise + Newton-Schulz iterations on `dtype` (MB_BF16 or MB_F16)
// operands; the last GEMM applies `upd`, or leaves the FP32 result in O.
int ns_core(const MuonSrc& t, const MuonParams& p, int gdt, int batch, int64_t rows, int64_t cols, int steps,
            const float* coeffs, int dtype, const Update* upd, char* ws, const Layout& L, int32_t* err,
            cudaStream_t s) {
  if (dtype != MB_BF16 && dtype != MB_F16) return MB_ERR_ARG;
  if (steps <= 0) return MB_ERR_ARG;
  const int64_t total = rows * cols;
  // vectorised pass: quads of elements, aligned pointers
  bool vec = total % 4 == 0;
  for (int b = 0; b < batch && vec; ++b) {
    const uintptr_t ga = t.mom[b] == nullptr || gdt == MB_F32 ? 16 : 8;
    vec = aligned(t.src[b], ga) && (t.mom[b] == nullptr || aligned(t.mom[b], 16));
  }
  const bool vec_rows = vec && cols % 4 == 0;  // every row starts on a 16-byte boundary
  if (cudaMemsetAsync(ws + L.tickets, 0, sizeof(unsigned) * batch, s) != cudaSuccess) return MB_ERR_CUDA;
  int rc;
  switch (gdt) {
    case MB_F32: rc = launch_sumsq<MB_F32>(t, p, batch, total, vec, ws, L, s); break;
    case MB_F16: rc = launch_sumsq<MB_F16>(t, p, batch, total, vec, ws, L, s); break;
    case MB_BF16: rc = launch_sumsq<MB_BF16>(t, p, batch, total, vec, ws, L, s); break;
    default: return MB_ERR_ARG;
  }
  if (rc) return rc;
  const int64_t m = rows < cols ? rows : cols;
  const float ps = prescale_for(m);
  switch (gdt) {
    case MB_F32: rc = launch_normalize_any<MB_F32>(dtype, t, p, batch, rows, cols, L, ws, ps, vec_rows, s); break;
    case MB_F16: rc = launch_normalize_any<MB_F16>(dtype, t, p, batch, rows, cols, L, ws, ps, vec_rows, s); break;
    default: rc = launch_normalize_any<MB_BF16>(dtype, t, p, batch, rows, cols, L, ws, ps, vec_rows, s); break;
  }
  if (rc) return rc;
  const int64_t mp = L.mp, np = L.np, sx = mp * np, sa = mp * mp;
  void* X = ws + L.x;
  void* A = ws + L.a;
  void* B = ws + L.b;
  void *XT = ws + L.t0, *XTn = ws + L.t1;
  for (int it = 0; it < steps; ++it) {
    const bool last = it == steps - 1;
    // the first iterate carries the prescale: undo it exactly in the FP32 epilogues
    const float s1 = it == 0 ? 1.0f / ps : 1.0f;
    // A = X X^T (symmetric: upper tiles only, lower triangle by transposition)
    GemmCall g1{};
    g1.dtype = dtype; g1.batch = batch; g1.sym = true;
    g1.a = X; g1.lda = np; g1.sa = sx;
    g1.b = X; g1.ldb = np; g1.sb = sx;
    g1.M = mp; g1.N = mp; g1.K = np;
    g1.alpha = s1 * s1;
    g1.d = A; g1.ldd = mp; g1.sd = sa;
    g1.dt = A; g1.lddt = mp; g1.sdt = sa;
    g1.err = err;
    g1.skip = p.skip;
    g1.max_sms = p.max_sms;
    if ((rc = gemm16(g1, s))) return rc;
    // M = a I + b A + c A A, formed in FP32 and rounded once: the reference's
    // a X + (b A + c A A) X would add two nearly cancelling products.
    GemmCall g2{};
    g2.dtype = dtype; g2.batch = batch; g2.sym = true;
    g2.a = A; g2.lda = mp; g2.sa = sa;
    g2.b = A; g2.ldb = mp; g2.sb = sa;
    g2.M = mp; g2.N = mp; g2.K = mp;
    g2.alpha = coeffs[2]; g2.beta = coeffs[1]; g2.diag = coeffs[0];
    g2.c = A; g2.ldc = mp; g2.sc = sa;
    g2.d = B; g2.ldd = mp; g2.sd = sa;
    g2.dt = B; g2.lddt = mp; g2.sdt = sa;
    g2.err = err;
    g2.skip = p.skip;
    g2.max_sms = p.max_sms;
    if ((rc = gemm16(g2, s))) return rc;
    // X' = M X: X^T is the K-major operand. X' overwrites X (no longer read);
    // X'^T goes to the other XT buffer. The last iteration applies the update
    // (or writes FP32 O).
    GemmCall g3{};
    g3.dtype = dtype; g3.batch = batch;
    g3.a = B; g3.lda = mp; g3.sa = sa;
    g3.b = XT; g3.ldb = mp; g3.sb = sx;
    g3.M = mp; g3.N = np; g3.K = mp;
    g3.alpha = s1;
    g3.err = err;
    g3.skip = p.skip;
    g3.max_sms = p.max_sms;
    if (!last) {
      g3.d = X; g3.ldd = np; g3.sd = sx;
      g3.dt = XTn; g3.lddt = mp; g3.sdt = sx;
    } else if (upd != nullptr) {
      g3.upd_w = upd->w; g3.upd_out = upd->out; g3.upd_odt = upd->odt;
      g3.upd_tall = rows > cols;
      g3.upd_m = m; g3.upd_n = rows < cols ? cols : rows; g3.upd_cols = cols;
      g3.upd_scale = upd->shape_scale; g3.upd_cwd = upd->cwd; g3.upd_neglr = upd->neg_lr;
    } else {
      g3.df = reinterpret_cast<float*>(ws + L.o); g3.lddf = np; g3.sdf = sx;
    }
    if ((rc = gemm16(g3, s))) return rc;
    void* tmp = XT; XT = XTn; XTn = tmp;
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
  return layout_for(1, rows, cols, true).total;
}

MB_API size_t mb_muon_batch_workspace_bytes(int32_t batch, int64_t rows, int64_t cols) {
  if (batch < 1 || batch > kMaxBatch || check_dims(rows, cols)) return 0;
  return layout_for(batch, rows, cols, false).total;
}

MB_API int mb_newton_schulz(const float* x, int64_t rows, int64_t cols, int32_t steps, const float* coeffs,
                            int32_t ns_dtype, float* out, void* workspace, size_t workspace_bytes,
                            int32_t* err_flag, mb_stream_t stream) {
  if (!x || !out || !coeffs || !workspace || steps <= 0) return MB_ERR_ARG;
  int rc = check_dims(rows, cols);
  if (rc) return rc;
  Layout L = layout_for(1, rows, cols, true);
  if (workspace_bytes < L.total) return MB_ERR_ARG;
  if (!aligned(workspace, 256)) return MB_ERR_ALIGN;
  cudaStream_t s = (cudaStream_t)stream;
  char* ws = static_cast<char*>(workspace);
  MuonSrc t{};
  t.src[0] = x;
  MuonParams p{0.0f, 0.0f};
  rc = ns_core(t, p, MB_F32, 1, rows, cols, steps, coeffs, ns_dtype, nullptr, ws, L, err_flag, s);
  if (rc) return rc;
  dim3 blk(32, 32), grd((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32));
  k_ns_output<<<grd, blk, 0, s>>>(reinterpret_cast<const float*>(ws + L.o), out, rows, cols, L.np, rows > cols);
  return cudaGetLastError() == cudaSuccess ? MB_OK : MB_ERR_CUDA;
}

MB_API int mb_muon_step_batched(float* const* w, float* const* momentum, const void* const* g, int32_t grad_dtype,
                                void* const* out, int32_t out_dtype, int32_t batch, int64_t rows, int64_t cols,
                                const mb_muon_args* args, void* workspace, size_t workspace_bytes,
                                int32_t* err_flag, mb_stream_t stream) {
  if (!w || !momentum || !g || !args || !workspace) return MB_ERR_ARG;
  if (batch < 1 || batch > kMaxBatch) return MB_ERR_ARG;
  if (grad_dtype < MB_F32 || grad_dtype > MB_BF16) return MB_ERR_ARG;
  if (out_dtype != MB_NONE && out_dtype != MB_F16 && out_dtype != MB_BF16) return MB_ERR_ARG;
  if (out_dtype != MB_NONE && !out) return MB_ERR_ARG;
  if (args->ns_steps <= 0) return MB_ERR_ARG;
  int rc = check_dims(rows, cols);
  if (rc) return rc;
  MuonSrc t{};
  for (int b = 0; b < batch; ++b) {
    if (!w[b] || !momentum[b] || !g[b] || (out_dtype != MB_NONE && !out[b])) return MB_ERR_ARG;
    t.mom[b] = momentum[b];
    t.src[b] = g[b];
  }
  Layout L = layout_for(batch, rows, cols, false);
  if (workspace_bytes < L.total) return MB_ERR_ARG;
  if (!aligned(workspace, 256)) return MB_ERR_ALIGN;
  if (args->max_sms < 0) return MB_ERR_ARG;
  MuonParams p{args->beta_lerp, args->nesterov, args->skip, args->max_sms};
  const float coeffs[3] = {args->ns_a, args->ns_b, args->ns_c};
  Update upd{w, out_dtype == MB_NONE ? nullptr : out, out_dtype, args->shape_scale, args->cwd, args->neg_lr};
  return ns_core(t, p, grad_dtype, batch, rows, cols, args->ns_steps, coeffs, args->ns_dtype, &upd,
                 static_cast<char*>(workspace), L, err_flag, (cudaStream_t)stream);
}

MB_API int mb_muon_step(float* w, float* momentum, const void* g, int32_t grad_dtype, void* out, int32_t out_dtype,
                        int64_t rows, int64_t cols, const mb_muon_args* args, void* workspace,
                        size_t workspace_bytes, int32_t* err_flag, mb_stream_t stream) {
  if (!w || !momentum || !g) return MB_ERR_ARG;
  if (out_dtype != MB_NONE && !out) return MB_ERR_ARG;
  return mb_muon_step_batched(&w, &momentum, &g, grad_dtype, &out, out_dtype, 1, rows, cols, args, workspace,
                              workspace_bytes, err_flag, stream);
}

}  // extern "C"
