// Kernel 4 building block: 16-bit (BF16 or FP16) GEMM on the sm_100a tensor
// cores (tcgen05), FP32 accumulation in TMEM.
//
//   out = alpha * (A . B^T) + beta * C + diag * I,   A [M, K], B [N, K], C/out [M, N]
//
// Both operands are K-major (row-major with K contiguous), which is what
// Newton-Schulz needs: X.X^T uses X for both; A.A uses the symmetric A for
// both; B.X reads X^T, which the previous GEMM writes as a second, transposed
// output. Outputs: BF16 row-major `d`, BF16 transposed `dt` (dt[j][i]) and/or
// FP32 row-major `df`.
//
// Persistent CTAs (one per SM) walk the 128 x 256 output tiles with 6 warps:
//   warp 0   TMA producer: 4-stage ring of 128x64 (A) and 256x64 (B) 16-bit
//            tiles, 128-byte swizzled, completion tracked by mbarrier
//            transaction bytes; the ring runs on across tiles;
//   warp 1   owns two 256-column TMEM accumulators (512 columns); one lane
//            issues tcgen05.mma (M=128, N=256, K=16, FP32 accumulate) per
//            16-wide K slice, tcgen05.commit releases each stage and, after a
//            tile's last slice, hands the accumulator to the epilogue;
//   warps 2-5 epilogue: tcgen05.ld 32 lanes x 32 columns at a time, scale, add
//            beta*C and diag*I, convert, store; then return the accumulator.
// While the epilogue drains tile i from one accumulator, the MMAs of tile
// i + 1 fill the other.
//
// Symmetric mode (the output is known symmetric, e.g. X X^T and polynomials
// of it): only tiles not entirely below the diagonal are computed; elements on
// or above the diagonal are stored directly and those strictly above are also
// stored transposed, so every element is written exactly once.
// Every mbarrier wait is bounded (about 2 s of %globaltimer): on expiry the CTA
// raises the error flag, stops issuing, waits (bounded) for its own loads in
// flight, frees its TMEM and returns.
//
// Shapes must be multiples of the tile (M % 128, N % 256, K % 64 == 0) and the
// row pitches multiples of 8 elements; callers pad with zeros (zero rows and
// columns stay zero through Newton-Schulz).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "mb_common.cuh"

namespace mb {
namespace gemm {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int kWarps = 6;
constexpr int kGemmThreads = kWarps * 32;
constexpr int A_STAGE = BM * BK * 2;   // 16 KiB
constexpr int B_STAGE = BN * BK * 2;   // 32 KiB
constexpr int kBarrierBytes = 256;  // full/empty rings, 2 x acc full/empty, TMEM slot, abort flag
constexpr int SMEM_BYTES = STAGES * (A_STAGE + B_STAGE) + 1024 + kBarrierBytes;
constexpr uint32_t TMEM_COLS = 512;  // two 256-column accumulators
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// Instruction descriptor, kind::f16: D FP32 (bits 4-5 = 1), A and B of one
// 16-bit type (bits 7-9 and 10-12: 1 = BF16, 0 = FP16), both K-major (bits 15,
// 16 = 0), N >> 3 at bits 17-22, M >> 4 at bits 24-28.
template <bool kF16>
__host__ __device__ constexpr uint32_t idesc() {
  return (1u << 4) | ((kF16 ? 0u : 1u) << 7) | ((kF16 ? 0u : 1u) << 10) | ((uint32_t)(BN >> 3) << 17) |
         ((uint32_t)(BM >> 4) << 24);
}

struct Args {
  int M, N, K;
  int n_tiles;  // tiles to compute (all, or the non-lower ones in symmetric mode)
  int sym;      // output symmetric: see the header comment
  float alpha, beta, diag;
  const uint16_t* c;
  int64_t ldc;
  uint16_t* d;
  int64_t ldd;
  uint16_t* dt;
  int64_t lddt;
  float* df;
  int64_t lddf;
  int32_t* err;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase of `parity` to complete; false on abort or time-out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > kWaitLimitNs) {
      *abort_flag = 1;
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 B apart (SBO), version 1 (bits 46-47), layout type 2 (bits 61-63).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void umma_16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t id,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(id), "r"(accumulate)
      : "memory");
}

template <bool kF16>
__device__ __forceinline__ float h2f(uint16_t h) {
  if constexpr (kF16) return __half2float(__ushort_as_half(h));
  else return __uint_as_float((uint32_t)h << 16);
}

template <bool kF16>
__device__ __forceinline__ uint16_t f2h(float x) {
  if constexpr (kF16) return __half_as_ushort(__float2half_rn(x));
  else return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Tile t -> (bm, bn). Plain: bm fastest (consecutive CTAs share the B tile).
// Symmetric: column bn holds the tiles bm < min(mt, 2 bn + 2), i.e. those not
// entirely below the diagonal (BN = 2 BM).
__device__ __forceinline__ void tile_coords(const Args& g, int t, int& bm, int& bn) {
  const int mt = g.M / BM;
  if (!g.sym) {
    bm = t % mt;
    bn = t / mt;
    return;
  }
  int c = 0;
  for (bn = 0;; ++bn) {
    const int h = mt < 2 * bn + 2 ? mt : 2 * bn + 2;
    if (t < c + h) {
      bm = t - c;
      return;
    }
    c += h;
  }
}

// Store one 32-column chunk of one row (thread's row `row`, columns col..col+31).
template <bool kF16>
__device__ __forceinline__ void store_chunk(const Args& g, float (&v)[32], int row, int col) {
  const bool all_upper = row < col;            // every element strictly above the diagonal
  const bool any_upper = row < col + 31;       // some element on/above (for direct stores: row <= col + j)
  if (g.d != nullptr) {
    if (!g.sym || all_upper) {
      uint4* dst = reinterpret_cast<uint4*>(g.d + (int64_t)row * g.ldd + col);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        uint32_t pk[4];
#pragma unroll
        for (int h = 0; h < 4; ++h)
          pk[h] = (uint32_t)f2h<kF16>(v[u * 8 + 2 * h]) | ((uint32_t)f2h<kF16>(v[u * 8 + 2 * h + 1]) << 16);
        dst[u] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
    } else if (any_upper || row == col + 31) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (row <= col + j) g.d[(int64_t)row * g.ldd + col + j] = f2h<kF16>(v[j]);
    }
  }
  if (g.dt != nullptr) {
    if (!g.sym) {
#pragma unroll
      for (int j = 0; j < 32; ++j) g.dt[(int64_t)(col + j) * g.lddt + row] = f2h<kF16>(v[j]);
    } else if (any_upper) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (row < col + j) g.dt[(int64_t)(col + j) * g.lddt + row] = f2h<kF16>(v[j]);
    }
  }
  if (g.df != nullptr) {
    float4* dst = reinterpret_cast<float4*>(g.df + (int64_t)row * g.lddf + col);
#pragma unroll
    for (int u = 0; u < 8; ++u) dst[u] = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
  }
}

template <bool kF16>
__global__ void __launch_bounds__(kGemmThreads, 1)
    k_gemm16(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Args g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;   // [2]: MMA -> epilogue
  uint64_t* acc_empty = acc_full + 2;    // [2]: epilogue -> MMA (4 arrivals: one per epilogue warp)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = g.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int kit = 0;  // k-blocks issued so far (the ring runs on across tiles)
      for (int t = blockIdx.x; t < g.n_tiles && !*abort_flag; t += gridDim.x) {
        int bm, bn;
        tile_coords(g, t, bm, bn);
        for (int kb = 0; kb < KB; ++kb, ++kit) {
          const int s = kit % STAGES;
          const uint32_t round = kit / STAGES;
          if (!mbar_wait(&empty[s], (round & 1) ^ 1, abort_flag)) break;
          mbar_expect_tx(&full[s], A_STAGE + B_STAGE);
          tma_load_2d(sA + s * A_STAGE, &tmA, &full[s], kb * BK, bm * BM);
          tma_load_2d(sB + s * B_STAGE, &tmB, &full[s], kb * BK, bn * BN);
        }
      }
      if (*abort_flag) {
        // Bounded wait for this CTA's own loads still in flight.
        const uint64_t t0 = globaltimer();
        for (int k = kit - STAGES > 0 ? kit - STAGES : 0; k < kit; ++k) {
          const int s = k % STAGES;
          const uint32_t round = k / STAGES;
          while (!mbar_try_wait(&full[s], round & 1) && globaltimer() - t0 < kWaitLimitNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int kit = 0, it = 0;
      for (int t = blockIdx.x; t < g.n_tiles && !*abort_flag; t += gridDim.x, ++it) {
        const int a = it & 1;
        const uint32_t use = it >> 1;
        if (!mbar_wait(&acc_empty[a], (use & 1) ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(a * BN);
        for (int kb = 0; kb < KB; ++kb, ++kit) {
          const int s = kit % STAGES;
          const uint32_t round = kit / STAGES;
          if (!mbar_wait(&full[s], round & 1, abort_flag)) break;
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * A_STAGE), b0 = smem_u32(sB + s * B_STAGE);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_16(acc, sw128_desc(a0 + k * 32), sw128_desc(b0 + k * 32), idesc<kF16>(), (kb | k) != 0 ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        umma_commit(&acc_full[a]);
      }
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may read
    int it = 0;
    for (int t = blockIdx.x; t < g.n_tiles; t += gridDim.x, ++it) {
      const int a = it & 1;
      const uint32_t use = it >> 1;
      int ok = 0;
      if (lane == 0) ok = mbar_wait(&acc_full[a], use & 1, abort_flag) && !*abort_flag;
      ok = __shfl_sync(0xffffffffu, ok, 0);  // warp-uniform: tcgen05.ld is .sync.aligned
      if (!ok) break;
      tc_fence_after();
      int bm, bn;
      tile_coords(g, t, bm, bn);
      const int row = bm * BM + q * 32 + lane;
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + (uint32_t)(a * BN) + ((uint32_t)(q * 32) << 16) + (uint32_t)c, r);
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = g.alpha * __uint_as_float(r[j]);
        const int col = bn * BN + c;
        if (g.diag != 0.0f && row >= col && row < col + 32) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col + j == row) v[j] += g.diag;  // compile-time index: v stays in registers
        }
        if (g.c != nullptr) {
          const uint4* src = reinterpret_cast<const uint4*>(g.c + (int64_t)row * g.ldc + col);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 w4 = src[u];
            const uint32_t ww[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              v[u * 8 + 2 * h] = fmaf(g.beta, h2f<kF16>((uint16_t)(ww[h] & 0xffffu)), v[u * 8 + 2 * h]);
              v[u * 8 + 2 * h + 1] = fmaf(g.beta, h2f<kF16>((uint16_t)(ww[h] >> 16)), v[u * 8 + 2 * h + 1]);
            }
          }
        }
        store_chunk<kF16>(g, v, row, col);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
  if (threadIdx.x == 0 && *abort_flag && g.err != nullptr) atomicExch(g.err, 1);
}

// ------------------------------------------------------------------ host --

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D 16-bit row-major [rows, cols] with row pitch `ld` elements; box = 64 x box_rows, 128B swizzle.
bool make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows, bool f16) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace gemm

int gemm16_nt(int dtype, const void* a, int64_t lda, const void* b, int64_t ldb, int64_t M, int64_t N, int64_t K,
              float alpha, float beta, float diag, const void* c, int64_t ldc, void* d, int64_t ldd, void* dt,
              int64_t lddt, float* df, int64_t lddf, int32_t* err, cudaStream_t stream, bool sym) {
  using namespace gemm;
  if (dtype != MB_BF16 && dtype != MB_F16) return MB_ERR_ARG;
  const bool f16 = dtype == MB_F16;
  if (!a || !b || M <= 0 || N <= 0 || K <= 0) return MB_ERR_ARG;
  if (M % BM || N % BN || K % BK || M > (1 << 30) || N > (1 << 30)) return MB_ERR_ARG;
  if (!d && !dt && !df) return MB_ERR_ARG;
  if (lda < K || ldb < K || (lda % 8) || (ldb % 8)) return MB_ERR_ALIGN;
  if (!aligned(a, 16) || !aligned(b, 16)) return MB_ERR_ALIGN;
  if (c && (ldc < N || ldc % 8 || !aligned(c, 16))) return MB_ERR_ALIGN;
  if (d && (ldd < N || ldd % 8 || !aligned(d, 16))) return MB_ERR_ALIGN;
  if (dt && (lddt < M || !aligned(dt, 2))) return MB_ERR_ALIGN;
  if (df && (lddf < N || lddf % 4 || !aligned(df, 16))) return MB_ERR_ALIGN;
  // symmetric mode writes the lower triangle through dt == d (square output, no FP32 copy)
  if (sym && (M != N || !d || dt != d || lddt != ldd || df)) return MB_ERR_ARG;
  CUtensorMap ma, mbm;
  if (!make_map(&ma, a, M, K, lda, BM, f16) || !make_map(&mbm, b, N, K, ldb, BN, f16)) return MB_ERR_CUDA;
  static std::once_flag attr_once;
  static cudaError_t attr_rc = cudaSuccess;
  std::call_once(attr_once, [] {
    attr_rc = cudaFuncSetAttribute(k_gemm16<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (attr_rc == cudaSuccess)
      attr_rc = cudaFuncSetAttribute(k_gemm16<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  });
  if (attr_rc != cudaSuccess) return MB_ERR_CUDA;
  const int mt = (int)(M / BM), nt = (int)(N / BN);
  int tiles = mt * nt;
  if (sym) {
    tiles = 0;
    for (int bn = 0; bn < nt; ++bn) tiles += mt < 2 * bn + 2 ? mt : 2 * bn + 2;
  }
  Args g{(int)M, (int)N, (int)K, tiles, sym ? 1 : 0, alpha, beta, diag, static_cast<const uint16_t*>(c), ldc,
         static_cast<uint16_t*>(d), ldd, static_cast<uint16_t*>(dt), lddt, df, lddf, err};
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  const int grid = tiles < sms ? tiles : sms;
  if (f16) k_gemm16<true><<<grid, kGemmThreads, SMEM_BYTES, stream>>>(ma, mbm, g);
  else k_gemm16<false><<<grid, kGemmThreads, SMEM_BYTES, stream>>>(ma, mbm, g);
  return cudaGetLastError() == cudaSuccess ? MB_OK : MB_ERR_CUDA;
}

}  // namespace mb

extern "C" MB_API int mb_gemm16(int32_t dtype, const void* a, int64_t lda, const void* b, int64_t ldb, int64_t m,
                                int64_t n, int64_t k, float alpha, float beta, const void* c, int64_t ldc, void* d,
                                int64_t ldd, void* dt, int64_t lddt, float* df, int64_t lddf, int32_t* err_flag,
                                mb_stream_t stream) {
  return mb::gemm16_nt(dtype, a, lda, b, ldb, m, n, k, alpha, beta, 0.0f, c, ldc, d, ldd, dt, lddt, df, lddf,
                       err_flag, (cudaStream_t)stream, false);
}
