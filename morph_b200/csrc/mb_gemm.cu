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
// Pair mode (the default when M % 256 == 0; MB_GEMM_PAIR=0 in the environment
// turns it off): clusters of two CTAs on two SMs share one 256 x 256 output
// tile through tcgen05.mma .cta_group::2 (M = 256). Each CTA loads its own 128
// rows of A and 128 of the 256 rows of B (no multicast) into a 6-stage ring, so
// an SM moves 32 KiB per 64-deep k-block instead of 48 KiB; the even CTA issues
// the MMAs and its commits arrive on both CTAs' barriers; each CTA's TMEM holds
// its 128 rows of the accumulator and its own epilogue drains them. The odd
// CTA's loads and epilogue signal the even CTA's barriers through their cluster
// addresses. The cluster barrier (not bounded) runs only at start-up and
// before TMEM is freed, after every bounded wait of both CTAs has ended.
// GemmCall.max_sms (0: all) caps the persistent grid, leaving SMs to kernels on
// other streams.
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

#include <cstdlib>
#include <mutex>

#include "mb_async.cuh"
#include "mb_common.cuh"

namespace mb {
namespace gemm {

// Tuning knob: K depth of a ring stage. 64 (default): 128-byte swizzled
// K-major tiles, 4 stages; 32: 64-byte swizzled tiles, 8 stages of half the
// size (the same shared memory, twice the stages in flight).
#ifndef MB_GEMM_BK
#define MB_GEMM_BK 64
#endif
constexpr int BM = 128, BN = 256, BK = MB_GEMM_BK, STAGES = BK == 64 ? 4 : 8;
static_assert(BK == 64 || BK == 32, "K stages of 64 or 32 elements");
constexpr int kRowBytes = BK * 2;  // one K-major row of a stage: the swizzle span
constexpr int kWarps = 6;
constexpr int kGemmThreads = kWarps * 32;
constexpr int A_STAGE = BM * BK * 2;   // 16 KiB
constexpr int B_STAGE = BN * BK * 2;   // 32 KiB
constexpr int kBarrierBytes = 256;  // full/empty rings, 2 x acc full/empty, TMEM slot, abort flag
// Epilogue staging: each epilogue warp owns 32 rows of 64 B (a 32 x 32 16-bit
// block) padded to 80 B, so a lane's own 16-byte row accesses are bank-conflict
// free while the warp's global accesses go out as 8 rows x 64 B per instruction.
constexpr int kStageRow = 80;
constexpr int kStageRowF = 144;  // the fused update's FP32 rows: 128 B + 16 B pad
constexpr int kStageWarp = 32 * kStageRowF;
constexpr int SMEM_BYTES = STAGES * (A_STAGE + B_STAGE) + 1024 + kBarrierBytes + 4 * kStageWarp;
constexpr uint32_t TMEM_COLS = 512;  // two 256-column accumulators
// pair mode: each CTA holds 128 of the tile's 256 B rows, so a stage is 32 KiB
// (BK = 64) and the same shared memory holds more stages
constexpr int B_STAGE_P = BM * BK * 2;
constexpr int STAGES_P = STAGES * (A_STAGE + B_STAGE) / (A_STAGE + B_STAGE_P);
static_assert(STAGES_P * (A_STAGE + B_STAGE_P) == STAGES * (A_STAGE + B_STAGE), "pair stages fill the same ring");
static_assert(2 * 8 * STAGES_P + 5 * 8 + 8 <= kBarrierBytes, "barrier area");

// Instruction descriptor, kind::f16: D FP32 (bits 4-5 = 1), A and B of one
// 16-bit type (bits 7-9 and 10-12: 1 = BF16, 0 = FP16), both K-major (bits 15,
// 16 = 0), N >> 3 at bits 17-22, M >> 4 at bits 24-28.
template <bool kF16, int kM = BM>
__host__ __device__ constexpr uint32_t idesc() {
  return (1u << 4) | ((kF16 ? 0u : 1u) << 7) | ((kF16 ? 0u : 1u) << 10) | ((uint32_t)(BN >> 3) << 17) |
         ((uint32_t)(kM >> 4) << 24);
}

struct Args {
  int M, N, K;
  int n_tiles;  // tiles per matrix (all, or the non-lower ones in symmetric mode)
  int batch;    // matrices; tile index t covers matrix t / n_tiles
  int sym;      // output symmetric: see the header comment
  float alpha, beta, diag;
  const uint16_t* c;
  int64_t ldc, sc;  // row pitch, matrix stride (elements)
  uint16_t* d;
  int64_t ldd, sd;
  uint16_t* dt;
  int64_t lddt, sdt;
  float* df;
  int64_t lddf, sdf;
  // Fused Muon update (upd): for each valid output element o of matrix b,
  // w = fma(o * upd_scale, upd_neglr, w * upd_cwd) on upd_w[b] (FP32
  // [rows, cols]); o[i][j] is w[i][j], or w[j][i] when upd_tall; upd_out[b]
  // (optional) receives w in upd_odt. upd_vec: w rows are 16-byte aligned
  // (cols % 4 == 0), so wide chunks move as float4.
  int upd, upd_odt, upd_tall, upd_vec;
  int64_t upd_m, upd_n, upd_cols;  // valid rows / columns of the output, w's row length
  float upd_scale, upd_cwd, upd_neglr;
  float* upd_w[kMaxBatch];
  void* upd_out[kMaxBatch];
  int32_t* err;
  int stage;  // d (and dt) 16-byte aligned with pitches in multiples of 8, no df / update: staged stores
  int upd_stage_out;  // the update's copy 16-byte aligned rows (cols % 8 == 0): staged too
  const int32_t* skip;  // optional device flag: nonzero = return at once (a refused optimizer step)
  FaultPlan fault;  // test-only: a tile whose first k-block is withheld, and the launch's wait bound
};

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Pair mode: the same load, completing on the barrier at cluster address `bar`
// (the even CTA's); no multicast.
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, uint32_t bar, int x, int y,
                                                 int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Cluster address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_u32(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

// Every thread of both CTAs of the pair (no early exits may precede it); the
// non-.aligned form, as the roles reach it from divergent branches.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// mbar_wait for a barrier that the other CTA of the pair also arrives on.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                  uint64_t limit_ns) {
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > limit_ns) {
      *abort_flag = 1;
      return false;
    }
  }
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, rows of kRowBytes swizzled over
// that span (layout type 2 = 128-byte, 4 = 64-byte swizzle, bits 61-63), 8-row
// groups 8 * kRowBytes apart (SBO), version 1 (bits 46-47).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  constexpr uint64_t layout = kRowBytes == 128 ? 2 : 4;
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(8 * kRowBytes >> 4) << 32) |
         ((uint64_t)1 << 46) | (layout << 61);
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

// Pair mode: one M = 256 MMA over both CTAs (A rows and B rows at the same
// shared offsets in each), accumulating into both CTAs' TMEM.
__device__ __forceinline__ void umma_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t id,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(id), "r"(accumulate)
      : "memory");
}

// Pair mode: arrive on this CTA's barrier `bar` once the pair MMAs issued so
// far complete.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ... on the barrier at the same offset in both CTAs of the pair (the commit's
// cluster-multicast form, CTA mask 0b11; an arrival, not a load).
__device__ __forceinline__ void umma_commit_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3)
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

// Tile t -> (matrix, bm, bn). Plain: bm fastest (consecutive CTAs share the B
// tile). Symmetric: column bn holds the tiles bm < min(mt, 2 bn + 2), i.e. those
// not entirely below the diagonal (BN = 2 BM).
__device__ __forceinline__ void tile_coords(const Args& g, int tb, int& mat, int& bm, int& bn) {
  mat = tb / g.n_tiles;
  const int t = tb - mat * g.n_tiles;
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

// Store one 32-column chunk of one row (thread's row `row`, columns col..col+31)
// of matrix `mat`.
template <bool kF16>
__device__ __forceinline__ void store_chunk(const Args& g, float (&v)[32], int mat, int row, int col) {
  const bool all_upper = row < col;            // every element strictly above the diagonal
  const bool any_upper = row < col + 31;       // some element strictly above
  if (g.d != nullptr) {
    uint16_t* d = g.d + (int64_t)mat * g.sd;
    if (!g.sym || all_upper) {
      uint4* dst = reinterpret_cast<uint4*>(d + (int64_t)row * g.ldd + col);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        uint32_t pk[4];
#pragma unroll
        for (int h = 0; h < 4; ++h)
          pk[h] = (uint32_t)f2h<kF16>(v[u * 8 + 2 * h]) | ((uint32_t)f2h<kF16>(v[u * 8 + 2 * h + 1]) << 16);
        dst[u] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
    } else if (row <= col + 31) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (row <= col + j) d[(int64_t)row * g.ldd + col + j] = f2h<kF16>(v[j]);
    }
  }
  if (g.dt != nullptr) {
    uint16_t* dt = g.dt + (int64_t)mat * g.sdt;
    if (!g.sym) {
#pragma unroll
      for (int j = 0; j < 32; ++j) dt[(int64_t)(col + j) * g.lddt + row] = f2h<kF16>(v[j]);
    } else if (any_upper) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (row < col + j) dt[(int64_t)(col + j) * g.lddt + row] = f2h<kF16>(v[j]);
    }
  }
  if (g.df != nullptr) {
    float4* dst = reinterpret_cast<float4*>(g.df + (int64_t)mat * g.sdf + (int64_t)row * g.lddf + col);
#pragma unroll
    for (int u = 0; u < 8; ++u) dst[u] = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
  }
  if (g.upd && row < g.upd_m) {
    // optimizer.py:60-61: u = o * shape_scale; w = w * (1 - lr wd) + (-lr) u
    float* w = g.upd_w[mat];
    void* out = g.upd_out[mat];
    if (!g.upd_tall && g.upd_vec && col + 32 <= g.upd_n) {
      float4* wp = reinterpret_cast<float4*>(w + (int64_t)row * g.upd_cols + col);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        float4 x = wp[u];
        float r[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int h = 0; h < 4; ++h)
          r[h] = __fmaf_rn(__fmul_rn(v[4 * u + h], g.upd_scale), g.upd_neglr, __fmul_rn(r[h], g.upd_cwd));
        wp[u] = make_float4(r[0], r[1], r[2], r[3]);
        if (out != nullptr) {
          const int64_t e = (int64_t)row * g.upd_cols + col + 4 * u;
          if (g.upd_odt == MB_BF16) store4<MB_BF16>(out, e, r);
          else store4<MB_F16>(out, e, r);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (col + j < g.upd_n) {
          const int64_t e =
              g.upd_tall ? (int64_t)(col + j) * g.upd_cols + row : (int64_t)row * g.upd_cols + col + j;
          const float wn = __fmaf_rn(__fmul_rn(v[j], g.upd_scale), g.upd_neglr, __fmul_rn(w[e], g.upd_cwd));
          w[e] = wn;
          if (out != nullptr) {
            if (g.upd_odt == MB_BF16) static_cast<__nv_bfloat16*>(out)[e] = __float2bfloat16_rn(wn);
            else static_cast<__half*>(out)[e] = __float2half_rn(wn);
          }
        }
      }
    }
  }
}

// Coalesced load of the 32 x 32 16-bit block at src (row pitch ld) into the
// warp's staging rows: lane l moves 16 B of rows l/4 + 8i.
__device__ __forceinline__ void stage_load_block(uint8_t* stg, const uint16_t* src, int64_t ld, int lane) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = (lane >> 2) + 8 * i, c4 = lane & 3;
    *reinterpret_cast<uint4*>(stg + r * kStageRow + c4 * 16) =
        *reinterpret_cast<const uint4*>(src + (int64_t)r * ld + c4 * 8);
  }
}

// The block of rows row0..row0+31 (lane = row - row0), columns col..col+31,
// stored through the warp's staging rows: d row-major, and dt (its transpose)
// with column j of the block as row col + j. Every element of the block is
// stored (callers use it for full blocks only).
template <bool kF16>
__device__ __forceinline__ void store_chunk_staged(const Args& g, const float (&v)[32], uint8_t* stg, int mat,
                                                   int row0, int col, int lane) {
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    uint32_t pk[4];
#pragma unroll
    for (int h = 0; h < 4; ++h)
      pk[h] = (uint32_t)f2h<kF16>(v[u * 8 + 2 * h]) | ((uint32_t)f2h<kF16>(v[u * 8 + 2 * h + 1]) << 16);
    *reinterpret_cast<uint4*>(stg + lane * kStageRow + u * 16) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
  }
  __syncwarp();
  if (g.d != nullptr) {
    uint16_t* d = g.d + (int64_t)mat * g.sd;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = (lane >> 2) + 8 * i, c4 = lane & 3;
      *reinterpret_cast<uint4*>(d + (int64_t)(row0 + r) * g.ldd + col + c4 * 8) =
          *reinterpret_cast<const uint4*>(stg + r * kStageRow + c4 * 16);
    }
  }
  if (g.dt != nullptr) {
    uint16_t* dt = g.dt + (int64_t)mat * g.sdt;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int j = (lane >> 2) + 8 * i, r8 = (lane & 3) * 8;
      uint32_t pk[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const uint32_t lo = *reinterpret_cast<const uint16_t*>(stg + (r8 + 2 * h) * kStageRow + j * 2);
        const uint32_t hi = *reinterpret_cast<const uint16_t*>(stg + (r8 + 2 * h + 1) * kStageRow + j * 2);
        pk[h] = lo | (hi << 16);
      }
      *reinterpret_cast<uint4*>(dt + (int64_t)(col + j) * g.lddt + row0 + r8) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
  }
  __syncwarp();  // the staging rows are rewritten by the next block
}

// The fused Muon update of a full 32 x 32 block of a wide matrix (o[i][j] is
// w[i][j]; rows row0.., columns col..), through the warp's staging rows: w is
// read and written back 8 rows x 128 B per instruction, the lane of row r
// applies w = fma(o * scale, -lr, w * (1 - lr wd)) to its own row in between
// (the same arithmetic as store_chunk), and the copy leaves 8 rows x 64 B.
__device__ __forceinline__ void update_chunk_staged(const Args& g, const float (&v)[32], uint8_t* stg, int mat,
                                                    int row0, int col, int lane) {
  float* w = g.upd_w[mat] + (int64_t)row0 * g.upd_cols + col;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = (lane >> 3) + 4 * i, c4 = (lane & 7) * 4;
    *reinterpret_cast<float4*>(stg + r * kStageRowF + c4 * 4) =
        *reinterpret_cast<const float4*>(w + (int64_t)r * g.upd_cols + c4);
  }
  __syncwarp();
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    float4* p = reinterpret_cast<float4*>(stg + lane * kStageRowF + u * 16);
    float4 x = *p;
    float rr[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
    for (int h = 0; h < 4; ++h)
      rr[h] = __fmaf_rn(__fmul_rn(v[4 * u + h], g.upd_scale), g.upd_neglr, __fmul_rn(rr[h], g.upd_cwd));
    *p = make_float4(rr[0], rr[1], rr[2], rr[3]);
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = (lane >> 3) + 4 * i, c4 = (lane & 7) * 4;
    *reinterpret_cast<float4*>(w + (int64_t)r * g.upd_cols + c4) =
        *reinterpret_cast<const float4*>(stg + r * kStageRowF + c4 * 4);
  }
  void* out = g.upd_out[mat];
  if (out != nullptr) {
    const int64_t base = (int64_t)row0 * g.upd_cols + col;
    if (g.upd_stage_out) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = (lane >> 2) + 8 * i, c8 = (lane & 3) * 8;
        const float4 x0 = *reinterpret_cast<const float4*>(stg + r * kStageRowF + c8 * 4);
        const float4 x1 = *reinterpret_cast<const float4*>(stg + r * kStageRowF + c8 * 4 + 16);
        const float a[4] = {x0.x, x0.y, x0.z, x0.w}, b[4] = {x1.x, x1.y, x1.z, x1.w};
        const int64_t e = base + (int64_t)r * g.upd_cols + c8;
        if (g.upd_odt == MB_BF16) {
          store4<MB_BF16>(out, e, a);
          store4<MB_BF16>(out, e + 4, b);
        } else {
          store4<MB_F16>(out, e, a);
          store4<MB_F16>(out, e + 4, b);
        }
      }
    } else {
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float4 x = *reinterpret_cast<const float4*>(stg + lane * kStageRowF + u * 16);
        const float a[4] = {x.x, x.y, x.z, x.w};
        const int64_t e = base + (int64_t)lane * g.upd_cols + 4 * u;
        if (g.upd_odt == MB_BF16) store4<MB_BF16>(out, e, a);
        else store4<MB_F16>(out, e, a);
      }
    }
  }
  __syncwarp();  // the staging rows are rewritten by the next block
}

// Pair mode: tile t -> (matrix, bm, bn) of 256 x 256 tiles (bm fastest);
// symmetric: column bn holds the tiles bm <= bn.
__device__ __forceinline__ void tile_coords_pair(const Args& g, int tb, int& mat, int& bm, int& bn) {
  mat = tb / g.n_tiles;
  const int t = tb - mat * g.n_tiles;
  const int mt = g.M / (2 * BM);
  if (!g.sym) {
    bm = t % mt;
    bn = t / mt;
    return;
  }
  int c = 0;
  for (bn = 0;; ++bn) {
    const int h = mt < bn + 1 ? mt : bn + 1;
    if (t < c + h) {
      bm = t - c;
      return;
    }
    c += h;
  }
}

template <bool kF16, bool kPair>
__global__ void __launch_bounds__(kGemmThreads, 1)
    k_gemm16(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Args g) {
  constexpr int ST = kPair ? STAGES_P : STAGES;
  constexpr int B_ST = kPair ? B_STAGE_P : B_STAGE;
  // both CTAs of a pair read the same flag, written before this launch: they return together
  if (g.skip != nullptr && *g.skip != 0) return;  // before any barrier or TMEM allocation
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + ST * A_STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + ST * B_ST);
  uint64_t* empty = full + ST;
  uint64_t* acc_full = empty + ST;       // [2]: MMA -> epilogue
  uint64_t* acc_empty = acc_full + 2;    // [2]: epilogue -> MMA (one arrival per epilogue warp, both CTAs in pairs)
  uint64_t* drain = acc_empty + 2;       // on abort: completion of every MMA issued
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* stage_rows = reinterpret_cast<uint8_t*>(smem + ST * (A_STAGE + B_ST)) + kBarrierBytes;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = g.K / BK;
  // pair mode: CTA rank in the pair, the pair's index and count
  const uint32_t rank = kPair ? cluster_rank() : 0;
  const int unit = kPair ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int n_units = kPair ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kPair ? 8 : 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    if constexpr (kPair) {
      // one warp of each CTA of the pair allocates together: the same columns in both
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"(TMEM_COLS)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"(TMEM_COLS)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
  }
  tc_fence_before();
  if constexpr (kPair) cluster_sync();  // both CTAs' barriers exist before either signals the other's
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int kit = 0;  // k-blocks issued so far (the ring runs on across tiles)
      const int total = g.n_tiles * g.batch;
      for (int t = unit; t < total && !*abort_flag; t += n_units) {
        int mat, bm, bn;
        if constexpr (kPair) tile_coords_pair(g, t, mat, bm, bn);
        else tile_coords(g, t, mat, bm, bn);
        for (int kb = 0; kb < KB; ++kb, ++kit) {
          const int s = kit % ST;
          const uint32_t round = kit / ST;
          if (!mbar_wait(&empty[s], (round & 1) ^ 1, abort_flag, g.fault.limit_ns)) break;
          if (t == g.fault.unit && kb == 0) continue;  // test-only: withhold; the MMA warp's wait expires
          if constexpr (kPair) {
            // both CTAs' loads complete on the even CTA's barrier, which expects the bytes of both
            const uint32_t bar = mapa_u32(smem_u32(&full[s]), 0);
            if (leader) mbar_expect_tx(&full[s], 2 * (A_STAGE + B_ST));
            tma_load_3d_pair(sA + s * A_STAGE, &tmA, bar, kb * BK, bm * 2 * BM + (int)rank * BM, mat);
            tma_load_3d_pair(sB + s * B_ST, &tmB, bar, kb * BK, bn * BN + (int)rank * BM, mat);
          } else {
            mbar_expect_tx(&full[s], A_STAGE + B_STAGE);
            tma_load_3d(sA + s * A_STAGE, &tmA, &full[s], kb * BK, bm * BM, mat);
            tma_load_3d(sB + s * B_STAGE, &tmB, &full[s], kb * BK, bn * BN, mat);
          }
        }
      }
      if (*abort_flag && (!kPair || leader)) {
        // Bounded wait for the loads still in flight (in pairs, both CTAs' land on the even CTA's barriers).
        const uint64_t t0 = globaltimer();
        for (int k = kit - ST > 0 ? kit - ST : 0; k < kit; ++k) {
          const int s = k % ST;
          const uint32_t round = k / ST;
          while (!mbar_try_wait(&full[s], round & 1) && globaltimer() - t0 < g.fault.limit_ns) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      int kit = 0, it = 0;
      const int total = g.n_tiles * g.batch;
      for (int t = unit; t < total && !*abort_flag; t += n_units, ++it) {
        const int a = it & 1;
        const uint32_t use = it >> 1;
        const bool free_acc = kPair ? mbar_wait_cluster(&acc_empty[a], (use & 1) ^ 1, abort_flag, g.fault.limit_ns)
                                    : mbar_wait(&acc_empty[a], (use & 1) ^ 1, abort_flag, g.fault.limit_ns);
        if (!free_acc) break;
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(a * BN);
        for (int kb = 0; kb < KB; ++kb, ++kit) {
          const int s = kit % ST;
          const uint32_t round = kit / ST;
          if (!mbar_wait(&full[s], round & 1, abort_flag, g.fault.limit_ns)) break;
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * A_STAGE), b0 = smem_u32(sB + s * B_ST);
          if constexpr (kPair) {
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              umma_pair(acc, sw128_desc(a0 + k * 32), sw128_desc(b0 + k * 32), idesc<kF16, 2 * BM>(),
                        (kb | k) != 0 ? 1u : 0u);
            umma_commit_both(&empty[s]);
          } else {
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              umma_16(acc, sw128_desc(a0 + k * 32), sw128_desc(b0 + k * 32), idesc<kF16>(), (kb | k) != 0 ? 1u : 0u);
            umma_commit(&empty[s]);
          }
        }
        if constexpr (kPair) {
          // an aborted tile is not handed over: the odd CTA cannot see this CTA's
          // abort flag, so its epilogue must time out rather than store the tile
          if (!*abort_flag) umma_commit_both(&acc_full[a]);
        } else {
          umma_commit(&acc_full[a]);
        }
      }
      if (*abort_flag) {
        // every MMA this thread issued completes (bounded) before the accumulators are freed
        if constexpr (kPair) umma_commit_pair(drain);
        else umma_commit(drain);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < g.fault.limit_ns) {
        }
      }
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may read
    uint8_t* stg = stage_rows + (warp - 2) * kStageWarp;
    int it = 0;
    const int total = g.n_tiles * g.batch;
    for (int t = unit; t < total; t += n_units, ++it) {
      const int a = it & 1;
      const uint32_t use = it >> 1;
      int ok = 0;
      if (lane == 0) ok = mbar_wait(&acc_full[a], use & 1, abort_flag, g.fault.limit_ns) && !*abort_flag;
      ok = __shfl_sync(0xffffffffu, ok, 0);  // warp-uniform: tcgen05.ld is .sync.aligned
      if (!ok) break;
      tc_fence_after();
      int mat, bm, bn;
      if constexpr (kPair) tile_coords_pair(g, t, mat, bm, bn);
      else tile_coords(g, t, mat, bm, bn);
      // this CTA's 128 rows of the tile (in pairs, the odd CTA holds rows 128..255)
      const int row0 = (kPair ? bm * 2 * BM + (int)rank * BM : bm * BM) + q * 32;
      const int row = row0 + lane;
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
          // the C block through the staging rows: coalesced in, one row per lane out
          stage_load_block(stg, g.c + (int64_t)mat * g.sc + (int64_t)row0 * g.ldc + col, g.ldc, lane);
          __syncwarp();
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 w4 = *reinterpret_cast<const uint4*>(stg + lane * kStageRow + u * 16);
            const uint32_t ww[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              v[u * 8 + 2 * h] = fmaf(g.beta, h2f<kF16>((uint16_t)(ww[h] & 0xffffu)), v[u * 8 + 2 * h]);
              v[u * 8 + 2 * h + 1] = fmaf(g.beta, h2f<kF16>((uint16_t)(ww[h] >> 16)), v[u * 8 + 2 * h + 1]);
            }
          }
          __syncwarp();  // every lane holds its C row: the staging rows may be rewritten
        }
        // symmetric outputs: a block entirely above the diagonal is stored whole
        // (and mirrored through dt), one entirely below is not stored at all
        const bool upper = row0 + 31 < col, lower = row0 > col + 31;
        if (g.stage && (!g.sym || upper)) {
          store_chunk_staged<kF16>(g, v, stg, mat, row0, col, lane);
        } else if (g.upd && !g.upd_tall && g.upd_vec && row0 + 32 <= g.upd_m && col + 32 <= g.upd_n) {
          update_chunk_staged(g, v, stg, mat, row0, col, lane);
        } else if (!(g.sym && lower)) {
          store_chunk<kF16>(g, v, mat, row, col);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (kPair) mbar_arrive_cluster(mapa_u32(smem_u32(&acc_empty[a]), 0));
        else mbar_arrive(&acc_empty[a]);
      }
    }
  }
  tc_fence_before();
  // pairs: neither CTA leaves (freeing shared memory that the pair's MMAs and
  // loads use) before the other is done; every wait before this is bounded
  if constexpr (kPair) cluster_sync();
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (kPair)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    else
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

// 3-D 16-bit tensor [batch][rows][cols], row pitch `ld` and matrix stride
// `bstride` (elements); box = 64 x box_rows x 1, 128B swizzle.
bool make_map(CUtensorMap* map, const void* base, int64_t batch, int64_t rows, int64_t cols, int64_t ld,
              int64_t bstride, int box_rows, bool f16) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(ld * 2), (cuuint64_t)((batch > 1 ? bstride : rows * ld) * 2)};
  cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base),
            dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            kRowBytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Pair mode unless MB_GEMM_PAIR=0 in the environment (read once per process).
bool pair_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("MB_GEMM_PAIR");
    return e == nullptr || e[0] != '0';
  }();
  return on;
}

// Co-resident CTA pairs of the pair kernel on this device (clusters of two live
// within one GPC), or 0 when none can be placed: the single-CTA kernel runs then.
int pair_units(bool f16, int sms) {
  static int units[2] = {-1, -1};
  int& n = units[f16 ? 1 : 0];
  if (n < 0) {
    cudaLaunchConfig_t occ = {};
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    occ.gridDim = dim3(2 * (sms / 2), 1, 1);
    occ.blockDim = dim3(kGemmThreads, 1, 1);
    occ.dynamicSmemBytes = SMEM_BYTES;
    occ.attrs = at;
    occ.numAttrs = 1;
    int c = 0;
    const cudaError_t rc =
        cudaOccupancyMaxActiveClusters(&c, f16 ? k_gemm16<true, true> : k_gemm16<false, true>, &occ);
    if (rc != cudaSuccess) cudaGetLastError();  // clear it: the single-CTA kernel takes over
    n = rc == cudaSuccess && c > 0 ? c : 0;
  }
  return n;
}

}  // namespace gemm

int gemm16(const GemmCall& q, cudaStream_t stream) {
  using namespace gemm;
  if (q.dtype != MB_BF16 && q.dtype != MB_F16) return MB_ERR_ARG;
  const bool f16 = q.dtype == MB_F16;
  const int64_t M = q.M, N = q.N, K = q.K;
  if (!q.a || !q.b || M <= 0 || N <= 0 || K <= 0 || q.batch <= 0) return MB_ERR_ARG;
  if (M % BM || N % BN || K % BK || M > (1 << 30) || N > (1 << 30)) return MB_ERR_ARG;
  if (!q.d && !q.dt && !q.df && !q.upd_w) return MB_ERR_ARG;
  if (q.batch > kMaxBatch) return MB_ERR_ARG;
  if (q.lda < K || q.ldb < K || (q.lda % 8) || (q.ldb % 8)) return MB_ERR_ALIGN;
  if (!aligned(q.a, 16) || !aligned(q.b, 16)) return MB_ERR_ALIGN;
  if (q.batch > 1 && (q.sa < M * q.lda || q.sb < N * q.ldb || q.sa % 8 || q.sb % 8)) return MB_ERR_ALIGN;
  if (q.c && (q.ldc < N || q.ldc % 8 || !aligned(q.c, 16) || q.sc % 8)) return MB_ERR_ALIGN;
  if (q.d && (q.ldd < N || q.ldd % 8 || !aligned(q.d, 16) || q.sd % 8)) return MB_ERR_ALIGN;
  if (q.dt && (q.lddt < M || !aligned(q.dt, 2))) return MB_ERR_ALIGN;
  if (q.df && (q.lddf < N || q.lddf % 4 || !aligned(q.df, 16) || q.sdf % 4)) return MB_ERR_ALIGN;
  bool upd_vec = q.upd_w != nullptr && q.upd_cols % 4 == 0;
  if (q.upd_w) {
    if (q.upd_m > M || q.upd_n > N || q.upd_cols <= 0) return MB_ERR_ARG;
    if (q.upd_out && q.upd_odt != MB_BF16 && q.upd_odt != MB_F16) return MB_ERR_ARG;
    for (int b = 0; b < q.batch; ++b) {
      if (!q.upd_w[b] || (q.upd_out && !q.upd_out[b])) return MB_ERR_ARG;
      upd_vec = upd_vec && aligned(q.upd_w[b], 16) && (!q.upd_out || aligned(q.upd_out[b], 8));
    }
  }
  // symmetric mode writes the lower triangle through dt == d (square output, no other outputs)
  if (q.sym && (M != N || !q.d || q.dt != q.d || q.lddt != q.ldd || q.sdt != q.sd || q.df || q.upd_w))
    return MB_ERR_ARG;
  static std::once_flag attr_once;
  static cudaError_t attr_rc = cudaSuccess;
  std::call_once(attr_once, [] {
    attr_rc = cudaFuncSetAttribute(k_gemm16<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (attr_rc == cudaSuccess)
      attr_rc = cudaFuncSetAttribute(k_gemm16<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (attr_rc == cudaSuccess)
      attr_rc = cudaFuncSetAttribute(k_gemm16<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (attr_rc == cudaSuccess)
      attr_rc = cudaFuncSetAttribute(k_gemm16<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  });
  if (attr_rc != cudaSuccess) return MB_ERR_CUDA;
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  // pair mode: 256-row tiles over CTA pairs
  const int pairs = pair_enabled() && M % (2 * BM) == 0 ? pair_units(f16, sms) : 0;
  const bool pair = pairs > 0;
  CUtensorMap ma, mbm;
  if (!make_map(&ma, q.a, q.batch, M, K, q.lda, q.sa, BM, f16) ||
      !make_map(&mbm, q.b, q.batch, N, K, q.ldb, q.sb, pair ? BM : BN, f16))
    return MB_ERR_CUDA;
  const int mt = (int)(M / (pair ? 2 * BM : BM)), nt = (int)(N / BN);
  int tiles = mt * nt;
  if (q.sym) {
    tiles = 0;
    for (int bn = 0; bn < nt; ++bn) {
      const int h = pair ? bn + 1 : 2 * bn + 2;  // tiles of column bn not entirely below the diagonal
      tiles += mt < h ? mt : h;
    }
  }
  if ((int64_t)tiles * q.batch > (int64_t)1 << 30) return MB_ERR_ARG;
  Args g{};
  g.M = (int)M; g.N = (int)N; g.K = (int)K;
  g.n_tiles = tiles; g.batch = q.batch; g.sym = q.sym ? 1 : 0;
  g.alpha = q.alpha; g.beta = q.beta; g.diag = q.diag;
  g.c = static_cast<const uint16_t*>(q.c); g.ldc = q.ldc; g.sc = q.sc;
  g.d = static_cast<uint16_t*>(q.d); g.ldd = q.ldd; g.sd = q.sd;
  g.dt = static_cast<uint16_t*>(q.dt); g.lddt = q.lddt; g.sdt = q.sdt;
  g.df = q.df; g.lddf = q.lddf; g.sdf = q.sdf;
  if (q.upd_w) {
    g.upd = 1; g.upd_odt = q.upd_odt; g.upd_tall = q.upd_tall ? 1 : 0; g.upd_vec = upd_vec ? 1 : 0;
    g.upd_m = q.upd_m; g.upd_n = q.upd_n; g.upd_cols = q.upd_cols;
    g.upd_scale = q.upd_scale; g.upd_cwd = q.upd_cwd; g.upd_neglr = q.upd_neglr;
    for (int b = 0; b < q.batch; ++b) {
      g.upd_w[b] = q.upd_w[b];
      g.upd_out[b] = q.upd_out ? q.upd_out[b] : nullptr;
    }
  }
  g.err = q.err;
  g.skip = q.skip;
  g.stage = q.d != nullptr && !q.df && !q.upd_w &&
            (q.dt == nullptr || (aligned(q.dt, 16) && q.lddt % 8 == 0 && q.sdt % 8 == 0));
  g.upd_stage_out = q.upd_out != nullptr && q.upd_cols % 8 == 0;
  for (int b = 0; b < q.batch && g.upd_stage_out; ++b) g.upd_stage_out = aligned(q.upd_out[b], 16);
  take_fault(kFaultGemm, &g.fault.unit, &g.fault.limit_ns);
  const int64_t work = (int64_t)tiles * q.batch;
  if (pair) {
    int units = (int)(work < pairs ? work : pairs);
    if (q.max_sms > 0 && units > q.max_sms / 2) units = q.max_sms / 2 > 0 ? q.max_sms / 2 : 1;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * units, 1, 1);
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cfg.stream = stream;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    const cudaError_t rc = f16 ? cudaLaunchKernelEx(&cfg, k_gemm16<true, true>, ma, mbm, g)
                               : cudaLaunchKernelEx(&cfg, k_gemm16<false, true>, ma, mbm, g);
    return rc == cudaSuccess && cudaGetLastError() == cudaSuccess ? MB_OK : MB_ERR_CUDA;
  }
  int grid = (int)(work < sms ? work : sms);
  if (q.max_sms > 0 && grid > q.max_sms) grid = q.max_sms;
  if (f16) k_gemm16<true, false><<<grid, kGemmThreads, SMEM_BYTES, stream>>>(ma, mbm, g);
  else k_gemm16<false, false><<<grid, kGemmThreads, SMEM_BYTES, stream>>>(ma, mbm, g);
  return cudaGetLastError() == cudaSuccess ? MB_OK : MB_ERR_CUDA;
}

}  // namespace mb

extern "C" MB_API int mb_gemm16(int32_t dtype, const void* a, int64_t lda, const void* b, int64_t ldb, int64_t m,
                                int64_t n, int64_t k, float alpha, float beta, const void* c, int64_t ldc, void* d,
                                int64_t ldd, void* dt, int64_t lddt, float* df, int64_t lddf, int32_t* err_flag,
                                mb_stream_t stream) {
  mb::GemmCall q{};
  q.dtype = dtype;
  q.a = a; q.lda = lda;
  q.b = b; q.ldb = ldb;
  q.M = m; q.N = n; q.K = k; q.batch = 1;
  q.alpha = alpha; q.beta = beta; q.diag = 0.0f;
  q.c = c; q.ldc = ldc;
  q.d = d; q.ldd = ldd;
  q.dt = dt; q.lddt = lddt;
  q.df = df; q.lddf = lddf;
  q.err = err_flag;
  return mb::gemm16(q, (cudaStream_t)stream);
}
