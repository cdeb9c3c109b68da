// Kernels 1 and 2 of the optimizer step: the fused multi-tensor AdamW update
// and the gradient statistics pass with its on-device finalize.
//
// Reference semantics (paths inside the MORPH project):
//   update     torch/optim/adam.py _single_tensor_adam (torch 2.11.0), as built at
//              streamtrain/optimizer.py:40 and stepped at optimizer.py:62 /
//              morph/training/runner.py:101; DiskState.update streamtrain/disk.py:207-215.
//   statistics streamtrain/disk.py:466-468 (FP64 squares), optimizer.py:50-51 (gate).
//   finalize   streamtrain/precision.py:9-14 (overflow/success), disk.py:482-489
//              (skip + backoff, clip), clip_grad.py:165-169 (torch clip coefficient).
//
// Layout: the plan's segments cover the parameters in a fixed order; each
// segment starts on a fresh 2048-element tile. A CTA sweeps a tile in two
// coalesced passes of 1024 elements (thread t owns elements 4t..4t+3 of each
// pass), so every warp-wide access is one contiguous 512 B (FP32) or 256 B
// (16-bit) run. The grid is persistent (CTAs resident on all SMs) and strides
// over tiles.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#include "mb_async.cuh"
#include "mb_common.cuh"

// Compile-time tuning knob: minimum resident CTAs per SM requested from ptxas
// for kernel 1 (caps its registers per thread).
#ifndef MB_APPLY_MIN_BLOCKS
#define MB_APPLY_MIN_BLOCKS 1
#endif

namespace mb {

int persistent_blocks(const void* kernel, int threads, size_t smem) {
  int dev = 0, sms = 0, per_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess) return 0;
  if (per_sm < 1) per_sm = 1;
  return sms * per_sm;
}

int grid_for(const void* fn, int64_t n_tiles) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  int blocks;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find({fn, dev});
    if (it == cache.end()) it = cache.emplace(std::make_pair(fn, dev), persistent_blocks(fn, kThreads, 0)).first;
    blocks = it->second;
  }
  int64_t b = blocks > 0 ? blocks : 148;
  if (b > n_tiles) b = n_tiles;
  return (int)(b < 1 ? 1 : b);
}

namespace {

constexpr int kMaxPeers = 15;  // other GPUs of one node a launch can write to

struct ApplyArgs {
  const mb_segment* segs;
  const mb_group* groups;
  const float2* seg_scal;  // per-segment {nss, bc2s} from the finalize
  const mb_step_state* state;
  int64_t tile_lo;         // first tile of the launch
  int64_t n_tiles;         // one past the last tile of the launch
  int32_t n_segs;
  // Peer copies (bulk kernel only): every low-precision value is also stored at
  // the same offset of n_peers other GPUs' buffers, i.e. at out + peer_delta[p]
  // bytes (the peers' buffers mapped into this process).
  int32_t n_peers;
  int64_t peer_delta[kMaxPeers];
  FaultPlan fault;  // test-only (bulk kernel): a withheld tile and the launch's wait bound
};

__device__ __forceinline__ StepScalars group_scalars(const mb_group& g, float2 ss) {
  StepScalars s;
  s.small = fabsf(g.omb1) < 0.5f;
  s.lw = s.small ? g.omb1 : __fsub_rn(g.omb1, 1.0f);
  s.cwd = g.cwd;
  s.b2 = g.beta2;
  s.omb2 = g.omb2;
  s.eps = g.eps;
  s.nss = ss.x;
  s.bc2s = ss.y;
  return s;
}

// Update the 4 elements at e (vector path) of one segment.
template <int GDT, int ODT>
__device__ __forceinline__ void apply_quad(const mb_segment& seg, int64_t e, const StepScalars& s,
                                           const GradPrep& prep) {
  float g[4];
  load4<GDT>(seg.g, e, g);
  float4 w = ld4f(seg.w + e), m = ld4f(seg.m + e), v = ld4f(seg.v + e);
  float ww[4] = {w.x, w.y, w.z, w.w}, mm[4] = {m.x, m.y, m.z, m.w}, vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) adam_elem(ww[j], mm[j], vv[j], prep(g[j]), s);
  st4f(seg.w + e, make_float4(ww[0], ww[1], ww[2], ww[3]));
  st4f(seg.m + e, make_float4(mm[0], mm[1], mm[2], mm[3]));
  st4f(seg.v + e, make_float4(vv[0], vv[1], vv[2], vv[3]));
  if constexpr (ODT != MB_NONE) store4<ODT>(seg.out, e, ww);
}

template <int GDT, int ODT>
__device__ __forceinline__ void apply_scalar(const mb_segment& seg, int64_t e, int64_t end,
                                             const StepScalars& s, const GradPrep& prep) {
  for (; e < end; ++e) {
    float w = seg.w[e], m = seg.m[e], v = seg.v[e];
    adam_elem(w, m, v, prep(load1<GDT>(seg.g, e)), s);
    seg.w[e] = w;
    seg.m[e] = m;
    seg.v[e] = v;
    if constexpr (ODT != MB_NONE) store1<ODT>(seg.out, e, w);
  }
}

__device__ __forceinline__ bool seg_vec_ok(const mb_segment& seg, int gdt, int odt) {
  bool ok = aligned(seg.w, 16) && aligned(seg.m, 16) && aligned(seg.v, 16);
  ok = ok && aligned(seg.g, gdt == MB_F32 ? 16 : 8);
  if (odt != MB_NONE) ok = ok && aligned(seg.out, 8);
  return ok;
}

// Process one tile of one segment: two coalesced sweeps of 1024 elements.
// When both of a thread's quads are in range, all eight loads are issued
// before any arithmetic or store (112 B in flight per thread for BF16 grads).
template <int GDT, int ODT>
__device__ __forceinline__ void apply_tile(const mb_segment& seg, int64_t tile_in_seg, bool vec,
                                           const StepScalars& s, const GradPrep& prep, int tid) {
  const int64_t e0 = tile_in_seg * kTile + tid * kQuad;
  const int64_t e1 = e0 + kHalf;
  if (vec && e1 + kQuad <= seg.numel) {
    float g0[4], g1[4];
    load4<GDT>(seg.g, e0, g0);
    load4<GDT>(seg.g, e1, g1);
    float4 w0 = ld4f(seg.w + e0), w1 = ld4f(seg.w + e1);
    float4 m0 = ld4f(seg.m + e0), m1 = ld4f(seg.m + e1);
    float4 v0 = ld4f(seg.v + e0), v1 = ld4f(seg.v + e1);
    float wa[4] = {w0.x, w0.y, w0.z, w0.w}, ma[4] = {m0.x, m0.y, m0.z, m0.w}, va[4] = {v0.x, v0.y, v0.z, v0.w};
    float wb[4] = {w1.x, w1.y, w1.z, w1.w}, mb_[4] = {m1.x, m1.y, m1.z, m1.w}, vb[4] = {v1.x, v1.y, v1.z, v1.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      adam_elem(wa[j], ma[j], va[j], prep(g0[j]), s);
      adam_elem(wb[j], mb_[j], vb[j], prep(g1[j]), s);
    }
    st4f(seg.w + e0, make_float4(wa[0], wa[1], wa[2], wa[3]));
    st4f(seg.m + e0, make_float4(ma[0], ma[1], ma[2], ma[3]));
    st4f(seg.v + e0, make_float4(va[0], va[1], va[2], va[3]));
    st4f(seg.w + e1, make_float4(wb[0], wb[1], wb[2], wb[3]));
    st4f(seg.m + e1, make_float4(mb_[0], mb_[1], mb_[2], mb_[3]));
    st4f(seg.v + e1, make_float4(vb[0], vb[1], vb[2], vb[3]));
    if constexpr (ODT != MB_NONE) {
      store4<ODT>(seg.out, e0, wa);
      store4<ODT>(seg.out, e1, wb);
    }
    return;
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    int64_t e = h ? e1 : e0;
    if (e >= seg.numel) continue;
    int64_t end = e + kQuad < seg.numel ? e + kQuad : seg.numel;
    if (vec && end - e == kQuad) apply_quad<GDT, ODT>(seg, e, s, prep);
    else apply_scalar<GDT, ODT>(seg, e, end, s, prep);
  }
}

// Kernel 1 (plan mode): every segment's scalars come from the finalize.
template <int GDT, int ODT>
__global__ void __launch_bounds__(kThreads, MB_APPLY_MIN_BLOCKS) k_adamw_apply(ApplyArgs a) {
  const mb_step_state* st = a.state;
  if (st->skip) return;
  GradPrep prep = make_prep(__double2float_rn(st->step_scale), st->clip_coef);
  int cur = -1;
  mb_segment seg;
  StepScalars s;
  bool vec = false;
  for (int64_t tile = a.tile_lo + blockIdx.x; tile < a.n_tiles; tile += gridDim.x) {
    int si = cur < 0 ? find_segment(a.segs, a.n_segs, tile) : cur;
    while (si + 1 < a.n_segs && __ldg(&a.segs[si + 1].tile_begin) <= tile) ++si;
    if (si != cur) {
      cur = si;
      seg = a.segs[si];
      s = group_scalars(a.groups[seg.group], a.seg_scal[si]);
      vec = seg_vec_ok(seg, GDT, ODT);
    }
    apply_tile<GDT, ODT>(seg, tile - seg.tile_begin, vec, s, prep, threadIdx.x);
  }
}

// Kernel 1, bulk-staged form (plan mode). One persistent CTA per SM: warp 0's
// lane 0 streams each tile's w, m, v and gradient into a ring of shared-memory
// stages with cp.async.bulk (completion counted in mbarrier transaction
// bytes); eight consumer warps read a stage into registers, release it, run
// the same element arithmetic and store w, m, v (and the low-precision copy)
// straight to global memory. The ring keeps up to kBulkStages tiles of reads in
// flight per SM independent of the consumers' registers. Tiles whose segment
// is not 16-byte aligned, or whose partial length is not a multiple of 8, take
// the direct-load path inside the consumers (the producer only signals them).
// Every wait is bounded; on expiry the CTA stops and records MB_ERR_TIMEOUT in
// the step state.
#ifndef MB_BULK_STAGES
#define MB_BULK_STAGES 3
#endif
#ifndef MB_BULK_WARPS
#define MB_BULK_WARPS 4
#endif
#ifndef MB_BULK_CTAS
#define MB_BULK_CTAS 2
#endif
#ifndef MB_BULK_L2_HINT
#define MB_BULK_L2_HINT 0  // 1: the producer's copies carry an L2 evict-first policy
#endif
constexpr int kBulkStages = MB_BULK_STAGES;        // ring depth (tiles)
constexpr int kBulkConsumerWarps = MB_BULK_WARPS;  // consumers; each thread takes kBulkQuads quads of a tile
constexpr int kBulkCtasPerSm = MB_BULK_CTAS;
constexpr int kBulkThreads = 32 * (kBulkConsumerWarps + 1);
constexpr int kBulkQuads = kTile / (kQuad * 32 * kBulkConsumerWarps);
static_assert(kBulkQuads * kQuad * 32 * kBulkConsumerWarps == kTile, "consumers must tile a tile exactly");

template <int GDT>
__host__ __device__ constexpr int bulk_stage_bytes() {
  return kTile * (12 + (GDT == MB_F32 ? 4 : 2));
}
template <int GDT>
__host__ __device__ constexpr int bulk_smem_bytes() {
  return kBulkStages * bulk_stage_bytes<GDT>() + 2 * kBulkStages * 8 + 16;
}

// Segment cursor of a CTA role: tiles only grow, so the segment advances; the
// next segment's first tile is cached, so most tiles touch no table entry.
struct SegCursor {
  int cur = -1;
  int64_t next_begin = -1;  // first tile of segment cur + 1 (INT64_MAX past the last)
  template <class Args>
  __device__ __forceinline__ bool advance(const Args& a, int64_t tile) {
    if (cur >= 0 && tile < next_begin) return false;
    int si = cur < 0 ? find_segment(a.segs, a.n_segs, tile) : cur;
    while (si + 1 < a.n_segs && __ldg(&a.segs[si + 1].tile_begin) <= tile) ++si;
    next_begin = si + 1 < a.n_segs ? __ldg(&a.segs[si + 1].tile_begin) : INT64_MAX;
    const bool changed = si != cur;
    cur = si;
    return changed;
  }
};

__device__ __forceinline__ bool bulk_ok(const mb_segment& seg, int gdt, int odt, int64_t n) {
  return seg_vec_ok(seg, gdt, odt) && aligned(seg.g, 16) && (n == kTile || n % 8 == 0);
}

template <int GDT, int ODT>
__global__ void __launch_bounds__(kBulkThreads, kBulkCtasPerSm) k_adamw_apply_bulk(ApplyArgs a) {
  constexpr int GB = GDT == MB_F32 ? 4 : 2;
  constexpr int STAGE = bulk_stage_bytes<GDT>();
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBulkStages * STAGE);
  uint64_t* empty = full + kBulkStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kBulkStages);
  mb_step_state* st = const_cast<mb_step_state*>(a.state);  // the plan's device record
  if (st->skip) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kBulkStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kBulkConsumerWarps);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();
  if (warp == 0) {
    if (lane == 0) {
      SegCursor sc_;
      mb_segment seg;
      int k = 0;
      int last_bulk[kBulkStages];  // per stage, the tile count k of its last bulk fill (-1: none)
#pragma unroll
      for (int i = 0; i < kBulkStages; ++i) last_bulk[i] = -1;
      for (int64_t tile = a.tile_lo + blockIdx.x; tile < a.n_tiles; tile += gridDim.x, ++k) {
        if (sc_.advance(a, tile)) seg = a.segs[sc_.cur];
        const int s = k % kBulkStages;
        if (!mbar_wait(&empty[s], ((k / kBulkStages) & 1) ^ 1, abort_flag, a.fault.limit_ns)) break;
        if (tile == a.fault.unit) continue;  // test-only: withhold this tile; its consumers' wait expires
        const int64_t t = tile - seg.tile_begin;
        const int64_t e = t * kTile;
        const int64_t rest = seg.numel - e;
        const int n = (int)(rest < kTile ? rest : kTile);
        if (bulk_ok(seg, GDT, ODT, n)) {
          uint8_t* base = smem + s * STAGE;
          mbar_expect_tx(&full[s], (uint32_t)n * (12 + GB));
#if MB_BULK_L2_HINT
          const uint64_t pol = l2_evict_first();
          bulk_load_hint(base, seg.w + e, n * 4, &full[s], pol);
          bulk_load_hint(base + kTile * 4, seg.m + e, n * 4, &full[s], pol);
          bulk_load_hint(base + kTile * 8, seg.v + e, n * 4, &full[s], pol);
          bulk_load_hint(base + kTile * 12, static_cast<const uint8_t*>(seg.g) + e * GB, n * GB, &full[s], pol);
#else
          bulk_load(base, seg.w + e, n * 4, &full[s]);
          bulk_load(base + kTile * 4, seg.m + e, n * 4, &full[s]);
          bulk_load(base + kTile * 8, seg.v + e, n * 4, &full[s]);
          bulk_load(base + kTile * 12, static_cast<const uint8_t*>(seg.g) + e * GB, n * GB, &full[s]);
#endif
          last_bulk[s] = k;
        } else {
          mbar_arrive(&full[s]);
        }
      }
      if (*abort_flag) {
        // give the copies still in flight (bounded) time to land before the CTA's shared memory goes away
#pragma unroll
        for (int i = 0; i < kBulkStages; ++i) {
          if (last_bulk[i] < 0) continue;
          const uint32_t parity = (last_bulk[i] / kBulkStages) & 1;
          const uint64_t t0 = globaltimer();
          while (!mbar_try_wait(&full[i], parity) && globaltimer() - t0 < a.fault.limit_ns) {
          }
        }
      }
    }
  } else {
    const int ct = threadIdx.x - 32;
    GradPrep prep = make_prep(__double2float_rn(st->step_scale), st->clip_coef);
    SegCursor sc_;
    mb_segment seg;
    StepScalars sc;
    int k = 0;
    for (int64_t tile = a.tile_lo + blockIdx.x; tile < a.n_tiles; tile += gridDim.x, ++k) {
      if (sc_.advance(a, tile)) {
        seg = a.segs[sc_.cur];
        sc = group_scalars(a.groups[seg.group], a.seg_scal[sc_.cur]);
      }
      const int s = k % kBulkStages;
      if (!mbar_wait(&full[s], (k / kBulkStages) & 1, abort_flag, a.fault.limit_ns)) break;
      const int64_t t = tile - seg.tile_begin;
      const int64_t e = t * kTile;
      const int64_t rest = seg.numel - e;
      const int n = (int)(rest < kTile ? rest : kTile);
      if (!bulk_ok(seg, GDT, ODT, n)) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        // the direct path covers a tile with 256 threads x 2 quads
        for (int part = ct; part < kThreads; part += 32 * kBulkConsumerWarps) {
          apply_tile<GDT, ODT>(seg, t, seg_vec_ok(seg, GDT, ODT), sc, prep, part);
          if constexpr (ODT != MB_NONE) {
            // replicate the copies this thread just wrote
            uint16_t* o = static_cast<uint16_t*>(seg.out);
            for (int h = 0; h < 2 && a.n_peers > 0; ++h) {
              const int64_t q = t * kTile + part * kQuad + h * kHalf;
              for (int64_t j = q; j < q + kQuad && j < seg.numel; ++j) {
                const uint16_t val = o[j];
                for (int pr = 0; pr < a.n_peers; ++pr)
                  *reinterpret_cast<uint16_t*>(reinterpret_cast<char*>(o + j) + a.peer_delta[pr]) = val;
              }
            }
          }
        }
        continue;
      }
      const uint8_t* base = smem + s * STAGE;
      float4 w4[kBulkQuads], m4[kBulkQuads], v4[kBulkQuads];
      float g4[kBulkQuads][4];
      bool in[kBulkQuads];
#pragma unroll
      for (int q = 0; q < kBulkQuads; ++q) {
        const int qe = (q * 32 * kBulkConsumerWarps + ct) * kQuad;  // element offset in the tile
        in[q] = qe < n;  // n % 8 == 0 or a full tile: a quad is all in or all out
        if (in[q]) {
          w4[q] = *reinterpret_cast<const float4*>(base + qe * 4);
          m4[q] = *reinterpret_cast<const float4*>(base + kTile * 4 + qe * 4);
          v4[q] = *reinterpret_cast<const float4*>(base + kTile * 8 + qe * 4);
          load4_any<GDT>(base + kTile * 12, qe, g4[q]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
      for (int q = 0; q < kBulkQuads; ++q) {
        if (!in[q]) continue;
        const int64_t ge = e + (q * 32 * kBulkConsumerWarps + ct) * kQuad;
        float ww[4] = {w4[q].x, w4[q].y, w4[q].z, w4[q].w}, mm[4] = {m4[q].x, m4[q].y, m4[q].z, m4[q].w};
        float vv[4] = {v4[q].x, v4[q].y, v4[q].z, v4[q].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) adam_elem(ww[j], mm[j], vv[j], prep(g4[q][j]), sc);
        st4f(seg.w + ge, make_float4(ww[0], ww[1], ww[2], ww[3]));
        st4f(seg.m + ge, make_float4(mm[0], mm[1], mm[2], mm[3]));
        st4f(seg.v + ge, make_float4(vv[0], vv[1], vv[2], vv[3]));
        if constexpr (ODT != MB_NONE) {
          store4<ODT>(seg.out, ge, ww);
          for (int pr = 0; pr < a.n_peers; ++pr)
            store4<ODT>(static_cast<char*>(seg.out) + a.peer_delta[pr], ge, ww);
        }
      }
    }
    if (a.n_peers > 0) __threadfence_system();  // peer stores ordered before whatever signals completion
  }
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) atomicExch(&st->status, MB_ERR_TIMEOUT);
}

// Kernel 1 (single tensor, host scalars): DiskState.update on device memory.
template <int GDT, int ODT>
__global__ void __launch_bounds__(kThreads) k_adamw_update(mb_segment seg, int64_t n_tiles,
                                                            mb_host_scalars hs) {
  StepScalars s;
  s.small = fabsf(hs.omb1) < 0.5f;
  s.lw = s.small ? hs.omb1 : __fsub_rn(hs.omb1, 1.0f);
  s.cwd = hs.cwd; s.b2 = hs.beta2; s.omb2 = hs.omb2; s.eps = hs.eps; s.nss = hs.nss; s.bc2s = hs.bc2s;
  GradPrep prep = make_prep(hs.scale, hs.coef);
  bool vec = seg_vec_ok(seg, GDT, ODT);
  for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x)
    apply_tile<GDT, ODT>(seg, tile, vec, s, prep, threadIdx.x);
}

// ------------------------------------------------------------- kernel 2 --

struct StatsArgs {
  const mb_segment* segs;
  int64_t n_tiles;
  int32_t n_segs;
  mb_adamw_plan plan;      // for the fused finalize
  mb_finalize_opts fin;
  int32_t fuse_finalize;
  int32_t unscale;         // divide by state.scale
  FaultPlan fault;         // test-only (bulk kernel): a withheld chunk and the launch's wait bound
};

// A CTA of kernel 2 whose bounded wait expired reports this many nonfinite
// elements; the finalize reads any count at or above it as a time-out (sums of
// real counts over ranks stay far below it).
constexpr double kTimeoutMark = 1099511627776.0;  // 2^40

// Block-wide sum of (a, b) in a fixed order; result valid in thread 0. Any
// block size that is a multiple of 32, up to 1024.
__device__ __forceinline__ double2 block_sum2(double a, double b) {
  __shared__ double2 red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_down_sync(0xffffffffu, a, o);
    b += __shfl_down_sync(0xffffffffu, b, o);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  if (lane == 0) red[warp] = make_double2(a, b);
  __syncthreads();
  double2 r = make_double2(0.0, 0.0);
  if (warp == 0) {
    r = lane < warps ? red[lane] : make_double2(0.0, 0.0);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      r.x += __shfl_down_sync(0xffffffffu, r.x, o);
      r.y += __shfl_down_sync(0xffffffffu, r.y, o);
    }
  }
  __syncthreads();
  return r;
}

// Loss-scale transition, skip decision, clip coefficient (thread 0), then clock
// advance and per-segment scalars (all threads). One CTA runs this.
__device__ void finalize_block(const mb_adamw_plan& p, const mb_finalize_opts& f) {
  __shared__ int s_skip;
  mb_step_state* st = p.state;
  if (threadIdx.x == 0) {
    double sumsq = st->sumsq;
    bool found = st->nonfinite != 0.0 || !isfinite(sumsq);
    int skip = 0, status = MB_OK;
    double used = (f.flags & MB_FIN_LOSS_SCALE) ? st->scale : 1.0;
    if (st->nonfinite >= kTimeoutMark) {
      skip = 1;  // the statistics pass gave up: no norm, no update, loss scale unchanged
      status = MB_ERR_TIMEOUT;
    } else if (f.flags & MB_FIN_LOSS_SCALE) {
      if (found) {
        skip = 1;
        if (st->scale <= 1.0) {
          status = MB_ERR_OVERFLOW_MIN_SCALE;  // precision.py:10: state unchanged
        } else {
          st->scale = fmax(1.0, st->scale * f.backoff);  // precision.py:11
          st->good_steps = 0;
        }
      } else {
        st->good_steps += 1;  // precision.py:13-14
        if (st->good_steps >= st->growth_interval) {
          st->scale = fmin(st->scale * f.growth, st->max_scale);
          st->good_steps = 0;
        }
      }
    } else if (found && (f.flags & MB_FIN_GATE)) {
      skip = 1;
      status = MB_ERR_NONFINITE;  // optimizer.py:50-51
    }
    double norm = sqrt(sumsq);
    float coef = 1.0f;
    if (!skip && (f.flags & MB_FIN_CLIP_TORCH)) {
      // clip_grad.py:165-169: (norm + 1e-6).reciprocal() * max_norm, clamp(max=1)
      float t = __fadd_rn(__double2float_rn(norm), 1e-6f);
      float c = __fmul_rn(__frcp_rn(t), __double2float_rn(f.max_norm));
      coef = c < 1.0f ? c : 1.0f;
    } else if (!skip && (f.flags & MB_FIN_CLIP_DISK)) {
      double c = fmin(1.0, f.max_norm / (norm + 1e-6));  // disk.py:489
      coef = __double2float_rn(c);
    }
    st->norm = norm;
    st->step_scale = used;
    st->clip_coef = coef;
    st->skip = skip;
    st->status = status;
    if (skip) st->steps_skipped += 1; else st->steps_applied += 1;
    s_skip = skip;
  }
  __syncthreads();
  float2* seg_scal = reinterpret_cast<float2*>(static_cast<char*>(p.workspace) + kSegScalOffset);
  for (int i = threadIdx.x; i < p.n_segs; i += blockDim.x) {
    mb_segment seg = p.segs[i];
    int32_t t = p.clocks[seg.clock];
    if (!s_skip) {
      t += 1;
      p.clocks[seg.clock] = t;
    }
    mb_group g = p.groups[seg.group];
    int64_t tt = t < p.bc_len ? t : p.bc_len - 1;
    if (tt < 0) tt = 0;
    double bc1 = p.bc[(2 * (int64_t)g.table) * p.bc_len + tt];
    double bc2s = p.bc[(2 * (int64_t)g.table + 1) * p.bc_len + tt];
    seg_scal[i] = make_float2(__double2float_rn(-(g.lr / bc1)), __double2float_rn(bc2s));
  }
}

// Kernel 2. Each CTA owns a contiguous run of tiles and reads it with one
// 16-byte load per thread per tile (8 BF16/FP16 or 4+4 FP32 elements), four
// tiles in flight per iteration. Squares are accumulated in FP64; a nonfinite
// gradient makes the FP64 sum nonfinite (finite squares cannot overflow it:
// 2^33 elements x FLT_MAX^2 < DBL_MAX), so finiteness is tested once per
// partial instead of per element.
template <int GDT>
__device__ __forceinline__ void stats_elems(const uint4& q, bool unscale, const GradPrep& prep, double& acc) {
  float x[8];
  int n = 8;
  if (GDT == MB_BF16) {
    const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      x[2 * j] = __uint_as_float(u[j] << 16);
      x[2 * j + 1] = __uint_as_float(u[j] & 0xffff0000u);
    }
  } else if (GDT == MB_F16) {
    const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[j]));
      x[2 * j] = f.x;
      x[2 * j + 1] = f.y;
    }
  } else {
    x[0] = __uint_as_float(q.x); x[1] = __uint_as_float(q.y);
    x[2] = __uint_as_float(q.z); x[3] = __uint_as_float(q.w);
    n = 4;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (j < n) {
      float y = unscale ? prep(x[j]) : x[j];
      double d = (double)y;
      acc = __fma_rn(d, d, acc);
    }
  }
}

// Per-CTA partial {sum of squares, nonfinite} of kernel 2, the last CTA's
// fixed-order reduction into the step state, and the optional fused finalize.
__device__ void stats_tail(const StatsArgs& a, double acc, bool aborted = false) {
  mb_step_state* st = a.plan.state;
  double2 r = block_sum2(acc, 0.0);
  char* ws = static_cast<char*>(a.plan.workspace);
  double2* partials = reinterpret_cast<double2*>(ws);
  unsigned int* ticket = reinterpret_cast<unsigned int*>(ws + kTicketOffset);
  __shared__ unsigned int s_last;
  if (threadIdx.x == 0) {
    r.y = aborted ? kTimeoutMark : (isfinite(r.x) ? 0.0 : 1.0);
    partials[blockIdx.x] = r;
    __threadfence();
    s_last = (atomicAdd(ticket, 1u) == gridDim.x - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // Last CTA: fixed-order reduction of the partials (deterministic for a grid).
  double a0 = 0.0, b0 = 0.0;
  for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) {
    double2 qq = __ldcg(&partials[i]);
    a0 += qq.x;
    b0 += qq.y;
  }
  double2 tot = block_sum2(a0, b0);
  if (threadIdx.x == 0) {
    st->sumsq = tot.x;
    st->nonfinite = tot.y;
    *ticket = 0u;
  }
  __syncthreads();
  if (a.fuse_finalize) {
    __threadfence_block();
    finalize_block(a.plan, a.fin);
  }
}

#ifndef MB_STATS_U
#define MB_STATS_U 4
#endif
template <int GDT, bool UNSCALE>
__global__ void __launch_bounds__(kThreads) k_grad_stats(StatsArgs a) {
  constexpr int kU = MB_STATS_U;                         // tiles in flight per iteration
  constexpr int kEpl = GDT == MB_F32 ? 4 : 8;            // elements per 16-byte load
  constexpr int kLoads = (kTile / kThreads) / kEpl;      // 16-byte loads per thread per tile
  using T = typename Elem<GDT>::T;
  mb_step_state* st = a.plan.state;
  GradPrep prep = make_prep(UNSCALE ? __double2float_rn(st->scale) : 1.0f, 1.0f);
  double acc = 0.0;
  const int64_t per = (a.n_tiles + gridDim.x - 1) / gridDim.x;
  const int64_t t0 = (int64_t)blockIdx.x * per;
  const int64_t t1 = t0 + per < a.n_tiles ? t0 + per : a.n_tiles;
  int si = t0 < a.n_tiles ? find_segment(a.segs, a.n_segs, t0) : 0;
  for (int64_t t = t0; t < t1; t += kU) {
    uint4 q[kU][kLoads];
    const T* gp[kU];
    int64_t base[kU], nel[kU];
    bool full[kU];
#pragma unroll
    for (int k = 0; k < kU; ++k) {
      const int64_t tile = t + k;
      gp[k] = nullptr;
      full[k] = false;
      base[k] = 0;
      nel[k] = 0;
      if (tile < t1) {
        while (si + 1 < a.n_segs && __ldg(&a.segs[si + 1].tile_begin) <= tile) ++si;
        const mb_segment* sg = &a.segs[si];
        gp[k] = reinterpret_cast<const T*>(__ldg(reinterpret_cast<const unsigned long long*>(&sg->g)));
        nel[k] = __ldg(&sg->numel);
        base[k] = (tile - __ldg(&sg->tile_begin)) * kTile;  // first element of the tile
        full[k] = base[k] + kTile <= nel[k] && aligned(gp[k], 16);
        if (full[k]) {
          // load l of thread t covers elements base + (l*kThreads + t)*kEpl .. +kEpl
#pragma unroll
          for (int l = 0; l < kLoads; ++l)
            q[k][l] = __ldcs(reinterpret_cast<const uint4*>(gp[k] + base[k] + (int64_t)(l * kThreads + threadIdx.x) * kEpl));
        }
      }
    }
#pragma unroll
    for (int k = 0; k < kU; ++k) {
      if (full[k]) {
#pragma unroll
        for (int l = 0; l < kLoads; ++l) stats_elems<GDT>(q[k][l], UNSCALE, prep, acc);
      } else if (gp[k] != nullptr) {
        for (int l = 0; l < kLoads; ++l) {
          int64_t e = base[k] + (int64_t)(l * kThreads + threadIdx.x) * kEpl;
          int64_t end = e + kEpl < nel[k] ? e + kEpl : nel[k];
          for (; e < end; ++e) {
            float y = to_f32(gp[k][e]);
            if (UNSCALE) y = prep(y);
            double d = (double)y;
            acc = __fma_rn(d, d, acc);
          }
        }
      }
    }
  }
  stats_tail(a, acc);
}

// Kernel 2, bulk-staged form (the default). One persistent CTA per SM (two
// when shared memory allows) walks a contiguous run of tiles. Lane 0 of warp 0
// streams chunks -- up to kSBTiles tiles of one segment -- of gradient bytes
// into a ring of shared-memory stages with cp.async.bulk; the consumer warps
// read 16-byte words from the stage and accumulate the FP64 sum of squares
// (the same per-element arithmetic as k_grad_stats). Chunks that are not
// 16-byte aligned or sized are read directly from global memory. Every wait is
// bounded; a CTA that gives up counts its partial as nonfinite, so the step is
// refused rather than clipped with a wrong norm.
constexpr int kSBStages = 4;
constexpr int kSBTiles = 4;
constexpr int kSBWarps = 8;
constexpr int kSBThreads = 32 * (kSBWarps + 1);

template <int GDT>
__host__ __device__ constexpr int sb_stage_bytes() {
  return kSBTiles * kTile * (GDT == MB_F32 ? 4 : 2);
}
template <int GDT>
__host__ __device__ constexpr int sb_smem_bytes() {
  return kSBStages * sb_stage_bytes<GDT>() + 2 * kSBStages * 8 + 16;
}

struct StatsChunk {
  const uint8_t* g;  // first byte of the chunk
  int64_t n;         // elements
  int tiles;         // tiles covered
  bool bulk;
};

// The chunk starting at tile t of this CTA's run [.., t1) (same on both roles).
template <int GDT>
__device__ __forceinline__ StatsChunk stats_chunk(const StatsArgs& a, SegCursor& cur, mb_segment& seg,
                                                  int64_t t, int64_t t1) {
  constexpr int GB = GDT == MB_F32 ? 4 : 2;
  if (cur.advance(a, t)) seg = a.segs[cur.cur];
  int64_t tiles = cur.next_begin - t;
  if (t1 - t < tiles) tiles = t1 - t;
  if (tiles > kSBTiles) tiles = kSBTiles;
  const int64_t e0 = (t - seg.tile_begin) * kTile;
  int64_t n = seg.numel - e0;
  if (n > tiles * kTile) n = tiles * kTile;
  StatsChunk c;
  c.g = static_cast<const uint8_t*>(seg.g) + e0 * GB;
  c.n = n;
  c.tiles = (int)tiles;
  c.bulk = aligned(c.g, 16) && (n * GB) % 16 == 0 && n > 0;
  return c;
}

template <int GDT, bool UNSCALE>
__global__ void __launch_bounds__(kSBThreads) k_grad_stats_bulk(StatsArgs a) {
  constexpr int GB = GDT == MB_F32 ? 4 : 2;
  constexpr int STAGE = sb_stage_bytes<GDT>();
  using T = typename Elem<GDT>::T;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kSBStages * STAGE);
  uint64_t* empty = full + kSBStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kSBStages);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kSBStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kSBWarps);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();
  const int64_t per = (a.n_tiles + gridDim.x - 1) / gridDim.x;
  const int64_t t0 = (int64_t)blockIdx.x * per;
  const int64_t t1 = t0 + per < a.n_tiles ? t0 + per : a.n_tiles;
  double acc = 0.0;
  if (warp == 0) {
    if (lane == 0) {
      SegCursor cur;
      mb_segment seg;
      int k = 0;
      int last_bulk[kSBStages];
#pragma unroll
      for (int i = 0; i < kSBStages; ++i) last_bulk[i] = -1;
      for (int64_t t = t0; t < t1; ++k) {
        const StatsChunk c = stats_chunk<GDT>(a, cur, seg, t, t1);
        const int64_t first = t;
        t += c.tiles;
        const int s = k % kSBStages;
        if (!mbar_wait(&empty[s], ((k / kSBStages) & 1) ^ 1, abort_flag, a.fault.limit_ns)) break;
        if (first == a.fault.unit) continue;  // test-only: withhold this chunk; its consumers' wait expires
        if (c.bulk) {
          mbar_expect_tx(&full[s], (uint32_t)(c.n * GB));
          bulk_load(smem + s * STAGE, c.g, (uint32_t)(c.n * GB), &full[s]);
          last_bulk[s] = k;
        } else {
          mbar_arrive(&full[s]);
        }
      }
      if (*abort_flag) {
#pragma unroll
        for (int i = 0; i < kSBStages; ++i) {
          if (last_bulk[i] < 0) continue;
          const uint32_t parity = (last_bulk[i] / kSBStages) & 1;
          const uint64_t w0 = globaltimer();
          while (!mbar_try_wait(&full[i], parity) && globaltimer() - w0 < a.fault.limit_ns) {
          }
        }
      }
    }
  } else {
    const int ct = threadIdx.x - 32;
    constexpr int nthr = 32 * kSBWarps;
    mb_step_state* st = a.plan.state;
    const GradPrep prep = make_prep(UNSCALE ? __double2float_rn(st->scale) : 1.0f, 1.0f);
    SegCursor cur;
    mb_segment seg;
    int k = 0;
    for (int64_t t = t0; t < t1; ++k) {
      const StatsChunk c = stats_chunk<GDT>(a, cur, seg, t, t1);
      t += c.tiles;
      const int s = k % kSBStages;
      if (!mbar_wait(&full[s], (k / kSBStages) & 1, abort_flag, a.fault.limit_ns)) break;
      if (c.bulk) {
        const uint4* words = reinterpret_cast<const uint4*>(smem + s * STAGE);
        const int nw = (int)(c.n * GB / 16);
        for (int w = ct; w < nw; w += nthr) stats_elems<GDT>(words[w], UNSCALE, prep, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      } else {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        const T* gp = reinterpret_cast<const T*>(c.g);
        for (int64_t e = ct; e < c.n; e += nthr) {
          float y = to_f32(gp[e]);
          if (UNSCALE) y = prep(y);
          const double d = (double)y;
          acc = __fma_rn(d, d, acc);
        }
      }
    }
  }
  __syncthreads();
  // a CTA that gave up refuses the step: its partial reports a time-out (see kTimeoutMark)
  const bool aborted = *abort_flag != 0;
  stats_tail(a, aborted ? 0.0 : acc, aborted);
}

__global__ void __launch_bounds__(kThreads) k_step_finalize(mb_adamw_plan p, mb_finalize_opts f) {
  finalize_block(p, f);
}

// ----------------------------------------------------------- dispatch ----

using ApplyFn = void (*)(ApplyArgs);
using UpdateFn = void (*)(mb_segment, int64_t, mb_host_scalars);

template <int GDT>
ApplyFn pick_apply(int odt) {
  switch (odt) {
    case MB_NONE: return &k_adamw_apply<GDT, MB_NONE>;
    case MB_F16: return &k_adamw_apply<GDT, MB_F16>;
    case MB_BF16: return &k_adamw_apply<GDT, MB_BF16>;
    default: return nullptr;
  }
}
ApplyFn pick_apply(int gdt, int odt) {
  switch (gdt) {
    case MB_F32: return pick_apply<MB_F32>(odt);
    case MB_F16: return pick_apply<MB_F16>(odt);
    case MB_BF16: return pick_apply<MB_BF16>(odt);
    default: return nullptr;
  }
}
struct BulkFn {
  ApplyFn fn;
  int smem;
};
template <int GDT>
BulkFn pick_apply_bulk(int odt) {
  switch (odt) {
    case MB_NONE: return {&k_adamw_apply_bulk<GDT, MB_NONE>, bulk_smem_bytes<GDT>()};
    case MB_F16: return {&k_adamw_apply_bulk<GDT, MB_F16>, bulk_smem_bytes<GDT>()};
    case MB_BF16: return {&k_adamw_apply_bulk<GDT, MB_BF16>, bulk_smem_bytes<GDT>()};
    default: return {nullptr, 0};
  }
}
BulkFn pick_apply_bulk(int gdt, int odt) {
  switch (gdt) {
    case MB_F32: return pick_apply_bulk<MB_F32>(odt);
    case MB_F16: return pick_apply_bulk<MB_F16>(odt);
    case MB_BF16: return pick_apply_bulk<MB_BF16>(odt);
    default: return {nullptr, 0};
  }
}

// Kernel 1's form: the bulk-staged kernel unless MB_APPLY_KERNEL=direct
// selects the register-staged one (read once).
bool use_bulk_apply() {
  static const bool bulk = [] {
    const char* e = getenv("MB_APPLY_KERNEL");
    return !(e && strcmp(e, "direct") == 0);
  }();
  return bulk;
}

// Opt a bulk kernel into its dynamic shared memory (once per kernel and device).
bool bulk_ready(const void* fn, int smem) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, bool> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_pair(fn, dev);
  auto it = done.find(key);
  if (it != done.end()) return it->second;
  bool ok = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) == cudaSuccess;
  done[key] = ok;
  return ok;
}

int sm_count() {
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (sms[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    sms[dev] = n > 0 ? n : 148;
  }
  return sms[dev];
}

template <int GDT>
UpdateFn pick_update(int odt) {
  switch (odt) {
    case MB_NONE: return &k_adamw_update<GDT, MB_NONE>;
    case MB_F16: return &k_adamw_update<GDT, MB_F16>;
    case MB_BF16: return &k_adamw_update<GDT, MB_BF16>;
    default: return nullptr;
  }
}
UpdateFn pick_update(int gdt, int odt) {
  switch (gdt) {
    case MB_F32: return pick_update<MB_F32>(odt);
    case MB_F16: return pick_update<MB_F16>(odt);
    case MB_BF16: return pick_update<MB_BF16>(odt);
    default: return nullptr;
  }
}
using StatsFn = void (*)(StatsArgs);

struct StatsBulk {
  StatsFn fn;
  int smem;
};
StatsBulk pick_stats_bulk(int gdt, bool unscale) {
  switch (gdt) {
    case MB_F32:
      return {unscale ? &k_grad_stats_bulk<MB_F32, true> : &k_grad_stats_bulk<MB_F32, false>, sb_smem_bytes<MB_F32>()};
    case MB_F16:
      return {unscale ? &k_grad_stats_bulk<MB_F16, true> : &k_grad_stats_bulk<MB_F16, false>, sb_smem_bytes<MB_F16>()};
    case MB_BF16:
      return {unscale ? &k_grad_stats_bulk<MB_BF16, true> : &k_grad_stats_bulk<MB_BF16, false>,
              sb_smem_bytes<MB_BF16>()};
    default: return {nullptr, 0};
  }
}

// Kernel 2's form: bulk-staged unless MB_STATS_KERNEL=direct (read once).
bool use_bulk_stats() {
  static const bool bulk = [] {
    const char* e = getenv("MB_STATS_KERNEL");
    return !(e && strcmp(e, "direct") == 0);
  }();
  return bulk;
}
StatsFn pick_stats(int gdt, bool unscale) {
  switch (gdt) {
    case MB_F32: return unscale ? &k_grad_stats<MB_F32, true> : &k_grad_stats<MB_F32, false>;
    case MB_F16: return unscale ? &k_grad_stats<MB_F16, true> : &k_grad_stats<MB_F16, false>;
    case MB_BF16: return unscale ? &k_grad_stats<MB_BF16, true> : &k_grad_stats<MB_BF16, false>;
    default: return nullptr;
  }
}

int launch_status() { return cudaGetLastError() == cudaSuccess ? MB_OK : MB_ERR_CUDA; }

}  // namespace

int check_plan(const mb_adamw_plan* p) {
  if (!p || !p->segs || !p->groups || !p->bc || !p->clocks || !p->workspace || !p->state) return MB_ERR_ARG;
  if (p->n_segs <= 0 || p->n_groups <= 0 || p->n_tiles <= 0 || p->bc_len <= 0) return MB_ERR_ARG;
  if (p->grad_dtype < MB_F32 || p->grad_dtype > MB_BF16) return MB_ERR_ARG;
  if (p->out_dtype != MB_NONE && p->out_dtype != MB_F16 && p->out_dtype != MB_BF16) return MB_ERR_ARG;
  if (!aligned(p->workspace, 256) || !aligned(p->state, 16)) return MB_ERR_ALIGN;
  return MB_OK;
}

int check_fin(const mb_finalize_opts* f) {
  if (!f) return MB_ERR_ARG;
  if (f->flags & ~(MB_FIN_LOSS_SCALE | MB_FIN_GATE | MB_FIN_CLIP_TORCH | MB_FIN_CLIP_DISK)) return MB_ERR_ARG;
  if ((f->flags & MB_FIN_CLIP_TORCH) && (f->flags & MB_FIN_CLIP_DISK)) return MB_ERR_ARG;
  if ((f->flags & (MB_FIN_CLIP_TORCH | MB_FIN_CLIP_DISK)) && !(f->max_norm > 0)) return MB_ERR_ARG;
  if ((f->flags & MB_FIN_LOSS_SCALE) && !(f->backoff > 0 && f->growth >= 1)) return MB_ERR_ARG;
  return MB_OK;
}

}  // namespace mb

using namespace mb;

extern "C" {

MB_API int mb_version(void) { return 1; }

MB_API const char* mb_status_string(int status) {
  switch (status) {
    case MB_OK: return "ok";
    case MB_ERR_ARG: return "invalid argument";
    case MB_ERR_ALIGN: return "misaligned pointer";
    case MB_ERR_CUDA: return "CUDA error";
    case MB_ERR_OVERFLOW_MIN_SCALE: return "FP16 overflow at minimum loss scale; state unchanged";
    case MB_ERR_NONFINITE: return "nonfinite gradient; optimizer not updated";
    case MB_ERR_TIMEOUT: return "bounded wait expired";
    case MB_ERR_INDEX: return "row index out of range";
    case MB_ERR_UNREPRESENTABLE: return "weights cannot be represented by finite FP16";
    case MB_ERR_TOO_LARGE: return "plan exceeds the 8192-segment no-allocation scratch";
    default: return "unknown status";
  }
}

MB_API int mb_segments_plan(mb_segment* segs, int32_t n, int64_t* n_tiles) {
  if (!segs || n <= 0 || !n_tiles) return MB_ERR_ARG;
  int64_t t = 0;
  for (int32_t i = 0; i < n; ++i) {
    if (segs[i].numel <= 0 || !segs[i].w || !segs[i].m || !segs[i].v || !segs[i].g) return MB_ERR_ARG;
    segs[i].tile_begin = t;
    t += (segs[i].numel + kTile - 1) / kTile;
  }
  *n_tiles = t;
  return MB_OK;
}

MB_API size_t mb_workspace_bytes(int32_t n_segs) { return workspace_bytes(n_segs); }

MB_API int mb_step_state_init(mb_step_state* s, double scale, int64_t growth_interval) {
  if (!s || !(scale > 0) || growth_interval <= 0) return MB_ERR_ARG;
  *s = mb_step_state{};
  s->scale = scale;
  s->step_scale = 1.0;
  s->growth_interval = growth_interval;
  s->max_scale = 65536.0;
  s->clip_coef = 1.0f;
  return MB_OK;
}

MB_API int mb_grad_stats(const mb_adamw_plan* p, const mb_finalize_opts* fin, mb_stream_t stream) {
  int rc = check_plan(p);
  if (rc) return rc;
  if (fin && (rc = check_fin(fin))) return rc;
  const bool unscale = fin ? (fin->flags & MB_FIN_LOSS_SCALE) != 0 : false;
  StatsFn fn = pick_stats(p->grad_dtype, unscale);
  StatsArgs a{};
  take_fault(kFaultStats, &a.fault.unit, &a.fault.limit_ns);
  a.segs = p->segs;
  a.n_tiles = p->n_tiles;
  a.n_segs = p->n_segs;
  a.plan = *p;
  a.fin = fin ? *fin : mb_finalize_opts{};
  a.fuse_finalize = fin != nullptr;
  a.unscale = unscale;
  StatsBulk bulk = pick_stats_bulk(p->grad_dtype, unscale);
  if (use_bulk_stats() && bulk.fn && bulk_ready(reinterpret_cast<const void*>(bulk.fn), bulk.smem)) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, bulk.fn, kSBThreads, bulk.smem) != cudaSuccess ||
        per_sm < 1)
      per_sm = 1;
    int64_t grid = (int64_t)sm_count() * per_sm;
    if (grid > p->n_tiles) grid = p->n_tiles;
    if (grid > kMaxStatsBlocks) grid = kMaxStatsBlocks;
    if (grid < 1) grid = 1;
    bulk.fn<<<(int)grid, kSBThreads, bulk.smem, (cudaStream_t)stream>>>(a);
    return launch_status();
  }
  int grid = grid_for(reinterpret_cast<const void*>(fn), p->n_tiles);
  if (grid > kMaxStatsBlocks) grid = kMaxStatsBlocks;
  fn<<<grid, kThreads, 0, (cudaStream_t)stream>>>(a);
  return launch_status();
}

MB_API int mb_step_finalize(const mb_adamw_plan* p, const mb_finalize_opts* fin, mb_stream_t stream) {
  int rc = check_plan(p);
  if (rc) return rc;
  if ((rc = check_fin(fin))) return rc;
  k_step_finalize<<<1, kThreads, 0, (cudaStream_t)stream>>>(*p, *fin);
  return launch_status();
}

MB_API int mb_adamw_apply_tiles(const mb_adamw_plan* p, int64_t tile_lo, int64_t tile_hi, int32_t max_ctas,
                                mb_stream_t stream) {
  int rc = check_plan(p);
  if (rc) return rc;
  if (tile_lo < 0 || tile_hi > p->n_tiles || tile_lo > tile_hi) return MB_ERR_ARG;
  if (tile_lo == tile_hi) return MB_OK;
  ApplyFn fn = pick_apply(p->grad_dtype, p->out_dtype);
  if (!fn) return MB_ERR_ARG;
  BulkFn bulk = pick_apply_bulk(p->grad_dtype, p->out_dtype);
  ApplyArgs a{};
  a.segs = p->segs;
  a.groups = p->groups;
  a.seg_scal = reinterpret_cast<const float2*>(static_cast<const char*>(p->workspace) + kSegScalOffset);
  a.state = p->state;
  a.tile_lo = tile_lo;
  a.n_tiles = tile_hi;
  a.n_segs = p->n_segs;
  if (use_bulk_apply() && bulk.fn && bulk_ready(reinterpret_cast<const void*>(bulk.fn), bulk.smem)) {
    take_fault(kFaultApply, &a.fault.unit, &a.fault.limit_ns);
    // kBulkCtasPerSm CTAs per SM; max_ctas counts register-staged CTAs (3 per SM)
    int64_t grid = (int64_t)sm_count() * kBulkCtasPerSm;
    if (max_ctas > 0) grid = max_ctas * kBulkCtasPerSm / 3 > 0 ? max_ctas * kBulkCtasPerSm / 3 : 1;
    if (grid > tile_hi - tile_lo) grid = tile_hi - tile_lo;
    bulk.fn<<<(int)grid, kBulkThreads, bulk.smem, (cudaStream_t)stream>>>(a);
    return launch_status();
  }
  int grid = grid_for(reinterpret_cast<const void*>(fn), tile_hi - tile_lo);
  if (max_ctas > 0 && grid > max_ctas) grid = max_ctas;
  fn<<<grid, kThreads, 0, (cudaStream_t)stream>>>(a);
  return launch_status();
}

MB_API int mb_adamw_apply_tiles_peers(const mb_adamw_plan* p, int64_t tile_lo, int64_t tile_hi, int32_t max_ctas,
                                      const int64_t* peer_deltas, int32_t n_peers, mb_stream_t stream) {
  int rc = check_plan(p);
  if (rc) return rc;
  if (tile_lo < 0 || tile_hi > p->n_tiles || tile_lo > tile_hi) return MB_ERR_ARG;
  if (n_peers < 0 || n_peers > kMaxPeers || (n_peers > 0 && !peer_deltas)) return MB_ERR_ARG;
  if (n_peers > 0 && p->out_dtype == MB_NONE) return MB_ERR_ARG;
  for (int i = 0; i < n_peers; ++i)
    if (peer_deltas[i] % 16) return MB_ERR_ALIGN;  // keeps the copies' vector alignment
  if (tile_lo == tile_hi) return MB_OK;
  BulkFn bulk = pick_apply_bulk(p->grad_dtype, p->out_dtype);
  if (!bulk.fn || !bulk_ready(reinterpret_cast<const void*>(bulk.fn), bulk.smem)) return MB_ERR_CUDA;
  ApplyArgs a{};
  a.segs = p->segs;
  a.groups = p->groups;
  a.seg_scal = reinterpret_cast<const float2*>(static_cast<const char*>(p->workspace) + kSegScalOffset);
  a.state = p->state;
  a.tile_lo = tile_lo;
  a.n_tiles = tile_hi;
  a.n_segs = p->n_segs;
  a.n_peers = n_peers;
  for (int i = 0; i < n_peers; ++i) a.peer_delta[i] = peer_deltas[i];
  take_fault(kFaultApply, &a.fault.unit, &a.fault.limit_ns);
  int64_t grid = (int64_t)sm_count() * kBulkCtasPerSm;
  if (max_ctas > 0) grid = max_ctas * kBulkCtasPerSm / 3 > 0 ? max_ctas * kBulkCtasPerSm / 3 : 1;
  if (grid > tile_hi - tile_lo) grid = tile_hi - tile_lo;
  bulk.fn<<<(int)grid, kBulkThreads, bulk.smem, (cudaStream_t)stream>>>(a);
  return launch_status();
}

MB_API int mb_adamw_apply(const mb_adamw_plan* p, mb_stream_t stream) {
  if (!p) return MB_ERR_ARG;
  return mb_adamw_apply_tiles(p, 0, p->n_tiles, 0, stream);
}

MB_API int mb_adamw_step(const mb_adamw_plan* p, const mb_finalize_opts* fin, mb_stream_t stream) {
  int rc = mb_grad_stats(p, fin, stream);
  if (rc) return rc;
  return mb_adamw_apply(p, stream);
}

MB_API int mb_adamw_update(float* w, float* m, float* v, const void* g, int32_t gdt, void* out,
                           int32_t odt, int64_t numel, const mb_host_scalars* s, mb_stream_t stream) {
  if (!w || !m || !v || !g || !s || numel < 0) return MB_ERR_ARG;
  if (odt != MB_NONE && !out) return MB_ERR_ARG;
  UpdateFn fn = pick_update(gdt, odt);
  if (!fn) return MB_ERR_ARG;
  if (numel == 0) return MB_OK;
  mb_segment seg{};
  seg.w = w; seg.m = m; seg.v = v; seg.g = g; seg.out = out; seg.numel = numel;
  int64_t tiles = (numel + kTile - 1) / kTile;
  int grid = grid_for(reinterpret_cast<const void*>(fn), tiles);
  fn<<<grid, kThreads, 0, (cudaStream_t)stream>>>(seg, tiles, *s);
  return launch_status();
}

}  // extern "C"
