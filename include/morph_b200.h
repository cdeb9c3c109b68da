/*
 * morph_b200 — C ABI of the B200 optimizer-step kernels.
 *
 * Every entry point takes raw device pointers, element counts, dtype codes and
 * a CUDA stream, returns an int status (MB_OK = 0) and throws nothing. No entry
 * point allocates parameter memory or synchronises the host with the device,
 * except the two whose job that is: mb_ipc_alloc (peer-mapped buffers) and
 * mb_stream_wait (a bounded host wait). Callers own every buffer (state,
 * workspace, tables) and size the workspace with mb_workspace_bytes().
 *
 * Reference interfaces replaced (paths inside the everett6/MORPH project):
 *   mb_adamw_step / mb_grad_stats / mb_step_finalize / mb_adamw_apply
 *       torch.optim.AdamW(..., betas=(.9,.95), foreach=False).step() built at
 *       streamtrain/optimizer.py:40 and stepped at streamtrain/optimizer.py:62 and
 *       morph/training/runner.py:101; the finiteness gate at
 *       streamtrain/optimizer.py:50-51; clip_grad_norm_ at morph/training/runner.py:100;
 *       the FP64 norm pass at streamtrain/disk.py:466-468 and
 *       streamtrain/sparse_disk.py:136; DynamicLossScale.overflow/success at
 *       streamtrain/precision.py:9-14 as driven by streamtrain/disk.py:482-497.
 *   mb_adamw_update
 *       DiskState.update(name, gradient, step, lr, clip) at streamtrain/disk.py:203-223
 *       (and CachedDiskState.update at streamtrain/state_cache.py:103-140), with the
 *       gradient unscale g.float()/loss_scale of streamtrain/sparse_disk.py:107.
 *   mb_sparse_rows_update
 *       the conditional AdamW of streamtrain/sparse_disk.py:122-138 applied to the
 *       touched rows of one table (DiskState.update on the gathered rows).
 *   mb_grad_accumulate
 *       the microbatch accumulation g.float() / loss_scale into the FP32 gradient
 *       window of streamtrain/sparse_disk.py:82-110, with the norm statistics.
 *   mb_export_f16
 *       the FP16 export cast and range check of streamtrain/export.py:30-35.
 *   mb_cast_f32
 *       the FP32 -> BF16/FP16 compute copy (streamtrain/disk.py:320-326,351) and the
 *       FP16 export with its range check (streamtrain/export.py:32-34).
 */
#ifndef MORPH_B200_H
#define MORPH_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MB_API __attribute__((visibility("default")))

/* Same object as cudaStream_t; NULL is the legacy default stream. */
typedef struct CUstream_st* mb_stream_t;

/* ------------------------------------------------------------- status -- */
enum {
  MB_OK = 0,
  MB_ERR_ARG = 1,                /* null pointer, negative size, unknown dtype/flag  */
  MB_ERR_ALIGN = 2,              /* pointer alignment below the entry's contract     */
  MB_ERR_CUDA = 3,               /* a CUDA runtime call or launch failed             */
  MB_ERR_OVERFLOW_MIN_SCALE = 4, /* FP16 overflow while the loss scale is already 1  */
  MB_ERR_NONFINITE = 5,          /* nonfinite gradient with the finiteness gate on   */
  MB_ERR_TIMEOUT = 6,            /* a bounded wait expired                           */
  MB_ERR_INDEX = 7,              /* a row index outside the table                    */
  MB_ERR_UNREPRESENTABLE = 8,    /* FP16 export of a nonfinite value or |w| > 65504  */
  MB_ERR_TOO_LARGE = 9           /* plan larger than the fixed no-allocation scratch */
};

/* ------------------------------------------------------------- dtypes -- */
enum { MB_F32 = 0, MB_F16 = 1, MB_BF16 = 2, MB_NONE = 3 };

/* ------------------------------------------------- multi-tensor AdamW -- */

/* One contiguous run of elements of one parameter tensor. w, m, v are FP32;
 * g has the plan's grad dtype; out (optional) receives the updated w in the
 * plan's out dtype (round to nearest even). Vector loads are used when w, m,
 * v (and an FP32 g) are 16-byte aligned and a 16-bit g / out is 8-byte
 * aligned; other segments take the scalar path. */
typedef struct mb_segment {
  float* w;
  float* m;
  float* v;
  const void* g;
  void* out;
  int64_t numel;
  int64_t tile_begin; /* set by mb_segments_plan */
  int32_t clock;      /* index into the plan's clock array; unique per segment */
  int32_t group;      /* index into the plan's group array */
} mb_segment;

/* Hyperparameters of one parameter group. Float fields are the float32
 * roundings of the double expressions named, computed by the caller exactly as
 * the reference's Python does. */
typedef struct mb_group {
  double lr;    /* step size numerator: scalar = (float)(-(lr / bc1[t]))  */
  float cwd;    /* (float)(1 - lr * weight_decay)                         */
  float omb1;   /* (float)(1 - beta1): lerp weight of the first moment    */
  float beta2;  /* (float)beta2                                           */
  float omb2;   /* (float)(1 - beta2): addcmul value of the second moment */
  float eps;    /* (float)eps                                             */
  int32_t table;/* row of the bias-correction table                       */
} mb_group;

/* Device-resident step control, one per optimizer. sumsq and nonfinite come
 * first: that 16-byte record is what ranks all-reduce (SUM, FP64). */
typedef struct mb_step_state {
  double sumsq;           /* sum of squared unscaled gradients (FP64)           */
  double nonfinite;       /* number of nonfinite gradient elements              */
  double scale;           /* loss scale the next step's gradients carry         */
  double step_scale;      /* loss scale the last finalized step divided by      */
  int64_t good_steps;     /* DynamicLossScale.good_steps                        */
  int64_t growth_interval;/* DynamicLossScale.growth_interval                   */
  double max_scale;       /* growth cap (65536 in the reference)                */
  double norm;            /* sqrt(sumsq) of the last finalized step             */
  float clip_coef;        /* multiplier applied to unscaled gradients           */
  int32_t skip;           /* 1 if the last finalized step skips its update      */
  int32_t status;         /* MB_OK, MB_ERR_OVERFLOW_MIN_SCALE, MB_ERR_NONFINITE or MB_ERR_TIMEOUT */
  int32_t steps_applied;  /* updates applied so far                             */
  int32_t steps_skipped;  /* updates skipped so far                             */
  int32_t reserved[3];
} mb_step_state;

/* Finalize flags. */
enum {
  MB_FIN_LOSS_SCALE = 1, /* divide grads by state.scale; on nonfinite back off, else success() */
  MB_FIN_GATE = 2,       /* without loss scaling: nonfinite -> skip, status MB_ERR_NONFINITE   */
  MB_FIN_CLIP_TORCH = 4, /* coef = min(1, fl32(1/(fl32(norm) + 1e-6f)) * max_norm)           */
  MB_FIN_CLIP_DISK = 8   /* coef = (float)min(1, max_norm / (norm + 1e-6)) in double          */
};

typedef struct mb_finalize_opts {
  int32_t flags;
  int32_t reserved;
  double max_norm;  /* clip threshold (> 0 when a clip flag is set) */
  double backoff;   /* loss-scale factor on overflow (0.5 in the reference) */
  double growth;    /* loss-scale factor after growth_interval good steps (2.0) */
} mb_finalize_opts;

/* Everything one fused multi-tensor AdamW launch needs. All pointers are
 * device pointers except that the struct itself is read on the host. */
typedef struct mb_adamw_plan {
  const mb_segment* segs;  /* n_segs entries, tile_begin planned                   */
  const mb_group* groups;  /* n_groups entries                                     */
  const double* bc;        /* [tables][2][bc_len]: 1 - beta1**t, sqrt(1 - beta2**t)*/
  int32_t* clocks;         /* per-segment step counters (torch state['step'])      */
  void* workspace;         /* mb_workspace_bytes(n_segs) bytes, 256-byte aligned   */
  mb_step_state* state;
  int64_t n_tiles;         /* from mb_segments_plan                                */
  int64_t bc_len;          /* clocks beyond bc_len-1 read the last entry           */
  int32_t n_segs;
  int32_t n_groups;
  int32_t grad_dtype;      /* MB_F32, MB_F16 or MB_BF16                            */
  int32_t out_dtype;       /* MB_F16, MB_BF16 or MB_NONE                           */
} mb_adamw_plan;

MB_API int mb_version(void);
MB_API const char* mb_status_string(int status);

/* Host only: fills segs[i].tile_begin and returns the tile count. */
MB_API int mb_segments_plan(mb_segment* segs_host, int32_t n_segs, int64_t* n_tiles);

/* Bytes of device workspace a plan with n_segs segments needs. */
MB_API size_t mb_workspace_bytes(int32_t n_segs);

/* Host only: a fresh step state (scale, growth interval; everything else 0,
 * clip_coef 1, max_scale 65536). Copy it to the device yourself. */
MB_API int mb_step_state_init(mb_step_state* host_state, double scale, int64_t growth_interval);

/* Kernel 2: FP64 sum of squares and nonfinite count of all plan gradients
 * (unscaled by state.scale when fin has MB_FIN_LOSS_SCALE). Writes
 * state.sumsq/nonfinite; with fin != NULL it also finalizes in the same launch. */
MB_API int mb_grad_stats(const mb_adamw_plan* plan, const mb_finalize_opts* fin, mb_stream_t stream);

/* One block: loss-scale transition, skip decision, clip coefficient, clock
 * advance and per-segment step scalars, from state.sumsq/nonfinite. */
MB_API int mb_step_finalize(const mb_adamw_plan* plan, const mb_finalize_opts* fin, mb_stream_t stream);

/* Kernel 1: the fused AdamW update of every segment (early exit when
 * state.skip), writing the optional low-precision copy. */
MB_API int mb_adamw_apply(const mb_adamw_plan* plan, mb_stream_t stream);

/* Kernel 1 on the tiles [tile_lo, tile_hi) of a finalized plan only (segment
 * s covers tiles [s.tile_begin, next tile_begin)), with at most max_ctas CTAs
 * (<= 0: one persistent wave). Lets a caller update a shard in rounds and run
 * each round's all-gather, on SMs left free, while the next round updates. */
MB_API int mb_adamw_apply_tiles(const mb_adamw_plan* plan, int64_t tile_lo, int64_t tile_hi, int32_t max_ctas,
                                mb_stream_t stream);

/* mb_grad_stats (fused finalize) followed by mb_adamw_apply. */
MB_API int mb_adamw_step(const mb_adamw_plan* plan, const mb_finalize_opts* fin, mb_stream_t stream);

/* Kernel 1 over tiles [tile_lo, tile_hi) that also stores every low-precision
 * copy into n_peers other GPUs' buffers: the value written at address a is
 * also written at a + peer_deltas[i] (bytes; multiples of 16) for each i, where
 * the peer buffers are mapped into this process (mb_ipc_open). This fuses the
 * sharded step's update with its all-gather of the low-precision weights
 * (no counterpart in the reference, which is single-process). The stores are
 * ordered (system scope) before the kernel completes; a collective after it on
 * every rank (e.g. a one-element all-reduce) makes them complete everywhere.
 * Requires out_dtype != MB_NONE; n_peers <= 15. */
MB_API int mb_adamw_apply_tiles_peers(const mb_adamw_plan* plan, int64_t tile_lo, int64_t tile_hi, int32_t max_ctas,
                                      const int64_t* peer_deltas, int32_t n_peers, mb_stream_t stream);

/* Peer-writable buffers on one node (cudaMalloc + CUDA IPC). mb_ipc_alloc
 * allocates `bytes` on the current device and writes its 64-byte handle;
 * another process on the node maps it with mb_ipc_open (peer access enabled)
 * and unmaps it with mb_ipc_close before the owner calls mb_ipc_free. */
MB_API int mb_ipc_alloc(size_t bytes, void** ptr, void* handle);
MB_API int mb_ipc_free(void* ptr);
MB_API int mb_ipc_open(const void* handle, void** ptr);
MB_API int mb_ipc_close(void* ptr);

/* No counterpart in the reference. mb_adamw_step for callers that cannot
 * allocate device memory (a host framework whose allocator already holds the
 * whole GPU, or a binding handed fixed buffers with no allocator of its own).
 * plan->workspace is ignored and may be NULL: the kernels use one fixed
 * library-owned device array instead (about 129 KiB per GPU, held until exit).
 * At most 8192 segments; larger plans return MB_ERR_TOO_LARGE and nothing runs.
 * fin is required (NULL returns MB_ERR_ARG). The plan and fin are validated
 * before anything is queued. The first call on a device looks the array up
 * (cudaGetSymbolAddress) and caches it for the current CUDA context (a new
 * context, e.g. after cudaDeviceReset, is looked up again): make that first
 * call before any stream capture. Calls share the array; calls that may
 * overlap on the GPU race, so order them on one stream. Allocates nothing. */
MB_API int mb_adamw_step_noalloc(const mb_adamw_plan* plan, const mb_finalize_opts* fin, mb_stream_t stream);

/* Test-only, no counterpart in the reference: arms a fault for the next launch
 * in this process of one kernel whose waits are bounded, so a test can make a
 * bounded device wait expire without faulting anything. That launch withholds
 * one unit's copy (kernel 1 = MB_FAULT_APPLY: the bulk-staged update's tile
 * `unit`; MB_FAULT_STATS: the bulk-staged statistics pass's chunk starting at
 * tile `unit`; MB_FAULT_GEMM: the first k-block of output tile `unit` of the
 * kernel-4 GEMM) and bounds every wait of the launch by wait_limit_ns (1 us to
 * 2 s). The consumers' wait for that unit expires; the CTA stops, drains its own
 * copies in flight (bounded), frees what it holds and reports MB_ERR_TIMEOUT in
 * the step state (kernel 2: the step is refused, nothing changes) or raises the
 * GEMM's error flag. One arm is consumed by one launch; kernel 0 disarms all. */
enum { MB_FAULT_APPLY = 1, MB_FAULT_STATS = 2, MB_FAULT_GEMM = 4 };
MB_API int mb_debug_arm_fault(int32_t kernel, int64_t unit, int64_t wait_limit_ns);

/* --------------------------------------- single tensor, host scalars -- */

/* Step scalars computed on the host (float32 roundings of the reference's
 * double expressions). grad' = (g / scale) * coef before the update. */
typedef struct mb_host_scalars {
  float cwd, omb1, beta2, omb2, bc2s, eps, nss;
  float scale; /* loss-scale divisor (1 for none) */
  float coef;  /* clip multiplier (1 for none) */
} mb_host_scalars;

/* DiskState.update on one device-resident tensor (w, m, v FP32). */
MB_API int mb_adamw_update(float* w, float* m, float* v, const void* g, int32_t grad_dtype,
                           void* out, int32_t out_dtype, int64_t numel,
                           const mb_host_scalars* s, mb_stream_t stream);

/* Kernel 3: lazy row-sparse AdamW. Rows idx[0..k) of the [rows, cols] FP32
 * planes w, m, v take one step with gradient row r = grads[r*cols ..]. Rows not
 * listed are not read or written. An index outside [0, rows) is skipped and
 * sets *err_flag (device int32, may be NULL) to 1. Each row is listed at most
 * once (the reference's sorted, unique index sets); a row listed twice is
 * updated by two CTAs at once, in no defined order. Any cols >= 1 works; cols
 * a multiple of 4 with 16-byte aligned planes and gradients takes the vector path. */
MB_API int mb_sparse_rows_update(float* w, float* m, float* v, int64_t rows, int64_t cols,
                                 const int64_t* idx, int64_t k, const void* grads,
                                 int32_t grad_dtype, const mb_host_scalars* s,
                                 int32_t* err_flag, mb_stream_t stream);

/* ------------------------------------------------------ Muon (kernel 4) -- */

/* 16-bit GEMM on the tcgen05 tensor cores: out = alpha * (a . b^T) + beta * c,
 * FP32 accumulation. dtype (MB_BF16 or MB_F16) is the type of a, b, c, d, dt.
 * a is [m, k] and b is [n, k], both row-major (K contiguous) with row pitches
 * lda/ldb (elements, multiples of 8, 16-byte aligned bases); c and d are
 * [m, n] with pitches ldc/ldd; dt (optional) receives out^T as [n, m] with
 * pitch lddt; df (optional) receives out in FP32 with pitch lddf. m must be a
 * multiple of 128, n of 256 and k of 64 (pad with zeros). A wait that exceeds
 * its bound sets *err_flag (device int32) to 1. When m is a multiple of 256 the
 * launch runs as clusters of two CTAs (tcgen05 cta_group::2, M = 256 over two
 * SMs) unless MB_GEMM_PAIR=0 is set in the environment; the results are the
 * same bits either way. These are the matmuls of orthogonalize,
 * streamtrain/optimizer.py:20-21. */
MB_API int mb_gemm16(int32_t dtype, const void* a, int64_t lda, const void* b, int64_t ldb, int64_t m, int64_t n,
                     int64_t k, float alpha, float beta, const void* c, int64_t ldc, void* d, int64_t ldd, void* dt,
                     int64_t lddt, float* df, int64_t lddf, int32_t* err_flag, mb_stream_t stream);

/* Muon hyperparameters of one matrix (float roundings of the reference's
 * Python expressions, streamtrain/optimizer.py:58-61). */
typedef struct mb_muon_args {
  float beta_lerp;   /* momentum.lerp_(g, .05)                  */
  float nesterov;    /* g.lerp(momentum, .95)                   */
  float ns_a;        /* 3.4445                                  */
  float ns_b;        /* -4.775                                  */
  float ns_c;        /* 2.0315                                  */
  int32_t ns_steps;  /* 5                                       */
  float shape_scale; /* (float)(max(1, rows / cols) ** .5)      */
  float cwd;         /* (float)(1 - lr * weight_decay)          */
  float neg_lr;      /* (float)(-lr)                            */
  int32_t ns_dtype;  /* Newton-Schulz operands: MB_BF16 or MB_F16 */
  const int32_t* skip; /* optional device flag (e.g. &mb_step_state.skip of a gate
                          finalized earlier on the stream): nonzero = every launch
                          of the step returns at once and nothing changes */
  int32_t max_sms;     /* 0: the GEMMs use every SM; else at most this many, leaving
                          the rest to work on other streams (e.g. a collective) */
} mb_muon_args;

/* Most matrices one mb_muon_step_batched call takes. */
#define MB_MUON_MAX_BATCH 64

/* Device workspace for one [rows, cols] matrix, enough for mb_newton_schulz
 * and mb_muon_step (0 for invalid shapes). */
MB_API size_t mb_muon_workspace_bytes(int64_t rows, int64_t cols);

/* Device workspace for mb_muon_step_batched over `batch` [rows, cols]
 * matrices (0 for invalid shapes or batch outside 1..MB_MUON_MAX_BATCH). */
MB_API size_t mb_muon_batch_workspace_bytes(int32_t batch, int64_t rows, int64_t cols);

/* orthogonalize (streamtrain/optimizer.py:13-22) of an FP32 [rows, cols]
 * matrix into out (FP32, same shape): transpose when rows > cols, divide by
 * (Frobenius norm + 1e-7), `steps` quintic Newton-Schulz iterations with
 * coeffs {a, b, c} on ns_dtype (MB_BF16 or MB_F16) operands with FP32
 * accumulation; each iteration forms a I + b A + c A A in FP32 before one
 * rounding, so the a X and (b A + c A A) X terms never cancel in 16 bits. */
MB_API int mb_newton_schulz(const float* x, int64_t rows, int64_t cols, int32_t steps, const float* coeffs,
                            int32_t ns_dtype, float* out, void* workspace, size_t workspace_bytes,
                            int32_t* err_flag, mb_stream_t stream);

/* One Muon step of one matrix (streamtrain/optimizer.py:55-61): momentum
 * (FP32, updated in place) lerps toward g, the Nesterov blend is
 * orthogonalised, scaled by shape_scale and applied with decoupled weight
 * decay to w (FP32); out (optional) receives w in out_dtype. */
MB_API int mb_muon_step(float* w, float* momentum, const void* g, int32_t grad_dtype, void* out, int32_t out_dtype,
                        int64_t rows, int64_t cols, const mb_muon_args* args, void* workspace,
                        size_t workspace_bytes, int32_t* err_flag, mb_stream_t stream);

/* mb_muon_step over `batch` matrices of one shape (the per-parameter loop of
 * streamtrain/optimizer.py:52-61, which runs the matrices one after another):
 * w, momentum, g and out (null when out_dtype is MB_NONE) are HOST arrays of
 * `batch` device pointers; every launch of the step covers the whole batch.
 * Each matrix gets exactly the arithmetic of mb_muon_step. */
MB_API int mb_muon_step_batched(float* const* w, float* const* momentum, const void* const* g, int32_t grad_dtype,
                                void* const* out, int32_t out_dtype, int32_t batch, int64_t rows, int64_t cols,
                                const mb_muon_args* args, void* workspace, size_t workspace_bytes,
                                int32_t* err_flag, mb_stream_t stream);

/* Kernel 5: one row-sparse DiskState.update step on state held in pinned host
 * memory (streamtrain/engine.py:60-163 ping-pong slots, applied to
 * streamtrain/sparse_disk.py:122-138). host_w/m/v are [rows, cols] FP32 planes
 * allocated pinned and mapped (cudaHostAlloc); idx (device, k sorted unique
 * int64) and grads (device, [k, cols]) name the touched rows. The rows move
 * through two device windows of window_rows rows ([3][window_rows][cols] FP32
 * each): gathers on stream h2d, kernel-1 updates on stream compute, scatters
 * on stream d2h, ordered by events; on return the work is enqueued and the
 * compute stream is ordered after the last scatter. An out-of-range index is
 * skipped and sets *err_flag. Calls on one device must come from one thread,
 * in order (the events are shared per device). */
MB_API int mb_offload_rows_step(float* host_w, float* host_m, float* host_v, int64_t rows, int64_t cols,
                                const int64_t* idx, int64_t k, const void* grads, int32_t grad_dtype,
                                const mb_host_scalars* s, float* window0, float* window1, int64_t window_rows,
                                mb_stream_t compute, mb_stream_t h2d, mb_stream_t d2h, int32_t* err_flag);

/* Host wait with a bound (the "wait" of the reference's slot protocol,
 * streamtrain/engine.py:111-112, which blocks without one): returns MB_OK once
 * all work enqueued on `stream` has finished, MB_ERR_TIMEOUT when timeout_us
 * elapses first (the work keeps running; call again to keep waiting), or
 * MB_ERR_CUDA if the stream reported an error. Polls; never blocks the GPU. */
MB_API int mb_stream_wait(mb_stream_t stream, int64_t timeout_us);

/* Block-scaled FP8 transport (streamtrain/precision.py:24-37): per 256-element
 * block, scale = max(amax|x| / 448, 1e-30) and codes = e4m3fn(clamp(x / scale,
 * -448, 448)) (round to nearest even); codes has n bytes, scales
 * ceil(n / 256) floats. */
MB_API int mb_fp8_pack(const float* src, int64_t n, uint8_t* codes, float* scales, mb_stream_t stream);

/* Inverse of mb_fp8_pack: out[i] = (float(code[i]) * scale[i / 256]) rounded to
 * out_dtype (MB_F32, MB_F16 or MB_BF16). */
MB_API int mb_fp8_unpack(const uint8_t* codes, const float* scales, int64_t n, void* out, int32_t out_dtype,
                         mb_stream_t stream);

/* Microbatch gradient accumulation (streamtrain/sparse_disk.py:82-110):
 * acc = acc + f32(g) / loss_scale over n elements (first != 0: acc = 0 +
 * f32(g) / loss_scale, i.e. the window's zero_() fused in), IEEE division.
 * With record != NULL (device, 2 doubles) the call also adds
 * {sum of acc^2 in FP64, 1 if any acc value is nonfinite} of the updated acc
 * to record (the norm pass of sparse_disk.py:119-120 / disk.py:466-468), in a
 * fixed reduction order; workspace (device, mb_accumulate_workspace_bytes(),
 * zeroed once before first use) is then required. Calls that share a
 * workspace must be ordered on one stream. */
MB_API size_t mb_accumulate_workspace_bytes(void);
MB_API int mb_grad_accumulate(float* acc, const void* g, int32_t grad_dtype, int64_t n, float loss_scale,
                              int32_t first, double* record, void* workspace, mb_stream_t stream);

/* FP16 export of n FP32 values (streamtrain/export.py:30-35): dst (device
 * memory, or pinned host memory written through its device mapping) receives
 * the values rounded to nearest even; *first_bad (device memory, set by the
 * caller to UINT64_MAX beforehand) is lowered to the index of the first value
 * that is nonfinite or has |x| > 65504. Elements before that index are always
 * written. */
MB_API int mb_export_f16(const float* src, int64_t n, void* dst, uint64_t* first_bad, mb_stream_t stream);

/* FP32 -> F16/BF16 cast (round to nearest even). With check != 0 (F16 only)
 * a nonfinite value or |x| > 65504 sets *err_flag to 1 (export.py:33). */
MB_API int mb_cast_f32(const float* src, void* dst, int32_t dst_dtype, int64_t n, int32_t check,
                       int32_t* err_flag, mb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MORPH_B200_H */
