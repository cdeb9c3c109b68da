/*
 * TEST INFRASTRUCTURE — CPU restatement of MORPH's optimizer-step arithmetic.
 *
 * This file is the parity oracle. Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg may load it, and only as the checker or as the
 * timed CPU baseline. No product code path calls it.
 *
 * Compile with -ffp-contract=off: every rounding step below is explicit, and a
 * fused multiply-add appears only where the reference's own build fuses one.
 *
 * What is restated, and from where (paths inside the reference project):
 *  - AdamW, decoupled weight decay: torch.optim.AdamW(foreach=False) as built by
 *    streamtrain/optimizer.py:40 and stepped at streamtrain/optimizer.py:62 and
 *    morph/training/runner.py:101. The arithmetic itself lives in torch 2.11.0
 *    (third-party, not vendored in the reference): torch/optim/adam.py
 *    `_single_tensor_adam` (installed file, lines 414-547) over the ATen CPU
 *    kernels (LerpKernel.cpp lerp_vec = fmadd(coeff, end-start, base);
 *    PointwiseOpsKernel.cpp addcmul/addcdiv). The FMA placement was pinned
 *    against the installed torch bit for bit (tests/test_oracle_cpu.py).
 *  - DiskState.update: streamtrain/disk.py:203-223 (and the identical cached
 *    copy streamtrain/state_cache.py:119-127).
 *  - Gradient unscale g.float()/loss_scale: streamtrain/sparse_disk.py:107,
 *    streamtrain/disk.py:447, streamtrain/engine.py:207.
 *  - FP64 chunked norm: streamtrain/disk.py:466-468, streamtrain/sparse_disk.py:136.
 *  - Muon elementwise: streamtrain/optimizer.py:58-61.
 *  - FP16 export cast and its checks: streamtrain/export.py:32-34.
 *
 * One known, bounded difference from the reference: torch's CPU float sqrt on
 * large tensors goes through MKL VML and is not always correctly rounded (it is
 * off by one ulp on well under 1% of elements). This oracle uses the IEEE
 * square root, which is what the CUDA kernels use too.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define ORC_API __attribute__((visibility("default")))

/* ---------------------------------------------------------------- casts -- */

ORC_API void orc_f16_to_f32(const uint16_t* src, float* dst, int64_t n) {
  const _Float16* s = (const _Float16*)src;
  for (int64_t i = 0; i < n; ++i) dst[i] = (float)s[i];
}

ORC_API void orc_bf16_to_f32(const uint16_t* src, float* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    uint32_t bits = (uint32_t)src[i] << 16;
    memcpy(&dst[i], &bits, 4);
  }
}

/* Round-to-nearest-even float -> float16 (numpy astype('<f2'), Tensor.copy_). */
ORC_API void orc_f32_to_f16(const float* src, uint16_t* dst, int64_t n) {
  _Float16* d = (_Float16*)dst;
  for (int64_t i = 0; i < n; ++i) d[i] = (_Float16)src[i];
}

/* Round-to-nearest-even float -> bfloat16, NaN kept quiet (c10::BFloat16). */
ORC_API void orc_f32_to_bf16(const float* src, uint16_t* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    uint32_t u;
    memcpy(&u, &src[i], 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) {
      dst[i] = 0x7fc0;
      continue;
    }
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    dst[i] = (uint16_t)(u >> 16);
  }
}

/* export.py:33-34: refuse nonfinite values or |w| > 65504, else RNE to f16.
 * Returns 0 on success, 1 if the chunk cannot be represented. */
ORC_API int orc_export_f16(const float* src, uint16_t* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    float x = src[i];
    if (!isfinite(x) || fabsf(x) > 65504.0f) return 1;
  }
  orc_f32_to_f16(src, dst, n);
  return 0;
}

/* --------------------------------------------------------- grad inputs -- */

/* g32 = (float(g) / scale) * coef, each step rounded to float, as the
 * reference does: the unscale at sparse_disk.py:107 (true division by the
 * Python float scale), then the clip multiply (clip_grad.py _foreach_mul_, or
 * disk.py:210 `gradient * clip`). dtype: 0 f32, 1 f16, 2 bf16. */
ORC_API void orc_grad_prepare(const void* g, int dtype, int64_t n, float scale,
                              float coef, float* out) {
  for (int64_t i = 0; i < n; ++i) {
    float x;
    if (dtype == 0) {
      x = ((const float*)g)[i];
    } else if (dtype == 1) {
      x = (float)((const _Float16*)g)[i];
    } else {
      uint32_t bits = (uint32_t)((const uint16_t*)g)[i] << 16;
      memcpy(&x, &bits, 4);
    }
    x = x / scale;
    x = x * coef;
    out[i] = x;
  }
}

/* Sum of squares in FP64 over 1,048,576-element pieces, each piece summed and
 * then added to the running total (disk.py:466-468). Also counts nonfinite
 * elements, the finiteness gate of optimizer.py:50. */
ORC_API double orc_sumsq(const float* g, int64_t n, int64_t* nonfinite) {
  double total = 0.0;
  int64_t bad = 0;
  for (int64_t start = 0; start < n; start += 1048576) {
    int64_t end = start + 1048576 < n ? start + 1048576 : n;
    double piece = 0.0;
    for (int64_t i = start; i < end; ++i) {
      double x = (double)g[i];
      if (!isfinite(g[i])) ++bad;
      piece += x * x;
    }
    total += piece;
  }
  if (nonfinite) *nonfinite = bad;
  return total;
}

/* ---------------------------------------------------------------- AdamW -- */

/* Per-step float scalars. Derived in double on the host exactly as the
 * reference's Python does, then rounded once to float (ATen Scalar.to<float>). */
typedef struct {
  float cwd;  /* 1 - lr*wd                   (adam.py decoupled wd; disk.py:215) */
  float omb1; /* lerp weight 1 - beta1       (adam.py lerp_; disk.py:211 .1)      */
  float b2;   /* beta2                       (adam.py mul_; disk.py:212 .999)     */
  float omb2; /* addcmul value 1 - beta2     (adam.py; disk.py:212 .001)          */
  float bc2s; /* sqrt of 1 - beta2**t        (adam.py **0.5; disk.py:213 math.sqrt)*/
  float eps;  /* eps                         (adam.py; disk.py:213 1e-8)          */
  float nss;  /* -(lr / (1 - beta1**t))      (adam.py value=-step_size; disk.py:215)*/
} orc_scalars;

/* torch lerp_ with a scalar weight, ATen CPU vector path:
 *   small = |w| < 0.5; coeff = small ? w : w - 1; base = small ? start : end;
 *   result = fma(coeff, end - start, base). */
static inline float orc_lerp(float start, float end, float weight) {
  if (fabsf(weight) < 0.5f) return fmaf(weight, end - start, start);
  return fmaf(weight - 1.0f, end - start, end);
}

/* One AdamW step on float arrays, in place. The op order is that of
 * _single_tensor_adam with decoupled weight decay, which DiskState.update
 * repeats with fixed hyperparameters:
 *   w *= cwd
 *   m  = lerp(m, g, omb1)
 *   v  = v*b2 ; v = fma(omb2*g, g, v)     (addcmul_, fused in torch's build)
 *   d  = sqrt(v) / bc2s + eps
 *   w  = w + (nss*m) / d                  (addcdiv_) */
ORC_API void orc_adamw(float* w, float* m, float* v, const float* g, int64_t n,
                       const orc_scalars* s) {
  for (int64_t i = 0; i < n; ++i) {
    float gi = g[i];
    float wi = w[i] * s->cwd;
    float mi = orc_lerp(m[i], gi, s->omb1);
    float vi = v[i] * s->b2;
    vi = fmaf(s->omb2 * gi, gi, vi);
    float d = sqrtf(vi) / s->bc2s + s->eps;
    wi = wi + (s->nss * mi) / d;
    w[i] = wi;
    m[i] = mi;
    v[i] = vi;
  }
}

/* Lazy row-sparse AdamW: rows idx[0..k) of the [rows x cols] planes w/m/v take
 * one DiskState.update step with gradient row r = grads[r*cols .. +cols)
 * (already unscaled and clipped, float). Rows outside idx are not touched.
 * Returns 0, or 1 if an index is out of range (nothing is written then). */
ORC_API int orc_sparse_rows(float* w, float* m, float* v, int64_t rows, int64_t cols,
                            const int64_t* idx, int64_t k, const float* grads,
                            const orc_scalars* s) {
  for (int64_t r = 0; r < k; ++r)
    if (idx[r] < 0 || idx[r] >= rows) return 1;
  for (int64_t r = 0; r < k; ++r) {
    int64_t base = idx[r] * cols;
    orc_adamw(w + base, m + base, v + base, grads + r * cols, cols, s);
  }
  return 0;
}

/* ----------------------------------------------------------------- Muon -- */

/* optimizer.py:58-59: momentum.lerp_(g, .05); u = g.lerp(momentum, .95).
 * Writes the new momentum in place and the Nesterov input u (float). */
ORC_API void orc_muon_momentum(float* mom, const float* g, float* u, int64_t n,
                               float beta_lerp, float nesterov_w) {
  for (int64_t i = 0; i < n; ++i) {
    float mo = orc_lerp(mom[i], g[i], beta_lerp);
    mom[i] = mo;
    u[i] = orc_lerp(g[i], mo, nesterov_w);
  }
}

/* optimizer.py:60-61: u *= shape_scale; p.mul_(1 - lr*wd).add_(u, alpha=-lr).
 * ATen add with alpha on the CPU vector path is fmadd(other, alpha, self). */
ORC_API void orc_muon_apply(float* w, const float* o, int64_t n, float shape_scale,
                            float cwd, float neg_lr) {
  for (int64_t i = 0; i < n; ++i) {
    float u = o[i] * shape_scale;
    float wi = w[i] * cwd;
    w[i] = fmaf(u, neg_lr, wi);
  }
}
