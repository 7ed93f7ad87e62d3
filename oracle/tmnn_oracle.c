/*
 * tmnn_oracle.c -- CPU restatement of tiny-metal-nn's hot path (TEST
 * INFRASTRUCTURE: parity checker and timed CPU baseline, never product code).
 *
 * Build: oracle/Makefile (gcc -O3 -fopenmp -ffp-contract=off).  Every
 * multiply and add is a separately rounded fp32 operation so the CUDA fp32
 * kernels (which use __fmul_rn/__fadd_rn in the same order) can be compared
 * bit for bit where the reference's arithmetic is deterministic.
 *
 * Parity pins (what ties this restatement to the reference itself):
 *  - tests/golden/ holds the reference's own known answers: the 0.34
 *    forward of tests/unit/tmnn/test_default_trainer.cpp:2260-2336, the
 *    mlpWeightCount values of tests/unit/tmnn/test_kernel_generation.cpp,
 *    the Adam-parameter split of tests/unit/tmnn/test_training_step_execution.cpp.
 *  - oracle/ref_build.py compiles the reference's own host code
 *    (morton_sort.h, kernel_spec.cpp, adam_params.h arithmetic) and the MSL
 *    text the reference's MLPKernelEmitter generates (run as C++ through a
 *    small Metal-language shim) into oracle/_ref; tests compare this file
 *    against those outputs on seeded inputs.
 *  - Philox-4x32-10 is checked against the published Random123 known-answer
 *    vectors (Salmon et al., SC'11).
 *
 * Deliberate restatement choices (documented, applied identically in CUDA):
 *  - Level resolution: one fp32 table res[l] built by iterative
 *    multiplication from the 6-decimal literals the emitter bakes
 *    (mlp_kernel_emitter.cpp:91-92, :224-236 "resolution *= PER_LEVEL_SCALE").
 *    The reference's scalar-train and scatter paths use
 *    BASE*pow(SCALE, l) (mlp_kernel_emitter.cpp:2907-2912, :677) which
 *    Metal evaluates with fast-math pow; that can differ by an ulp.
 *  - No fused multiply-add anywhere (Metal may contract; it is not
 *    observable here).
 *  - MLP gradients are summed in point order (the reference uses device
 *    float atomics in arbitrary order, mlp_kernel_emitter.cpp:2829-2836).
 */
#include "tmnn_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* mlp_kernel_emitter.cpp:16-18 (hash primes, instant-NGP) */
#define PRIME_Y 2654435761u
#define PRIME_Z 805459861u
#define PRIME_W 56711039u
/* mlp_kernel_emitter.cpp:20, :2741 */
#define GRAD_SCALE 65536.0f

#define MAX_W 512
#define MAX_O 64
#define MAX_H 8

/* ---------------------------------------------------------------- geometry */

/* The emitter prints BASE/SCALE with std::fixed << setprecision(6)
 * (mlp_kernel_emitter.cpp:91-92) and Metal parses the literal as float. */
float tmo_round6(float x) {
  char buf[64];
  snprintf(buf, sizeof buf, "%.6f", (double)x);
  return strtof(buf, NULL);
}

void tmo_level_resolutions(const tmo_spec *s, float *res) {
  float r = tmo_round6(s->base);
  const float sc = tmo_round6(s->scale);
  for (int l = 0; l < s->L; ++l) {
    if (s->res_mode == 1) {
      /* BASE_RESOLUTION * pow(PER_LEVEL_SCALE, float(l))
       * (mlp_kernel_emitter.cpp:2907, :677) */
      res[l] = tmo_round6(s->base) * powf(sc, (float)l);
    } else {
      res[l] = r;
      r = r * sc;
    }
  }
}

uint64_t tmo_hash_grid_size(const tmo_spec *s) {
  return (uint64_t)s->L * ((uint64_t)1 << s->log2T) * (uint64_t)s->F;
}

/* kernel_spec.cpp:65-71 */
int64_t tmo_mlp_weight_count(const tmo_spec *s) {
  const int64_t In = (int64_t)s->L * s->F, W = s->W, O = s->O;
  int64_t c = In * W + W;
  for (int i = 1; i < s->H; ++i) c += W * W + W;
  return c + W * O + O;
}

/* mlp_kernel_emitter.cpp:144-161: uint(x)*1 ^ uint(y)*P_Y ^ uint(z)*P_Z
 * [^ uint(w)*P_W], then % table_size (a power of two). */
uint32_t tmo_hash3(int32_t x, int32_t y, int32_t z, uint32_t T) {
  uint32_t h = (uint32_t)x * 1u ^ (uint32_t)y * PRIME_Y ^ (uint32_t)z * PRIME_Z;
  return h % T;
}
uint32_t tmo_hash4(int32_t x, int32_t y, int32_t z, int32_t w, uint32_t T) {
  uint32_t h = (uint32_t)x * 1u ^ (uint32_t)y * PRIME_Y ^
               (uint32_t)z * PRIME_Z ^ (uint32_t)w * PRIME_W;
  return h % T;
}

/* Corner enumeration of one level: dz, dy, dx nested with dx fastest, 4D adds
 * an outer dw (mlp_kernel_emitter.cpp:265-268, :305-308).  Weight product is
 * left to right: ((wx*wy)*wz)*wt. */
typedef struct {
  uint32_t off[16];  /* element offset of feature 0 */
  float w[16];       /* (wx*wy)*wz[*wt] */
  float wc[16][4];   /* per-axis weights, for the scalar scatter product */
  int32_t bc[4];
  int n;
} corners_t;

static void level_corners(const tmo_spec *s, const float *p, float res, int l,
                          corners_t *c) {
  const uint32_t T = 1u << s->log2T;
  float frac[4];
  for (int a = 0; a < s->d; ++a) {
    const float sa = p[a] * res;
    const float fl = floorf(sa);
    c->bc[a] = (int32_t)fl;
    frac[a] = sa - fl;
  }
  const uint64_t level_base = (uint64_t)l * T * (uint64_t)s->F;
  int k = 0;
  const int nw = (s->d == 4) ? 2 : 1;
  for (int dw = 0; dw < nw; ++dw)
    for (int dz = 0; dz < 2; ++dz)
      for (int dy = 0; dy < 2; ++dy)
        for (int dx = 0; dx < 2; ++dx) {
          uint32_t h;
          if (s->d == 4)
            h = tmo_hash4(c->bc[0] + dx, c->bc[1] + dy, c->bc[2] + dz,
                          c->bc[3] + dw, T);
          else
            h = tmo_hash3(c->bc[0] + dx, c->bc[1] + dy, c->bc[2] + dz, T);
          c->off[k] = (uint32_t)(level_base + (uint64_t)h * s->F);
          const float wx = dx == 0 ? 1.0f - frac[0] : frac[0];
          const float wy = dy == 0 ? 1.0f - frac[1] : frac[1];
          const float wz = dz == 0 ? 1.0f - frac[2] : frac[2];
          float w = wx * wy;
          w = w * wz;
          c->wc[k][0] = wx;
          c->wc[k][1] = wy;
          c->wc[k][2] = wz;
          if (s->d == 4) {
            const float wt = dw == 0 ? 1.0f - frac[3] : frac[3];
            w = w * wt;
            c->wc[k][3] = wt;
          }
          c->w[k] = w;
          ++k;
        }
  c->n = k;
}

/* Interpolated features of one level.  F==2 in 3D follows the float2 path
 * (mlp_kernel_emitter.cpp:264-278: feat2 += w * table2); every other case the
 * scalar path (:319-331 / 4D :305-317: feat += wx*wy*wz[*wt]*table). */
static void level_features(const tmo_spec *s, const float *table,
                           const corners_t *c, float *feat /* [F] */) {
  for (int f = 0; f < s->F; ++f) {
    float acc = 0.0f;
    for (int k = 0; k < c->n; ++k) {
      const float t = table[c->off[k] + f];
      acc = acc + c->w[k] * t;
    }
    feat[f] = acc;
  }
}

void tmo_encode(const tmo_spec *s, const float *table, const float *pos,
                int64_t N, float *feat, uint32_t *corner_idx, int32_t *cells) {
  float res[32];
  tmo_level_resolutions(s, res);
  const int In = s->L * s->F, nc = 1 << s->d;
  for (int64_t i = 0; i < N; ++i) {
    for (int l = 0; l < s->L; ++l) {
      corners_t c;
      level_corners(s, pos + i * s->d, res[l], l, &c);
      level_features(s, table, &c, feat + i * In + l * s->F);
      if (corner_idx)
        for (int k = 0; k < nc; ++k)
          corner_idx[(i * s->L + l) * nc + k] = c.off[k];
      if (cells)
        for (int a = 0; a < s->d; ++a)
          cells[(i * s->L + l) * s->d + a] = c.bc[a];
    }
  }
}

/* ------------------------------------------------------------ MLP pieces */

typedef struct {
  int64_t w_off[MAX_H + 1], b_off[MAX_H + 1]; /* [0..H-1] hidden, [H] output */
} offsets_t;

/* mlp_kernel_emitter.cpp:163-191 */
static void mlp_offsets(const tmo_spec *s, offsets_t *o) {
  const int64_t In = (int64_t)s->L * s->F, W = s->W;
  int64_t off = 0;
  o->w_off[0] = off; off += In * W;
  o->b_off[0] = off; off += W;
  for (int i = 1; i < s->H; ++i) {
    o->w_off[i] = off; off += W * W;
    o->b_off[i] = off; off += W;
  }
  o->w_off[s->H] = off; off += W * s->O;
  o->b_off[s->H] = off;
}

/* Encode fused with W0 (mlp_kernel_emitter.cpp:279-296 float2 path:
 * h0[j] += f.x*W0[2l][j] + f.y*W0[2l+1][j]; scalar path :343-358:
 * h0[j] += feat*W0[row][j]); then h0 = max(h0 + b0, 0) (:2950-2951). */
/* fp16 operand rounding of the tensor-core emulation mode (identity
 * otherwise). */
static inline float r16(int on, float x) { return on ? (float)(_Float16)x : x; }

static void forward_point(const tmo_spec *s, const float *res,
                          const float *table, const float *mlp,
                          const offsets_t *o, const float *p,
                          float acts[MAX_H][MAX_W], float *y) {
  const int W = s->W, e = s->fp16_operands;
  float *h0 = acts[0];
  for (int j = 0; j < W; ++j) h0[j] = 0.0f;
  const int vec2 = (s->F == 2 && s->d == 3);
  for (int l = 0; l < s->L; ++l) {
    corners_t c;
    float feat[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    level_corners(s, p, res[l], l, &c);
    level_features(s, table, &c, feat);
    for (int f = 0; f < s->F; ++f) feat[f] = r16(e, feat[f]);
    if (vec2) {
      const float *wa = mlp + o->w_off[0] + (int64_t)(2 * l) * W;
      const float *wb = wa + W;
      for (int j = 0; j < W; ++j) {
        const float t = feat[0] * r16(e, wa[j]) + feat[1] * r16(e, wb[j]);
        h0[j] = h0[j] + t;
      }
    } else {
      for (int f = 0; f < s->F; ++f) {
        const float *wr = mlp + o->w_off[0] + (int64_t)(l * s->F + f) * W;
        for (int j = 0; j < W; ++j) h0[j] = h0[j] + feat[f] * r16(e, wr[j]);
      }
    }
  }
  for (int j = 0; j < W; ++j) {
    const float t = h0[j] + mlp[o->b_off[0] + j];
    h0[j] = r16(e, t > 0.0f ? t : 0.0f);
  }
  /* hidden layers (mlp_kernel_emitter.cpp:2962-2970): acc = sum_i h[i]*W[i][j]
   * from 0, then max(acc + b, 0) */
  for (int k = 1; k < s->H; ++k) {
    const float *hin = acts[k - 1];
    float *hout = acts[k];
    const float *Wk = mlp + o->w_off[k];
    for (int j = 0; j < W; ++j) {
      float acc = 0.0f;
      for (int i = 0; i < W; ++i)
        acc = acc + hin[i] * r16(e, Wk[(int64_t)i * W + j]);
      const float t = acc + mlp[o->b_off[k] + j];
      hout[j] = r16(e, t > 0.0f ? t : 0.0f);
    }
  }
  /* output (mlp_kernel_emitter.cpp:2983-2997): acc starts at the bias */
  const float *hl = acts[s->H - 1];
  const float *Wo = mlp + o->w_off[s->H];
  for (int m = 0; m < s->O; ++m) {
    float acc = mlp[o->b_off[s->H] + m];
    for (int j = 0; j < W; ++j)
      acc = acc + hl[j] * r16(e, Wo[(int64_t)j * s->O + m]);
    y[m] = acc;
  }
}

void tmo_forward(const tmo_spec *s, const float *table, const float *mlp,
                 const float *pos, int64_t N, float *out) {
  float res[32];
  offsets_t o;
  tmo_level_resolutions(s, res);
  mlp_offsets(s, &o);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < N; ++i) {
    float acts[MAX_H][MAX_W];
    forward_point(s, res, table, mlp, &o, pos + i * s->d, acts,
                  out + i * s->O);
  }
}

/* Loss and dL/dy (mlp_kernel_emitter.cpp:562-670).  Multi-output loss is the
 * SUM over outputs.  Returns the per-point loss. */
static float point_loss(const tmo_spec *s, const float *y, const float *t,
                        float inv_N, float *d) {
  const int O = s->O;
  if (s->loss == TMO_LOSS_COSINE) {
    float dot = 0.0f, pn = 0.0f, tn = 0.0f;
    for (int m = 0; m < O; ++m) {
      dot = dot + y[m] * t[m];
      pn = pn + y[m] * y[m];
      tn = tn + t[m] * t[m];
    }
    const float pred_norm = sqrtf(pn + 1e-8f);
    const float target_norm = sqrtf(tn + 1e-8f);
    const float denom = pred_norm * target_norm;
    const float cosine = dot / denom;
    const float pnd = pn + 1e-8f;
    for (int m = 0; m < O; ++m) {
      const float a = (cosine * y[m]) / pnd;
      const float b = t[m] / denom;
      d[m] = (a - b) * inv_N;
    }
    return 1.0f - cosine;
  }
  float loss = 0.0f;
  for (int m = 0; m < O; ++m) {
    const float r = y[m] - t[m];
    float term;
    if (s->loss == TMO_LOSS_L2) {
      term = r * r;
      d[m] = (2.0f * r) * inv_N;
    } else if (s->loss == TMO_LOSS_L1) {
      term = fabsf(r);
      d[m] = (r > 0.0f ? 1.0f : (r < 0.0f ? -1.0f : 0.0f)) * inv_N;
    } else {
      const float ar = fabsf(r), delta = tmo_round6(s->huber_delta);
      if (ar <= delta) {
        term = (0.5f * r) * r;
        d[m] = r * inv_N;
      } else {
        term = delta * (ar - 0.5f * delta);
        d[m] = (delta * (r > 0.0f ? 1.0f : -1.0f)) * inv_N;
      }
    }
    loss = loss + term;
  }
  return loss;
}

static int32_t fixed_trunc(float x) {
  /* int(x) truncates toward zero; out-of-range saturates, NaN -> 0 (the
   * CUDA cvt.rzi.s32.f32 behaviour, used identically in the kernels). */
  if (x != x) return 0;
  if (x >= 2147483648.0f) return 2147483647;
  if (x <= -2147483648.0f) return (int32_t)0x80000000u;
  return (int32_t)x;
}

typedef struct {
  int32_t *gh_fixed;
  float *gh_float;
  uint8_t *touched;
  int atomic; /* parallel caller: use atomics on shared hash grads */
} scatter_t;

static void atomic_add_float(float *p, float v) {
  union { float f; uint32_t u; } cur, nxt;
  do {
    cur.u = __atomic_load_n((uint32_t *)p, __ATOMIC_RELAXED);
    nxt.f = cur.f + v;
  } while (!__atomic_compare_exchange_n((uint32_t *)p, &cur.u, nxt.u, 0,
                                        __ATOMIC_RELAXED, __ATOMIC_RELAXED));
}

static void scatter_one(const tmo_spec *s, scatter_t *sc, uint32_t off,
                        float v) {
  if (s->grad_mode == TMO_GRAD_FIXED16) {
    const int32_t q = fixed_trunc(v * GRAD_SCALE);
    if (sc->atomic)
      __atomic_fetch_add(&sc->gh_fixed[off], q, __ATOMIC_RELAXED);
    else
      sc->gh_fixed[off] += q;
  } else {
    if (sc->atomic)
      atomic_add_float(&sc->gh_float[off], v);
    else
      sc->gh_float[off] = sc->gh_float[off] + v;
  }
}

/* Fused forward + loss + backward + scatter of one point: the scalar train
 * kernel body (mlp_kernel_emitter.cpp:2875-3155). */
/* The fused tensor-core step with fp16 operands (tmo_spec.fp16_operands):
 * dL/dy is scaled by dscale and rounded to fp16; every pre-activation
 * gradient is rounded to fp16 after its ReLU mask; products accumulate in
 * fp32; weight and table gradients are divided by dscale; the output-bias
 * gradient uses the unscaled fp32 dL/dy. */
static float fwd_bwd_point_f16(const tmo_spec *s, const float *res,
                               const float *table, const float *mlp,
                               const offsets_t *o, const float *p,
                               const float *t, const float *dext, float inv_N,
                               float *gm, scatter_t *sc, float *yout) {
  const int W = s->W, O = s->O, H = s->H;
  const float S = s->dscale > 0.0f ? s->dscale : 1.0f, iS = 1.0f / S;
  float acts[MAX_H][MAX_W], dh[MAX_W], dn[MAX_W];
  float y[MAX_O], d[MAX_O], ds[MAX_O];
  forward_point(s, res, table, mlp, o, p, acts, y);
  if (yout)
    for (int m = 0; m < O; ++m) yout[m] = y[m];
  float loss = 0.0f;
  if (dext) {
    for (int m = 0; m < O; ++m) d[m] = dext[m];
  } else {
    loss = point_loss(s, y, t, inv_N, d);
  }
  for (int m = 0; m < O; ++m) ds[m] = r16(1, d[m] * S);
  const float *hl = acts[H - 1];
  const float *Wo = mlp + o->w_off[H];
  for (int j = 0; j < W; ++j) {
    float acc = 0.0f;
    for (int m = 0; m < O; ++m) {
      gm[o->w_off[H] + (int64_t)j * O + m] += (hl[j] * ds[m]) * iS;
      acc = acc + ds[m] * r16(1, Wo[(int64_t)j * O + m]);
    }
    dh[j] = r16(1, hl[j] > 0.0f ? acc : 0.0f);
  }
  for (int m = 0; m < O; ++m) gm[o->b_off[H] + m] += d[m];
  for (int k = H - 1; k >= 1; --k) {
    const float *hin = acts[k - 1];
    const float *Wk = mlp + o->w_off[k];
    for (int i = 0; i < W; ++i) {
      float acc = 0.0f;
      for (int j = 0; j < W; ++j) {
        gm[o->w_off[k] + (int64_t)i * W + j] += (hin[i] * dh[j]) * iS;
        acc = acc + dh[j] * r16(1, Wk[(int64_t)i * W + j]);
      }
      dn[i] = r16(1, hin[i] > 0.0f ? acc : 0.0f);
    }
    for (int j = 0; j < W; ++j) gm[o->b_off[k] + j] += dh[j] * iS;
    for (int i = 0; i < W; ++i) dh[i] = dn[i];
  }
  int levels = s->active_levels > 0 ? s->active_levels : s->L;
  if (levels > s->L) levels = s->L;
  for (int l = 0; l < levels; ++l) {
    corners_t c;
    float feat[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    level_corners(s, p, res[l], l, &c);
    level_features(s, table, &c, feat);
    for (int f = 0; f < s->F; ++f) {
      const int64_t r = o->w_off[0] + (int64_t)(l * s->F + f) * W;
      const float xf = r16(1, feat[f]);
      float df = 0.0f;
      for (int j = 0; j < W; ++j) {
        gm[r + j] += (xf * dh[j]) * iS;
        df = df + dh[j] * r16(1, mlp[r + j]);
      }
      df = df * iS;
      for (int k = 0; k < c.n; ++k) {
        const uint32_t e = c.off[k] + f;
        scatter_one(s, sc, e, df * c.w[k]);
        if (sc->touched) sc->touched[s->F == 2 ? e >> 1 : e] = 1;
      }
    }
  }
  for (int j = 0; j < W; ++j) gm[o->b_off[0] + j] += dh[j] * iS;
  return loss;
}

static float fwd_bwd_point(const tmo_spec *s, const float *res,
                           const float *table, const float *mlp,
                           const offsets_t *o, const float *p, const float *t,
                           const float *dext, float inv_N, float *gm,
                           scatter_t *sc, float *yout) {
  if (s->fp16_operands)
    return fwd_bwd_point_f16(s, res, table, mlp, o, p, t, dext, inv_N, gm, sc,
                             yout);
  const int W = s->W, O = s->O, H = s->H;
  float acts[MAX_H][MAX_W];
  float y[MAX_O], d[MAX_O];
  forward_point(s, res, table, mlp, o, p, acts, y);
  if (yout)
    for (int m = 0; m < O; ++m) yout[m] = y[m];
  float loss = 0.0f;
  if (dext) {
    for (int m = 0; m < O; ++m) d[m] = dext[m];
  } else {
    loss = point_loss(s, y, t, inv_N, d);
  }
  /* output layer backward (:3061-3086): dWo[j][m] += d_m*h_j;
   * d_pre_j = (sum_m d_m*Wo[j][m]) * relu'(h_j) */
  float *hl = acts[H - 1];
  const float *Wo = mlp + o->w_off[H];
  for (int j = 0; j < W; ++j) {
    const float hv = hl[j];
    float dpre = 0.0f;
    for (int m = 0; m < O; ++m) {
      gm[o->w_off[H] + (int64_t)j * O + m] += d[m] * hv;
      if (O == 1)
        dpre = d[m] * Wo[j];
      else
        dpre = dpre + d[m] * Wo[(int64_t)j * O + m];
    }
    hl[j] = dpre * (hv > 0.0f ? 1.0f : 0.0f);
  }
  for (int m = 0; m < O; ++m) gm[o->b_off[H] + m] += d[m];
  /* hidden layers backward (:3098-3113) */
  for (int k = H - 1; k >= 1; --k) {
    const float *dk = acts[k];
    float *hin = acts[k - 1];
    const float *Wk = mlp + o->w_off[k];
    for (int i = 0; i < W; ++i) {
      const float hv = hin[i];
      for (int j = 0; j < W; ++j)
        gm[o->w_off[k] + (int64_t)i * W + j] += dk[j] * hv;
      float acc = 0.0f;
      for (int j = 0; j < W; ++j) acc = acc + dk[j] * Wk[(int64_t)i * W + j];
      hin[i] = acc * (hv > 0.0f ? 1.0f : 0.0f);
    }
    for (int j = 0; j < W; ++j) gm[o->b_off[k] + j] += dk[j];
  }
  /* layer 0 + hash scatter (emitHashScatter :672-901) */
  const float *h0 = acts[0]; /* now d_pre of layer 0 */
  int levels = s->active_levels > 0 ? s->active_levels : s->L;
  if (levels > s->L) levels = s->L;
  const int vec2 = (s->F == 2 && s->d == 3);
  for (int l = 0; l < levels; ++l) {
    corners_t c;
    float feat[4];
    level_corners(s, p, res[l], l, &c);
    level_features(s, table, &c, feat);
    if (vec2) {
      const int64_t r0 = o->w_off[0] + (int64_t)(2 * l) * W, r1 = r0 + W;
      for (int j = 0; j < W; ++j) {
        gm[r0 + j] += h0[j] * feat[0];
        gm[r1 + j] += h0[j] * feat[1];
      }
      float dfx = 0.0f, dfy = 0.0f;
      for (int j = 0; j < W; ++j) {
        dfx = dfx + h0[j] * mlp[r0 + j];
        dfy = dfy + h0[j] * mlp[r1 + j];
      }
      for (int k = 0; k < c.n; ++k) {
        /* int(d_feat2.x * w * GRAD_SCALE) (:735-738) */
        scatter_one(s, sc, c.off[k], dfx * c.w[k]);
        scatter_one(s, sc, c.off[k] + 1, dfy * c.w[k]);
        if (sc->touched) sc->touched[c.off[k] >> 1] = 1;
      }
    } else {
      for (int f = 0; f < s->F; ++f) {
        const int64_t r = o->w_off[0] + (int64_t)(l * s->F + f) * W;
        for (int j = 0; j < W; ++j) gm[r + j] += h0[j] * feat[f];
        float df = 0.0f;
        for (int j = 0; j < W; ++j) df = df + h0[j] * mlp[r + j];
        for (int k = 0; k < c.n; ++k) {
          /* int(d_feat * wx * wy * wz [* wt] * GRAD_SCALE) (:853-861) */
          float v = df * c.wc[k][0];
          v = v * c.wc[k][1];
          v = v * c.wc[k][2];
          if (s->d == 4) v = v * c.wc[k][3];
          scatter_one(s, sc, c.off[k] + f, v);
          if (sc->touched) {
            const uint32_t e = c.off[k] + f;
            sc->touched[s->F == 2 ? e >> 1 : e] = 1;
          }
        }
      }
    }
  }
  for (int j = 0; j < W; ++j) gm[o->b_off[0] + j] += h0[j];
  return loss;
}

double tmo_fwd_bwd(const tmo_spec *s, const float *table, const float *mlp,
                   const float *pos, const float *tgt, const float *d_out_ext,
                   int64_t N, int64_t inv_count, float *grad_mlp,
                   int32_t *grad_hash_fixed, float *grad_hash_float,
                   uint8_t *touched, float *out) {
  if (N <= 0) return 0.0;
  float res[32];
  offsets_t o;
  tmo_level_resolutions(s, res);
  mlp_offsets(s, &o);
  const float inv_N = 1.0f / (float)(inv_count > 0 ? inv_count : N);
  scatter_t sc = {grad_hash_fixed, grad_hash_float, touched, 0};
  double total = 0.0;
  for (int64_t i = 0; i < N; ++i) {
    total += fwd_bwd_point(s, res, table, mlp, &o, pos + i * s->d,
                           tgt ? tgt + i * s->O : NULL,
                           d_out_ext ? d_out_ext + i * s->O : NULL, inv_N,
                           grad_mlp, &sc, out ? out + i * s->O : NULL);
  }
  return total;
}

double tmo_fwd_bwd_par(const tmo_spec *s, const float *table, const float *mlp,
                       const float *pos, const float *tgt, int64_t N,
                       int64_t inv_count, float *grad_mlp,
                       int32_t *grad_hash_fixed, float *grad_hash_float,
                       uint8_t *touched, int nthreads) {
  if (N <= 0) return 0.0;
  float res[32];
  offsets_t o;
  tmo_level_resolutions(s, res);
  mlp_offsets(s, &o);
  const float inv_N = 1.0f / (float)(inv_count > 0 ? inv_count : N);
  const int64_t nm = tmo_mlp_weight_count(s);
  double total = 0.0;
#ifdef _OPENMP
  if (nthreads <= 0) nthreads = omp_get_max_threads();
#else
  nthreads = 1;
#endif
  float *part = (float *)calloc((size_t)nthreads * (size_t)nm, sizeof(float));
#pragma omp parallel num_threads(nthreads) reduction(+ : total)
  {
    int tid = 0;
#ifdef _OPENMP
    tid = omp_get_thread_num();
#endif
    float *gm = part + (size_t)tid * (size_t)nm;
    scatter_t sc = {grad_hash_fixed, grad_hash_float, touched, 1};
#pragma omp for schedule(static)
    for (int64_t i = 0; i < N; ++i)
      total += fwd_bwd_point(s, res, table, mlp, &o, pos + i * s->d,
                             tgt + i * s->O, NULL, inv_N, gm, &sc, NULL);
  }
  for (int t = 0; t < nthreads; ++t)
    for (int64_t k = 0; k < nm; ++k) grad_mlp[k] += part[(size_t)t * nm + k];
  free(part);
  return total;
}

/* ------------------------------------------------------------------- Adam */

/* adam_params.h:33-52: bc_k = 1 - pow(beta_k, step+1) in float. */
void tmo_adam_bias_corrections(float beta1, float beta2, uint32_t step,
                               float *bc1, float *bc2) {
  const float sf = (float)(step + 1u);
  *bc1 = 1.0f - powf(beta1, sf);
  *bc2 = 1.0f - powf(beta2, sf);
}

/* adam_kernel_msl.h:37-109 (unified) and :120-203 (sparse hash / dense MLP). */
static void adam_elem(float *w, float *m, float *v, float g, float lr,
                      float b1, float b2, float eps, float bc1, float bc2,
                      float clip, float wd, float reg, int is_mlp) {
  if (clip > 0.0f) g = g < -clip ? -clip : (g > clip ? clip : g);
  if (wd > 0.0f) {
    const float t = (lr * wd) * (*w);
    *w = *w - t;
  } else if (reg > 0.0f) {
    if (is_mlp) {
      g = g + reg * (*w);
    } else {
      const float wv = *w;
      g = g + reg * (wv > 0.0f ? 1.0f : (wv < 0.0f ? -1.0f : 0.0f));
    }
  }
  const float mn = b1 * (*m) + (1.0f - b1) * g;
  const float vn = b2 * (*v) + ((1.0f - b2) * g) * g;
  *m = mn;
  *v = vn;
  const float mh = mn / bc1;
  const float vh = vn / bc2;
  const float upd = (lr * mh) / (sqrtf(vh) + eps);
  *w = *w - upd;
}

void tmo_adam(const tmo_adam_cfg *c, float *w, float *m, float *v,
              uint64_t hash_count, uint64_t mlp_count,
              const int32_t *grad_hash_fixed, const float *grad_hash_float,
              const float *grad_mlp, const uint8_t *touched, int nthreads) {
  float bc1, bc2;
  tmo_adam_bias_corrections(c->beta1, c->beta2, c->step, &bc1, &bc2);
  const uint64_t total = hash_count + mlp_count;
  const int ew = c->entry_width > 0 ? c->entry_width : 1;
#ifdef _OPENMP
  if (nthreads <= 0) nthreads = omp_get_max_threads();
#else
  (void)nthreads;
#endif
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
  for (int64_t i = 0; i < (int64_t)total; ++i) {
    const int is_mlp = (uint64_t)i >= hash_count;
    float g;
    if (is_mlp) {
      g = grad_mlp[i - hash_count];
    } else {
      if (c->sparse_hash && !touched[i / ew]) continue;
      g = grad_hash_fixed ? (float)grad_hash_fixed[i] * (1.0f / 65536.0f)
                          : grad_hash_float[i];
    }
    adam_elem(&w[i], &m[i], &v[i], g, is_mlp ? c->lr_mlp : c->lr_hash,
              c->beta1, c->beta2, c->eps, bc1, bc2, c->grad_clip,
              c->weight_decay, is_mlp ? c->l2_mlp : c->l1_hash, is_mlp);
  }
}

/* ------------------------------------------------------------- Philox init */

/* metal_context.cpp:737-756: standard Philox-4x32-10 (Salmon et al. 2011). */
void tmo_philox4x32_10(const uint32_t ctr_in[4], const uint32_t key_in[2],
                       uint32_t out[4]) {
  uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
  uint32_t k0 = key_in[0], k1 = key_in[1];
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c0;
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    c0 = hi1 ^ c1 ^ k0;
    c1 = lo1;
    c2 = hi0 ^ c3 ^ k1;
    c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* metal_context.cpp:765-790: thread t draws ctr=(base+t,0,0,0), key=seed;
 * u = float(r) * 2^-32; v = low + u*(high-low). */
void tmo_init_uniform(float *out, uint64_t count, float low, float high,
                      uint64_t seed, uint32_t counter_base) {
  const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  const uint64_t threads = (count + 3) / 4;
  const float kScale = 1.0f / 4294967296.0f;
  const float span = high - low;
  for (uint64_t t = 0; t < threads; ++t) {
    const uint32_t ctr[4] = {counter_base + (uint32_t)t, 0u, 0u, 0u};
    uint32_t r[4];
    tmo_philox4x32_10(ctr, key, r);
    for (int k = 0; k < 4; ++k) {
      const uint64_t e = t * 4 + (uint64_t)k;
      if (e >= count) break;
      const float u = (float)r[k] * kScale;
      out[e] = low + u * span;
    }
  }
}

/* metal_context.cpp:837-873: Box-Muller pairs (u1,u2), (u3,u4). */
void tmo_init_normal(float *out, uint64_t count, float mean, float stddev,
                     uint64_t seed, uint32_t counter_base) {
  const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  const uint64_t threads = (count + 3) / 4;
  const float kScale = 1.0f / 4294967296.0f;
  const float TWO_PI = 6.28318530718f;
  for (uint64_t t = 0; t < threads; ++t) {
    const uint32_t ctr[4] = {counter_base + (uint32_t)t, 0u, 0u, 0u};
    uint32_t r[4];
    tmo_philox4x32_10(ctr, key, r);
    float u1 = (float)r[0] * kScale, u2 = (float)r[1] * kScale;
    float u3 = (float)r[2] * kScale, u4 = (float)r[3] * kScale;
    if (u1 < 1.0e-30f) u1 = 1.0e-30f;
    if (u3 < 1.0e-30f) u3 = 1.0e-30f;
    const float r1 = sqrtf(-2.0f * logf(u1)), r2 = sqrtf(-2.0f * logf(u3));
    const float z[4] = {r1 * cosf(TWO_PI * u2), r1 * sinf(TWO_PI * u2),
                        r2 * cosf(TWO_PI * u4), r2 * sinf(TWO_PI * u4)};
    for (int k = 0; k < 4; ++k) {
      const uint64_t e = t * 4 + (uint64_t)k;
      if (e >= count) break;
      out[e] = mean + stddev * z[k];
    }
  }
}

/* default_trainer.cpp:1978-2180: hash U(-r, r) at counter 0; MLP per layer,
 * weights then bias, each advancing the counter by ceil(count/4). */
void tmo_init_weights(const tmo_spec *s, const tmo_init_cfg *c, float *hash,
                      float *mlp) {
  const uint64_t hc = tmo_hash_grid_size(s);
  if (c->hash_zero)
    memset(hash, 0, hc * sizeof(float));
  else
    tmo_init_uniform(hash, hc, -c->hash_range, c->hash_range, c->seed, 0u);
  uint32_t cb = (uint32_t)((hc + 3) / 4);
  const int64_t nm = tmo_mlp_weight_count(s);
  if (c->mlp_mode == TMO_MLP_UNIFORM) {
    tmo_init_uniform(mlp, (uint64_t)nm, -c->mlp_uniform_range,
                     c->mlp_uniform_range, c->seed, cb);
    return;
  }
  if (c->mlp_mode == TMO_MLP_NORMAL) {
    tmo_init_normal(mlp, (uint64_t)nm, 0.0f, c->mlp_normal_stddev, c->seed, cb);
    return;
  }
  if (c->mlp_mode == TMO_MLP_ZERO) {
    memset(mlp, 0, (size_t)nm * sizeof(float));
    return;
  }
  const int In = s->L * s->F, W = s->W;
  int64_t off = 0;
  for (int layer = 0; layer <= s->H; ++layer) {
    const int fin = layer == 0 ? In : W;
    const int fout = layer == s->H ? s->O : W;
    const int64_t wc = (int64_t)fin * fout;
    const float fi = (float)fin, fo = (float)fout;
    switch (c->mlp_mode) {
      case TMO_MLP_KAIMING_UNIFORM: {
        const float b = c->gain * sqrtf(3.0f / fi);
        tmo_init_uniform(mlp + off, (uint64_t)wc, -b, b, c->seed, cb);
        break;
      }
      case TMO_MLP_KAIMING_NORMAL:
        tmo_init_normal(mlp + off, (uint64_t)wc, 0.0f, c->gain / sqrtf(fi),
                        c->seed, cb);
        break;
      case TMO_MLP_XAVIER_UNIFORM: {
        const float b = sqrtf(6.0f / (fi + fo));
        tmo_init_uniform(mlp + off, (uint64_t)wc, -b, b, c->seed, cb);
        break;
      }
      default:
        tmo_init_normal(mlp + off, (uint64_t)wc, 0.0f, sqrtf(2.0f / (fi + fo)),
                        c->seed, cb);
        break;
    }
    cb += (uint32_t)((wc + 3) / 4);
    off += wc;
    const float bb = 1.0f / sqrtf(fi);
    tmo_init_uniform(mlp + off, (uint64_t)fout, -bb, bb, c->seed, cb);
    cb += (uint32_t)((fout + 3) / 4);
    off += fout;
  }
}

/* ------------------------------------------------------------------ Morton */

/* morton_sort.h:14-58 */
static uint32_t expand3(uint32_t v) {
  v = (v | (v << 16)) & 0x030000FFu;
  v = (v | (v << 8)) & 0x0300F00Fu;
  v = (v | (v << 4)) & 0x030C30C3u;
  v = (v | (v << 2)) & 0x09249249u;
  return v;
}
static uint32_t expand4(uint32_t v) {
  v &= 0xFFu;
  v = (v | (v << 16)) & 0x000F000Fu;
  v = (v | (v << 8)) & 0x00C30C03u;
  v = (v | (v << 4)) & 0x09090909u;
  v = (v | (v << 2)) & 0x11111111u;
  return v;
}
static uint32_t quant(float v, float cells) {
  const float mapped = (v * 0.5f + 0.5f) * cells;
  return (uint32_t)fminf(fmaxf(mapped, 0.0f), cells - 1.0f);
}
uint32_t tmo_morton3(float x, float y, float z) {
  return (expand3(quant(z, 1024.0f)) << 2) | (expand3(quant(y, 1024.0f)) << 1) |
         expand3(quant(x, 1024.0f));
}
uint32_t tmo_morton4(float x, float y, float z, float w) {
  return (expand4(quant(w, 256.0f)) << 3) | (expand4(quant(z, 256.0f)) << 2) |
         (expand4(quant(y, 256.0f)) << 1) | expand4(quant(x, 256.0f));
}

static const uint32_t *g_codes;
static int cmp_code(const void *a, const void *b) {
  const uint32_t ia = *(const uint32_t *)a, ib = *(const uint32_t *)b;
  if (g_codes[ia] != g_codes[ib]) return g_codes[ia] < g_codes[ib] ? -1 : 1;
  return ia < ib ? -1 : (ia > ib ? 1 : 0);
}

void tmo_morton_order(const float *pos, int64_t N, int d, uint32_t *perm) {
  uint32_t *codes = (uint32_t *)malloc((size_t)(N > 0 ? N : 1) * 4);
  for (int64_t i = 0; i < N; ++i) {
    const float *p = pos + i * d;
    codes[i] = d == 4 ? tmo_morton4(p[0], p[1], p[2], p[3])
                      : tmo_morton3(p[0], p[1], p[2]);
    perm[i] = (uint32_t)i;
  }
  g_codes = codes;
  qsort(perm, (size_t)N, sizeof(uint32_t), cmp_code);
  free(codes);
}

/* ------------------------------------------------- plain MLP (no encoding) */

/* FullyFusedMLP evaluated on given input features x [N x In] (In = L*F):
 * the layer loops of forward_point (mlp_kernel_emitter.cpp:362-480) without
 * the hash encode.  With fp16_operands the inputs, weights and activations
 * are rounded to fp16 as a tensor-core kernel consumes them. */
void tmo_mlp_forward(const tmo_spec *s, const float *mlp, const float *x,
                     int64_t N, float *out) {
  offsets_t o;
  mlp_offsets(s, &o);
  const int In = s->L * s->F, W = s->W, e = s->fp16_operands;
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    float a[MAX_W], b[MAX_W];
    const float *xi = x + n * In;
    for (int j = 0; j < W; ++j) {
      float acc = 0.0f;
      for (int i = 0; i < In; ++i)
        acc = acc + r16(e, xi[i]) * r16(e, mlp[o.w_off[0] + (int64_t)i * W + j]);
      const float t = acc + mlp[o.b_off[0] + j];
      a[j] = r16(e, t > 0.0f ? t : 0.0f);
    }
    for (int k = 1; k < s->H; ++k) {
      for (int j = 0; j < W; ++j) {
        float acc = 0.0f;
        for (int i = 0; i < W; ++i)
          acc = acc + a[i] * r16(e, mlp[o.w_off[k] + (int64_t)i * W + j]);
        const float t = acc + mlp[o.b_off[k] + j];
        b[j] = r16(e, t > 0.0f ? t : 0.0f);
      }
      for (int j = 0; j < W; ++j) a[j] = b[j];
    }
    for (int m = 0; m < s->O; ++m) {
      float acc = mlp[o.b_off[s->H] + m];
      for (int j = 0; j < W; ++j)
        acc = acc + a[j] * r16(e, mlp[o.w_off[s->H] + (int64_t)j * s->O + m]);
      out[n * s->O + m] = acc;
    }
  }
}

/* ------------------------------------------- analytic input gradient */

/* Table value of one corner: hash_grid_lookup (mlp_kernel_emitter.cpp:1663-1671). */
static float corner_value(const tmo_spec *s, const float *table, int l, int f,
                          const int32_t *bc, int dx, int dy, int dz, int dw) {
  const uint32_t T = 1u << s->log2T;
  const uint32_t h = s->d == 4
      ? tmo_hash4(bc[0] + dx, bc[1] + dy, bc[2] + dz, bc[3] + dw, T)
      : tmo_hash3(bc[0] + dx, bc[1] + dy, bc[2] + dz, T);
  return table[(uint64_t)l * T * s->F + (uint64_t)h * s->F + f];
}

/* trilinear_feature_grad (mlp_kernel_emitter.cpp:1674-1705): the value by
 * lerps along x, then y, then z; the three partial derivatives of the
 * trilinear interpolant w.r.t. the cell fraction. */
static float trilinear_grad(const tmo_spec *s, const float *table, int l,
                            int f, const int32_t *bc, const float *fr,
                            float *g) {
  const float fx = fr[0], fy = fr[1], fz = fr[2];
  const float c000 = corner_value(s, table, l, f, bc, 0, 0, 0, 0);
  const float c001 = corner_value(s, table, l, f, bc, 0, 0, 1, 0);
  const float c010 = corner_value(s, table, l, f, bc, 0, 1, 0, 0);
  const float c011 = corner_value(s, table, l, f, bc, 0, 1, 1, 0);
  const float c100 = corner_value(s, table, l, f, bc, 1, 0, 0, 0);
  const float c101 = corner_value(s, table, l, f, bc, 1, 0, 1, 0);
  const float c110 = corner_value(s, table, l, f, bc, 1, 1, 0, 0);
  const float c111 = corner_value(s, table, l, f, bc, 1, 1, 1, 0);
  const float ox = 1.0f - fx, oy = 1.0f - fy, oz = 1.0f - fz;
  const float c00 = c000 * ox + c100 * fx;
  const float c01 = c001 * ox + c101 * fx;
  const float c10 = c010 * ox + c110 * fx;
  const float c11 = c011 * ox + c111 * fx;
  const float c0 = c00 * oy + c10 * fy;
  const float c1 = c01 * oy + c11 * fy;
  const float val = c0 * oz + c1 * fz;
  g[0] = oz * (oy * (c100 - c000) + fy * (c110 - c010)) +
         fz * (oy * (c101 - c001) + fy * (c111 - c011));
  g[1] = oz * (ox * (c010 - c000) + fx * (c110 - c100)) +
         fz * (ox * (c011 - c001) + fx * (c111 - c101));
  g[2] = oy * (ox * (c001 - c000) + fx * (c101 - c100)) +
         fy * (ox * (c011 - c010) + fx * (c111 - c110));
  return val;
}

/* Partial derivatives of the quadrilinear interpolant (4D branch of
 * emitGradientKernelImpl, mlp_kernel_emitter.cpp:1996-2024): each is a sum
 * over the other three axes, loops nested in the order written there, of
 * ((w_a*w_b)*w_c) * (upper - lower). */
static void quadrilinear_grad(const tmo_spec *s, const float *table, int l,
                              int f, const int32_t *bc, const float *fr,
                              float *g) {
  float c[2][2][2][2]; /* [dw][dz][dy][dx] */
  for (int dw = 0; dw < 2; ++dw)
    for (int dz = 0; dz < 2; ++dz)
      for (int dy = 0; dy < 2; ++dy)
        for (int dx = 0; dx < 2; ++dx)
          c[dw][dz][dy][dx] = corner_value(s, table, l, f, bc, dx, dy, dz, dw);
#define W_(a, k) ((k) == 0 ? 1.0f - fr[a] : fr[a])
  float gx = 0, gy = 0, gz = 0, gt = 0;
  for (int dw = 0; dw < 2; ++dw)
    for (int dz = 0; dz < 2; ++dz)
      for (int dy = 0; dy < 2; ++dy)
        gx += ((W_(1, dy) * W_(2, dz)) * W_(3, dw)) *
              (c[dw][dz][dy][1] - c[dw][dz][dy][0]);
  for (int dw = 0; dw < 2; ++dw)
    for (int dz = 0; dz < 2; ++dz)
      for (int dx = 0; dx < 2; ++dx)
        gy += ((W_(0, dx) * W_(2, dz)) * W_(3, dw)) *
              (c[dw][dz][1][dx] - c[dw][dz][0][dx]);
  for (int dw = 0; dw < 2; ++dw)
    for (int dy = 0; dy < 2; ++dy)
      for (int dx = 0; dx < 2; ++dx)
        gz += ((W_(0, dx) * W_(1, dy)) * W_(3, dw)) *
              (c[dw][1][dy][dx] - c[dw][0][dy][dx]);
  for (int dz = 0; dz < 2; ++dz)
    for (int dy = 0; dy < 2; ++dy)
      for (int dx = 0; dx < 2; ++dx)
        gt += ((W_(0, dx) * W_(1, dy)) * W_(2, dz)) *
              (c[1][dz][dy][dx] - c[0][dz][dy][dx]);
#undef W_
  g[0] = gx; g[1] = gy; g[2] = gz; g[3] = gt;
}

static void cell_of(const tmo_spec *s, const float *p, float res, int32_t *bc,
                    float *fr) {
  for (int a = 0; a < s->d; ++a) {
    const float sa = p[a] * res;
    const float fl = floorf(sa);
    bc[a] = (int32_t)fl;
    fr[a] = sa - fl;
  }
}

void tmo_eval_gradient(const tmo_spec *s, const float *table, const float *mlp,
                       const float *pos, int64_t N, float *out, float *grad) {
  float res[32];
  offsets_t o;
  tmo_level_resolutions(s, res);
  mlp_offsets(s, &o);
  const int W = s->W, F = s->F, H = s->H, d = s->d;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < N; ++i) {
    const float *p = pos + i * d;
    float acts[MAX_H][MAX_W], ga[MAX_W], gb[MAX_W];
    int32_t bc[4];
    float fr[4], tg[4];
    /* forward (mlp_kernel_emitter.cpp:1892-1945): per level and feature the
     * interpolated value times the W0 row, accumulated into h0 */
    float *h0 = acts[0];
    for (int j = 0; j < W; ++j) h0[j] = 0.0f;
    for (int l = 0; l < s->L; ++l) {
      cell_of(s, p, res[l], bc, fr);
      for (int f = 0; f < F; ++f) {
        float feat;
        if (d == 4) {
          corners_t c;
          level_corners(s, p, res[l], l, &c);
          feat = 0.0f;
          for (int k = 0; k < c.n; ++k)
            feat = feat + c.w[k] * table[c.off[k] + f];
        } else {
          feat = trilinear_grad(s, table, l, f, bc, fr, tg);
        }
        const float *wr = mlp + o.w_off[0] + (int64_t)(l * F + f) * W;
        for (int j = 0; j < W; ++j) h0[j] = h0[j] + feat * wr[j];
      }
    }
    for (int j = 0; j < W; ++j) {
      const float t = h0[j] + mlp[o.b_off[0] + j];
      h0[j] = t > 0.0f ? t : 0.0f;
    }
    for (int k = 1; k < H; ++k)
      for (int j = 0; j < W; ++j) {
        float acc = 0.0f;
        for (int q = 0; q < W; ++q)
          acc = acc + acts[k - 1][q] * mlp[o.w_off[k] + (int64_t)q * W + j];
        const float t = acc + mlp[o.b_off[k] + j];
        acts[k][j] = t > 0.0f ? t : 0.0f;
      }
    /* backward from d(out)/d(out) = 1 (:1947-1971): the output row masked by
     * the last activation, then through the hidden layers */
    float *cur = ga, *nxt = gb;
    for (int j = 0; j < W; ++j)
      cur[j] = mlp[o.w_off[H] + j] * (acts[H - 1][j] > 0.0f ? 1.0f : 0.0f);
    for (int k = H - 1; k >= 1; --k) {
      for (int q = 0; q < W; ++q) {
        float acc = 0.0f;
        for (int j = 0; j < W; ++j)
          acc = acc + cur[j] * mlp[o.w_off[k] + (int64_t)q * W + j];
        nxt[q] = acc * (acts[k - 1][q] > 0.0f ? 1.0f : 0.0f);
      }
      float *t = cur; cur = nxt; nxt = t;
    }
    /* position gradient (:1973-2033): sum over levels and features of
     * (grad_feat * resolution) * d(interpolant)/d(frac) */
    float gp[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int l = 0; l < s->L; ++l) {
      cell_of(s, p, res[l], bc, fr);
      for (int f = 0; f < F; ++f) {
        const float *wr = mlp + o.w_off[0] + (int64_t)(l * F + f) * W;
        float gf = 0.0f;
        for (int j = 0; j < W; ++j) gf = gf + cur[j] * wr[j];
        if (d == 4)
          quadrilinear_grad(s, table, l, f, bc, fr, tg);
        else
          trilinear_grad(s, table, l, f, bc, fr, tg);
        const float sc = gf * res[l];
        for (int a = 0; a < d; ++a) gp[a] = gp[a] + sc * tg[a];
      }
    }
    /* output (:2064-2070): bias plus the last activations times the output
     * column */
    float y = mlp[o.b_off[H]];
    for (int j = 0; j < W; ++j) y = y + acts[H - 1][j] * mlp[o.w_off[H] + j];
    out[i] = y;
    for (int a = 0; a < d; ++a) grad[i * d + a] = gp[a];
  }
}

/* ------------------------------------------- plain MLP training, SH */

/* Forward, loss and backward of a plain MLP (no encoding) on inputs x
 * [N x In] (In = L*F), the arithmetic of forward_point / backward without
 * the hash parts.  out_act 1 applies a sigmoid to every output; the loss
 * (point_loss against tgt) is then on the activated outputs and its
 * gradient passes through y (1 - y).  Accumulates grad_mlp, writes dL/dx to
 * dx [N x In] when non-NULL, returns the summed loss. */
double tmo_mlp_train(const tmo_spec *s, const float *mlp, const float *x,
                     const float *tgt, int64_t N, int64_t inv_count,
                     int out_act, float *grad_mlp, float *dx) {
  offsets_t o;
  mlp_offsets(s, &o);
  const int In = s->L * s->F, W = s->W, H = s->H, O = s->O;
  const float inv_N = inv_count > 0 ? 1.0f / (float)inv_count : 0.0f;
  double loss = 0.0;
  for (int64_t n = 0; n < N; ++n) {
    float acts[MAX_H][MAX_W], y[MAX_O], d[MAX_O], g[MAX_W], g2[MAX_W];
    const float *xi = x + n * In;
    for (int j = 0; j < W; ++j) {
      float acc = 0.0f;
      for (int i = 0; i < In; ++i)
        acc = acc + xi[i] * mlp[o.w_off[0] + (int64_t)i * W + j];
      const float t = acc + mlp[o.b_off[0] + j];
      acts[0][j] = t > 0.0f ? t : 0.0f;
    }
    for (int k = 1; k < H; ++k)
      for (int j = 0; j < W; ++j) {
        float acc = 0.0f;
        for (int i = 0; i < W; ++i)
          acc = acc + acts[k - 1][i] * mlp[o.w_off[k] + (int64_t)i * W + j];
        const float t = acc + mlp[o.b_off[k] + j];
        acts[k][j] = t > 0.0f ? t : 0.0f;
      }
    for (int m = 0; m < O; ++m) {
      float acc = mlp[o.b_off[H] + m];
      for (int j = 0; j < W; ++j)
        acc = acc + acts[H - 1][j] * mlp[o.w_off[H] + (int64_t)j * O + m];
      y[m] = out_act == 1 ? 1.0f / (1.0f + expf(-acc)) : acc;
    }
    loss += point_loss(s, y, tgt + n * O, inv_N, d);
    if (out_act == 1)
      for (int m = 0; m < O; ++m) d[m] = d[m] * (y[m] * (1.0f - y[m]));
    /* output layer */
    for (int j = 0; j < W; ++j) {
      float acc = 0.0f;
      for (int m = 0; m < O; ++m) {
        grad_mlp[o.w_off[H] + (int64_t)j * O + m] += d[m] * acts[H - 1][j];
        acc = acc + d[m] * mlp[o.w_off[H] + (int64_t)j * O + m];
      }
      g[j] = acts[H - 1][j] > 0.0f ? acc : 0.0f;
    }
    for (int m = 0; m < O; ++m) grad_mlp[o.b_off[H] + m] += d[m];
    for (int k = H - 1; k >= 1; --k) {
      for (int i = 0; i < W; ++i) {
        float acc = 0.0f;
        for (int j = 0; j < W; ++j) {
          grad_mlp[o.w_off[k] + (int64_t)i * W + j] += g[j] * acts[k - 1][i];
          acc = acc + g[j] * mlp[o.w_off[k] + (int64_t)i * W + j];
        }
        g2[i] = acts[k - 1][i] > 0.0f ? acc : 0.0f;
      }
      for (int j = 0; j < W; ++j) {
        grad_mlp[o.b_off[k] + j] += g[j];
        g[j] = g2[j];
      }
    }
    for (int i = 0; i < In; ++i) {
      float acc = 0.0f;
      for (int j = 0; j < W; ++j) {
        grad_mlp[o.w_off[0] + (int64_t)i * W + j] += g[j] * xi[i];
        acc = acc + g[j] * mlp[o.w_off[0] + (int64_t)i * W + j];
      }
      if (dx) dx[n * In + i] = acc;
    }
    for (int j = 0; j < W; ++j) grad_mlp[o.b_off[0] + j] += g[j];
  }
  return loss;
}

/* Real spherical harmonics of degree < 4 (16 coefficients) of a unit
 * direction, graphics sign convention (Sloan 2008, appendix). */
void tmo_sh4(float x, float y, float z, float *o) {
  const float xx = x * x, yy = y * y, zz = z * z;
  o[0] = 0.28209479177387814f;
  o[1] = -0.48860251190291987f * y;
  o[2] = 0.48860251190291987f * z;
  o[3] = -0.48860251190291987f * x;
  o[4] = 1.0925484305920792f * (x * y);
  o[5] = -1.0925484305920792f * (y * z);
  o[6] = 0.94617469575755997f * zz - 0.31539156525251999f;
  o[7] = -1.0925484305920792f * (x * z);
  o[8] = 0.54627421529603959f * (xx - yy);
  o[9] = 0.59004358992664352f * y * (yy - 3.0f * xx);
  o[10] = 2.8906114426405538f * (x * y) * z;
  o[11] = 0.45704579946446572f * y * (1.0f - 5.0f * zz);
  o[12] = 0.3731763325901154f * z * (5.0f * zz - 3.0f);
  o[13] = 0.45704579946446572f * x * (1.0f - 5.0f * zz);
  o[14] = 1.4453057213202769f * z * (xx - yy);
  o[15] = 0.59004358992664352f * x * (3.0f * yy - xx);
}
