/*
 * tmnn_oracle.h -- CPU restatement of tiny-metal-nn's neural-field hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * CUDA implementation and the timed CPU baseline of bench.py.  Nothing in
 * the product (the CUDA library, its C ABI, the Python wrapper) may link,
 * load or call it.
 *
 * Every function restates the arithmetic of the MSL that tmnn generates
 * (src/tiny_metal_nn/kernels/mlp_kernel_emitter.cpp) or its static MSL
 * (include/tiny-metal-nn/kernels/adam_kernel_msl.h,
 *  src/tiny_metal_nn/runtime/metal_context.cpp) in plain C, operation by
 * operation, with every multiply and add rounded separately (the library is
 * compiled with -ffp-contract=off).  Citations are file:line into the
 * reference project.
 *
 * Parity pins: see oracle/tmnn_oracle.c header.
 */
#ifndef TMNN_ORACLE_H
#define TMNN_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { TMO_LOSS_L2 = 0, TMO_LOSS_L1 = 1, TMO_LOSS_HUBER = 2, TMO_LOSS_COSINE = 3 };
enum { TMO_GRAD_FIXED16 = 0, TMO_GRAD_FLOAT = 1 };

typedef struct tmo_spec {
  int32_t L;          /* levels */
  int32_t F;          /* features per level (1, 2, 4) */
  int32_t log2T;      /* log2 hashmap size */
  int32_t d;          /* spatial dims (3, 4) */
  int32_t W;          /* hidden width */
  int32_t H;          /* hidden layers */
  int32_t O;          /* outputs */
  int32_t loss;       /* TMO_LOSS_* */
  float base;         /* base_resolution as configured */
  float scale;        /* per_level_scale as configured */
  float huber_delta;
  int32_t active_levels; /* <= 0 means L */
  int32_t grad_mode;  /* TMO_GRAD_* */
  int32_t res_mode;   /* 0: iterative res*=scale (eval kernel, default);
                         1: base*powf(scale,l) (scalar train kernel) */
  int32_t fp16_operands; /* 1: round every matrix-product operand to fp16
                            as a tensor-core kernel consumes it (features,
                            weights, activations, dL/dy scaled by dscale,
                            pre-activation gradients); accumulate in fp32 */
  float dscale;          /* power-of-two dL/dy scale of the fp16 mode */
} tmo_spec;

/* ---- geometry --------------------------------------------------------- */
float tmo_round6(float x);
void tmo_level_resolutions(const tmo_spec *s, float *res_out /* [L] */);
uint64_t tmo_hash_grid_size(const tmo_spec *s);
int64_t tmo_mlp_weight_count(const tmo_spec *s);
uint32_t tmo_hash3(int32_t x, int32_t y, int32_t z, uint32_t T);
uint32_t tmo_hash4(int32_t x, int32_t y, int32_t z, int32_t w, uint32_t T);

/* ---- encode / forward ------------------------------------------------- */
/* feat [N x L*F]; corner_idx [N x L x 2^d] (table element offset of feature 0,
 * may be NULL); cells [N x L x d] (may be NULL). */
void tmo_encode(const tmo_spec *s, const float *table, const float *pos,
                int64_t N, float *feat, uint32_t *corner_idx, int32_t *cells);
/* Inference: encode fused with W0, hidden layers, output layer. out [N x O]. */
void tmo_forward(const tmo_spec *s, const float *table, const float *mlp,
                 const float *pos, int64_t N, float *out);

/* Analytic input gradient of a single-output field (the EvalGradient kernel,
 * mlp_kernel_emitter.cpp:1716-2090, scalar path): out [N] = the field value,
 * grad [N x d] = d(out)/d(pos).  Requires O == 1.  The 3D value uses the
 * lerp form of trilinear_feature_grad, so it can differ from tmo_forward by
 * rounding. */
void tmo_eval_gradient(const tmo_spec *s, const float *table, const float *mlp,
                       const float *pos, int64_t N, float *out, float *grad);

/* Plain MLP training pass on inputs x [N x L*F]: forward, loss of the spec
 * against tgt (after a sigmoid on every output when out_act == 1), backward;
 * accumulates grad_mlp, writes dL/dx [N x L*F] to dx when non-NULL and
 * returns the summed loss.  dL/dy uses 1/inv_count. */
double tmo_mlp_train(const tmo_spec *s, const float *mlp, const float *x,
                     const float *tgt, int64_t N, int64_t inv_count,
                     int out_act, float *grad_mlp, float *dx);
/* Real spherical harmonics of degree < 4 (16 values) of a unit direction. */
void tmo_sh4(float x, float y, float z, float *out);

/* Plain MLP on given features x [N x L*F] (no encoding). */
void tmo_mlp_forward(const tmo_spec *s, const float *mlp, const float *x,
                     int64_t N, float *out);

/* ---- training --------------------------------------------------------- */
/* One fused forward+backward over N points (the scalar train kernel).
 * inv_count: divisor used for dL/dy (the kernel's inv_N); pass the global
 * batch under data parallelism.  d_out_ext != NULL selects the ExternalGrad
 * mode (loss not computed).  grad_hash_fixed (int32, TMO_GRAD_FIXED16) or
 * grad_hash_float (TMO_GRAD_FLOAT) and grad_mlp are ACCUMULATED into.
 * touched [tracked slots] gets 1 for every slot a scatter wrote.
 * out (may be NULL) receives the outputs [N x O].  Returns the summed loss. */
double tmo_fwd_bwd(const tmo_spec *s, const float *table, const float *mlp,
                   const float *pos, const float *tgt, const float *d_out_ext,
                   int64_t N, int64_t inv_count, float *grad_mlp,
                   int32_t *grad_hash_fixed, float *grad_hash_float,
                   uint8_t *touched, float *out);
/* Same, parallel over points with OpenMP (nthreads <= 0: all cores).  MLP
 * gradients are summed per thread then reduced; fixed-point hash grads use
 * integer atomics (order independent), float hash grads use CAS adds. */
double tmo_fwd_bwd_par(const tmo_spec *s, const float *table, const float *mlp,
                       const float *pos, const float *tgt, int64_t N,
                       int64_t inv_count, float *grad_mlp,
                       int32_t *grad_hash_fixed, float *grad_hash_float,
                       uint8_t *touched, int nthreads);

typedef struct tmo_adam_cfg {
  float lr_hash, lr_mlp, beta1, beta2, eps, l1_hash, l2_mlp, grad_clip,
      weight_decay;
  uint32_t step; /* logical step before increment */
  int32_t sparse_hash; /* 1: update only touched hash slots */
  int32_t entry_width; /* tracked slot width: 2 when F==2 else 1 */
} tmo_adam_cfg;
void tmo_adam_bias_corrections(float beta1, float beta2, uint32_t step,
                               float *bc1, float *bc2);
/* w, m, v: flat [hash | mlp]. */
void tmo_adam(const tmo_adam_cfg *c, float *w, float *m, float *v,
              uint64_t hash_count, uint64_t mlp_count,
              const int32_t *grad_hash_fixed, const float *grad_hash_float,
              const float *grad_mlp, const uint8_t *touched, int nthreads);

/* ---- weight init (Philox-4x32-10) ------------------------------------- */
void tmo_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2],
                       uint32_t out[4]);
void tmo_init_uniform(float *out, uint64_t count, float low, float high,
                      uint64_t seed, uint32_t counter_base);
void tmo_init_normal(float *out, uint64_t count, float mean, float stddev,
                     uint64_t seed, uint32_t counter_base);
enum { TMO_MLP_KAIMING_UNIFORM = 0, TMO_MLP_KAIMING_NORMAL = 1,
       TMO_MLP_XAVIER_UNIFORM = 2, TMO_MLP_XAVIER_NORMAL = 3,
       TMO_MLP_UNIFORM = 4, TMO_MLP_NORMAL = 5, TMO_MLP_ZERO = 6 };
typedef struct tmo_init_cfg {
  int32_t hash_zero;       /* 0 uniform, 1 zero */
  float hash_range;
  int32_t mlp_mode;        /* TMO_MLP_* */
  float gain;              /* Kaiming gain (sqrt 2 for ReLU) */
  float mlp_uniform_range;
  float mlp_normal_stddev;
  uint64_t seed;
} tmo_init_cfg;
void tmo_init_weights(const tmo_spec *s, const tmo_init_cfg *c, float *hash,
                      float *mlp);

/* ---- Morton ordering -------------------------------------------------- */
uint32_t tmo_morton3(float x, float y, float z);
uint32_t tmo_morton4(float x, float y, float z, float w);
/* perm[i] = source index of the i-th point in ascending code order (ties by
 * source index). */
void tmo_morton_order(const float *pos, int64_t N, int d, uint32_t *perm);

#ifdef __cplusplus
}
#endif
#endif
