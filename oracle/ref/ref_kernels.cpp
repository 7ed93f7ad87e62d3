// Entry points that execute the reference's generated MSL (compiled as C++
// through metal_shim.h) on the CPU.  One translation unit per kernel role;
// the build defines ROLE_* and MSL_FILE.  Test infrastructure only.
#include "tg_runner.h"
#include <cstdint>

#if defined(ROLE_TRAIN_LANES)
// REF_LANES copies of the training kernel, one per namespace, so that each
// lane of run_threadgroups_lanes has its own threadgroup (static) arrays.
namespace ref_k0 {
#include MSL_FILE
}
namespace ref_k1 {
#include MSL_FILE
}
namespace ref_k2 {
#include MSL_FILE
}
namespace ref_k3 {
#include MSL_FILE
}
namespace ref_k4 {
#include MSL_FILE
}
namespace ref_k5 {
#include MSL_FILE
}
namespace ref_k6 {
#include MSL_FILE
}
namespace ref_k7 {
#include MSL_FILE
}
#define REF_LANES 8u
#else
namespace ref_k {
#include MSL_FILE
}
#endif
using namespace metal;

extern "C" {
#if defined(ROLE_TRAIN)
// neural_sdf_train_forward_backward (scalar, int atomics, active-hash mask)
void tmnn_ref_train(const float *pos, const float *tgt, const float *cfg,
                    const float *hash, int32_t *grad_hash, float *grad_mlp,
                    float *loss_partials, const float *train_params,
                    uint32_t *mask, uint32_t *summary, const float *mlp,
                    uint32_t N) {
  const uint32_t tgs = (N + 127) / 128;
  for (uint32_t tg = 0; tg < tgs; ++tg)
    run_threadgroup(128, [&](unsigned lid) {
      ref_k::neural_sdf_train_forward_backward(
          pos, tgt, cfg, hash, reinterpret_cast<atomic_int *>(grad_hash),
          reinterpret_cast<atomic_float *>(grad_mlp), loss_partials,
          train_params, reinterpret_cast<atomic_uint *>(mask),
          reinterpret_cast<atomic_uint *>(summary), mlp, tg * 128 + lid, tg,
          lid);
    });
}
#elif defined(ROLE_TRAIN_SIMD)
// neural_sdf_train_forward_backward, simdgroup-matrix variant: threadgroups
// of SIMD_TG_SIZE threads over TOTAL_PTS_PER_TG points (batches of
// POINTS_PER_TG rows)
void tmnn_ref_train_simd(const float *pos, const float *tgt, const float *cfg,
                         const float *hash, int32_t *grad_hash, float *grad_mlp,
                         float *loss_partials, const float *train_params,
                         uint32_t *mask, uint32_t *summary, const float *mlp,
                         uint32_t N) {
  const uint32_t tgs = (N + TOTAL_PTS_PER_TG - 1) / TOTAL_PTS_PER_TG;
  for (uint32_t tg = 0; tg < tgs; ++tg)
    run_threadgroup(SIMD_TG_SIZE, [&](unsigned lid) {
      ref_k::neural_sdf_train_forward_backward(
          pos, tgt, cfg, hash, reinterpret_cast<atomic_int *>(grad_hash),
          reinterpret_cast<atomic_float *>(grad_mlp), loss_partials,
          train_params, reinterpret_cast<atomic_uint *>(mask),
          reinterpret_cast<atomic_uint *>(summary), mlp, tg, lid);
    });
}
uint32_t tmnn_ref_train_simd_points_per_tg() { return TOTAL_PTS_PER_TG; }
#elif defined(ROLE_TRAIN_LANES)
// The reference's scalar training kernel with up to REF_LANES threadgroups
// running at once (emulated on the host, the scalar kernel is several times
// faster than the simdgroup-matrix one, whose matrix ops are emulated).
// Same arguments and outputs as tmnn_ref_train; the float accumulations into
// grad_mlp and the fixed-point hash gradients are atomic, so only the order
// of the float sums varies.
typedef decltype(&ref_k0::neural_sdf_train_forward_backward) train_fn;
static const train_fn k_lane_fns[REF_LANES] = {
    ref_k0::neural_sdf_train_forward_backward,
    ref_k1::neural_sdf_train_forward_backward,
    ref_k2::neural_sdf_train_forward_backward,
    ref_k3::neural_sdf_train_forward_backward,
    ref_k4::neural_sdf_train_forward_backward,
    ref_k5::neural_sdf_train_forward_backward,
    ref_k6::neural_sdf_train_forward_backward,
    ref_k7::neural_sdf_train_forward_backward};
uint32_t tmnn_ref_train_lanes_max() { return REF_LANES; }
void tmnn_ref_train_lanes(const float *pos, const float *tgt, const float *cfg,
                          const float *hash, int32_t *grad_hash,
                          float *grad_mlp, float *loss_partials,
                          const float *train_params, uint32_t *mask,
                          uint32_t *summary, const float *mlp, uint32_t N,
                          uint32_t lanes) {
  const uint32_t tgs = (N + 127) / 128;
  if (lanes < 1) lanes = 1;
  if (lanes > REF_LANES) lanes = REF_LANES;
  run_threadgroups_lanes(lanes, 128, tgs,
                         [&](unsigned ln, unsigned tg, unsigned lid) {
    k_lane_fns[ln](pos, tgt, cfg, hash,
                   reinterpret_cast<atomic_int *>(grad_hash),
                   reinterpret_cast<atomic_float *>(grad_mlp), loss_partials,
                   train_params, reinterpret_cast<atomic_uint *>(mask),
                   reinterpret_cast<atomic_uint *>(summary), mlp,
                   tg * 128 + lid, tg, lid);
  });
}
#elif defined(ROLE_EXTGRAD)
void tmnn_ref_extgrad(const float *pos, const float *tgt, const float *cfg,
                      const float *hash, int32_t *grad_hash, float *grad_mlp,
                      float *loss_partials, const float *train_params,
                      const float *d_out, uint32_t *mask, uint32_t *summary,
                      const float *mlp, uint32_t N) {
  const uint32_t tgs = (N + 127) / 128;
  for (uint32_t tg = 0; tg < tgs; ++tg)
    run_threadgroup(128, [&](unsigned lid) {
      ref_k::neural_sdf_train_external_grad(
          pos, tgt, cfg, hash, reinterpret_cast<atomic_int *>(grad_hash),
          reinterpret_cast<atomic_float *>(grad_mlp), loss_partials,
          train_params, d_out, reinterpret_cast<atomic_uint *>(mask),
          reinterpret_cast<atomic_uint *>(summary), mlp, tg * 128 + lid, tg,
          lid);
    });
}
#elif defined(ROLE_EVAL)
void tmnn_ref_eval(const float *pos, float *out, const float *cfg,
                   const float *hash, const float *mlp, uint32_t N) {
  for (uint32_t t = 0; t < N; ++t)
    ref_k::neural_sdf_eval_points(pos, out, cfg, hash, mlp, t);
}
#elif defined(ROLE_EVALGRAD)
// neural_sdf_analytical_eval_gradient_points: out [N x 4] = value, then the
// first three position-gradient components.
void tmnn_ref_eval_gradient(const float *pos, float *out, const float *cfg,
                            const float *hash, const float *mlp, uint32_t N) {
  for (uint32_t t = 0; t < N; ++t)
    ref_k::neural_sdf_analytical_eval_gradient_points(pos, out, cfg, hash, mlp,
                                                      t);
}
#elif defined(ROLE_ADAM)
// neural_sdf_adam_unified / _hash_sparse / _mlp_dense (USE_INT_ATOMICS_HASH)
void tmnn_ref_adam_unified(float *w, int32_t *gh, float *gm, float *m,
                           float *v, const float *params, uint32_t total) {
  for (uint32_t t = 0; t < total; ++t)
    ref_k::neural_sdf_adam_unified(w, gh, gm, m, v, params, t);
}
void tmnn_ref_adam_sparse(float *w, int32_t *gh, float *m, float *v,
                          const float *params, const uint32_t *idx,
                          uint32_t count) {
  for (uint32_t t = 0; t < count; ++t)
    ref_k::neural_sdf_adam_hash_sparse(w, gh, m, v, params, idx, t);
}
void tmnn_ref_adam_dense(float *w, float *g, float *m, float *v,
                         const float *params, uint32_t count) {
  for (uint32_t t = 0; t < count; ++t)
    ref_k::neural_sdf_adam_mlp_dense(w, g, m, v, params, t);
}
#elif defined(ROLE_INIT)
void tmnn_ref_init_uniform(float *out, uint32_t key0, uint32_t key1,
                           uint32_t counter_base, uint32_t count, float low,
                           float high) {
  ref_k::InitParams p{key0, key1, counter_base, count, low, high};
  for (uint32_t t = 0; t < (count + 3) / 4; ++t)
    ref_k::init_uniform_philox(out, p, t);
}
#elif defined(ROLE_NORMAL)
void tmnn_ref_init_normal(float *out, uint32_t key0, uint32_t key1,
                          uint32_t counter_base, uint32_t count, float mean,
                          float stddev) {
  ref_k::InitNormalParams p{key0, key1, counter_base, count, mean, stddev};
  for (uint32_t t = 0; t < (count + 3) / 4; ++t)
    ref_k::init_normal_philox(out, p, t);
}
#endif
}
