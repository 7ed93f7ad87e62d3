// kernels.h -- host-side launchers of the hot-path kernels.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "common.cuh"

namespace tmnn {

// ---- reference-order fp32 kernels (kernels_exact.cu) ----
size_t exact_scratch_floats(const NetDims &nd, int num_sms);
void launch_train_exact(const NetDims &nd, const float *table,
                        const float *mlp, const float *pos, const float *tgt,
                        const float *dext, float inv_N, float *grad_mlp,
                        int32_t *gh_fixed, float *gh_float, uint8_t *touched,
                        double *loss_acc, uint32_t N, float *scratch,
                        int num_sms, cudaStream_t st, ProbeAcc *probe = nullptr);
void launch_forward_exact(const NetDims &nd, const float *table,
                          const float *mlp, const float *pos, float *out,
                          uint32_t N, float *scratch, int num_sms,
                          cudaStream_t st);
size_t eval_gradient_scratch_floats(const NetDims &nd, int num_sms);
// Value [N] and d(value)/d(pos) [N x d] of a single-output field.
void launch_eval_gradient(const NetDims &nd, const float *table,
                          const float *mlp, const float *pos, float *out,
                          float *grad, uint32_t N, float *scratch, int num_sms,
                          cudaStream_t st);
void launch_encode_debug(const NetDims &nd, const float *table,
                         const float *pos, float *feat, uint32_t *corner_idx,
                         int32_t *cells, uint32_t N, cudaStream_t st);
void launch_adam(const AdamArgs &a, float *w, float *m, float *v,
                 int32_t *gh_fixed, float *gh_float, float *gm,
                 uint8_t *touched, __half *table_h, int num_sms,
                 cudaStream_t st);
// Numerics probe over [hash (a.hash_count from w/m/v/grads) | mlp (gm; w, m,
// v at mlp_base)] into st; see kernels_exact.cu.
void launch_numerics_probe(const AdamArgs &a, const float *w, const float *m,
                           const float *v, const int32_t *gh_fixed,
                           const float *gh_float, const float *gm,
                           uint64_t mlp_base, StepStats *st, int force,
                           int gate, int num_sms, cudaStream_t st_);
void launch_touched_from_grads(const float *g, uint8_t *touched, uint64_t slots,
                               int entry_width, bool half, int num_sms,
                               cudaStream_t st);
// Data-parallel ranks on one node whose buffers this process maps (CUDA
// IPC): every rank's hash-gradient buffer, fp16 gather copy of the table and
// barrier flags (one uint32 slot per rank), indexed by rank.
constexpr int kMaxPeers = 8;
struct PeerTable {
  const void *grad[kMaxPeers];
  __half *table_h[kMaxPeers];
  uint32_t *flags[kMaxPeers];
};
// Sharded update of table elements [off, off + a.hash_count) owned by this
// rank, over peer memory: barrier, sum of the ranks' partial gradients +
// sparse Adam on this rank's w/m/v + fp16 copy stored to every rank,
// barrier.  Advances epoch by two (every rank runs the same sequence).
// A barrier that times out sets *err.  Returns the kernels launched.
int launch_peer_exchange(const AdamArgs &a, const PeerTable &pt, int rank,
                         int world, uint64_t off, float *w, float *m, float *v,
                         uint32_t &epoch, int32_t *err, int num_sms,
                         cudaStream_t st);
void launch_adam_mlp(const AdamArgs &a, float *w, float *m, float *v,
                     float *gm, int num_sms, cudaStream_t st);
void launch_to_half(const float *src, __half *dst, uint64_t n, int num_sms,
                    cudaStream_t st);
void launch_init_uniform(float *out, uint64_t count, float low, float high,
                         uint64_t seed, uint32_t counter_base, cudaStream_t st);
void launch_init_normal(float *out, uint64_t count, float mean, float stddev,
                        uint64_t seed, uint32_t counter_base, cudaStream_t st);
size_t morton_temp_bytes(uint32_t N);
void launch_morton_order(const float *pos, int d, uint32_t N, uint32_t *codes,
                         uint32_t *codes_alt, uint32_t *idx,
                         uint32_t *perm_out, void *temp, size_t temp_bytes,
                         cudaStream_t st, int key_bits = 0,
                         float *pos_dst = nullptr, const float *rows = nullptr,
                         int width = 0, float *rows_dst = nullptr,
                         bool *gathered = nullptr);
// (With pos_dst and a short key the sort also writes the sorted position rows
// and, when rows_dst is given, the sorted rows of `rows`; *gathered reports
// whether it did, otherwise the caller gathers by perm.)
void launch_gather_rows(const float *src, int width, const uint32_t *perm,
                        float *dst, uint32_t N, cudaStream_t st);
void launch_scatter_rows(const float *src, int width, const uint32_t *perm,
                         float *dst, uint32_t N, cudaStream_t st);

// ---- plain MLP helpers (mlp.cu) ----
void mlp_layout(NetDims &nd);
void mlp_init_xavier(const NetDims &nd, float *w, uint64_t seed,
                     cudaStream_t st);

}  // namespace tmnn
