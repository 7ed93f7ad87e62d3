// The reference's own host-side arithmetic for the hot path, compiled from
// its sources: Morton codes/sort (morton_sort.h), KernelSpec limits and
// mlpWeightCount (kernel_spec.cpp), Adam parameter packing (adam_params.h).
// Test infrastructure only.
#include "tiny_metal_nn/runtime/adam_params.h"
#include "tiny_metal_nn/runtime/morton_sort.h"
#include "tiny-metal-nn/kernels/kernel_spec.h"
#include <cstring>
#include <string>

extern "C" {
uint32_t tmnn_ref_morton3(float x, float y, float z) {
  return tmnn::detail::morton_code_3d(x, y, z);
}
uint32_t tmnn_ref_morton4(float x, float y, float z, float w) {
  return tmnn::detail::morton_code_4d(x, y, z, w);
}
// Sorted positions/targets as the reference produces them (std::sort).
void tmnn_ref_morton_sort(const float *in, const float *tgt, int N, int d,
                          int td, float *pos_out, float *tgt_out) {
  std::vector<uint32_t> idx, codes;
  std::vector<float> sp, st;
  tmnn::detail::morton_sort_batch(in, tgt, N, d, td, idx, codes, sp, st);
  std::memcpy(pos_out, sp.data(), sp.size() * 4);
  std::memcpy(tgt_out, st.data(), st.size() * 4);
}
int tmnn_ref_mlp_weight_count(int in, int W, int H, int O) {
  tmnn::KernelSpec s;
  s.input_dim = in;
  s.hidden_dim = W;
  s.num_hidden_layers = H;
  s.num_outputs = O;
  return s.mlpWeightCount();
}
// 0 if KernelSpec::validate accepts, 1 otherwise (message into buf).
int tmnn_ref_validate(int L, int F, int log2T, int d, int W, int H, int O,
                      int loss, float huber, char *buf, int cap) {
  tmnn::KernelSpec s;
  s.num_levels = L;
  s.features_per_level = F;
  s.log2_hashmap_size = log2T;
  s.spatial_dims = d;
  s.encoding = d == 4 ? tmnn::KernelSpec::FourD : tmnn::KernelSpec::Standard;
  s.hidden_dim = W;
  s.num_hidden_layers = H;
  s.num_outputs = O;
  s.input_dim = L * F;
  s.loss = static_cast<tmnn::KernelSpec::LossType>(loss);
  s.huber_delta = huber;
  try {
    s.validate();
    return 0;
  } catch (const std::exception &e) {
    std::strncpy(buf, e.what(), cap - 1);
    buf[cap - 1] = 0;
    return 1;
  }
}
void tmnn_ref_adam_params(float *out13, float lr_enc, float lr_net, float b1,
                          float b2, float eps, float l1, float l2,
                          uint32_t hash_size, uint32_t mlp_count,
                          uint32_t step, float clip, float wd) {
  tmnn::TrainerConfig cfg;
  cfg.lr_encoding = lr_enc;
  cfg.lr_network = lr_net;
  cfg.beta1 = b1;
  cfg.beta2 = b2;
  cfg.epsilon = eps;
  cfg.l1_reg = l1;
  cfg.l2_reg = l2;
  tmnn::ParameterStoreDesc desc;
  desc.hash_grid_size = hash_size;
  desc.mlp_weight_count = mlp_count;
  tmnn::detail::fill_unified_adam_params(out13, cfg, desc, step, clip, wd);
}
}
