// Runs the reference's own MSL generator (tmnn::KernelCompiler /
// MLPKernelEmitter, compiled from the reference sources) and prints the
// kernel text for one spec.  Test infrastructure: its output is compiled as
// C++ by oracle/ref_build.py through oracle/ref/metal_shim.h.
//
// usage: gen_msl ROLE L F log2T d W H O loss base scale huber active_mask [simd]
//   ROLE: train | eval | fwd | extgrad | evalgrad
//   simd: 1 lets the compiler realise the simdgroup-matrix training kernel
//   (the reference's default for the shapes that allow it); default 0.
#include "tiny-metal-nn/kernels/kernel_compiler.h"
#include <cstdio>
#include <cstdlib>
#include <cstring>

int main(int argc, char **argv) {
  if (argc < 14) { std::fprintf(stderr, "usage\n"); return 2; }
  tmnn::KernelSpec s;
  s.num_levels = std::atoi(argv[2]);
  s.features_per_level = std::atoi(argv[3]);
  s.log2_hashmap_size = std::atoi(argv[4]);
  s.spatial_dims = std::atoi(argv[5]);
  s.encoding = s.spatial_dims == 4 ? tmnn::KernelSpec::FourD : tmnn::KernelSpec::Standard;
  s.hidden_dim = std::atoi(argv[6]);
  s.num_hidden_layers = std::atoi(argv[7]);
  s.num_outputs = std::atoi(argv[8]);
  s.input_dim = s.num_levels * s.features_per_level;
  s.loss = static_cast<tmnn::KernelSpec::LossType>(std::atoi(argv[9]));
  s.base_resolution = std::strtof(argv[10], nullptr);
  s.per_level_scale = std::strtof(argv[11], nullptr);
  s.huber_delta = std::strtof(argv[12], nullptr);
  s.emit_active_hash_mask = std::atoi(argv[13]) != 0;
  auto schema = tmnn::KernelCompiler::makeDefaultSchema(s);
  tmnn::extension::KernelCompileSpec cs;
  cs.allow_simd = argc > 14 && std::atoi(argv[14]) != 0;
  cs.allow_fp16 = false;
  cs.allow_tg_weight_cache = false;
  cs.loss_kind = static_cast<tmnn::extension::LossKind>(std::atoi(argv[9]));
  cs.huber_delta = s.huber_delta;
  tmnn::KernelRole role = tmnn::KernelRole::TrainForwardBackward;
  if (!std::strcmp(argv[1], "eval")) role = tmnn::KernelRole::Eval;
  if (!std::strcmp(argv[1], "fwd")) role = tmnn::KernelRole::ForwardForTraining;
  if (!std::strcmp(argv[1], "extgrad")) role = tmnn::KernelRole::BackwardFromExternalGrad;
  if (!std::strcmp(argv[1], "evalgrad")) role = tmnn::KernelRole::EvalGradient;
  auto r = tmnn::KernelCompiler::compile({role, s, schema, cs});
  std::fprintf(stderr, "entry=%s simd=%d fp16=%d\n", r.entry_point.c_str(),
               (int)r.decision.realized_simd, (int)r.decision.realized_fp16);
  std::fwrite(r.source.data(), 1, r.source.size(), stdout);
  return 0;
}
