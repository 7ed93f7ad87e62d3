// fused.h -- the FullyFused family: one persistent sm_100a kernel per step
// that encodes, runs the MLP forward and backward on tcgen05 tensor cores,
// evaluates the loss and scatters the hash-table gradients.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/tmnn_cuda.h"
#include "common.cuh"

namespace tmnn {

// Device-side state of the family: the fp16 weight image (rebuilt lazily
// after every weight change) and an error word the kernels set when a
// bounded wait on the tensor-core pipeline gives up.
struct FusedWorkspace {
  void *wpack = nullptr;
  size_t wpack_bytes = 0;
  bool dirty = true;        // training image out of date
  bool dirty_infer = true;  // inference image out of date
  int ctas_per_sm = 0;
  int *err = nullptr;
  bool no_pipe = false;  // plain-MLP inference: force the one-tile kernel
};

bool fused_supported(const tmnn_spec &spec, const tmnn_train_cfg &cfg,
                     std::string *why);
void fused_weights_changed(FusedWorkspace &ws);
void fused_release(FusedWorkspace &ws);
// Each returns the number of kernels it launched.
int fused_train(FusedWorkspace &ws, const NetDims &nd, const tmnn_spec &spec,
                const float *params, const __half *table_h, const float *pos,
                const float *tgt, const float *dext, float inv_N, float *gm,
                int32_t *gh_fixed, float *gh_float, uint8_t *touched,
                double *loss_acc, uint32_t N, int num_sms, cudaStream_t st,
                bool implicit_touch);
int fused_forward(FusedWorkspace &ws, const NetDims &nd, const tmnn_spec &spec,
                  const float *params, const __half *table_h, const float *pos,
                  float *out, uint32_t N, int num_sms, cudaStream_t st);
// Plain FullyFusedMLP inference (no encoding): x fp16 [N x nd.In], mlp the
// fp32 weights in the reference layout, out fp32 [N x nd.O].
// out_act 1 applies a sigmoid to every output.
int fused_mlp_forward(FusedWorkspace &ws, const NetDims &nd, const float *mlp,
                      const __half *x, float *out, uint32_t N, int num_sms,
                      cudaStream_t st, int out_act = 0);
bool fused_mlp_supported(const NetDims &nd, std::string *why);
// Plain FullyFusedMLP training pass: forward, loss (internal, from tgt with
// the spec's loss) or the caller's dL/d(output) (dext), backward; weight
// gradients accumulate into gm, the summed loss into *loss_acc, and dL/dx
// [N x In] fp32 is written to dx when non-null.  With out_act 1 the outputs
// (and the loss / dext) are those after a sigmoid.
int fused_mlp_train(FusedWorkspace &ws, const NetDims &nd, const float *mlp,
                    const __half *x, const float *tgt, const float *dext,
                    float inv_N, float *gm, double *loss_acc, float *dx,
                    uint32_t N, int num_sms, cudaStream_t st, int out_act = 0);
bool fused_mlp_train_supported(const NetDims &nd, std::string *why);
// Nonzero when a fused kernel reported a timed-out pipeline wait.
int fused_error(FusedWorkspace &ws, cudaStream_t st);

}  // namespace tmnn
