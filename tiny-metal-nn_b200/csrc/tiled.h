// tiled.h -- the Tiled family: the training step as separate launches
//   encode (level-major) -> tcgen05 MLP forward/backward -> scatter
//   (level-major),
// for tables whose fp16/fp32 gather copy plus fp32 gradients overflow the
// L2.  The hash-grid kernels sweep one level at a time over the whole batch,
// so the level's slice of the table (and of the gradients) is the only part
// of them in use and stays resident in L2 while every point visits it.
// The MLP stage is the FullyFused family's plain-MLP training kernel, fed
// the encoded features and writing dL/d(features).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/tmnn_cuda.h"
#include "common.cuh"
#include "fused.h"

namespace tmnn {

// Shapes the family can run (those of the plain-MLP tensor-core kernel).
bool tiled_supported(const NetDims &nd, std::string *why);

// Encoded features, fp16 [N x In] row-major (column l*F + f): every level
// of every point, interpolated in fp32 in the reference's corner order and
// rounded to fp16.  table16 (non-null) selects the fp16 gather copy.
// Returns the kernels launched.
int tiled_encode(const NetDims &nd, const float *table32,
                 const __half *table16, const float *pos, __half *feat,
                 uint32_t N, cudaStream_t st);

// Hash-table gradients of dL/d(features) dfeat fp32 [N x In]: every
// corner's weight times the feature gradient, into gh_fixed (int32 fixed
// point x 2^16, truncated) or gh_float (vector float reductions), marking
// touched slots unless implicit_touch (float gradients: a nonzero sum marks
// the slot).  Levels >= nd.active_levels receive nothing.
// Levels [l0, l1) only (l1 < 0: up to the active levels), so that a
// data-parallel step can exchange a finished group of levels while the next
// group is being scattered.
int tiled_scatter(const NetDims &nd, const float *pos, const float *dfeat,
                  int32_t *gh_fixed, float *gh_float, uint8_t *touched,
                  uint32_t N, bool implicit_touch, cudaStream_t st, int l0 = 0,
                  int l1 = -1);

// One training pass: encode, MLP forward + loss (tgt) or the caller's
// dL/dy (dext) + backward (weight gradients into gm, summed loss into
// loss_acc), scatter.  feat / dfeat are batch scratch of N * In elements.
int tiled_train(FusedWorkspace &ws, const NetDims &nd, const float *params,
                const __half *table_h, const float *pos, const float *tgt,
                const float *dext, float inv_N, float *gm, int32_t *gh_fixed,
                float *gh_float, uint8_t *touched, double *loss_acc,
                __half *feat, float *dfeat, uint32_t N, int num_sms,
                cudaStream_t st, bool implicit_touch);

// Inference: encode, then the pipelined tcgen05 MLP forward into out.
int tiled_forward(FusedWorkspace &ws, const NetDims &nd, const float *params,
                  const __half *table_h, const float *pos, float *out,
                  __half *feat, uint32_t N, int num_sms, cudaStream_t st);

}  // namespace tmnn
