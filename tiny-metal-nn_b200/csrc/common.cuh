// common.cuh -- shared definitions of the B200 hot-path kernels.
//
// Data layout in HBM (one context):
//   params  f32 [hash_count | mlp_count]   flat master weights; the hash part
//           is level-major [L][T][F] (element l*T*F + h*F + f,
//           mlp_kernel_emitter.cpp:272, :311); the MLP part is
//           [W0 In x W][b0 W][W1..W(H-1) W x W][b_i W][Wout W x O][bout O]
//           (mlp_kernel_emitter.cpp:163-191).
//   m, v    f32, same shape (Adam moments of the fused [hash|mlp] buffer).
//   table_h f16 [hash_count]  gather copy of the hash part (table_dtype F16).
//   grad_hash  i32 fixed point (x 2^16), f32, or f16 (x 2^18) [hash_count].
//   grad_mlp   f32 [mlp_count].
//   touched    u8 per tracked slot (a feature pair when F == 2, else one
//              element): the reference's active-hash bitmask
//              (mlp_kernel_emitter.cpp:48-71) as bytes.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace tmnn {

constexpr int kMaxLevels = 32;
constexpr int kMaxHidden = 8;
constexpr float kGradScale = 65536.0f;  // mlp_kernel_emitter.cpp:20
constexpr float kInvGradScale = 1.0f / 65536.0f;
// fp16 hash gradients hold d*w*2^18: per-slot sums of mean-loss gradients
// at the benchmark batches lie within ~1e-10..5e-4, so the scaled values are
// mostly normal fp16 numbers with >2^17 headroom below the fp16 maximum
constexpr float kHalfGradScale = 262144.0f;
constexpr float kInvHalfGradScale = 1.0f / 262144.0f;

// hash primes (mlp_kernel_emitter.cpp:16-18)
constexpr uint32_t kPrimeY = 2654435761u;
constexpr uint32_t kPrimeZ = 805459861u;
constexpr uint32_t kPrimeW = 56711039u;

// Geometry of one network, passed by value to every kernel.
struct NetDims {
  int32_t L, F, log2T, d, W, H, O, In;
  int32_t loss;          // tmnn_loss
  float huber_delta;     // already rounded to 6 decimals
  int32_t active_levels; // levels receiving gradients
  int32_t grad_fixed;    // 1: int32 fixed-point hash gradients
  int32_t grad_half;     // 1: fp16 hash gradients (x kHalfGradScale)
  uint32_t T;            // 1 << log2T
  uint32_t mlp_count;
  uint64_t hash_count;
  int64_t w_off[kMaxHidden + 1];  // [0..H-1] hidden layers, [H] output
  int64_t b_off[kMaxHidden + 1];
  float res[kMaxLevels];          // per-level grid resolution
};

__host__ __device__ inline uint32_t hash3(int32_t x, int32_t y, int32_t z,
                                          uint32_t mask) {
  return ((uint32_t)x ^ (uint32_t)y * kPrimeY ^ (uint32_t)z * kPrimeZ) & mask;
}
__host__ __device__ inline uint32_t hash4(int32_t x, int32_t y, int32_t z,
                                          int32_t w, uint32_t mask) {
  return ((uint32_t)x ^ (uint32_t)y * kPrimeY ^ (uint32_t)z * kPrimeZ ^
          (uint32_t)w * kPrimeW) &
         mask;
}

// int(x) of the reference's fixed-point scatter: truncation toward zero,
// saturating, NaN -> 0.
__device__ inline int32_t fixed_trunc(float x) {
  if (x != x) return 0;
  if (x >= 2147483648.0f) return 2147483647;
  if (x <= -2147483648.0f) return (int32_t)0x80000000u;
  return (int32_t)x;
}

// Per-step device statistics: the summed loss (written by the forward/backward
// kernels) followed by the numerics probe's results.  One memset clears it,
// one copy reads it back.
struct StepStats {
  double loss;            // sum of per-point losses
  double grad_l2;         // sum of squared finite gradients
  float max_abs_grad;     // max |g| over finite gradients
  float max_abs_update;   // max |w - w'| of the would-be Adam update
  float nonfinite_bwd;    // 1 when a gradient is NaN/Inf
  float nonfinite_upd;    // 1 when a would-be update quantity is NaN/Inf
  int32_t probed;         // 1 when the probe scanned the gradients
  int32_t gate;           // 1: Adam skips the update on an anomaly
  int32_t exchange_err;   // 1: a rank did not reach a peer-exchange barrier
  int32_t reserved;
};

// In-kernel training probes (ProbeResult, include/tiny-metal-nn/common.h:
// 78-94), accumulated by the fp32 training kernel over all its points:
// maxima of non-negative values (atomicMax on the float bits) and sums.
struct ProbeAcc {
  float fwd_nan, bwd_nan;   // 1 when a NaN was seen
  float out_abs_max;        // max |output|
  float out_neg_min;        // max(0, max -output), one-output networks
  float act_max[kMaxHidden];
  float grad_l2[kMaxHidden];
};

struct AdamArgs {
  float lr_hash, lr_mlp, beta1, beta2, eps, bc1, bc2, l1_hash, l2_mlp,
      grad_clip, weight_decay;
  uint64_t hash_count;
  uint32_t mlp_count;
  uint64_t slots;       // tracked hash slots
  int32_t entry_width;  // elements per tracked slot
  int32_t sparse;       // update only touched hash slots
  int32_t grad_fixed;
  int32_t grad_half;       // gh_float points at fp16 values x kHalfGradScale
  int32_t implicit_touch;  // touched = byte set or nonzero float gradient
  const StepStats *guard;  // non-null: skip the update when the gated probe
                           // found an anomaly (gradients are still cleared)
};

// Whether the numerics guard vetoes this step's update.
__device__ inline bool adam_vetoed(const AdamArgs &a) {
  if (!a.guard || !a.guard->gate) return false;
  const double l = a.guard->loss;
  return a.guard->nonfinite_bwd != 0.0f || a.guard->nonfinite_upd != 0.0f ||
         !(l - l == 0.0);
}

}  // namespace tmnn
