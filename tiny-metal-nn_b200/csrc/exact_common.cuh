// exact_common.cuh -- device helpers shared by the reference-order fp32
// kernels (kernels_exact.cu, kernels_evalgrad.cu): the corners of one level
// and their interpolated features, in the reference's operation order.  The
// including files are compiled with --fmad=false.
#pragma once
#include "common.cuh"

namespace tmnn {

constexpr int kExactBlock = 128;

inline int wmax_for(int W) {
  return W <= 16 ? 16 : W <= 32 ? 32 : W <= 64 ? 64 : W <= 128 ? 128 : 0;
}

int exact_grid(uint32_t N, int num_sms);

// ------------------------------------------------------------ corners

struct Corners {
  uint32_t off[16];  // element offset of feature 0 of the corner's entry
  float w[16];       // (wx*wy)*wz[*wt]
  float wc[16][4];   // per-axis weights (scalar scatter product order)
  int32_t bc[4];
};

// One level's 2^d corners: cell = floor(p*res), frac = p*res - cell; corners
// enumerated dz, dy, dx (dx fastest) with dw outermost in 4D
// (mlp_kernel_emitter.cpp:224-255, :265-268, :305-308).
__device__ inline void level_corners(const NetDims &nd, const float *p, int l,
                                     Corners &c) {
  const float res = nd.res[l];
  float frac[4];
  for (int a = 0; a < nd.d; ++a) {
    const float s = p[a] * res;
    const float fl = floorf(s);
    c.bc[a] = (int32_t)fl;
    frac[a] = s - fl;
  }
  const uint64_t base = (uint64_t)l * nd.T * (uint64_t)nd.F;
  const uint32_t mask = nd.T - 1u;
  const int nw = nd.d == 4 ? 2 : 1;
  int k = 0;
  for (int dw = 0; dw < nw; ++dw)
    for (int dz = 0; dz < 2; ++dz)
      for (int dy = 0; dy < 2; ++dy)
        for (int dx = 0; dx < 2; ++dx) {
          const uint32_t h =
              nd.d == 4 ? hash4(c.bc[0] + dx, c.bc[1] + dy, c.bc[2] + dz,
                                c.bc[3] + dw, mask)
                        : hash3(c.bc[0] + dx, c.bc[1] + dy, c.bc[2] + dz, mask);
          c.off[k] = (uint32_t)(base + (uint64_t)h * nd.F);
          const float wx = dx == 0 ? 1.0f - frac[0] : frac[0];
          const float wy = dy == 0 ? 1.0f - frac[1] : frac[1];
          const float wz = dz == 0 ? 1.0f - frac[2] : frac[2];
          float w = wx * wy;
          w = w * wz;
          c.wc[k][0] = wx;
          c.wc[k][1] = wy;
          c.wc[k][2] = wz;
          if (nd.d == 4) {
            const float wt = dw == 0 ? 1.0f - frac[3] : frac[3];
            w = w * wt;
            c.wc[k][3] = wt;
          }
          c.w[k] = w;
          ++k;
        }
}

__device__ inline void level_features(const NetDims &nd, const float *table,
                                      const Corners &c, float *feat) {
  const int nc = 1 << nd.d;
  for (int f = 0; f < nd.F; ++f) {
    float acc = 0.0f;
    for (int k = 0; k < nc; ++k) acc = acc + c.w[k] * table[c.off[k] + f];
    feat[f] = acc;
  }
}

}  // namespace tmnn
