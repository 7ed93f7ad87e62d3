// kernels_evalgrad.cu -- the analytic input gradient (value and
// d(value)/d(position) of a single-output field) in the reference's
// operation order, compiled with --fmad=false like kernels_exact.cu; a
// translation unit of its own so the two build in parallel.
#include "common.cuh"
#include "exact_common.cuh"
#include "kernels.h"

namespace tmnn {

// ------------------------------------------------------------ input gradient

// Cell and fraction of one level (mlp_kernel_emitter.cpp:1904-1910, :1930-1933).
__device__ inline void level_cell(const NetDims &nd, const float *p, int l,
                                  int32_t *bc, float *fr) {
  const float res = nd.res[l];
  for (int a = 0; a < nd.d; ++a) {
    const float s = p[a] * res;
    const float fl = floorf(s);
    bc[a] = (int32_t)fl;
    fr[a] = s - fl;
  }
}

// Element offset of feature 0 of one corner (hash_grid_lookup,
// mlp_kernel_emitter.cpp:1663-1671).
__device__ inline uint32_t corner_offset(const NetDims &nd, int l,
                                         const int32_t *bc, int dx, int dy,
                                         int dz, int dw) {
  const uint32_t mask = nd.T - 1u;
  const uint32_t h = nd.d == 4 ? hash4(bc[0] + dx, bc[1] + dy, bc[2] + dz,
                                       bc[3] + dw, mask)
                               : hash3(bc[0] + dx, bc[1] + dy, bc[2] + dz, mask);
  return (uint32_t)((uint64_t)l * nd.T * (uint64_t)nd.F + (uint64_t)h * nd.F);
}

// Trilinear value (lerps along x, y, z) and its partial derivatives w.r.t.
// the cell fraction, for corner values c[dz][dy][dx]
// (trilinear_feature_grad, mlp_kernel_emitter.cpp:1674-1705).
__device__ inline float trilinear_value_grad(const float c[2][2][2],
                                             const float *fr, float *g) {
  const float fx = fr[0], fy = fr[1], fz = fr[2];
  const float ox = 1.0f - fx, oy = 1.0f - fy, oz = 1.0f - fz;
  const float c000 = c[0][0][0], c001 = c[1][0][0], c010 = c[0][1][0],
              c011 = c[1][1][0], c100 = c[0][0][1], c101 = c[1][0][1],
              c110 = c[0][1][1], c111 = c[1][1][1];
  const float c00 = c000 * ox + c100 * fx;
  const float c01 = c001 * ox + c101 * fx;
  const float c10 = c010 * ox + c110 * fx;
  const float c11 = c011 * ox + c111 * fx;
  const float c0 = c00 * oy + c10 * fy;
  const float c1 = c01 * oy + c11 * fy;
  if (g) {
    g[0] = oz * (oy * (c100 - c000) + fy * (c110 - c010)) +
           fz * (oy * (c101 - c001) + fy * (c111 - c011));
    g[1] = oz * (ox * (c010 - c000) + fx * (c110 - c100)) +
           fz * (ox * (c011 - c001) + fx * (c111 - c101));
    g[2] = oy * (ox * (c001 - c000) + fx * (c101 - c100)) +
           fy * (ox * (c011 - c010) + fx * (c111 - c110));
  }
  return c0 * oz + c1 * fz;
}

// Partial derivatives of the quadrilinear interpolant for corner values
// c[dw][dz][dy][dx] (mlp_kernel_emitter.cpp:1996-2024): each a sum, loops
// nested as there, of ((w_a*w_b)*w_c) * (upper - lower).
__device__ inline void quadrilinear_grad(const float c[2][2][2][2],
                                         const float *fr, float *g) {
  float w[4][2];
  for (int a = 0; a < 4; ++a) {
    w[a][0] = 1.0f - fr[a];
    w[a][1] = fr[a];
  }
  float gx = 0.0f, gy = 0.0f, gz = 0.0f, gt = 0.0f;
  for (int dw = 0; dw < 2; ++dw)
    for (int dz = 0; dz < 2; ++dz)
      for (int dy = 0; dy < 2; ++dy)
        gx = gx + ((w[1][dy] * w[2][dz]) * w[3][dw]) *
                      (c[dw][dz][dy][1] - c[dw][dz][dy][0]);
  for (int dw = 0; dw < 2; ++dw)
    for (int dz = 0; dz < 2; ++dz)
      for (int dx = 0; dx < 2; ++dx)
        gy = gy + ((w[0][dx] * w[2][dz]) * w[3][dw]) *
                      (c[dw][dz][1][dx] - c[dw][dz][0][dx]);
  for (int dw = 0; dw < 2; ++dw)
    for (int dy = 0; dy < 2; ++dy)
      for (int dx = 0; dx < 2; ++dx)
        gz = gz + ((w[0][dx] * w[1][dy]) * w[3][dw]) *
                      (c[dw][1][dy][dx] - c[dw][0][dy][dx]);
  for (int dz = 0; dz < 2; ++dz)
    for (int dy = 0; dy < 2; ++dy)
      for (int dx = 0; dx < 2; ++dx)
        gt = gt + ((w[0][dx] * w[1][dy]) * w[2][dz]) *
                      (c[1][dz][dy][dx] - c[0][dz][dy][dx]);
  g[0] = gx;
  g[1] = gy;
  g[2] = gz;
  g[3] = gt;
}

// Value and analytic position gradient of a single-output field, one thread
// per point (the EvalGradient kernel, mlp_kernel_emitter.cpp:1855-2090,
// scalar path): forward with the W0 product accumulated per level and
// feature, backward from d(out)/d(out) = 1 through the ReLU masks, then
// sum over levels and features of (dfeat * res) * d(interp)/d(frac).
// Corners are gathered once per level for all F features (the reference
// loads them per feature; the values are the same).
template <int WMAX>
__global__ void __launch_bounds__(kExactBlock)
    k_eval_gradient(NetDims nd, const float *__restrict__ table,
                    const float *__restrict__ mlp,
                    const float *__restrict__ pos, float *__restrict__ out,
                    float *__restrict__ grad, uint32_t N, float *scratch) {
  float local_acts[WMAX > 0 ? (kMaxHidden + 2) * WMAX : 1];
  float *acts = WMAX > 0 ? local_acts
                         : scratch + (size_t)(blockIdx.x * blockDim.x +
                                              threadIdx.x) * (nd.H + 2) * nd.W;
  const int W = nd.W, H = nd.H, F = nd.F, d = nd.d;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < N;
       i += gridDim.x * blockDim.x) {
    float p[4];
    for (int a = 0; a < d; ++a) p[a] = pos[(size_t)i * d + a];
    float *h0 = acts;
    for (int j = 0; j < W; ++j) h0[j] = 0.0f;
    for (int l = 0; l < nd.L; ++l) {
      float feat[4];
      if (d == 4) {
        Corners c;
        level_corners(nd, p, l, c);
        level_features(nd, table, c, feat);
      } else {
        int32_t bc[4];
        float fr[4];
        level_cell(nd, p, l, bc, fr);
        float cv[4][2][2][2];
        for (int dz = 0; dz < 2; ++dz)
          for (int dy = 0; dy < 2; ++dy)
            for (int dx = 0; dx < 2; ++dx) {
              const float *e = table + corner_offset(nd, l, bc, dx, dy, dz, 0);
              for (int f = 0; f < F; ++f) cv[f][dz][dy][dx] = e[f];
            }
        for (int f = 0; f < F; ++f)
          feat[f] = trilinear_value_grad(cv[f], fr, nullptr);
      }
      for (int f = 0; f < F; ++f) {
        const float *wr = mlp + nd.w_off[0] + (int64_t)(l * F + f) * W;
        for (int j = 0; j < W; ++j) h0[j] = h0[j] + feat[f] * wr[j];
      }
    }
    for (int j = 0; j < W; ++j) {
      const float t = h0[j] + mlp[nd.b_off[0] + j];
      h0[j] = t > 0.0f ? t : 0.0f;
    }
    for (int k = 1; k < H; ++k) {
      const float *hin = acts + (k - 1) * W;
      float *hout = acts + k * W;
      const float *Wk = mlp + nd.w_off[k];
      for (int j = 0; j < W; ++j) {
        float acc = 0.0f;
        for (int q = 0; q < W; ++q) acc = acc + hin[q] * Wk[(int64_t)q * W + j];
        const float t = acc + mlp[nd.b_off[k] + j];
        hout[j] = t > 0.0f ? t : 0.0f;
      }
    }
    const float *hl = acts + (H - 1) * W;
    float *cur = acts + H * W, *nxt = cur + W;
    const float *wo = mlp + nd.w_off[H];
    float y = mlp[nd.b_off[H]];
    for (int j = 0; j < W; ++j) {
      y = y + hl[j] * wo[j];
      cur[j] = wo[j] * (hl[j] > 0.0f ? 1.0f : 0.0f);
    }
    for (int k = H - 1; k >= 1; --k) {
      const float *hprev = acts + (k - 1) * W;
      const float *Wk = mlp + nd.w_off[k];
      for (int q = 0; q < W; ++q) {
        float acc = 0.0f;
        for (int j = 0; j < W; ++j) acc = acc + cur[j] * Wk[(int64_t)q * W + j];
        nxt[q] = acc * (hprev[q] > 0.0f ? 1.0f : 0.0f);
      }
      float *t = cur;
      cur = nxt;
      nxt = t;
    }
    float gp[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int l = 0; l < nd.L; ++l) {
      int32_t bc[4];
      float fr[4];
      level_cell(nd, p, l, bc, fr);
      float dfeat[4];
      for (int f = 0; f < F; ++f) {
        const float *wr = mlp + nd.w_off[0] + (int64_t)(l * F + f) * W;
        float gf = 0.0f;
        for (int j = 0; j < W; ++j) gf = gf + cur[j] * wr[j];
        dfeat[f] = gf * nd.res[l];
      }
      if (d == 4) {
        float cv[2][2][2][2];
        for (int f = 0; f < F; ++f) {
          for (int dw = 0; dw < 2; ++dw)
            for (int dz = 0; dz < 2; ++dz)
              for (int dy = 0; dy < 2; ++dy)
                for (int dx = 0; dx < 2; ++dx)
                  cv[dw][dz][dy][dx] =
                      table[corner_offset(nd, l, bc, dx, dy, dz, dw) + f];
          float tg[4];
          quadrilinear_grad(cv, fr, tg);
          for (int a = 0; a < 4; ++a) gp[a] = gp[a] + dfeat[f] * tg[a];
        }
      } else {
        float cv[4][2][2][2];
        for (int dz = 0; dz < 2; ++dz)
          for (int dy = 0; dy < 2; ++dy)
            for (int dx = 0; dx < 2; ++dx) {
              const float *e = table + corner_offset(nd, l, bc, dx, dy, dz, 0);
              for (int f = 0; f < F; ++f) cv[f][dz][dy][dx] = e[f];
            }
        for (int f = 0; f < F; ++f) {
          float tg[3];
          trilinear_value_grad(cv[f], fr, tg);
          for (int a = 0; a < 3; ++a) gp[a] = gp[a] + dfeat[f] * tg[a];
        }
      }
    }
    out[i] = y;
    for (int a = 0; a < d; ++a) grad[(size_t)i * d + a] = gp[a];
  }
}

// Register-resident variant of k_eval_gradient for the common shapes
// (W <= 64, H <= 2 supported by the template): the weights sit in shared memory (broadcast reads), the
// activations and back-propagated gradients in registers (the layer loops
// are unrolled at compile time), ReLU masks as bits.  Same operations in the
// same order as k_eval_gradient, so the results are identical.
template <int W, int H, int F, int D>
__global__ void __launch_bounds__(kExactBlock)
    k_eval_gradient_reg(NetDims nd, const float *__restrict__ table,
                        const float *__restrict__ mlp,
                        const float *__restrict__ pos, float *__restrict__ out,
                        float *__restrict__ grad, uint32_t N) {
  extern __shared__ float sw[];
  for (uint32_t i = threadIdx.x; i < nd.mlp_count; i += blockDim.x) sw[i] = mlp[i];
  __syncthreads();
  constexpr int MW = (W + 31) / 32;
  const float *W0 = sw + nd.w_off[0];
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < N;
       i += gridDim.x * blockDim.x) {
    float p[4];
#pragma unroll
    for (int a = 0; a < D; ++a) p[a] = pos[(size_t)i * D + a];
    float ha[W], hb[W];
    uint32_t m0[MW];
#pragma unroll
    for (int j = 0; j < W; ++j) ha[j] = 0.0f;
    for (int l = 0; l < nd.L; ++l) {
      float feat[F];
      if (D == 4) {
        Corners c;
        level_corners(nd, p, l, c);
        level_features(nd, table, c, feat);
      } else {
        int32_t bc[4];
        float fr[4];
        level_cell(nd, p, l, bc, fr);
        float cv[F][2][2][2];
#pragma unroll
        for (int dz = 0; dz < 2; ++dz)
#pragma unroll
          for (int dy = 0; dy < 2; ++dy)
#pragma unroll
            for (int dx = 0; dx < 2; ++dx) {
              const float *e = table + corner_offset(nd, l, bc, dx, dy, dz, 0);
#pragma unroll
              for (int f = 0; f < F; ++f) cv[f][dz][dy][dx] = e[f];
            }
#pragma unroll
        for (int f = 0; f < F; ++f) feat[f] = trilinear_value_grad(cv[f], fr, nullptr);
      }
#pragma unroll
      for (int f = 0; f < F; ++f) {
        const float *wr = W0 + (l * F + f) * W;
#pragma unroll
        for (int j = 0; j < W; ++j) ha[j] = ha[j] + feat[f] * wr[j];
      }
    }
#pragma unroll
    for (int j = 0; j < W; ++j) {
      const float t = ha[j] + sw[nd.b_off[0] + j];
      ha[j] = t > 0.0f ? t : 0.0f;
    }
    // ha = h0; for H == 2 hb = h1 and ha keeps only its mask
    if (H == 2) {
#pragma unroll
      for (int w = 0; w < MW; ++w) m0[w] = 0u;
      const float *W1 = sw + nd.w_off[1];
#pragma unroll
      for (int j = 0; j < W; ++j) hb[j] = 0.0f;
#pragma unroll
      for (int q = 0; q < W; ++q) {
        const float hq = ha[q];
        if (hq > 0.0f) m0[q >> 5] |= 1u << (q & 31);
#pragma unroll
        for (int j = 0; j < W; ++j) hb[j] = hb[j] + hq * W1[q * W + j];
      }
#pragma unroll
      for (int j = 0; j < W; ++j) {
        const float t = hb[j] + sw[nd.b_off[1] + j];
        hb[j] = t > 0.0f ? t : 0.0f;
      }
    }
    const float *wo = sw + nd.w_off[H];
    float y = sw[nd.b_off[H]];
    float cur[W];
#pragma unroll
    for (int j = 0; j < W; ++j) {
      const float hv = H == 2 ? hb[j] : ha[j];
      y = y + hv * wo[j];
      cur[j] = wo[j] * (hv > 0.0f ? 1.0f : 0.0f);
    }
    if (H == 2) {
      const float *W1 = sw + nd.w_off[1];
#pragma unroll
      for (int q = 0; q < W; ++q) {
        float acc = 0.0f;
#pragma unroll
        for (int j = 0; j < W; ++j) acc = acc + cur[j] * W1[q * W + j];
        hb[q] = acc * (((m0[q >> 5] >> (q & 31)) & 1u) ? 1.0f : 0.0f);
      }
#pragma unroll
      for (int j = 0; j < W; ++j) cur[j] = hb[j];
    }
    float gp[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int l = 0; l < nd.L; ++l) {
      int32_t bc[4];
      float fr[4];
      level_cell(nd, p, l, bc, fr);
      float dfeat[F];
#pragma unroll
      for (int f = 0; f < F; ++f) {
        const float *wr = W0 + (l * F + f) * W;
        float gf = 0.0f;
#pragma unroll
        for (int j = 0; j < W; ++j) gf = gf + cur[j] * wr[j];
        dfeat[f] = gf * nd.res[l];
      }
      if (D == 4) {
#pragma unroll
        for (int f = 0; f < F; ++f) {
          float cv[2][2][2][2];
#pragma unroll
          for (int dw = 0; dw < 2; ++dw)
#pragma unroll
            for (int dz = 0; dz < 2; ++dz)
#pragma unroll
              for (int dy = 0; dy < 2; ++dy)
#pragma unroll
                for (int dx = 0; dx < 2; ++dx)
                  cv[dw][dz][dy][dx] =
                      table[corner_offset(nd, l, bc, dx, dy, dz, dw) + f];
          float tg[4];
          quadrilinear_grad(cv, fr, tg);
#pragma unroll
          for (int a = 0; a < 4; ++a) gp[a] = gp[a] + dfeat[f] * tg[a];
        }
      } else {
        float cv[F][2][2][2];
#pragma unroll
        for (int dz = 0; dz < 2; ++dz)
#pragma unroll
          for (int dy = 0; dy < 2; ++dy)
#pragma unroll
            for (int dx = 0; dx < 2; ++dx) {
              const float *e = table + corner_offset(nd, l, bc, dx, dy, dz, 0);
#pragma unroll
              for (int f = 0; f < F; ++f) cv[f][dz][dy][dx] = e[f];
            }
#pragma unroll
        for (int f = 0; f < F; ++f) {
          float tg[3];
          trilinear_value_grad(cv[f], fr, tg);
#pragma unroll
          for (int a = 0; a < 3; ++a) gp[a] = gp[a] + dfeat[f] * tg[a];
        }
      }
    }
    out[i] = y;
#pragma unroll
    for (int a = 0; a < D; ++a) grad[(size_t)i * D + a] = gp[a];
  }
}

using EvalGradFn = void (*)(NetDims, const float *, const float *,
                            const float *, float *, float *, uint32_t);

// Instantiated for the shapes of the benchmark configurations (two
// features per level, 64 wide, one hidden layer -- the single-output SDF
// shape -- 3D or 4D; with two hidden layers the unrolled code spills); other
// shapes run k_eval_gradient.
EvalGradFn pick_eval_grad(const NetDims &nd) {
  if (nd.F != 2 || nd.W != 64) return nullptr;
  if (nd.H == 1) return nd.d == 3 ? k_eval_gradient_reg<64, 1, 2, 3>
                                  : k_eval_gradient_reg<64, 1, 2, 4>;
  return nullptr;
}

size_t eval_gradient_scratch_floats(const NetDims &nd, int num_sms) {
  return wmax_for(nd.W) ? 0
                        : (size_t)num_sms * 8 * kExactBlock * (nd.H + 2) * nd.W;
}

void launch_eval_gradient(const NetDims &nd, const float *table,
                          const float *mlp, const float *pos, float *out,
                          float *grad, uint32_t N, float *scratch, int num_sms,
                          cudaStream_t st) {
  if (N == 0) return;
  const int grid = exact_grid(N, num_sms);
  const size_t wbytes = (size_t)nd.mlp_count * sizeof(float);
  if (EvalGradFn fn = pick_eval_grad(nd); fn && wbytes <= 96 * 1024) {
    if (wbytes > 48 * 1024)
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)wbytes);
    fn<<<grid, kExactBlock, wbytes, st>>>(nd, table, mlp, pos, out, grad, N);
    return;
  }
#define TMNN_EG_CASE(WM)                                                     \
  k_eval_gradient<WM><<<grid, kExactBlock, 0, st>>>(nd, table, mlp, pos, out, \
                                                    grad, N, scratch);
  switch (wmax_for(nd.W)) {
    case 16: TMNN_EG_CASE(16) break;
    case 32: TMNN_EG_CASE(32) break;
    case 64: TMNN_EG_CASE(64) break;
    case 128: TMNN_EG_CASE(128) break;
    default: TMNN_EG_CASE(0) break;
  }
#undef TMNN_EG_CASE
}

}  // namespace tmnn
