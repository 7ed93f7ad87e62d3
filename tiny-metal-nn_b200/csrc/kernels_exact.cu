// kernels_exact.cu -- fp32 CUDA-core kernels that evaluate tmnn's hot path in
// the reference's operation order.  Compiled with --fmad=false: every
// multiply and add is rounded separately, exactly as the CPU restatement of
// the reference, so encodings, fixed-point hash gradients and Adam updates
// agree bit for bit.  These kernels are the SafeDebug family, the inference
// path's reference-order variant, and the weight initialiser / optimizer of
// every family.
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>
#include <cub/block/block_radix_sort.cuh>

#include "common.cuh"
#include "exact_common.cuh"
#include "kernels.h"

namespace tmnn {

// ------------------------------------------------------------ forward

// acts: [H][W] activations (row k = output of hidden layer k); y: [O].
// Encode fused with W0 level by level (mlp_kernel_emitter.cpp:279-296,
// :343-358), bias+ReLU, hidden layers (:2962-2970), output from the bias
// (:2983-2997).
__device__ void forward_point(const NetDims &nd, const float *table,
                              const float *mlp, const float *p, float *acts,
                              float *y) {
  const int W = nd.W;
  float *h0 = acts;
  for (int j = 0; j < W; ++j) h0[j] = 0.0f;
  const bool vec2 = nd.F == 2 && nd.d == 3;
  for (int l = 0; l < nd.L; ++l) {
    Corners c;
    float feat[4];
    level_corners(nd, p, l, c);
    level_features(nd, table, c, feat);
    if (vec2) {
      const float *wa = mlp + nd.w_off[0] + (int64_t)(2 * l) * W;
      const float *wb = wa + W;
      for (int j = 0; j < W; ++j) {
        const float t = feat[0] * wa[j] + feat[1] * wb[j];
        h0[j] = h0[j] + t;
      }
    } else {
      for (int f = 0; f < nd.F; ++f) {
        const float *wr = mlp + nd.w_off[0] + (int64_t)(l * nd.F + f) * W;
        for (int j = 0; j < W; ++j) h0[j] = h0[j] + feat[f] * wr[j];
      }
    }
  }
  for (int j = 0; j < W; ++j) {
    const float t = h0[j] + mlp[nd.b_off[0] + j];
    h0[j] = t > 0.0f ? t : 0.0f;
  }
  for (int k = 1; k < nd.H; ++k) {
    const float *hin = acts + (k - 1) * W;
    float *hout = acts + k * W;
    const float *Wk = mlp + nd.w_off[k];
    for (int j = 0; j < W; ++j) {
      float acc = 0.0f;
      for (int i = 0; i < W; ++i) acc = acc + hin[i] * Wk[(int64_t)i * W + j];
      const float t = acc + mlp[nd.b_off[k] + j];
      hout[j] = t > 0.0f ? t : 0.0f;
    }
  }
  const float *hl = acts + (nd.H - 1) * W;
  const float *Wo = mlp + nd.w_off[nd.H];
  for (int m = 0; m < nd.O; ++m) {
    float acc = mlp[nd.b_off[nd.H] + m];
    for (int j = 0; j < W; ++j) acc = acc + hl[j] * Wo[(int64_t)j * nd.O + m];
    y[m] = acc;
  }
}

// Loss and dL/dy (mlp_kernel_emitter.cpp:562-670); multi-output loss is the
// sum over outputs.
__device__ float point_loss(const NetDims &nd, const float *y, const float *t,
                            float inv_N, float *d) {
  const int O = nd.O;
  if (nd.loss == 3) {
    float dot = 0.0f, pn = 0.0f, tn = 0.0f;
    for (int m = 0; m < O; ++m) {
      dot = dot + y[m] * t[m];
      pn = pn + y[m] * y[m];
      tn = tn + t[m] * t[m];
    }
    const float pred_norm = sqrtf(pn + 1e-8f);
    const float target_norm = sqrtf(tn + 1e-8f);
    const float denom = pred_norm * target_norm;
    const float cosine = dot / denom;
    const float pnd = pn + 1e-8f;
    for (int m = 0; m < O; ++m) {
      const float a = (cosine * y[m]) / pnd;
      const float b = t[m] / denom;
      d[m] = (a - b) * inv_N;
    }
    return 1.0f - cosine;
  }
  float loss = 0.0f;
  for (int m = 0; m < O; ++m) {
    const float r = y[m] - t[m];
    float term;
    if (nd.loss == 0) {
      term = r * r;
      d[m] = (2.0f * r) * inv_N;
    } else if (nd.loss == 1) {
      term = fabsf(r);
      d[m] = (r > 0.0f ? 1.0f : (r < 0.0f ? -1.0f : 0.0f)) * inv_N;
    } else {
      const float ar = fabsf(r), delta = nd.huber_delta;
      if (ar <= delta) {
        term = (0.5f * r) * r;
        d[m] = r * inv_N;
      } else {
        term = delta * (ar - 0.5f * delta);
        d[m] = (delta * (r > 0.0f ? 1.0f : -1.0f)) * inv_N;
      }
    }
    loss = loss + term;
  }
  return loss;
}

struct GradSink {
  float *gm;          // MLP gradient accumulator (shared or global)
  int32_t *gh_fixed;  // fixed-point hash gradients
  float *gh_float;    // float hash gradients
  uint8_t *touched;
};

__device__ inline void scatter_one(const NetDims &nd, const GradSink &g,
                                   uint32_t off, float v) {
  if (nd.grad_fixed)
    atomicAdd(g.gh_fixed + off, fixed_trunc(v * kGradScale));
  else if (nd.grad_half)
    atomicAdd(reinterpret_cast<__half *>(g.gh_float) + off,
              __float2half_rn(v * kHalfGradScale));
  else
    atomicAdd(g.gh_float + off, v);
}

// Backward of one point (mlp_kernel_emitter.cpp:3061-3155 with
// emitHashScatter :672-901).  d: dL/dy [O]; acts hold the forward
// activations and are overwritten with pre-activation gradients.
__device__ void backward_point(const NetDims &nd, const float *table,
                               const float *mlp, const float *p, float *acts,
                               const float *d, const GradSink &g) {
  const int W = nd.W, O = nd.O, H = nd.H;
  float *hl = acts + (H - 1) * W;
  const float *Wo = mlp + nd.w_off[H];
  for (int j = 0; j < W; ++j) {
    const float hv = hl[j];
    float dpre = 0.0f;
    for (int m = 0; m < O; ++m) {
      atomicAdd(g.gm + nd.w_off[H] + (int64_t)j * O + m, d[m] * hv);
      dpre = dpre + d[m] * Wo[(int64_t)j * O + m];
    }
    hl[j] = dpre * (hv > 0.0f ? 1.0f : 0.0f);
  }
  for (int m = 0; m < O; ++m) atomicAdd(g.gm + nd.b_off[H] + m, d[m]);
  for (int k = H - 1; k >= 1; --k) {
    const float *dk = acts + k * W;
    float *hin = acts + (k - 1) * W;
    const float *Wk = mlp + nd.w_off[k];
    for (int i = 0; i < W; ++i) {
      const float hv = hin[i];
      for (int j = 0; j < W; ++j)
        atomicAdd(g.gm + nd.w_off[k] + (int64_t)i * W + j, dk[j] * hv);
      float acc = 0.0f;
      for (int j = 0; j < W; ++j) acc = acc + dk[j] * Wk[(int64_t)i * W + j];
      hin[i] = acc * (hv > 0.0f ? 1.0f : 0.0f);
    }
    for (int j = 0; j < W; ++j) atomicAdd(g.gm + nd.b_off[k] + j, dk[j]);
  }
  const float *h0 = acts;
  const bool vec2 = nd.F == 2 && nd.d == 3;
  const int nc = 1 << nd.d;
  for (int l = 0; l < nd.active_levels; ++l) {
    Corners c;
    float feat[4];
    level_corners(nd, p, l, c);
    level_features(nd, table, c, feat);
    if (vec2) {
      const int64_t r0 = nd.w_off[0] + (int64_t)(2 * l) * W, r1 = r0 + W;
      for (int j = 0; j < W; ++j) {
        atomicAdd(g.gm + r0 + j, h0[j] * feat[0]);
        atomicAdd(g.gm + r1 + j, h0[j] * feat[1]);
      }
      float dfx = 0.0f, dfy = 0.0f;
      for (int j = 0; j < W; ++j) {
        dfx = dfx + h0[j] * mlp[r0 + j];
        dfy = dfy + h0[j] * mlp[r1 + j];
      }
      for (int k = 0; k < nc; ++k) {
        scatter_one(nd, g, c.off[k], dfx * c.w[k]);
        scatter_one(nd, g, c.off[k] + 1, dfy * c.w[k]);
        g.touched[c.off[k] >> 1] = 1;
      }
    } else {
      for (int f = 0; f < nd.F; ++f) {
        const int64_t r = nd.w_off[0] + (int64_t)(l * nd.F + f) * W;
        for (int j = 0; j < W; ++j) atomicAdd(g.gm + r + j, h0[j] * feat[f]);
        float df = 0.0f;
        for (int j = 0; j < W; ++j) df = df + h0[j] * mlp[r + j];
        for (int k = 0; k < nc; ++k) {
          float v = df * c.wc[k][0];
          v = v * c.wc[k][1];
          v = v * c.wc[k][2];
          if (nd.d == 4) v = v * c.wc[k][3];
          const uint32_t e = c.off[k] + f;
          scatter_one(nd, g, e, v);
          g.touched[nd.F == 2 ? e >> 1 : e] = 1;
        }
      }
    }
  }
  for (int j = 0; j < W; ++j) atomicAdd(g.gm + nd.b_off[0] + j, h0[j]);
}

// ------------------------------------------------------------ kernels


// Probe statistics of one thread's points (the reference's emitted probe
// code, mlp_kernel_emitter.cpp:2879-2886, :2993-3050, :3105-3155): forward
// maxima and NaN flags after the forward pass, gradient sums of squares of
// every hidden layer's pre-activation gradient after the backward pass.
struct ProbeLocal {
  float fwd_nan = 0.f, bwd_nan = 0.f, out_abs_max = 0.f, out_neg_min = 0.f;
  float act_max[kMaxHidden] = {};
  float grad_l2[kMaxHidden] = {};
};

__device__ void probe_forward(const NetDims &nd, const float *acts,
                              const float *y, ProbeLocal &pl) {
  for (int k = 0; k < nd.H; ++k)
    for (int j = 0; j < nd.W; ++j) {
      const float h = acts[k * nd.W + j];
      pl.act_max[k] = fmaxf(pl.act_max[k], fabsf(h));
      if (isnan(h)) pl.fwd_nan = 1.f;
    }
  if (nd.O == 1) {
    // the reference assigns (one point per thread there): max over points
    pl.out_abs_max = fmaxf(pl.out_abs_max, fabsf(y[0]));
    pl.out_neg_min = fmaxf(pl.out_neg_min, -y[0]);
    if (isnan(y[0])) pl.fwd_nan = 1.f;
  } else {
    for (int m = 0; m < nd.O; ++m) {
      pl.out_abs_max = fmaxf(pl.out_abs_max, fabsf(y[m]));
      if (isnan(y[m])) pl.fwd_nan = 1.f;
    }
  }
}

__device__ void probe_backward(const NetDims &nd, const float *dacts,
                               const float *d, ProbeLocal &pl) {
  for (int m = 0; m < nd.O; ++m)
    if (isnan(d[m])) pl.bwd_nan = 1.f;
  for (int k = 0; k < nd.H; ++k)
    for (int j = 0; j < nd.W; ++j) {
      const float g = dacts[k * nd.W + j];
      pl.grad_l2[k] = pl.grad_l2[k] + g * g;
      if (isnan(g)) pl.bwd_nan = 1.f;
    }
}

__device__ __forceinline__ void probe_max(float *addr, float v) {
  if (v > 0.f) atomicMax(reinterpret_cast<int *>(addr), __float_as_int(v));
}

// Warp reduction of the thread statistics, one set of atomics per warp.
__device__ void probe_flush(const NetDims &nd, ProbeLocal &pl, ProbeAcc *acc) {
  const unsigned full = 0xffffffffu;
  auto wmax = [&](float v) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(full, v, o));
    return v;
  };
  auto wsum = [&](float v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(full, v, o);
    return v;
  };
  const bool lead = (threadIdx.x & 31) == 0;
  const float fn = wmax(pl.fwd_nan), bn = wmax(pl.bwd_nan);
  const float oa = wmax(pl.out_abs_max), on = wmax(pl.out_neg_min);
  if (lead) {
    probe_max(&acc->fwd_nan, fn);
    probe_max(&acc->bwd_nan, bn);
    probe_max(&acc->out_abs_max, oa);
    probe_max(&acc->out_neg_min, on);
  }
  for (int k = 0; k < nd.H; ++k) {
    const float am = wmax(pl.act_max[k]), gs = wsum(pl.grad_l2[k]);
    if (lead) {
      probe_max(&acc->act_max[k], am);
      if (gs != 0.f) atomicAdd(&acc->grad_l2[k], gs);
    }
  }
}

template <int WMAX>
__global__ void __launch_bounds__(kExactBlock)
    k_train_exact(NetDims nd, const float *__restrict__ table,
                  const float *__restrict__ mlp, const float *__restrict__ pos,
                  const float *__restrict__ tgt, const float *__restrict__ dext,
                  float inv_N, float *grad_mlp, int32_t *gh_fixed,
                  float *gh_float, uint8_t *touched, double *loss_acc,
                  uint32_t N, int use_smem_grads, float *scratch,
                  ProbeAcc *probe) {
  extern __shared__ float s_grad[];
  __shared__ double s_loss[kExactBlock / 32];
  if (use_smem_grads) {
    for (uint32_t i = threadIdx.x; i < nd.mlp_count; i += blockDim.x)
      s_grad[i] = 0.0f;
    __syncthreads();
  }
  GradSink g{use_smem_grads ? s_grad : grad_mlp, gh_fixed, gh_float, touched};
  float local_acts[WMAX > 0 ? kMaxHidden * WMAX : 1];
  float *acts = WMAX > 0 ? local_acts
                         : scratch + (size_t)(blockIdx.x * blockDim.x +
                                              threadIdx.x) * nd.H * nd.W;
  float loss = 0.0f;
  ProbeLocal pl;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < N;
       i += gridDim.x * blockDim.x) {
    const float *p = pos + (size_t)i * nd.d;
    float y[64], d[64];
    forward_point(nd, table, mlp, p, acts, y);
    if (probe) probe_forward(nd, acts, y, pl);
    if (dext) {
      for (int m = 0; m < nd.O; ++m) d[m] = dext[(size_t)i * nd.O + m];
    } else {
      loss = loss + point_loss(nd, y, tgt + (size_t)i * nd.O, inv_N, d);
    }
    backward_point(nd, table, mlp, p, acts, d, g);
    // backward_point leaves each hidden layer's pre-activation gradient in
    // acts
    if (probe) probe_backward(nd, acts, d, pl);
  }
  if (probe) probe_flush(nd, pl, probe);
  // block loss reduction in double, one atomic per block
  double lv = loss;
  for (int o = 16; o > 0; o >>= 1) lv += __shfl_down_sync(0xffffffffu, lv, o);
  if ((threadIdx.x & 31) == 0) s_loss[threadIdx.x >> 5] = lv;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < kExactBlock / 32; ++w) t += s_loss[w];
    if (!dext) atomicAdd(loss_acc, t);
  }
  if (use_smem_grads) {
    for (uint32_t i = threadIdx.x; i < nd.mlp_count; i += blockDim.x) {
      const float v = s_grad[i];
      if (v != 0.0f) atomicAdd(grad_mlp + i, v);
    }
  }
}

template <int WMAX>
__global__ void __launch_bounds__(kExactBlock)
    k_forward_exact(NetDims nd, const float *__restrict__ table,
                    const float *__restrict__ mlp, const float *__restrict__ pos,
                    float *__restrict__ out, uint32_t N, float *scratch) {
  float local_acts[WMAX > 0 ? kMaxHidden * WMAX : 1];
  float *acts = WMAX > 0 ? local_acts
                         : scratch + (size_t)(blockIdx.x * blockDim.x +
                                              threadIdx.x) * nd.H * nd.W;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < N;
       i += gridDim.x * blockDim.x) {
    float y[64];
    forward_point(nd, table, mlp, pos + (size_t)i * nd.d, acts, y);
    for (int m = 0; m < nd.O; ++m) out[(size_t)i * nd.O + m] = y[m];
  }
}

__global__ void k_encode_debug(NetDims nd, const float *__restrict__ table,
                               const float *__restrict__ pos, float *feat,
                               uint32_t *corner_idx, int32_t *cells,
                               uint32_t N) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N) return;
  const int nc = 1 << nd.d;
  for (int l = 0; l < nd.L; ++l) {
    Corners c;
    level_corners(nd, pos + (size_t)i * nd.d, l, c);
    level_features(nd, table, c, feat + (size_t)i * nd.In + l * nd.F);
    if (corner_idx)
      for (int k = 0; k < nc; ++k)
        corner_idx[((size_t)i * nd.L + l) * nc + k] = c.off[k];
    if (cells)
      for (int a = 0; a < nd.d; ++a)
        cells[((size_t)i * nd.L + l) * nd.d + a] = c.bc[a];
  }
}

// ------------------------------------------------------------ Adam

// adam_kernel_msl.h:37-109 (unified) and :120-203 (sparse hash + dense MLP),
// fused with the post-Adam gradient reset of the reference's step
// (training_step_execution.cpp:1285-1294) and the refresh of the fp16
// gather copy.  One thread per tracked hash slot (entry_width elements)
// or per MLP weight.
__device__ inline void adam_elem(float &w, float &m, float &v, float g,
                                 float lr, const AdamArgs &a, float reg,
                                 bool is_mlp) {
  if (a.grad_clip > 0.0f)
    g = g < -a.grad_clip ? -a.grad_clip : (g > a.grad_clip ? a.grad_clip : g);
  if (a.weight_decay > 0.0f) {
    const float t = (lr * a.weight_decay) * w;
    w = w - t;
  } else if (reg > 0.0f) {
    if (is_mlp)
      g = g + reg * w;
    else
      g = g + reg * (w > 0.0f ? 1.0f : (w < 0.0f ? -1.0f : 0.0f));
  }
  const float mn = a.beta1 * m + (1.0f - a.beta1) * g;
  const float vn = a.beta2 * v + ((1.0f - a.beta2) * g) * g;
  m = mn;
  v = vn;
  const float mh = mn / a.bc1;
  const float vh = vn / a.bc2;
  const float upd = (lr * mh) / (sqrtf(vh) + a.eps);
  w = w - upd;
}

__global__ void k_adam(AdamArgs a, float *__restrict__ w, float *__restrict__ m,
                       float *__restrict__ v, int32_t *gh_fixed,
                       float *gh_float, float *__restrict__ gm,
                       uint8_t *__restrict__ touched, __half *table_h) {
  const uint64_t total = a.slots + a.mlp_count;
  const bool veto = adam_vetoed(a);
  for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (uint64_t)gridDim.x * blockDim.x) {
    if (t < a.slots) {
      const bool on = !a.sparse || touched[t];
      if (a.sparse) touched[t] = 0;
      for (int k = 0; k < a.entry_width; ++k) {
        const uint64_t e = t * a.entry_width + k;
        float g;
        if (a.grad_fixed) {
          g = (float)gh_fixed[e] * kInvGradScale;
          gh_fixed[e] = 0;
        } else if (a.grad_half) {
          __half *gh = reinterpret_cast<__half *>(gh_float);
          g = __half2float(gh[e]) * kInvHalfGradScale;
          gh[e] = __float2half_rn(0.0f);
        } else {
          g = gh_float[e];
          gh_float[e] = 0.0f;
        }
        if (!on || veto) continue;
        float wv = w[e], mv = m[e], vv = v[e];
        adam_elem(wv, mv, vv, g, a.lr_hash, a, a.l1_hash, false);
        w[e] = wv;
        m[e] = mv;
        v[e] = vv;
        if (table_h) table_h[e] = __float2half_rn(wv);
      }
    } else {
      const uint64_t j = t - a.slots;
      const uint64_t e = a.hash_count + j;
      const float g = gm[j];
      gm[j] = 0.0f;
      if (veto) continue;
      float wv = w[e], mv = m[e], vv = v[e];
      adam_elem(wv, mv, vv, g, a.lr_mlp, a, a.l2_mlp, true);
      w[e] = wv;
      m[e] = mv;
      v[e] = vv;
    }
  }
}

// MLP part (a.mlp_count weights at w + a.hash_count, gradients gm), one
// element per thread of the grid; same arithmetic as k_adam.
__device__ inline void adam_mlp_range(const AdamArgs &a, float *w, float *m,
                                      float *v, float *gm, bool veto) {
  for (uint64_t j = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
       j < a.mlp_count; j += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t e = a.hash_count + j;
    const float g = gm[j];
    gm[j] = 0.0f;
    if (veto) continue;
    float wv = w[e], mv = m[e], vv = v[e];
    adam_elem(wv, mv, vv, g, a.lr_mlp, a, a.l2_mlp, true);
    w[e] = wv;
    m[e] = mv;
    v[e] = vv;
  }
}

// Hash part of the same update, four elements per thread with 16-byte
// accesses (the table size L*T*F is a multiple of 4), followed by the MLP
// weights (gm non-null) in the same launch.  Same arithmetic per element as
// k_adam.
__global__ void __launch_bounds__(256, 4)
    k_adam_hash4(AdamArgs a, float *__restrict__ w, float *__restrict__ m,
                 float *__restrict__ v, int32_t *gh_fixed, float *gh_float,
                 uint8_t *__restrict__ touched, __half *table_h, float *gm) {
  const uint64_t n4 = a.hash_count / 4;
  if (adam_vetoed(a)) {
    // the numerics guard rejected the step: only reset gradients and marks
    for (uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n4;
         q += (uint64_t)gridDim.x * blockDim.x) {
      if (a.sparse) {
        if (a.entry_width == 2)
          reinterpret_cast<uchar2 *>(touched)[q] = make_uchar2(0, 0);
        else
          reinterpret_cast<uchar4 *>(touched)[q] = make_uchar4(0, 0, 0, 0);
      }
      if (a.grad_fixed)
        reinterpret_cast<int4 *>(gh_fixed)[q] = make_int4(0, 0, 0, 0);
      else if (a.grad_half)
        reinterpret_cast<uint2 *>(gh_float)[q] = make_uint2(0u, 0u);
      else
        reinterpret_cast<float4 *>(gh_float)[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (gm) adam_mlp_range(a, w, m, v, gm, true);
    return;
  }
  // Software-pipelined by one group: the touched bytes and gradients of
  // the thread's next group are loaded before the current group's w, m, v
  // are, so a gradient load is always in flight beside them.
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  uint32_t tt = 0u;
  int4 gi = make_int4(0, 0, 0, 0);
  uint4 gf = make_uint4(0u, 0u, 0u, 0u);  // fp32 gradients (bits), or fp16 in .x, .y
  auto load_next = [&](uint64_t qq, uint32_t &t_, int4 &i_, uint4 &f_) {
    if (qq >= n4) return;
    if (a.sparse)
      t_ = a.entry_width == 2 ? (uint32_t)reinterpret_cast<uint16_t *>(touched)[qq]
                              : reinterpret_cast<uint32_t *>(touched)[qq];
    if (a.grad_fixed) {
      i_ = reinterpret_cast<int4 *>(gh_fixed)[qq];
    } else if (a.grad_half) {
      const uint2 r = reinterpret_cast<uint2 *>(gh_float)[qq];
      f_ = make_uint4(r.x, r.y, 0u, 0u);
    } else {
      f_ = reinterpret_cast<uint4 *>(gh_float)[qq];
    }
  };
  load_next(q, tt, gi, gf);
#pragma unroll 1
  for (; q < n4; q += stride) {
    const uint32_t tc = tt;
    const int4 gic = gi;
    const uint4 gfc = gf;
    load_next(q + stride, tt, gi, gf);
    bool on[4] = {true, true, true, true};
    if (a.sparse) {
      // touched bytes: one per pair (entry width 2) or per element
      if (a.entry_width == 2) {
        on[0] = on[1] = (tc & 0xffu) != 0;
        on[2] = on[3] = (tc >> 8) != 0;
        if (tc) reinterpret_cast<uint16_t *>(touched)[q] = 0;
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) on[k] = ((tc >> (8 * k)) & 0xffu) != 0;
        if (tc) reinterpret_cast<uint32_t *>(touched)[q] = 0u;
      }
    }
    float g[4];
    if (a.grad_fixed) {
      g[0] = (float)gic.x * kInvGradScale;
      g[1] = (float)gic.y * kInvGradScale;
      g[2] = (float)gic.z * kInvGradScale;
      g[3] = (float)gic.w * kInvGradScale;
      if (gic.x | gic.y | gic.z | gic.w)
        reinterpret_cast<int4 *>(gh_fixed)[q] = make_int4(0, 0, 0, 0);
    } else {
      if (a.grad_half) {
        const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&gfc.x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&gfc.y));
        g[0] = lo.x * kInvHalfGradScale;
        g[1] = lo.y * kInvHalfGradScale;
        g[2] = hi.x * kInvHalfGradScale;
        g[3] = hi.y * kInvHalfGradScale;
        // a subnormal fp16 touch mark scales to a nonzero float (2^-42)
        if (gfc.x | gfc.y) reinterpret_cast<uint2 *>(gh_float)[q] = make_uint2(0u, 0u);
      } else {
        g[0] = __uint_as_float(gfc.x);
        g[1] = __uint_as_float(gfc.y);
        g[2] = __uint_as_float(gfc.z);
        g[3] = __uint_as_float(gfc.w);
        if (g[0] != 0.f || g[1] != 0.f || g[2] != 0.f || g[3] != 0.f)
          reinterpret_cast<float4 *>(gh_float)[q] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      if (a.sparse && a.implicit_touch) {
        if (a.entry_width == 2) {
          on[0] = on[1] = on[0] || g[0] != 0.f || g[1] != 0.f;
          on[2] = on[3] = on[2] || g[2] != 0.f || g[3] != 0.f;
        } else {
#pragma unroll
          for (int k = 0; k < 4; ++k) on[k] = on[k] || g[k] != 0.f;
        }
      }
    }
    if (!(on[0] | on[1] | on[2] | on[3])) continue;
    float4 wv = reinterpret_cast<float4 *>(w)[q];
    float4 mv = reinterpret_cast<float4 *>(m)[q];
    float4 vv = reinterpret_cast<float4 *>(v)[q];
    float *pw = &wv.x, *pm = &mv.x, *pv = &vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (on[k]) adam_elem(pw[k], pm[k], pv[k], g[k], a.lr_hash, a, a.l1_hash, false);
    reinterpret_cast<float4 *>(w)[q] = wv;
    reinterpret_cast<float4 *>(m)[q] = mv;
    reinterpret_cast<float4 *>(v)[q] = vv;
    if (table_h) {
      __half2 h[2] = {__floats2half2_rn(wv.x, wv.y), __floats2half2_rn(wv.z, wv.w)};
      reinterpret_cast<uint2 *>(table_h)[q] = *reinterpret_cast<uint2 *>(h);
    }
  }
  if (gm) adam_mlp_range(a, w, m, v, gm, false);
}

// ------------------------------------------------------------ peer exchange

// Sharded data-parallel update over NVLink peer memory, one launch per
// bucket of levels: the rank that owns a range of the table reads every
// rank's partial gradients of it with plain peer loads, sums them in rank
// order, runs the sparse Adam above on the sum (implicit touch marks: a
// nonzero sum marks its slot) and stores the updated fp16 gather copy into
// every rank's table with plain peer stores.  This replaces a reduce-scatter,
// the shard's Adam and an all-gather with one pass; the bytes on NVLink are
// the reduce-scatter's reads and the all-gather's writes.  `off` is the
// range's first element in every rank's buffers; a.hash_count its length (a
// multiple of 4).  Gradients are not cleared here: a peer may still be
// reading them until the closing barrier.
// Peer loads that go to the owning GPU every time (volatile: never served
// from a cache line filled by an earlier step).
__device__ __forceinline__ uint4 ld_peer_v4(const void *p) {
  uint4 r;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint2 ld_peer_v2(const void *p) {
  uint2 r;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];"
               : "=r"(r.x), "=r"(r.y)
               : "l"(p));
  return r;
}

__global__ void __launch_bounds__(256)
    k_peer_adam(AdamArgs a, PeerTable pt, int world, uint64_t off,
                float *__restrict__ w, float *__restrict__ m,
                float *__restrict__ v) {
  if (adam_vetoed(a)) return;
  const uint64_t n4 = a.hash_count / 4;
  const uint64_t q0 = off / 4;
  for (uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n4;
       q += (uint64_t)gridDim.x * blockDim.x) {
    float g[4] = {0.f, 0.f, 0.f, 0.f};
    if (a.grad_half) {
      uint2 r[kMaxPeers];
#pragma unroll
      for (int k = 0; k < kMaxPeers; ++k)
        if (k < world)
          r[k] = ld_peer_v2(reinterpret_cast<const uint2 *>(pt.grad[k]) + q0 + q);
#pragma unroll
      for (int k = 0; k < kMaxPeers; ++k) {
        if (k >= world) break;
        const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&r[k].x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&r[k].y));
        g[0] += lo.x;
        g[1] += lo.y;
        g[2] += hi.x;
        g[3] += hi.y;
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) g[k] *= kInvHalfGradScale;
    } else {
      uint4 r[kMaxPeers];
#pragma unroll
      for (int k = 0; k < kMaxPeers; ++k)
        if (k < world)
          r[k] = ld_peer_v4(reinterpret_cast<const uint4 *>(pt.grad[k]) + q0 + q);
#pragma unroll
      for (int k = 0; k < kMaxPeers; ++k) {
        if (k >= world) break;
        g[0] += __uint_as_float(r[k].x);
        g[1] += __uint_as_float(r[k].y);
        g[2] += __uint_as_float(r[k].z);
        g[3] += __uint_as_float(r[k].w);
      }
    }
    bool on[4];
    if (a.entry_width == 2) {
      on[0] = on[1] = g[0] != 0.f || g[1] != 0.f;
      on[2] = on[3] = g[2] != 0.f || g[3] != 0.f;
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) on[k] = g[k] != 0.f;
    }
    if (!(on[0] | on[1] | on[2] | on[3])) continue;
    float4 wv = reinterpret_cast<float4 *>(w)[q];
    float4 mv = reinterpret_cast<float4 *>(m)[q];
    float4 vv = reinterpret_cast<float4 *>(v)[q];
    float *pw = &wv.x, *pm = &mv.x, *pv = &vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (on[k]) adam_elem(pw[k], pm[k], pv[k], g[k], a.lr_hash, a, a.l1_hash, false);
    reinterpret_cast<float4 *>(w)[q] = wv;
    reinterpret_cast<float4 *>(m)[q] = mv;
    reinterpret_cast<float4 *>(v)[q] = vv;
    __half2 h[2] = {__floats2half2_rn(wv.x, wv.y), __floats2half2_rn(wv.z, wv.w)};
    const uint2 hb = *reinterpret_cast<uint2 *>(h);
#pragma unroll
    for (int k = 0; k < kMaxPeers; ++k)
      if (k < world) reinterpret_cast<uint2 *>(pt.table_h[k])[q0 + q] = hb;
  }
  // this thread's peer stores are ordered before the closing barrier's flag
  __threadfence_system();
}

// Barrier of the ranks over peer memory: thread t announces `epoch` in slot
// `rank` of rank t's flag array, then waits until rank t has announced it in
// this rank's array.  Epochs only grow, so the flags are never reset.  The
// wait gives up after about two seconds (a rank that never arrives): it sets
// *err and returns, the context stays usable and the host reports the error.
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void k_peer_barrier(PeerTable pt, int rank, int world,
                               uint32_t epoch, int32_t *err) {
  const int t = threadIdx.x;
  if (t >= world) return;
  __threadfence_system();
  st_release_sys(pt.flags[t] + rank, epoch);
  const uint32_t *f = pt.flags[rank] + t;
  const long long t0 = clock64();
  while ((int32_t)(ld_acquire_sys(f) - epoch) < 0) {
    if (clock64() - t0 > (1ll << 32)) {
      atomicExch(err, 1);
      return;
    }
    __nanosleep(256);
  }
}

// ------------------------------------------------------------ numerics probe

// The reference's sampled numerics probes (training_step_execution.cpp:
// 237-250 probe_backward_numerics, :290-340 accumulate_update_probe_for_range)
// evaluated on the device over the gradients before Adam: finiteness, max
// |g| and sum g^2 of the finite gradients; and, per element, the Adam update
// the step would apply (same arithmetic as the probe: clip, decay or L1/L2,
// moments, bias corrections, candidate weight), its finiteness and max
// |w - w'|.  Every parameter is scanned (dense), as the reference does.
// Unless `force`, the probe returns at once when the step's loss is finite,
// so launching it every step costs one empty launch.
__device__ inline void atomic_max_nonneg(float *p, float v) {
  atomicMax(reinterpret_cast<int *>(p), __float_as_int(v));
}

__device__ inline bool probe_elem(float g, float w, float m, float v, float lr,
                                  float reg, bool is_mlp, const AdamArgs &a,
                                  float &du) {
  if (a.grad_clip > 0.0f)
    g = g < -a.grad_clip ? -a.grad_clip : (g > a.grad_clip ? a.grad_clip : g);
  if (a.weight_decay > 0.0f) {
  } else if (!is_mlp && reg > 0.0f) {
    g = g + reg * (w > 0.0f ? 1.0f : (w < 0.0f ? -1.0f : 0.0f));
  } else if (is_mlp && reg > 0.0f) {
    g = g + reg * w;
  }
  const float mn = a.beta1 * m + (1.0f - a.beta1) * g;
  const float vn = a.beta2 * v + ((1.0f - a.beta2) * g) * g;
  const float mh = mn / a.bc1;
  const float vh = vn / a.bc2;
  const float ad = (lr * mh) / (sqrtf(vh) + a.eps);
  const float wd = a.weight_decay > 0.0f ? (lr * a.weight_decay) * w : 0.0f;
  const float cand = (w - wd) - ad;
  du = w - cand;
  return isfinite(g) && isfinite(mn) && isfinite(vn) && isfinite(mh) &&
         isfinite(vh) && isfinite(ad) && isfinite(wd) && isfinite(cand) &&
         isfinite(du);
}

__global__ void __launch_bounds__(256)
    k_numerics_probe(AdamArgs a, const float *__restrict__ w,
                     const float *__restrict__ m, const float *__restrict__ v,
                     const int32_t *__restrict__ gh_fixed,
                     const float *__restrict__ gh_float,
                     const float *__restrict__ gm, uint64_t mlp_base,
                     StepStats *st, int force, int gate) {
  const double loss = st->loss;
  if (!force && loss - loss == 0.0) return;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    st->probed = 1;
    st->gate = gate;
  }
  const uint64_t total = a.hash_count + a.mlp_count;
  double l2 = 0.0;
  float mg = 0.0f, mu = 0.0f;
  bool bad_g = false, bad_u = false;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const bool is_mlp = i >= a.hash_count;
    const uint64_t e = is_mlp ? mlp_base + (i - a.hash_count) : i;
    float g;
    if (is_mlp)
      g = gm[i - a.hash_count];
    else
      g = a.grad_fixed  ? (float)gh_fixed[i] * kInvGradScale
          : a.grad_half ? __half2float(reinterpret_cast<const __half *>(gh_float)[i]) *
                              kInvHalfGradScale
                        : gh_float[i];
    if (!isfinite(g)) {
      bad_g = true;
      continue;
    }
    mg = fmaxf(mg, fabsf(g));
    l2 += (double)g * (double)g;
    float du;
    if (probe_elem(g, w[e], m[e], v[e], is_mlp ? a.lr_mlp : a.lr_hash,
                   is_mlp ? a.l2_mlp : a.l1_hash, is_mlp, a, du))
      mu = fmaxf(mu, fabsf(du));
    else
      bad_u = true;
  }
  __shared__ double s_l2[8];
  __shared__ float s_mg[8], s_mu[8];
  __shared__ int s_bad;
  if (threadIdx.x == 0) s_bad = 0;
  for (int o = 16; o > 0; o >>= 1) {
    l2 += __shfl_down_sync(0xffffffffu, l2, o);
    mg = fmaxf(mg, __shfl_down_sync(0xffffffffu, mg, o));
    mu = fmaxf(mu, __shfl_down_sync(0xffffffffu, mu, o));
  }
  __syncthreads();
  if (bad_g) atomicOr(&s_bad, 1);
  if (bad_u) atomicOr(&s_bad, 2);
  const int wid = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    s_l2[wid] = l2;
    s_mg[wid] = mg;
    s_mu[wid] = mu;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < (int)(blockDim.x >> 5); ++k) {
      l2 += s_l2[k];
      mg = fmaxf(mg, s_mg[k]);
      mu = fmaxf(mu, s_mu[k]);
    }
    if (l2 != 0.0) atomicAdd(&st->grad_l2, l2);
    atomic_max_nonneg(&st->max_abs_grad, mg);
    atomic_max_nonneg(&st->max_abs_update, mu);
    if (s_bad & 1) st->nonfinite_bwd = 1.0f;
    if (s_bad & 2) st->nonfinite_upd = 1.0f;
  }
}

void launch_numerics_probe(const AdamArgs &a, const float *w, const float *m,
                           const float *v, const int32_t *gh_fixed,
                           const float *gh_float, const float *gm,
                           uint64_t mlp_base, StepStats *st, int force,
                           int gate, int num_sms, cudaStream_t st_) {
  // unforced: one block checks the loss and scans only when it is not
  // finite (rare, and then slow is fine); forced: the whole device
  k_numerics_probe<<<force ? num_sms * 8 : 1, 256, 0, st_>>>(a, w, m, v, gh_fixed,
                                                 gh_float, gm, mlp_base, st,
                                                 force, gate);
}

// Completes the touched map of the implicit-touch mode: a slot whose float
// gradient is nonzero is touched (read-back only).
__global__ void k_touched_from_grads(const float *__restrict__ g,
                                     uint8_t *touched, uint64_t slots, int ew,
                                     int half) {
  const __half *gh = reinterpret_cast<const __half *>(g);
  for (uint64_t s = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; s < slots;
       s += (uint64_t)gridDim.x * blockDim.x) {
    bool nz = false;
    for (int k = 0; k < ew; ++k)
      nz = nz || (half ? __half2float(gh[s * ew + k]) != 0.f : g[s * ew + k] != 0.f);
    if (nz) touched[s] = 1;
  }
}

void launch_touched_from_grads(const float *g, uint8_t *touched, uint64_t slots,
                               int entry_width, bool half, int num_sms,
                               cudaStream_t st) {
  if (slots)
    k_touched_from_grads<<<num_sms * 8, 256, 0, st>>>(g, touched, slots,
                                                      entry_width, half ? 1 : 0);
}

__global__ void k_to_half(const float *__restrict__ src, __half *dst,
                          uint64_t n) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    dst[i] = __float2half_rn(src[i]);
}

// ------------------------------------------------------------ Philox init

// Philox-4x32-10 (Salmon et al., SC'11); the reference's init kernels
// (metal_context.cpp:731-874) draw ctr = (counter_base + t, 0, 0, 0).
__device__ inline void philox(uint32_t c[4], uint32_t k0, uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = 0xD2511F53u * c[0], hi0 = __umulhi(0xD2511F53u, c[0]);
    const uint32_t lo1 = 0xCD9E8D57u * c[2], hi1 = __umulhi(0xCD9E8D57u, c[2]);
    const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0;
    c[1] = lo1;
    c[2] = n2;
    c[3] = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

__global__ void k_init_uniform(float *out, uint64_t count, float low,
                               float high, uint32_t k0, uint32_t k1,
                               uint32_t counter_base) {
  const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t * 4 >= count) return;
  uint32_t c[4] = {counter_base + (uint32_t)t, 0u, 0u, 0u};
  philox(c, k0, k1);
  const float span = high - low;
  for (int k = 0; k < 4; ++k) {
    const uint64_t e = t * 4 + k;
    if (e >= count) break;
    const float u = (float)c[k] * (1.0f / 4294967296.0f);
    out[e] = low + u * span;
  }
}

__global__ void k_init_normal(float *out, uint64_t count, float mean,
                              float stddev, uint32_t k0, uint32_t k1,
                              uint32_t counter_base) {
  const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t * 4 >= count) return;
  uint32_t c[4] = {counter_base + (uint32_t)t, 0u, 0u, 0u};
  philox(c, k0, k1);
  const float s = 1.0f / 4294967296.0f;
  float u1 = fmaxf((float)c[0] * s, 1.0e-30f), u2 = (float)c[1] * s;
  float u3 = fmaxf((float)c[2] * s, 1.0e-30f), u4 = (float)c[3] * s;
  const float TWO_PI = 6.28318530718f;
  const float r1 = sqrtf(-2.0f * logf(u1)), r2 = sqrtf(-2.0f * logf(u3));
  const float z[4] = {r1 * cosf(TWO_PI * u2), r1 * sinf(TWO_PI * u2),
                      r2 * cosf(TWO_PI * u4), r2 * sinf(TWO_PI * u4)};
  for (int k = 0; k < 4; ++k) {
    const uint64_t e = t * 4 + k;
    if (e >= count) break;
    out[e] = mean + stddev * z[k];
  }
}

// ------------------------------------------------------------ Morton order

__device__ inline uint32_t expand3(uint32_t v) {
  v = (v | (v << 16)) & 0x030000FFu;
  v = (v | (v << 8)) & 0x0300F00Fu;
  v = (v | (v << 4)) & 0x030C30C3u;
  v = (v | (v << 2)) & 0x09249249u;
  return v;
}
__device__ inline uint32_t expand4(uint32_t v) {
  v &= 0xFFu;
  v = (v | (v << 16)) & 0x000F000Fu;
  v = (v | (v << 8)) & 0x00C30C03u;
  v = (v | (v << 4)) & 0x09090909u;
  v = (v | (v << 2)) & 0x11111111u;
  return v;
}
__device__ inline uint32_t quant(float v, float cells) {
  const float mapped = (v * 0.5f + 0.5f) * cells;
  return (uint32_t)fminf(fmaxf(mapped, 0.0f), cells - 1.0f);
}

// morton_sort.h:14-58 codes.
__device__ inline uint32_t morton_code(const float *p, int d) {
  return d == 4 ? (expand4(quant(p[3], 256.f)) << 3) |
                      (expand4(quant(p[2], 256.f)) << 2) |
                      (expand4(quant(p[1], 256.f)) << 1) |
                      expand4(quant(p[0], 256.f))
                : (expand3(quant(p[2], 1024.f)) << 2) |
                      (expand3(quant(p[1], 1024.f)) << 1) |
                      expand3(quant(p[0], 1024.f));
}

// Codes and identity indices for CUB's stable radix sort (equal keys keep
// their input order).
__global__ void k_morton_codes(const float *__restrict__ pos, int d,
                               uint32_t *codes, uint32_t *idx, uint32_t N) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N) return;
  codes[i] = morton_code(pos + (size_t)i * d, d);
  idx[i] = i;
}

// Stable counting sort on short keys (the top <= 12 bits of the code): the
// same permutation as the stable radix sort, in three light passes.  Block b
// owns points [b*chunk, (b+1)*chunk).
constexpr int kCsBuckets = 4096;

__global__ void __launch_bounds__(256)
    k_count_hist(const float *__restrict__ pos, int d, uint32_t N,
                 uint32_t chunk, int shift, int nbuckets, uint32_t *hist) {
  __shared__ uint32_t cnt[kCsBuckets];
  for (int k = threadIdx.x; k < nbuckets; k += blockDim.x) cnt[k] = 0;
  __syncthreads();
  const uint32_t b0 = blockIdx.x * chunk;
  const uint32_t b1 = min(N, b0 + chunk);
  for (uint32_t i = b0 + threadIdx.x; i < b1; i += blockDim.x)
    atomicAdd(&cnt[morton_code(pos + (size_t)i * d, d) >> shift], 1u);
  __syncthreads();
  for (int k = threadIdx.x; k < nbuckets; k += blockDim.x)
    hist[(size_t)k * gridDim.x + blockIdx.x] = cnt[k];
}

// offs = exclusive scan of hist in (bucket, block) order: the first sorted
// slot of block b's points with key k.  The block sorts its chunk locally
// (CUB's stable block radix sort on the key), so a point's slot is
// offs[key][b] + its position among the block's points of that key; then
// it moves its index, position row and per-point row there.
constexpr int kCsThreads = 256, kCsItems = 8;

__global__ void __launch_bounds__(kCsThreads)
    k_count_scatter(const float *__restrict__ pos, int d, uint32_t N,
                    uint32_t chunk, int shift, int nbuckets,
                    const uint32_t *__restrict__ offs, uint32_t *perm,
                    float *pos_dst, const float *__restrict__ rows, int width,
                    float *rows_dst) {
  using BlockSort = cub::BlockRadixSort<uint32_t, kCsThreads, kCsItems, uint32_t>;
  __shared__ union {
    typename BlockSort::TempStorage sort;
    uint32_t keys[kCsThreads * kCsItems];
  } sh;
  __shared__ uint32_t first[kCsBuckets];  // local sorted position of a key's
                                          // first point (present keys only)
  const uint32_t b0 = blockIdx.x * chunk;
  uint32_t key[kCsItems], idx[kCsItems];
#pragma unroll
  for (int j = 0; j < kCsItems; ++j) {
    const uint32_t i = b0 + threadIdx.x * kCsItems + j;
    idx[j] = i;
    // points past the end sort last under the sentinel key nbuckets
    key[j] = i < N ? morton_code(pos + (size_t)i * d, d) >> shift
                   : (uint32_t)nbuckets;
  }
  int bits = 1;
  while ((1 << bits) <= nbuckets) ++bits;
  BlockSort(sh.sort).Sort(key, idx, 0, bits);  // stable, blocked result
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kCsItems; ++j) sh.keys[threadIdx.x * kCsItems + j] = key[j];
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kCsItems; ++j) {
    const int p = threadIdx.x * kCsItems + j;
    if (key[j] < (uint32_t)nbuckets && (p == 0 || sh.keys[p - 1] != key[j]))
      first[key[j]] = (uint32_t)p;
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kCsItems; ++j) {
    if (key[j] >= (uint32_t)nbuckets) continue;
    const int p = threadIdx.x * kCsItems + j;
    const uint32_t dst =
        offs[(size_t)key[j] * gridDim.x + blockIdx.x] + (uint32_t)p - first[key[j]];
    const uint32_t i = idx[j];
    perm[dst] = i;
    if (pos_dst)
      for (int a = 0; a < d; ++a)
        pos_dst[(size_t)dst * d + a] = pos[(size_t)i * d + a];
    if (rows_dst)
      for (int a = 0; a < width; ++a)
        rows_dst[(size_t)dst * width + a] = rows[(size_t)i * width + a];
  }
}

__host__ inline uint32_t count_chunk(uint32_t) {
  return (uint32_t)(kCsThreads * kCsItems);  // one block sort per chunk
}

__global__ void k_gather_rows(const float *__restrict__ src, int width,
                              const uint32_t *__restrict__ perm, float *dst,
                              uint32_t N) {
  const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (uint64_t)N * width) return;
  const uint64_t row = t / width, col = t % width;
  dst[t] = src[(uint64_t)perm[row] * width + col];
}

__global__ void k_scatter_rows(const float *__restrict__ src, int width,
                               const uint32_t *__restrict__ perm, float *dst,
                               uint32_t N) {
  const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (uint64_t)N * width) return;
  const uint64_t row = t / width, col = t % width;
  dst[(uint64_t)perm[row] * width + col] = src[t];
}

// ------------------------------------------------------------ launchers


int exact_grid(uint32_t N, int num_sms) {
  const uint32_t want = (N + kExactBlock - 1) / kExactBlock;
  const uint32_t cap = (uint32_t)num_sms * 8u;
  return (int)(want < cap ? (want > 0 ? want : 1) : cap);
}

size_t exact_scratch_floats(const NetDims &nd, int num_sms) {
  return wmax_for(nd.W) ? 0
                        : (size_t)num_sms * 8 * kExactBlock * nd.H * nd.W;
}

void launch_train_exact(const NetDims &nd, const float *table,
                        const float *mlp, const float *pos, const float *tgt,
                        const float *dext, float inv_N, float *grad_mlp,
                        int32_t *gh_fixed, float *gh_float, uint8_t *touched,
                        double *loss_acc, uint32_t N, float *scratch,
                        int num_sms, cudaStream_t st, ProbeAcc *probe) {
  if (N == 0) return;
  const int grid = exact_grid(N, num_sms);
  const size_t smem = (size_t)nd.mlp_count * sizeof(float);
  const int use_smem = smem <= 96 * 1024 ? 1 : 0;
  const size_t dyn = use_smem ? smem : 0;
#define TMNN_TRAIN_CASE(WM)                                                   \
  {                                                                           \
    if (dyn > 48 * 1024)                                                      \
      cudaFuncSetAttribute(k_train_exact<WM>,                                 \
                           cudaFuncAttributeMaxDynamicSharedMemorySize,       \
                           (int)dyn);                                         \
    k_train_exact<WM><<<grid, kExactBlock, dyn, st>>>(                        \
        nd, table, mlp, pos, tgt, dext, inv_N, grad_mlp, gh_fixed, gh_float,  \
        touched, loss_acc, N, use_smem, scratch, probe);                      \
  }
  switch (wmax_for(nd.W)) {
    case 16: TMNN_TRAIN_CASE(16) break;
    case 32: TMNN_TRAIN_CASE(32) break;
    case 64: TMNN_TRAIN_CASE(64) break;
    case 128: TMNN_TRAIN_CASE(128) break;
    default: TMNN_TRAIN_CASE(0) break;
  }
#undef TMNN_TRAIN_CASE
}

void launch_forward_exact(const NetDims &nd, const float *table,
                          const float *mlp, const float *pos, float *out,
                          uint32_t N, float *scratch, int num_sms,
                          cudaStream_t st) {
  if (N == 0) return;
  const int grid = exact_grid(N, num_sms);
  switch (wmax_for(nd.W)) {
    case 16: k_forward_exact<16><<<grid, kExactBlock, 0, st>>>(nd, table, mlp, pos, out, N, scratch); break;
    case 32: k_forward_exact<32><<<grid, kExactBlock, 0, st>>>(nd, table, mlp, pos, out, N, scratch); break;
    case 64: k_forward_exact<64><<<grid, kExactBlock, 0, st>>>(nd, table, mlp, pos, out, N, scratch); break;
    case 128: k_forward_exact<128><<<grid, kExactBlock, 0, st>>>(nd, table, mlp, pos, out, N, scratch); break;
    default: k_forward_exact<0><<<grid, kExactBlock, 0, st>>>(nd, table, mlp, pos, out, N, scratch); break;
  }
}

void launch_encode_debug(const NetDims &nd, const float *table,
                         const float *pos, float *feat, uint32_t *corner_idx,
                         int32_t *cells, uint32_t N, cudaStream_t st) {
  if (N == 0) return;
  k_encode_debug<<<(N + 127) / 128, 128, 0, st>>>(nd, table, pos, feat,
                                                  corner_idx, cells, N);
}

void launch_adam(const AdamArgs &a, float *w, float *m, float *v,
                 int32_t *gh_fixed, float *gh_float, float *gm,
                 uint8_t *touched, __half *table_h, int num_sms,
                 cudaStream_t st) {
  // hash table: 4 elements per thread, enough threads to keep HBM busy
  const uint64_t n4 = a.hash_count / 4;
  uint64_t blocks = (n4 + 255) / 256;
  const uint64_t cap = (uint64_t)num_sms * 64;
  if (blocks > cap) blocks = cap;
  if (blocks) {
    // the MLP weights ride along in the same launch
    k_adam_hash4<<<(unsigned)blocks, 256, 0, st>>>(a, w, m, v, gh_fixed,
                                                   gh_float, touched, table_h,
                                                   a.mlp_count ? gm : nullptr);
    return;
  }
  // MLP weights: one thread each (slots = 0 selects the MLP range)
  AdamArgs am = a;
  am.slots = 0;
  const uint64_t mb = (a.mlp_count + 255) / 256;
  if (mb)
    k_adam<<<(unsigned)mb, 256, 0, st>>>(am, w, m, v, gh_fixed, gh_float, gm,
                                         touched, table_h);
}

// MLP part of the update only (w, m, v, gm indexed from a.hash_count).
void launch_adam_mlp(const AdamArgs &a, float *w, float *m, float *v,
                     float *gm, int num_sms, cudaStream_t st) {
  (void)num_sms;
  AdamArgs am = a;
  am.slots = 0;
  const uint64_t mb = (a.mlp_count + 255) / 256;
  if (mb)
    k_adam<<<(unsigned)mb, 256, 0, st>>>(am, w, m, v, nullptr, nullptr, gm,
                                         nullptr, nullptr);
}

int launch_peer_exchange(const AdamArgs &a, const PeerTable &pt, int rank,
                         int world, uint64_t off, float *w, float *m, float *v,
                         uint32_t &epoch, int32_t *err, int num_sms,
                         cudaStream_t st) {
  k_peer_barrier<<<1, 32, 0, st>>>(pt, rank, world, ++epoch, err);
  const uint64_t n4 = a.hash_count / 4;
  uint64_t blocks = (n4 + 255) / 256;
  const uint64_t cap = (uint64_t)num_sms * 8;
  if (blocks > cap) blocks = cap;
  if (blocks)
    k_peer_adam<<<(unsigned)blocks, 256, 0, st>>>(a, pt, world, off, w + off,
                                                  m + off, v + off);
  k_peer_barrier<<<1, 32, 0, st>>>(pt, rank, world, ++epoch, err);
  return blocks ? 3 : 2;
}

void launch_to_half(const float *src, __half *dst, uint64_t n, int num_sms,
                    cudaStream_t st) {
  if (n == 0) return;
  k_to_half<<<num_sms * 8, 256, 0, st>>>(src, dst, n);
}

void launch_init_uniform(float *out, uint64_t count, float low, float high,
                         uint64_t seed, uint32_t counter_base,
                         cudaStream_t st) {
  const uint64_t threads = (count + 3) / 4;
  if (!threads) return;
  k_init_uniform<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
      out, count, low, high, (uint32_t)seed, (uint32_t)(seed >> 32),
      counter_base);
}

void launch_init_normal(float *out, uint64_t count, float mean, float stddev,
                        uint64_t seed, uint32_t counter_base,
                        cudaStream_t st) {
  const uint64_t threads = (count + 3) / 4;
  if (!threads) return;
  k_init_normal<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
      out, count, mean, stddev, (uint32_t)seed, (uint32_t)(seed >> 32),
      counter_base);
}

size_t morton_temp_bytes(uint32_t N) {
  size_t bytes = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, bytes, (uint32_t *)nullptr,
                                  (uint32_t *)nullptr, (uint32_t *)nullptr,
                                  (uint32_t *)nullptr, (int)N, 0, 32);
  const size_t nb = (N + count_chunk(N) - 1) / count_chunk(N);
  const size_t hist = ((size_t)kCsBuckets * nb * 4 + 255) & ~(size_t)255;
  size_t scan = 0;
  cub::DeviceScan::ExclusiveSum(nullptr, scan, (uint32_t *)nullptr,
                                (uint32_t *)nullptr, (int)(kCsBuckets * nb));
  return bytes > hist + scan ? bytes : hist + scan;
}

// Sorted permutation of the batch by Morton code; returns perm (input index
// of the i-th sorted point) in perm_out.
void launch_morton_order(const float *pos, int d, uint32_t N, uint32_t *codes,
                         uint32_t *codes_alt, uint32_t *idx,
                         uint32_t *perm_out, void *temp, size_t temp_bytes,
                         cudaStream_t st, int key_bits, float *pos_dst,
                         const float *rows, int width, float *rows_dst,
                         bool *gathered) {
  if (gathered) *gathered = false;
  if (N == 0) return;
  const int end = d == 4 ? 32 : 30;
  const int begin = key_bits > 0 && key_bits < end ? end - key_bits : 0;
  if (end - begin <= 12) {
    // short key: stable counting sort (the same permutation, fewer passes)
    const uint32_t chunk = count_chunk(N);
    const uint32_t nb = (N + chunk - 1) / chunk;
    const int nbuckets = 1 << (end - begin);
    uint32_t *hist = static_cast<uint32_t *>(temp);
    const size_t hbytes = ((size_t)nbuckets * nb * 4 + 255) & ~(size_t)255;
    size_t scan = temp_bytes - hbytes;
    k_count_hist<<<nb, 256, 0, st>>>(pos, d, N, chunk, begin, nbuckets, hist);
    cub::DeviceScan::ExclusiveSum(static_cast<uint8_t *>(temp) + hbytes, scan,
                                  hist, hist, (int)(nbuckets * nb), st);
    k_count_scatter<<<nb, 256, 0, st>>>(pos, d, N, chunk, begin, nbuckets,
                                        hist, perm_out, pos_dst, rows,
                                        width, rows_dst);
    if (gathered) *gathered = pos_dst != nullptr;
    return;
  }
  k_morton_codes<<<(N + 255) / 256, 256, 0, st>>>(pos, d, codes, idx, N);
  // stable radix sort on the top key_bits of the code: points of one coarse
  // Morton cell keep their input order
  cub::DeviceRadixSort::SortPairs(temp, temp_bytes, codes, codes_alt, idx,
                                  perm_out, (int)N, begin, end, st);
}

void launch_gather_rows(const float *src, int width, const uint32_t *perm,
                        float *dst, uint32_t N, cudaStream_t st) {
  const uint64_t n = (uint64_t)N * width;
  if (!n) return;
  k_gather_rows<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(src, width, perm,
                                                            dst, N);
}

void launch_scatter_rows(const float *src, int width, const uint32_t *perm,
                         float *dst, uint32_t N, cudaStream_t st) {
  const uint64_t n = (uint64_t)N * width;
  if (!n) return;
  k_scatter_rows<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(src, width, perm,
                                                             dst, N);
}

}  // namespace tmnn
