// nerf.cu -- the NeRF-style field of the benchmark configuration: a density
// network (HashGrid -> FullyFusedMLP with 16 outputs, exp on output 0) and a
// colour network (FullyFusedMLP on [SH degree-4 of the view direction (16) |
// geometry outputs 1..15 of the density network | one zero pad], sigmoid
// RGB).  tmnn composes no such pair (it has neither an SH encoding nor two
// chained networks); this is the composition of its split API
// (forward_for_training / backward_accumulate / adam_step,
// default_trainer.cpp:1047-1443) with a trainable plain MLP, on one stream:
//
//   density forward (fused tcgen05 kernel)
//   -> colour input: SH(dir) and the geometry features, fp16     (k_nerf_input)
//   -> colour forward + loss + backward, dL/dx to memory          (fused, D = 0)
//   -> density dL/dy: [2 (sigma - sigma_t) sigma / N | dL/dx geo] (k_nerf_dens)
//   -> density backward_accumulate (fused tcgen05 + hash scatter)
//   -> Adam on both.
//
// Loss per sample: sum over RGB of (rgb - rgb_t)^2 + (sigma - sigma_t)^2,
// averaged over the batch.
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <string>

#include "../../include/tmnn_cuda.h"
#include "fused.h"
#include "kernels.h"
#include "runtime.h"

using namespace tmnn;

namespace {

constexpr int kGeo = 15;    // density outputs 1..15 feed the colour network
constexpr int kColorIn = 32;  // 16 SH + 15 geometry + 1 zero pad

// Real spherical harmonics up to degree 3 (16 coefficients) of a unit
// direction, in the usual graphics order and sign convention (Sloan, "Stupid
// Spherical Harmonics Tricks", 2008, appendix): the constants are the
// normalisations sqrt((2l+1)/(4 pi) (l-|m|)!/(l+|m|)!) times the factors of
// the real basis, e.g. 0.2820947918 = 1/(2 sqrt(pi)).
__host__ __device__ inline void sh4(float x, float y, float z, float *o) {
  const float xx = x * x, yy = y * y, zz = z * z;
  o[0] = 0.28209479177387814f;
  o[1] = -0.48860251190291987f * y;
  o[2] = 0.48860251190291987f * z;
  o[3] = -0.48860251190291987f * x;
  o[4] = 1.0925484305920792f * (x * y);
  o[5] = -1.0925484305920792f * (y * z);
  o[6] = 0.94617469575755997f * zz - 0.31539156525251999f;
  o[7] = -1.0925484305920792f * (x * z);
  o[8] = 0.54627421529603959f * (xx - yy);
  o[9] = 0.59004358992664352f * y * (yy - 3.0f * xx);
  o[10] = 2.8906114426405538f * (x * y) * z;
  o[11] = 0.45704579946446572f * y * (1.0f - 5.0f * zz);
  o[12] = 0.3731763325901154f * z * (5.0f * zz - 3.0f);
  o[13] = 0.45704579946446572f * x * (1.0f - 5.0f * zz);
  o[14] = 1.4453057213202769f * z * (xx - yy);
  o[15] = 0.59004358992664352f * x * (3.0f * yy - xx);
}

// Colour-network input row: [SH(dir) | density outputs 1..15 | 0] as fp16.
__global__ void k_nerf_input(const float *__restrict__ dirs,
                             const float *__restrict__ dens,
                             __half *__restrict__ xin, uint32_t N) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N) return;
  float v[kColorIn];
  sh4(dirs[(size_t)i * 3], dirs[(size_t)i * 3 + 1], dirs[(size_t)i * 3 + 2], v);
#pragma unroll
  for (int k = 0; k < kGeo; ++k) v[16 + k] = dens[(size_t)i * 16 + 1 + k];
  v[31] = 0.0f;
  uint4 u[4];
  __half2 *h = reinterpret_cast<__half2 *>(u);
#pragma unroll
  for (int k = 0; k < 16; ++k) h[k] = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
  uint4 *dst = reinterpret_cast<uint4 *>(xin + (size_t)i * kColorIn);
#pragma unroll
  for (int k = 0; k < 4; ++k) dst[k] = u[k];
}

// Density-network dL/dy: output 0 through sigma = exp(y0) against the target
// density; outputs 1..15 receive the colour network's dL/dx of the geometry
// columns.  Sums the density loss.
__global__ void k_nerf_dens_grad(const float *__restrict__ dens,
                                 const float *__restrict__ sigma_t,
                                 const float *__restrict__ dx, float inv_N,
                                 float *__restrict__ dy, double *loss,
                                 uint32_t N) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  float l = 0.0f;
  if (i < N) {
    const float s = expf(dens[(size_t)i * 16]);
    const float r = s - sigma_t[i];
    l = r * r;
    float *o = dy + (size_t)i * 16;
    o[0] = (2.0f * r) * s * inv_N;
#pragma unroll
    for (int k = 0; k < kGeo; ++k) o[1 + k] = dx[(size_t)i * kColorIn + 16 + k];
  }
  for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
  if ((threadIdx.x & 31) == 0 && l != 0.0f) atomicAdd(loss, (double)l);
}

__global__ void k_nerf_sigma(const float *__restrict__ dens,
                             float *__restrict__ sigma, uint32_t N) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < N) sigma[i] = expf(dens[(size_t)i * 16]);
}

template <class T>
struct Buf {
  T *p = nullptr;
  size_t n = 0;
  void ensure(size_t count) {
    if (count <= n) return;
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
    if (cudaMalloc(&p, count * sizeof(T)) != cudaSuccess)
      throw std::runtime_error("nerf: cudaMalloc failed");
    n = count;
  }
  ~Buf() {
    if (p) cudaFree(p);
  }
};

thread_local std::string g_nerf_err;

#define CKN(x)                                                             \
  do {                                                                     \
    cudaError_t e_ = (x);                                                  \
    if (e_ != cudaSuccess)                                                 \
      throw std::runtime_error(std::string(#x) + ": " +                    \
                               cudaGetErrorString(e_));                    \
  } while (0)

void check(tmnn_status st, const char *what) {
  if (st == TMNN_OK) return;
  const std::string m = std::string(what) + ": " + tmnn_cuda_last_error();
  if (st == TMNN_ERR_INVALID_ARGUMENT) throw std::invalid_argument(m);
  throw std::runtime_error(m);
}

template <class F>
tmnn_status run(F &&f) {
  try {
    g_nerf_err.clear();
    f();
    return TMNN_OK;
  } catch (const std::invalid_argument &e) {
    g_nerf_err = e.what();
    return TMNN_ERR_INVALID_ARGUMENT;
  } catch (const std::exception &e) {
    g_nerf_err = e.what();
    return TMNN_ERR_OPERATION_FAILED;
  }
}

}  // namespace

struct tmnn_nerf {
  int device = 0, num_sms = 148;
  tmnn_ctx *density = nullptr;
  cudaStream_t stream = nullptr;  // the density context's stream
  NetDims cnd{};                  // colour network
  float lr = 1e-2f, beta1 = 0.9f, beta2 = 0.99f, eps = 1e-15f;
  uint32_t step = 0;
  Buf<float> cw, cm, cv, cg;  // colour weights, moments, gradients
  Buf<double> loss;           // [rgb, density]
  double *h_loss = nullptr;
  FusedWorkspace ws;
  Buf<float> pos_d, dirs_d, rgb_d, sig_d, dens, dx, dy, out_rgb, out_sig;
  Buf<__half> xin;
  uint64_t launches = 0;   // kernels launched by this object (not the density
                           // context's own, which it counts itself)
  cudaEvent_t ev[5] = {};  // phase boundaries of a profiled step
  float phase_ms[4] = {};  // density fwd, colour, density bwd, density Adam
  ~tmnn_nerf() {
    if (stream) cudaStreamSynchronize(stream);
    for (auto e : ev)
      if (e) cudaEventDestroy(e);
    fused_release(ws);
    if (h_loss) cudaFreeHost(h_loss);
    if (density) tmnn_cuda_ctx_destroy(density);
  }
};

namespace {

const float *stage(tmnn_nerf &n, const float *src, size_t count, Buf<float> &b,
                   uint32_t flags) {
  if (flags & TMNN_PTR_DEVICE) return src;
  b.ensure(count);
  CKN(cudaMemcpyAsync(b.p, src, count * 4, cudaMemcpyHostToDevice, n.stream));
  return b.p;
}

void colour_adam(tmnn_nerf &n) {
  AdamArgs a{};
  const float s = (float)(n.step + 1u);
  a.lr_hash = a.lr_mlp = n.lr;
  a.beta1 = n.beta1;
  a.beta2 = n.beta2;
  a.eps = n.eps;
  a.bc1 = 1.0f - std::pow(n.beta1, s);
  a.bc2 = 1.0f - std::pow(n.beta2, s);
  a.hash_count = 0;
  a.mlp_count = n.cnd.mlp_count;
  launch_adam_mlp(a, n.cw.p, n.cm.p, n.cv.p, n.cg.p, n.num_sms, n.stream);
  n.launches++;
  fused_weights_changed(n.ws);
  ++n.step;
}

// Density forward + colour input for N staged samples.
void front(tmnn_nerf &n, const float *pos, const float *dirs, uint32_t N) {
  n.dens.ensure((size_t)N * 16);
  n.xin.ensure((size_t)N * kColorIn);
  check(tmnn_cuda_forward(n.density, pos, n.dens.p, N, TMNN_PTR_DEVICE),
        "nerf: density forward");
  k_nerf_input<<<(N + 255) / 256, 256, 0, n.stream>>>(dirs, n.dens.p, n.xin.p,
                                                       N);
  n.launches++;
}

}  // namespace

extern "C" {

tmnn_status tmnn_cuda_nerf_create(int device, const tmnn_nerf_cfg *cfg,
                                  tmnn_nerf **out) {
  if (!cfg || !out) return TMNN_ERR_NULL_OBJECT;
  *out = nullptr;
  tmnn_nerf *n = new tmnn_nerf;
  tmnn_status st = run([&] {
    tmnn_spec spec = cfg->density;
    if (spec.num_outputs != 16 || spec.spatial_dims != 3)
      throw std::invalid_argument(
          "nerf_create: the density network maps 3D positions to 16 outputs");
    tmnn_train_cfg tc;
    tmnn_cuda_default_train_cfg(&tc);
    tc.lr_encoding = tc.lr_network = cfg->lr;
    tc.seed = cfg->seed;
    tc.family = cfg->family;
    tc.hash_grad_format = TMNN_GRAD_F32;
    tc.batch_size = 1 << 20;
    check(tmnn_cuda_ctx_create(device, &spec, &tc, &n->density),
          "nerf_create: density network");
    void *sp = nullptr;
    check(tmnn_cuda_get_stream(n->density, &sp), "nerf_create");
    n->stream = static_cast<cudaStream_t>(sp);
    n->device = device;
    n->lr = cfg->lr;
    CKN(cudaSetDevice(device));
    CKN(cudaDeviceGetAttribute(&n->num_sms, cudaDevAttrMultiProcessorCount,
                               device));
    NetDims &c = n->cnd;
    c.In = kColorIn;
    c.L = kColorIn;
    c.F = 1;
    c.W = (int)cfg->color_width;
    c.H = (int)cfg->color_hidden_layers;
    c.O = 3;
    c.loss = 0;  // L2 on the sigmoid outputs
    if (c.H < 1 || c.H > kMaxHidden)
      throw std::invalid_argument("nerf_create: color_hidden_layers out of range");
    std::string why;
    if (!fused_mlp_train_supported(c, &why))
      throw std::invalid_argument("nerf_create: colour network: " + why);
    mlp_layout(c);
    n->cw.ensure(c.mlp_count);
    n->cm.ensure(c.mlp_count);
    n->cv.ensure(c.mlp_count);
    n->cg.ensure(c.mlp_count);
    n->loss.ensure(2);
    CKN(cudaMallocHost(&n->h_loss, 2 * sizeof(double)));
    for (auto &e : n->ev) CKN(cudaEventCreate(&e));
    mlp_init_xavier(c, n->cw.p, cfg->seed ^ 0x9E3779B97F4A7C15ull, n->stream);
    CKN(cudaMemsetAsync(n->cm.p, 0, c.mlp_count * 4, n->stream));
    CKN(cudaMemsetAsync(n->cv.p, 0, c.mlp_count * 4, n->stream));
    CKN(cudaMemsetAsync(n->cg.p, 0, c.mlp_count * 4, n->stream));
    CKN(cudaStreamSynchronize(n->stream));
  });
  if (st == TMNN_OK)
    *out = n;
  else
    delete n;
  return st;
}

tmnn_status tmnn_cuda_nerf_destroy(tmnn_nerf *n) {
  if (!n) return TMNN_ERR_NULL_OBJECT;
  return run([&] {
    cudaSetDevice(n->device);
    delete n;
  });
}

tmnn_status tmnn_cuda_nerf_density(tmnn_nerf *n, tmnn_ctx **out) {
  if (!n || !out) return TMNN_ERR_NULL_OBJECT;
  *out = n->density;
  return TMNN_OK;
}

tmnn_status tmnn_cuda_nerf_color_weights(tmnn_nerf *n, const float *host_in,
                                         float *host_out, size_t count) {
  if (!n) return TMNN_ERR_NULL_OBJECT;
  return run([&] {
    if (count != n->cnd.mlp_count)
      throw std::invalid_argument("nerf_color_weights: count mismatch");
    CKN(cudaSetDevice(n->device));
    if (host_in) {
      CKN(cudaMemcpyAsync(n->cw.p, host_in, count * 4, cudaMemcpyHostToDevice,
                          n->stream));
      CKN(cudaMemsetAsync(n->cm.p, 0, count * 4, n->stream));
      CKN(cudaMemsetAsync(n->cv.p, 0, count * 4, n->stream));
      n->step = 0;
      fused_weights_changed(n->ws);
    }
    if (host_out)
      CKN(cudaMemcpyAsync(host_out, n->cw.p, count * 4, cudaMemcpyDeviceToHost,
                          n->stream));
    CKN(cudaStreamSynchronize(n->stream));
  });
}

tmnn_status tmnn_cuda_nerf_train_step(tmnn_nerf *n, const float *pos,
                                      const float *dirs, const float *rgb,
                                      const float *sigma, uint32_t N,
                                      uint32_t flags, float *loss) {
  if (!n) return TMNN_ERR_NULL_OBJECT;
  return run([&] {
    if (N > 0 && (!pos || !dirs || !rgb || !sigma))
      throw std::invalid_argument("nerf_train_step: null arguments");
    CKN(cudaSetDevice(n->device));
    if (N == 0) {
      if (loss) *loss = 0.0f;
      return;
    }
    const float *p = stage(*n, pos, (size_t)N * 3, n->pos_d, flags);
    const float *d = stage(*n, dirs, (size_t)N * 3, n->dirs_d, flags);
    const float *c = stage(*n, rgb, (size_t)N * 3, n->rgb_d, flags);
    const float *s = stage(*n, sigma, N, n->sig_d, flags);
    // data parallel: every mean is over the global batch (equal shards)
    const uint64_t global_n = (uint64_t)N * (uint64_t)ctx_world(n->density);
    const float inv_N = 1.0f / (float)global_n;
    const bool prof = flags & TMNN_PROFILE;
    if (prof) CKN(cudaEventRecord(n->ev[0], n->stream));
    front(*n, p, d, N);
    if (prof) CKN(cudaEventRecord(n->ev[1], n->stream));
    n->dx.ensure((size_t)N * kColorIn);
    n->dy.ensure((size_t)N * 16);
    CKN(cudaMemsetAsync(n->loss.p, 0, 2 * sizeof(double), n->stream));
    n->launches += fused_mlp_train(n->ws, n->cnd, n->cw.p, n->xin.p, c, nullptr,
                                   inv_N, n->cg.p, n->loss.p, n->dx.p, N,
                                   n->num_sms, n->stream, 1);
    k_nerf_dens_grad<<<(N + 255) / 256, 256, 0, n->stream>>>(
        n->dens.p, s, n->dx.p, inv_N, n->dy.p, n->loss.p + 1, N);
    n->launches++;
    // colour gradients and both losses summed over the ranks (the density
    // network's gradients are exchanged by its own adam_step)
    ctx_allreduce_sum(n->density, n->cg.p, n->cnd.mlp_count, n->loss.p, 2);
    colour_adam(*n);
    CKN(cudaMemcpyAsync(n->h_loss, n->loss.p, 2 * sizeof(double),
                        cudaMemcpyDeviceToHost, n->stream));
    if (prof) CKN(cudaEventRecord(n->ev[2], n->stream));
    check(tmnn_cuda_backward_accumulate(n->density, p, n->dy.p, N,
                                        TMNN_PTR_DEVICE),
          "nerf: density backward");
    if (prof) CKN(cudaEventRecord(n->ev[3], n->stream));
    check(tmnn_cuda_adam_step(n->density), "nerf: density adam");
    if (prof) {
      CKN(cudaEventRecord(n->ev[4], n->stream));
      CKN(cudaEventSynchronize(n->ev[4]));
      for (int k = 0; k < 4; ++k)
        CKN(cudaEventElapsedTime(&n->phase_ms[k], n->ev[k], n->ev[k + 1]));
    }
    CKN(cudaGetLastError());
    if (fused_error(n->ws, n->stream))
      throw std::runtime_error("nerf: colour kernel pipeline wait timed out");
    if (loss)
      *loss = (float)((n->h_loss[0] + n->h_loss[1]) / (double)global_n);
  });
}

tmnn_status tmnn_cuda_nerf_dp_init(tmnn_nerf *n, const uint8_t unique_id[128],
                                   int rank, int world) {
  if (!n) return TMNN_ERR_NULL_OBJECT;
  return tmnn_cuda_dp_init(n->density, unique_id, rank, world);
}

tmnn_status tmnn_cuda_nerf_inference(tmnn_nerf *n, const float *pos,
                                     const float *dirs, float *rgb,
                                     float *sigma, uint32_t N, uint32_t flags) {
  if (!n) return TMNN_ERR_NULL_OBJECT;
  return run([&] {
    if (N > 0 && (!pos || !dirs || !rgb || !sigma))
      throw std::invalid_argument("nerf_inference: null arguments");
    CKN(cudaSetDevice(n->device));
    if (N == 0) return;
    const float *p = stage(*n, pos, (size_t)N * 3, n->pos_d, flags);
    const float *d = stage(*n, dirs, (size_t)N * 3, n->dirs_d, flags);
    front(*n, p, d, N);
    const bool dev = flags & TMNN_PTR_DEVICE;
    float *o_rgb = rgb, *o_sig = sigma;
    if (!dev) {
      n->out_rgb.ensure((size_t)N * 3);
      n->out_sig.ensure(N);
      o_rgb = n->out_rgb.p;
      o_sig = n->out_sig.p;
    }
    n->launches += fused_mlp_forward(n->ws, n->cnd, n->cw.p, n->xin.p, o_rgb, N,
                                     n->num_sms, n->stream, 1);
    k_nerf_sigma<<<(N + 255) / 256, 256, 0, n->stream>>>(n->dens.p, o_sig, N);
    n->launches++;
    if (!dev) {
      CKN(cudaMemcpyAsync(rgb, o_rgb, (size_t)N * 12, cudaMemcpyDeviceToHost,
                          n->stream));
      CKN(cudaMemcpyAsync(sigma, o_sig, (size_t)N * 4, cudaMemcpyDeviceToHost,
                          n->stream));
    }
    CKN(cudaStreamSynchronize(n->stream));
    CKN(cudaGetLastError());
  });
}

tmnn_status tmnn_cuda_nerf_profile(tmnn_nerf *n, float *phase_ms,
                                   uint64_t *launches) {
  if (!n) return TMNN_ERR_NULL_OBJECT;
  if (phase_ms)
    for (int k = 0; k < 4; ++k) phase_ms[k] = n->phase_ms[k];
  if (launches) {
    uint64_t d = 0;
    tmnn_cuda_launch_count(n->density, &d);
    *launches = n->launches + d;
  }
  return TMNN_OK;
}

const char *tmnn_cuda_nerf_last_error(void) { return g_nerf_err.c_str(); }

}  // extern "C"
