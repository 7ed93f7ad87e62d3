// mlp.cu -- standalone FullyFusedMLP inference (no input encoding) through
// the C ABI: the tcnn/tmnn `FullyFusedMLP` module (include/tiny-metal-nn/
// fully_fused_mlp.h) evaluated on fp16 inputs with the same tcgen05 kernel
// as the fused training step, minus the hash-grid gather.
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <string>

#include "../../include/tmnn_cuda.h"
#include "fused.h"
#include "kernels.h"

using namespace tmnn;

struct tmnn_mlp {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  NetDims nd{};
  float *w = nullptr;
  FusedWorkspace ws;
  ~tmnn_mlp() {
    if (stream) cudaStreamSynchronize(stream);
    if (w) cudaFree(w);
    fused_release(ws);
    if (stream) cudaStreamDestroy(stream);
  }
};

namespace tmnn {

// Reference weight layout (mlp_kernel_emitter.cpp:163-191) of a plain MLP
// with nd.In inputs: offsets and the total count.
void mlp_layout(NetDims &nd) {
  int64_t off = 0;
  nd.w_off[0] = off;
  off += (int64_t)nd.In * nd.W;
  nd.b_off[0] = off;
  off += nd.W;
  for (int i = 1; i < nd.H; ++i) {
    nd.w_off[i] = off;
    off += (int64_t)nd.W * nd.W;
    nd.b_off[i] = off;
    off += nd.W;
  }
  nd.w_off[nd.H] = off;
  off += (int64_t)nd.W * nd.O;
  nd.b_off[nd.H] = off;
  off += nd.O;
  nd.mlp_count = (uint32_t)off;
}

// Xavier-uniform weights and U(-1/sqrt(fan_in), ...) biases from the Philox
// stream (the XavierUniform mode of default_trainer.cpp:2090-2096).
void mlp_init_xavier(const NetDims &nd, float *w, uint64_t seed,
                     cudaStream_t st) {
  uint32_t cb = 0;
  for (int layer = 0; layer <= nd.H; ++layer) {
    const int fin = layer == 0 ? nd.In : nd.W;
    const int fout = layer == nd.H ? nd.O : nd.W;
    const uint64_t wc = (uint64_t)fin * fout;
    const float b = std::sqrt(6.0f / (float)(fin + fout));
    launch_init_uniform(w + nd.w_off[layer], wc, -b, b, seed, cb, st);
    cb += (uint32_t)((wc + 3) / 4);
    const float bb = 1.0f / std::sqrt((float)fin);
    launch_init_uniform(w + nd.b_off[layer], (uint64_t)fout, -bb, bb, seed, cb,
                        st);
    cb += (uint32_t)((fout + 3) / 4);
  }
}

}  // namespace tmnn

namespace {
thread_local std::string g_mlp_err;

#define CKM(x)                                                             \
  do {                                                                     \
    cudaError_t e_ = (x);                                                  \
    if (e_ != cudaSuccess)                                                 \
      throw std::runtime_error(std::string(#x) + ": " +                    \
                               cudaGetErrorString(e_));                    \
  } while (0)

template <class F>
tmnn_status run(F &&f) {
  try {
    f();
    return TMNN_OK;
  } catch (const std::invalid_argument &e) {
    g_mlp_err = e.what();
    return TMNN_ERR_INVALID_ARGUMENT;
  } catch (const std::exception &e) {
    g_mlp_err = e.what();
    return TMNN_ERR_OPERATION_FAILED;
  }
}
}  // namespace

extern "C" {

tmnn_status tmnn_cuda_mlp_create(int device, uint32_t n_input, uint32_t width,
                                 uint32_t hidden_layers, uint32_t n_output,
                                 uint64_t seed, tmnn_mlp **out) {
  if (!out) return TMNN_ERR_NULL_OBJECT;
  *out = nullptr;
  tmnn_mlp *m = new tmnn_mlp;
  tmnn_status st = run([&] {
    NetDims &nd = m->nd;
    nd.In = (int)n_input;
    nd.W = (int)width;
    nd.H = (int)hidden_layers;
    nd.O = (int)n_output;
    if (hidden_layers < 1 || hidden_layers > kMaxHidden)
      throw std::invalid_argument("mlp_create: hidden_layers must be in [1, 8]");
    std::string why;
    if (!fused_mlp_supported(nd, &why))
      throw std::invalid_argument("mlp_create: " + why);
    mlp_layout(nd);
    m->device = device;
    CKM(cudaSetDevice(device));
    CKM(cudaDeviceGetAttribute(&m->num_sms, cudaDevAttrMultiProcessorCount, device));
    CKM(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
    CKM(cudaMalloc(&m->w, (size_t)nd.mlp_count * 4));
    mlp_init_xavier(nd, m->w, seed, m->stream);
    CKM(cudaStreamSynchronize(m->stream));
  });
  if (st == TMNN_OK)
    *out = m;
  else
    delete m;
  return st;
}

tmnn_status tmnn_cuda_mlp_destroy(tmnn_mlp *m) {
  if (!m) return TMNN_ERR_NULL_OBJECT;
  return run([&] {
    cudaSetDevice(m->device);
    delete m;
  });
}

tmnn_status tmnn_cuda_mlp_weights(tmnn_mlp *m, const float *host_in, float *host_out,
                                  size_t count) {
  if (!m) return TMNN_ERR_NULL_OBJECT;
  return run([&] {
    if (count != m->nd.mlp_count)
      throw std::invalid_argument("mlp_weights: count mismatch");
    CKM(cudaSetDevice(m->device));
    if (host_in) {
      CKM(cudaMemcpyAsync(m->w, host_in, count * 4, cudaMemcpyHostToDevice,
                          m->stream));
      fused_weights_changed(m->ws);
    }
    if (host_out)
      CKM(cudaMemcpyAsync(host_out, m->w, count * 4, cudaMemcpyDeviceToHost,
                          m->stream));
    CKM(cudaStreamSynchronize(m->stream));
  });
}

tmnn_status tmnn_cuda_mlp_forward(tmnn_mlp *m, const void *input_f16,
                                  float *output, uint32_t n) {
  if (!m) return TMNN_ERR_NULL_OBJECT;
  return run([&] {
    if (n && (!input_f16 || !output))
      throw std::invalid_argument("mlp_forward: null arguments");
    if (((uintptr_t)input_f16 & 15u) != 0)
      throw std::invalid_argument("mlp_forward: input must be 16-byte aligned");
    CKM(cudaSetDevice(m->device));
    fused_mlp_forward(m->ws, m->nd, m->w,
                      static_cast<const __half *>(input_f16), output, n,
                      m->num_sms, m->stream);
    CKM(cudaStreamSynchronize(m->stream));
    CKM(cudaGetLastError());
  });
}

const char *tmnn_cuda_mlp_last_error(void) { return g_mlp_err.c_str(); }

tmnn_status tmnn_cuda_mlp_stream(tmnn_mlp *m, void **stream) {
  if (!m || !stream) return TMNN_ERR_NULL_OBJECT;
  *stream = m->stream;
  return TMNN_OK;
}

}  // extern "C"
