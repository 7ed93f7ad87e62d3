// runtime.cu -- the host runtime behind the C ABI (include/tmnn_cuda.h).
//
// Plays the part of tmnn's DefaultRuntime (src/tiny_metal_nn/runtime/
// default_trainer.cpp:836-2414) and ParameterStore (parameter_store.cpp) on a
// CUDA stream: owns the device parameter store, runs the weight init,
// sequences one training step (Morton sort -> forward/backward/scatter ->
// [NCCL allreduce] -> Adam with gradient reset -> loss read-back), and
// implements the split / accumulation API, evaluation, the optimizer
// checkpoint blob and the network plan.
#include <nccl.h>

#include <atomic>
#include <cctype>
#include <cstdlib>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/tmnn_cuda.h"
#include "fused.h"
#include "kernels.h"
#include "tiled.h"
#include "runtime.h"

using namespace tmnn;

namespace {

thread_local std::string g_last_error;

struct CapacityError : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct ConcurrentCall : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct OperationFailed : std::runtime_error {
  using std::runtime_error::runtime_error;
};

#define CK(x)                                                              \
  do {                                                                     \
    cudaError_t e_ = (x);                                                  \
    if (e_ != cudaSuccess)                                                 \
      throw std::runtime_error(std::string(#x) + ": " +                    \
                               cudaGetErrorString(e_));                    \
  } while (0)
#define NK(x)                                                              \
  do {                                                                     \
    ncclResult_t r_ = (x);                                                 \
    if (r_ != ncclSuccess)                                                 \
      throw std::runtime_error(std::string(#x) + ": " +                    \
                               ncclGetErrorString(r_));                    \
  } while (0)

// The emitter prints BASE/SCALE/huber with std::fixed << setprecision(6)
// (mlp_kernel_emitter.cpp:91-92) and the kernel parses them as float.
float round6(float x) {
  char buf[64];
  std::snprintf(buf, sizeof buf, "%.6f", (double)x);
  return std::strtof(buf, nullptr);
}

template <class T>
struct DevBuf {
  T *p = nullptr;
  size_t n = 0;
  ~DevBuf() { release(); }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
  }
  void alloc(size_t count) {
    release();
    if (count) CK(cudaMalloc(&p, count * sizeof(T)));
    n = count;
  }
  void ensure(size_t count) {
    if (count > n) alloc(count);
  }
  size_t bytes() const { return n * sizeof(T); }
};

// NumericsGuard (src/tiny_metal_nn/runtime/numerics_guard.cpp:12-48): which
// steps the probe records, and the anomaly bookkeeping.
struct NumericsGuard {
  int mode = TMNN_NUMERICS_SAMPLED;
  uint32_t interval = 128;
  uint32_t anomaly_count = 0, last_anomaly_step = 0;
  uint64_t report_count = 0;
  bool should_sample(uint32_t step, bool force) const {
    if (force) return true;
    switch (mode) {
      case TMNN_NUMERICS_DISABLED:
        return false;
      case TMNN_NUMERICS_FULL:
        return true;
      case TMNN_NUMERICS_PERIODIC:
        if (anomaly_count > 0 && step == last_anomaly_step + 1) return true;
        return step != 0 && step % interval == 0;
      default:
        if (step == 0 || step == 1) return true;
        if (anomaly_count > 0 && step == last_anomaly_step + 1) return true;
        return step % interval == 0;
    }
  }
  void record(uint32_t step, bool anomaly) {
    ++report_count;
    if (anomaly) {
      ++anomaly_count;
      last_anomaly_step = step;
    }
  }
};

}  // namespace

struct tmnn_ctx {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  tmnn_spec spec{};
  tmnn_train_cfg cfg{};
  NetDims nd{};
  uint64_t hash_count = 0;
  uint32_t mlp_count = 0;
  uint64_t slots = 0;
  int entry_width = 1;
  int family = TMNN_FAMILY_SAFE_DEBUG;
  int fallback_reason = kReasonNone;
  std::string plan_text;
  bool sparse = true;
  // float gradients of the fused family: a nonzero gradient marks its slot
  // touched, so the kernel stores touched bytes only for zero contributions
  bool implicit_touch = false;
  uint32_t step = 0;
  uint64_t launches = 0;
  std::atomic<bool> busy{false};
  // parameter store
  DevBuf<float> params, m, v;
  DevBuf<__half> table_h;
  DevBuf<int32_t> gh_fixed;
  DevBuf<float> gh_float, gm;
  DevBuf<uint8_t> touched;
  DevBuf<double> loss_acc;  // a StepStats (loss first), see stats()
  DevBuf<float> scratch;
  // enable_probes: statistics of the last forward/backward pass
  DevBuf<float> probe;
  bool probe_ran = false;
  // batch staging
  DevBuf<float> pos_in, tgt_in, pos_s, tgt_s, out_buf, out_s;
  DevBuf<float> grad_out, eg_scratch;  // evaluate_with_gradient
  DevBuf<uint32_t> codes, codes_alt, idx, perm;
  DevBuf<uint8_t> sort_tmp;
  DevBuf<__half> feat;   // Tiled family: encoded features [N x In]
  DevBuf<float> dfeat;   // Tiled family: dL/d(features) [N x In]
  StepStats *h_stats = nullptr;  // pinned copy of the step statistics
  double *h_loss = nullptr;      // &h_stats->loss
  // numerics guard
  NumericsGuard guard;
  uint64_t n_skipped = 0, n_rolled_back = 0, n_safe_recoveries = 0;
  bool safe_family_active = false;
  StepStats *stats() { return reinterpret_cast<StepStats *>(loss_acc.p); }
  cudaEvent_t ev[6] = {};
  // two-lane step ring of the enqueue / finalize API: each lane holds its
  // batch's device copy of the inputs and its pinned step statistics, so the
  // upload of step k+1 overlaps the device work of step k
  struct StepLane {
    DevBuf<float> pos, tgt;
    StepStats *h_stats = nullptr;
    cudaEvent_t copied = nullptr, consumed = nullptr, done = nullptr;
    uint32_t N = 0, step = 0;
    bool used = false;
  };
  StepLane lanes[2];
  int lane_next = 0, lane_oldest = 0, n_pending = 0;
  cudaStream_t copy_stream = nullptr;
  FusedWorkspace fws;
  // data parallelism
  ncclComm_t comm = nullptr;
  // bucketed exchange (Tiled family): the gradient collectives run on
  // comm_stream, one bucket of levels at a time, behind the scatter
  cudaStream_t comm_stream = nullptr;
  // [0] MLP done, [1 + g] bucket g scattered, [kMaxLevels + 1] exchange
  // done (main stream); ev_comm[g] bucket g reduced, ev_comm[kMaxLevels]
  // MLP/loss reduced (comm stream); ev_adam[g] bucket g updated
  cudaEvent_t dp_ev[kMaxLevels + 2] = {};
  cudaEvent_t ev_comm[kMaxLevels + 1] = {};
  cudaEvent_t ev_adam[kMaxLevels + 1] = {};
  int dp_buckets = 4;
  int rank = 0, world = 1;
  // sharded data-parallel optimizer: this rank's copies of the fp32 table
  // outside its shard, and of m and v outside its shard, are out of date
  // until tmnn_cuda_dp_sync_state gathers them
  bool stale = false;
  // level ranges [l0, l1) whose per-rank shards the stale state follows
  std::vector<std::pair<int, int>> stale_layout;
  // sharded update over NVLink peer memory (TMNN_DP_P2P=1, opt-in): the
  // ranks' gradient buffers, fp16 tables and barrier flags mapped into this
  // process; decided once, by all ranks together, at the first bucketed
  // sharded step
  bool p2p_decided = false, p2p = false;
  PeerTable peers{};
  DevBuf<uint32_t> p2p_flags;
  std::vector<void *> p2p_opened;
  uint32_t p2p_epoch = 0;

  float *hash_w() { return params.p; }
  float *mlp_w() { return params.p + hash_count; }
  const float *gather_table() const { return params.p; }
  // the fp16 gather copy the tensor-core families read (null: fp32 table)
  const __half *gather_half() const {
    return spec.table_dtype == TMNN_DTYPE_F16 ? table_h.p : nullptr;
  }
  bool tensor_core_family() const {
    return family == TMNN_FAMILY_FULLY_FUSED || family == TMNN_FAMILY_TILED;
  }
  // the float-format hash gradients (fp32, or fp16 held in the same
  // allocation) from element `off`, their element size and NCCL type
  bool grad_half() const { return nd.grad_half != 0; }
  float *ghf(uint64_t off) {
    if (!gh_float.p) return nullptr;
    return grad_half() ? reinterpret_cast<float *>(
                             reinterpret_cast<__half *>(gh_float.p) + off)
                       : gh_float.p + off;
  }
  size_t gh_elem() const { return grad_half() ? 2 : 4; }
  ncclDataType_t gh_type() const { return grad_half() ? ncclFloat16 : ncclFloat32; }

  ~tmnn_ctx() {
    if (stream) cudaStreamSynchronize(stream);
    if (comm_stream) cudaStreamSynchronize(comm_stream);
    for (void *q : p2p_opened) cudaIpcCloseMemHandle(q);
    if (comm) ncclCommDestroy(comm);
    if (comm_stream) {
      cudaStreamSynchronize(comm_stream);
      cudaStreamDestroy(comm_stream);
    }
    for (auto e : dp_ev)
      if (e) cudaEventDestroy(e);
    for (auto e : ev_comm)
      if (e) cudaEventDestroy(e);
    for (auto e : ev_adam)
      if (e) cudaEventDestroy(e);
    if (h_stats) cudaFreeHost(h_stats);
    for (auto &l : lanes) {
      if (l.h_stats) cudaFreeHost(l.h_stats);
      for (cudaEvent_t e : {l.copied, l.consumed, l.done})
        if (e) cudaEventDestroy(e);
    }
    if (copy_stream) {
      cudaStreamSynchronize(copy_stream);
      cudaStreamDestroy(copy_stream);
    }
    for (auto e : ev)
      if (e) cudaEventDestroy(e);
    fused_release(fws);
    if (stream) cudaStreamDestroy(stream);
  }
};

namespace {

struct BusyGuard {
  tmnn_ctx *c;
  explicit BusyGuard(tmnn_ctx *ctx) : c(ctx) {
    bool expected = false;
    if (!c->busy.compare_exchange_strong(expected, true))
      throw ConcurrentCall(
          "another call is in progress on this context; a context is "
          "single-threaded (use one context per thread)");
  }
  ~BusyGuard() { c->busy.store(false); }
};

template <class F>
tmnn_status guarded(F &&f) {
  try {
    g_last_error.clear();
    f();
    return TMNN_OK;
  } catch (const ConcurrentCall &e) {
    g_last_error = e.what();
    return TMNN_ERR_CONCURRENT_CALL;
  } catch (const CapacityError &e) {
    g_last_error = e.what();
    return TMNN_ERR_CAPACITY;
  } catch (const std::invalid_argument &e) {
    g_last_error = e.what();
    return TMNN_ERR_INVALID_ARGUMENT;
  } catch (const std::exception &e) {
    g_last_error = e.what();
    return TMNN_ERR_OPERATION_FAILED;
  } catch (...) {
    g_last_error = "unknown error";
    return TMNN_ERR_OPERATION_FAILED;
  }
}

#define REQUIRE_CTX(c) \
  if (!(c)) {          \
    g_last_error = "null context"; \
    return TMNN_ERR_NULL_OBJECT;   \
  }

// The numerics-policy environment variables of load_runtime_policy
// (src/tiny_metal_nn/runtime/runtime_policy.h:78-140, :155-161), same
// spellings; an unknown value leaves the default (the reference throws from
// its constructor; here defaults are filled by a function that cannot fail).
bool env_is(const char *v, const char *a) {
  for (; *v && *a; ++v, ++a)
    if (std::tolower((unsigned char)*v) != std::tolower((unsigned char)*a))
      return false;
  return *v == 0 && *a == 0;
}

std::string env_trim(const char *name) {
  const char *v = std::getenv(name);
  if (!v) return {};
  std::string s(v);
  const size_t b = s.find_first_not_of(" \t\n\r");
  const size_t e = s.find_last_not_of(" \t\n\r");
  return b == std::string::npos ? std::string() : s.substr(b, e - b + 1);
}

void apply_policy_env(tmnn_train_cfg &c) {
  std::string v = env_trim("TMNN_NUMERICS_SAMPLING_MODE");
  if (!v.empty()) {
    const char *x = v.c_str();
    if (env_is(x, "sampled") || env_is(x, "default"))
      c.numerics_sampling_mode = TMNN_NUMERICS_SAMPLED;
    else if (env_is(x, "periodic") || env_is(x, "steady-state") ||
             env_is(x, "interval-only"))
      c.numerics_sampling_mode = TMNN_NUMERICS_PERIODIC;
    else if (env_is(x, "full") || env_is(x, "full-per-step"))
      c.numerics_sampling_mode = TMNN_NUMERICS_FULL;
    else if (env_is(x, "disabled") || env_is(x, "off"))
      c.numerics_sampling_mode = TMNN_NUMERICS_DISABLED;
  }
  v = env_trim("TMNN_NUMERICS_SAMPLE_INTERVAL");
  if (!v.empty()) {
    char *end = nullptr;
    const unsigned long n = std::strtoul(v.c_str(), &end, 10);
    if (end != v.c_str() && *end == 0 && n <= 0xFFFFFFFFul)
      c.numerics_sample_interval = (int32_t)(n > 0 ? (n > 0x7FFFFFFF ? 0x7FFFFFFF : n) : 1);
  }
  v = env_trim("TMNN_BAD_STEP_MODE");
  if (!v.empty()) {
    const char *x = v.c_str();
    if (env_is(x, "signal") || env_is(x, "signal-only"))
      c.bad_step_recovery = TMNN_BAD_STEP_SIGNAL_ONLY;
    else if (env_is(x, "throw") || env_is(x, "strict"))
      c.bad_step_recovery = TMNN_BAD_STEP_THROW;
    else if (env_is(x, "skip"))
      c.bad_step_recovery = TMNN_BAD_STEP_SKIP;
    else if (env_is(x, "rollback") || env_is(x, "revert"))
      c.bad_step_recovery = TMNN_BAD_STEP_ROLLBACK;
    else if (env_is(x, "fallback") || env_is(x, "fallback-and-retry") ||
             env_is(x, "fallback-and-retry-with-safe-family") ||
             env_is(x, "safe-family-fallback"))
      c.bad_step_recovery = TMNN_BAD_STEP_SAFE_FAMILY_RETRY;
  }
}

// KernelSpec::validate (kernel_spec.cpp:12-44) plus this build's limits.
void validate(const tmnn_spec &s) {
  auto bad = [](const char *m) { throw std::invalid_argument(m); };
  if (s.hidden_dim <= 0 || s.hidden_dim > 512)
    bad("KernelSpec: hidden_dim must be in (0, 512]");
  if (s.num_hidden_layers < 1 || s.num_hidden_layers > 8)
    bad("KernelSpec: num_hidden_layers must be in [1, 8]");
  if (s.n_levels < 1 || s.n_levels > 32)
    bad("KernelSpec: num_levels must be in [1, 32]");
  if (s.log2_hashmap_size < 10 || s.log2_hashmap_size > 24)
    bad("KernelSpec: log2_hashmap_size must be in [10, 24]");
  if (s.n_features_per_level != 1 && s.n_features_per_level != 2 &&
      s.n_features_per_level != 4)
    bad("KernelSpec: features_per_level must be 1, 2, or 4");
  if (s.spatial_dims != 3 && s.spatial_dims != 4)
    bad("KernelSpec: spatial_dims must be 3 or 4");
  if (s.loss < TMNN_LOSS_L2 || s.loss > TMNN_LOSS_COSINE)
    bad("KernelSpec: invalid loss type");
  if (s.loss == TMNN_LOSS_HUBER && !(s.huber_delta > 0.0f))
    bad("KernelSpec: Huber loss requires huber_delta > 0");
  if (s.loss == TMNN_LOSS_COSINE && s.num_outputs < 2)
    bad("KernelSpec: Cosine loss requires num_outputs >= 2");
  if (s.num_outputs < 1 || s.num_outputs > 64)
    bad("KernelSpec: num_outputs must be in [1, 64]");
  if (!(s.base_resolution > 0.0f) || !(s.per_level_scale > 0.0f))
    bad("KernelSpec: base_resolution and per_level_scale must be positive");
  if (s.table_dtype != TMNN_DTYPE_F32 && s.table_dtype != TMNN_DTYPE_F16)
    bad("tmnn_spec: table_dtype must be F32 or F16");
}

NetDims make_dims(const tmnn_spec &s, const tmnn_train_cfg &c) {
  NetDims nd{};
  nd.L = s.n_levels;
  nd.F = s.n_features_per_level;
  nd.log2T = s.log2_hashmap_size;
  nd.d = s.spatial_dims;
  nd.W = s.hidden_dim;
  nd.H = s.num_hidden_layers;
  nd.O = s.num_outputs;
  nd.In = nd.L * nd.F;
  nd.loss = s.loss;
  nd.huber_delta = round6(s.huber_delta);
  nd.active_levels =
      c.active_levels > 0 && c.active_levels < nd.L ? c.active_levels : nd.L;
  nd.grad_fixed = c.hash_grad_format == TMNN_GRAD_FIXED16 ? 1 : 0;
  nd.grad_half = c.hash_grad_format == TMNN_GRAD_F16 ? 1 : 0;
  nd.T = 1u << nd.log2T;
  nd.hash_count = (uint64_t)nd.L * nd.T * nd.F;
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
  // One fp32 resolution table for every kernel: iterative res *= scale from
  // the 6-decimal literals (mlp_kernel_emitter.cpp:224-236).
  float r = round6(s.base_resolution);
  const float sc = round6(s.per_level_scale);
  for (int l = 0; l < nd.L; ++l) {
    nd.res[l] = r;
    r = r * sc;
  }
  return nd;
}

// NetworkPlanner::plan_with_capabilities (network_planner.cpp:132-290):
// forced families win; Auto takes FullyFused when its kernel supports the
// shape, except that when the table's gather copy plus its fp32 gradients
// take more than a quarter of the L2 the level-major Tiled family is
// selected (the fused kernel's point-major gathers and reductions then
// spill out of L2, or compete for it).  When the
// tensor-core kernels cannot run the shape at all, SafeDebug (fp32 CUDA
// cores) runs it, with the reason recorded and a warning on stderr.
void plan_family(tmnn_ctx &c) {
  std::string why, why_t;
  const bool fused_ok = fused_supported(c.spec, c.cfg, &why);
  const bool tiled_ok = tiled_supported(c.nd, &why_t);
  const int want = c.cfg.family;
  int l2 = 0;
  cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, c.device);
  const uint64_t tbytes = c.spec.table_dtype == TMNN_DTYPE_F16 ? 2 : 4;
  const uint64_t resident = c.nd.hash_count * (tbytes + 4);
  // measured: the level-major family wins once table + gradients take more
  // than a quarter of the L2 (sdf3d, 100 MB: fwd/bwd 0.303 against 0.322 ms)
  // and loses on small tables (image, 8 MB: 0.365 against 0.325 ms)
  const bool overflows_l2 = l2 > 0 && resident > (uint64_t)l2 / 4;
  auto fallback_reason = [](const std::string &w) {
    return w.find("hidden") != std::string::npos   ? kReasonHiddenDimUnsupported
           : w.find("output") != std::string::npos ? kReasonUnsupportedOutputDims
                                                   : kReasonUnsupportedInputDims;
  };
  if (c.cfg.enable_probes) {
    // TrainerConfig::enable_probes disables the reference's SIMD training
    // kernels (include/tiny-metal-nn/trainer.h:51-54): the probes are
    // emitted into its scalar kernel.  The same here: the fp32
    // reference-order kernels carry them.
    c.family = TMNN_FAMILY_SAFE_DEBUG;
    c.fallback_reason = kReasonForcedSafeDebug;
    c.plan_text = "SafeDebug: enable_probes (the probes ride in the fp32 "
                  "reference-order training kernel)";
  } else if (want == TMNN_FAMILY_SAFE_DEBUG) {
    c.family = TMNN_FAMILY_SAFE_DEBUG;
    c.fallback_reason = kReasonForcedSafeDebug;
    c.plan_text = "SafeDebug requested";
  } else if (want == TMNN_FAMILY_TILED) {
    if (!tiled_ok)
      throw std::invalid_argument("Tiled family unavailable: " + why_t);
    c.family = TMNN_FAMILY_TILED;
    c.fallback_reason = kReasonForcedTiled;
    c.plan_text = "Tiled requested: level-major encode, tcgen05 MLP, "
                  "level-major scatter";
  } else if (want == TMNN_FAMILY_FULLY_FUSED) {
    if (!fused_ok)
      throw std::invalid_argument("FullyFused family unavailable: " + why);
    c.family = TMNN_FAMILY_FULLY_FUSED;
    c.fallback_reason = kReasonNone;
    c.plan_text = "FullyFused requested: tcgen05 fused step";
  } else if (fused_ok && tiled_ok && overflows_l2) {
    c.family = TMNN_FAMILY_TILED;
    c.fallback_reason = kReasonNone;
    c.plan_text = "Tiled: gather table + gradients (" +
                  std::to_string(resident >> 20) + " MiB) exceed a quarter "
                  "of the L2 (" + std::to_string((uint64_t)l2 >> 20) +
                  " MiB): level-major encode and scatter";
  } else if (fused_ok) {
    c.family = TMNN_FAMILY_FULLY_FUSED;
    c.fallback_reason = kReasonNone;
    c.plan_text = "FullyFused: tcgen05 fused step";
  } else {
    c.family = TMNN_FAMILY_SAFE_DEBUG;
    c.fallback_reason = fallback_reason(why);
    c.plan_text = "SafeDebug fallback (fp32 CUDA cores, no tensor cores): " + why;
    std::fprintf(stderr,
                 "tmnn: warning: this network shape leaves the tensor-core "
                 "path (%s); training runs on the fp32 SafeDebug kernels\n",
                 why.c_str());
  }
}

float kaiming_gain(const tmnn_train_cfg &c) {
  // default_trainer.cpp:2037-2049
  switch (c.mlp_nonlinearity) {
    case 0:
    case 4:
      return 1.0f;
    case 2:
      return std::sqrt(2.0f / (1.0f + c.mlp_kaiming_a * c.mlp_kaiming_a));
    case 3:
      return 5.0f / 3.0f;
    default:
      return std::sqrt(2.0f);
  }
}

// Philox weight init (default_trainer.cpp:1978-2180): hash U(-r, r) at
// counter 0; the MLP per layer, weights then bias, each slice advancing the
// counter by ceil(count / 4).
void init_weights(tmnn_ctx &c) {
  const tmnn_train_cfg &w = c.cfg;
  cudaStream_t st = c.stream;
  if (w.hash_init == 1)
    CK(cudaMemsetAsync(c.hash_w(), 0, c.hash_count * sizeof(float), st));
  else
    launch_init_uniform(c.hash_w(), c.hash_count, -w.hash_init_range,
                        w.hash_init_range, w.seed, 0u, st);
  c.launches++;
  uint32_t cb = (uint32_t)((c.hash_count + 3) / 4);
  float *mlp = c.mlp_w();
  if (w.mlp_init == 4 || w.mlp_init == 5 || w.mlp_init == 6) {
    if (w.mlp_init == 4)
      launch_init_uniform(mlp, c.mlp_count, -w.mlp_uniform_range,
                          w.mlp_uniform_range, w.seed, cb, st);
    else if (w.mlp_init == 5)
      launch_init_normal(mlp, c.mlp_count, 0.0f, w.mlp_normal_stddev, w.seed,
                         cb, st);
    else
      CK(cudaMemsetAsync(mlp, 0, c.mlp_count * sizeof(float), st));
    c.launches++;
    return;
  }
  const float gain = kaiming_gain(w);
  const NetDims &nd = c.nd;
  int64_t off = 0;
  for (int layer = 0; layer <= nd.H; ++layer) {
    const int fin = layer == 0 ? nd.In : nd.W;
    const int fout = layer == nd.H ? nd.O : nd.W;
    const uint64_t wc = (uint64_t)fin * fout;
    const float fi = (float)fin, fo = (float)fout;
    switch (w.mlp_init) {
      case 0: {
        const float b = gain * std::sqrt(3.0f / fi);
        launch_init_uniform(mlp + off, wc, -b, b, w.seed, cb, st);
        break;
      }
      case 1:
        launch_init_normal(mlp + off, wc, 0.0f, gain / std::sqrt(fi), w.seed,
                           cb, st);
        break;
      case 2: {
        const float b = std::sqrt(6.0f / (fi + fo));
        launch_init_uniform(mlp + off, wc, -b, b, w.seed, cb, st);
        break;
      }
      default:
        launch_init_normal(mlp + off, wc, 0.0f, std::sqrt(2.0f / (fi + fo)),
                           w.seed, cb, st);
    }
    cb += (uint32_t)((wc + 3) / 4);
    off += (int64_t)wc;
    const float bb = 1.0f / std::sqrt(fi);
    launch_init_uniform(mlp + off, (uint64_t)fout, -bb, bb, w.seed, cb, st);
    cb += (uint32_t)((fout + 3) / 4);
    off += fout;
    c.launches += 2;
  }
}

void refresh_gather_copy(tmnn_ctx &c) {
  if (c.table_h.p) {
    launch_to_half(c.hash_w(), c.table_h.p, c.hash_count, c.num_sms, c.stream);
    c.launches++;
  }
  fused_weights_changed(c.fws);
}

void zero_grads(tmnn_ctx &c) {
  if (c.gh_fixed.p)
    CK(cudaMemsetAsync(c.gh_fixed.p, 0, c.gh_fixed.bytes(), c.stream));
  if (c.gh_float.p)
    CK(cudaMemsetAsync(c.gh_float.p, 0, c.gh_float.bytes(), c.stream));
  CK(cudaMemsetAsync(c.gm.p, 0, c.gm.bytes(), c.stream));
  CK(cudaMemsetAsync(c.touched.p, 0, c.touched.bytes(), c.stream));
}

void reset_optimizer(tmnn_ctx &c) {
  CK(cudaMemsetAsync(c.m.p, 0, c.m.bytes(), c.stream));
  CK(cudaMemsetAsync(c.v.p, 0, c.v.bytes(), c.stream));
  c.step = 0;
}

void ensure_batch(tmnn_ctx &c, uint32_t N) {
  const size_t d = c.nd.d, O = c.nd.O;
  if (c.family == TMNN_FAMILY_TILED) {
    c.feat.ensure((size_t)N * c.nd.In);
    c.dfeat.ensure((size_t)N * c.nd.In);
  }
  c.pos_in.ensure(N * d);
  c.tgt_in.ensure(N * O);
  c.pos_s.ensure(N * d);
  c.tgt_s.ensure(N * O);
  c.out_buf.ensure(N * O);
  c.out_s.ensure(N * O);
  c.codes.ensure(N);
  c.codes_alt.ensure(N);
  c.idx.ensure(N);
  c.perm.ensure(N);
  const size_t tb = morton_temp_bytes(N);
  c.sort_tmp.ensure(tb);
}

// Copies a caller array of `count` floats into `staging` (host pointer) or
// passes a device pointer through.
const float *stage_in(tmnn_ctx &c, const float *src, size_t count,
                      DevBuf<float> &staging, uint32_t flags) {
  if (!src) return nullptr;
  if (flags & TMNN_PTR_DEVICE) return src;
  if (count)
    CK(cudaMemcpyAsync(staging.p, src, count * sizeof(float),
                       cudaMemcpyHostToDevice, c.stream));
  return staging.p;
}

// Morton order of the batch (morton_sort.h:60-110) on the device: codes,
// stable sort (counting sort for short keys, which also moves the rows),
// then row gathers of positions and the per-point array where needed.
void morton_sort(tmnn_ctx &c, const float *pos, const float *per_point,
                 uint32_t N, const float **pos_out, const float **pp_out) {
  bool gathered = false;
  launch_morton_order(pos, c.nd.d, N, c.codes.p, c.codes_alt.p, c.idx.p,
                      c.perm.p, c.sort_tmp.p, c.sort_tmp.n, c.stream,
                      c.cfg.morton_key_bits, c.pos_s.p, per_point, c.nd.O,
                      per_point ? c.tgt_s.p : nullptr, &gathered);
  c.launches += 3;
  *pos_out = c.pos_s.p;
  if (!gathered) {
    launch_gather_rows(pos, c.nd.d, c.perm.p, c.pos_s.p, N, c.stream);
    c.launches++;
  }
  if (per_point) {
    if (!gathered) {
      launch_gather_rows(per_point, c.nd.O, c.perm.p, c.tgt_s.p, N, c.stream);
      c.launches++;
    }
    *pp_out = c.tgt_s.p;
  }
}

// Forward + backward + scatter of one batch with the context's family.
void fwd_bwd(tmnn_ctx &c, const float *pos, const float *tgt,
             const float *dext, uint32_t N, float inv_N) {
  if (N == 0) return;
  if (c.family == TMNN_FAMILY_FULLY_FUSED) {
    c.launches += fused_train(c.fws, c.nd, c.spec, c.params.p, c.table_h.p,
                              pos, tgt, dext, inv_N, c.gm.p, c.gh_fixed.p,
                              c.gh_float.p, c.touched.p, c.loss_acc.p, N,
                              c.num_sms, c.stream, c.implicit_touch);
    return;
  }
  if (c.family == TMNN_FAMILY_TILED) {
    c.launches += tiled_train(c.fws, c.nd, c.params.p, c.gather_half(), pos,
                              tgt, dext, inv_N, c.gm.p, c.gh_fixed.p,
                              c.gh_float.p, c.touched.p, c.loss_acc.p,
                              c.feat.p, c.dfeat.p, N, c.num_sms, c.stream,
                              c.implicit_touch);
    return;
  }
  ProbeAcc *pa = nullptr;
  if (c.cfg.enable_probes) {
    pa = reinterpret_cast<ProbeAcc *>(c.probe.p);
    CK(cudaMemsetAsync(pa, 0, sizeof(ProbeAcc), c.stream));
    c.probe_ran = true;
  }
  launch_train_exact(c.nd, c.hash_w(), c.mlp_w(), pos, tgt, dext, inv_N,
                     c.gm.p, c.gh_fixed.p, c.gh_float.p, c.touched.p,
                     c.loss_acc.p, N, c.scratch.p, c.num_sms, c.stream, pa);
  c.launches++;
}

void forward_dev(tmnn_ctx &c, const float *pos, float *out, uint32_t N) {
  if (N == 0) return;
  if (c.family == TMNN_FAMILY_FULLY_FUSED) {
    c.launches += fused_forward(c.fws, c.nd, c.spec, c.params.p, c.table_h.p,
                                pos, out, N, c.num_sms, c.stream);
    return;
  }
  if (c.family == TMNN_FAMILY_TILED) {
    c.launches += tiled_forward(c.fws, c.nd, c.params.p, c.gather_half(), pos,
                                out, c.feat.p, N, c.num_sms, c.stream);
    return;
  }
  launch_forward_exact(c.nd, c.hash_w(), c.mlp_w(), pos, out, N, c.scratch.p,
                       c.num_sms, c.stream);
  c.launches++;
}

void allreduce_grads(tmnn_ctx &c, bool with_loss) {
  if (!c.comm || c.world <= 1) return;
  NK(ncclGroupStart());
  if (c.nd.grad_fixed)
    NK(ncclAllReduce(c.gh_fixed.p, c.gh_fixed.p, c.hash_count, ncclInt32,
                     ncclSum, c.comm, c.stream));
  else
    NK(ncclAllReduce(c.gh_float.p, c.gh_float.p, c.hash_count, c.gh_type(),
                     ncclSum, c.comm, c.stream));
  NK(ncclAllReduce(c.gm.p, c.gm.p, c.mlp_count, ncclFloat32, ncclSum, c.comm,
                   c.stream));
  if (c.sparse && !c.implicit_touch)  // implicit: the gradient sum decides
    NK(ncclAllReduce(c.touched.p, c.touched.p, c.slots, ncclUint8, ncclMax,
                     c.comm, c.stream));
  if (with_loss)
    NK(ncclAllReduce(c.loss_acc.p, c.loss_acc.p, 1, ncclFloat64, ncclSum,
                     c.comm, c.stream));
  NK(ncclGroupEnd());
}

// Adam over the fused [hash | mlp] buffer with the reference's bias
// corrections bc_k = 1 - pow(beta_k, step + 1) in float (adam_params.h:33-52),
// then the gradient reset; advances the step counter.
AdamArgs adam_args(const tmnn_ctx &c) {
  AdamArgs a{};
  const float s = (float)(c.step + 1u);
  a.lr_hash = c.cfg.lr_encoding;
  a.lr_mlp = c.cfg.lr_network;
  a.beta1 = c.cfg.beta1;
  a.beta2 = c.cfg.beta2;
  a.eps = c.cfg.epsilon;
  a.bc1 = 1.0f - std::pow(c.cfg.beta1, s);
  a.bc2 = 1.0f - std::pow(c.cfg.beta2, s);
  a.l1_hash = c.cfg.l1_reg;
  a.l2_mlp = c.cfg.l2_reg;
  a.grad_clip = c.cfg.grad_clip;
  a.weight_decay = c.cfg.weight_decay;
  a.hash_count = c.hash_count;
  a.mlp_count = c.mlp_count;
  a.slots = c.slots;
  a.entry_width = c.entry_width;
  a.sparse = c.sparse ? 1 : 0;
  a.grad_fixed = c.nd.grad_fixed;
  a.grad_half = c.nd.grad_half;
  a.implicit_touch = c.implicit_touch ? 1 : 0;
  return a;
}

// Launches the numerics probe over the (reduced) gradients of this rank's
// parameters, before Adam; see k_numerics_probe.
void probe_numerics(tmnn_ctx &c, bool force, bool gate) {
  launch_numerics_probe(adam_args(c), c.params.p, c.m.p, c.v.p, c.gh_fixed.p,
                        c.gh_float.p, c.gm.p, c.hash_count, c.stats(),
                        force ? 1 : 0, gate ? 1 : 0, c.num_sms, c.stream);
  c.launches++;
}

void adam(tmnn_ctx &c, const StepStats *guard = nullptr) {
  AdamArgs a = adam_args(c);
  a.guard = guard;
  launch_adam(a, c.params.p, c.m.p, c.v.p, c.gh_fixed.p, c.gh_float.p, c.gm.p,
              c.touched.p, c.table_h.p, c.num_sms, c.stream);
  c.launches += 1;
  fused_weights_changed(c.fws);
  if (!c.sparse)  // the dense path leaves the touched map unused
    CK(cudaMemsetAsync(c.touched.p, 0, c.touched.bytes(), c.stream));
  c.step++;
}

// Data-parallel update with the optimizer sharded over the ranks (ZeRO-1
// style): reduce-scatter the hash gradients and touched map so each rank
// owns 1/world of the table, Adam on that shard only (MLP replicated after an
// allreduce), then all-gather the updated fp32 table.  Same bytes on NVLink
// as one allreduce, 1/world of the table's Adam work per rank.
bool can_shard(const tmnn_ctx &c) {
  // at 2 ranks the extra memsets and fp16 refresh cost more than the halved
  // Adam saves (measured); from 4 ranks on the sharded update is cheaper
  return c.comm && c.cfg.dp_replicated_optimizer <= 0 &&
         (c.world >= 4 || (c.world >= 2 && c.cfg.dp_replicated_optimizer < 0)) &&
         c.hash_count % (4ull * (uint64_t)c.world) == 0 &&
         c.slots % (uint64_t)c.world == 0;
}

// ---- bucketed data-parallel exchange (Tiled family) ----------------------
//
// The Tiled family scatters the hash gradients level by level, so a group
// of levels is final while later levels are still being scattered.  The
// step then runs its collectives on a second stream, bucket by bucket: the
// MLP gradients and the loss as soon as the MLP kernel is done, each
// bucket's reduce-scatter (sharded optimizer) or allreduce right after that
// bucket's scatter launch.  The exchange overlaps the scatter of the later
// buckets instead of following the whole backward pass.
struct Bucket {
  int l0, l1;      // levels
  uint64_t e0, n;  // table elements of the levels
};

std::vector<Bucket> dp_bucket_list(const tmnn_ctx &c) {
  const int L = c.nd.L;
  int G = c.dp_buckets < 1 ? 1 : (c.dp_buckets > L ? L : c.dp_buckets);
  std::vector<Bucket> b;
  const uint64_t per = (uint64_t)c.nd.T * c.nd.F;
  for (int g = 0; g < G; ++g) {
    const int l0 = g * L / G, l1 = (g + 1) * L / G;
    if (l1 > l0) b.push_back({l0, l1, per * l0, per * (uint64_t)(l1 - l0)});
  }
  return b;
}

bool can_overlap(const tmnn_ctx &c) {
  return c.comm && c.world > 1 && c.comm_stream &&
         c.family == TMNN_FAMILY_TILED && c.dp_buckets > 1;
}

// Every bucket splits evenly into groups of four elements per rank (the
// sharded Adam works on groups of four) and into whole tracked slots.
bool buckets_shardable(const tmnn_ctx &c, const std::vector<Bucket> &bs) {
  if (!can_shard(c)) return false;
  for (const Bucket &b : bs)
    if (b.n % (4ull * (uint64_t)c.world) != 0 ||
        (b.n / c.entry_width) % (uint64_t)c.world != 0 ||
        b.e0 % (uint64_t)c.entry_width != 0)
      return false;
  return true;
}

// Whether every rank can run the sharded update over peer memory, decided
// once by all ranks together (two tiny allreduces, so that no rank takes
// the peer path alone): requested by TMNN_DP_P2P=1 (on every rank), float
// gradients with implicit touch marks, an fp16 gather table, at most
// kMaxPeers ranks, and the CUDA IPC mapping of every rank's gradient
// buffer, fp16 table and barrier flags succeeding everywhere.
int p2p_vote(tmnn_ctx &c, int mine) {
  DevBuf<int32_t> v;
  v.alloc(1);
  CK(cudaMemcpyAsync(v.p, &mine, sizeof(int), cudaMemcpyHostToDevice, c.stream));
  NK(ncclAllReduce(v.p, v.p, 1, ncclInt32, ncclMin, c.comm, c.stream));
  int all = 0;
  CK(cudaMemcpyAsync(&all, v.p, sizeof(int), cudaMemcpyDeviceToHost, c.stream));
  CK(cudaStreamSynchronize(c.stream));
  return all;
}

bool p2p_requested() {
  const char *e = std::getenv("TMNN_DP_P2P");
  return e && e[0] == '1';
}

// Every rank must set TMNN_DP_P2P alike: the vote below is a collective.
void p2p_setup(tmnn_ctx &c) {
  c.p2p = false;
  const int want = c.world <= kMaxPeers && c.gh_float.p &&
                   c.gather_half() && c.sparse && c.implicit_touch &&
                   !c.gh_fixed.p;
  if (!p2p_vote(c, want)) return;
  struct Handles { cudaIpcMemHandle_t grad, half, flags; };
  int ok = 1;
  Handles mine{};
  c.p2p_flags.alloc(kMaxPeers);
  CK(cudaMemsetAsync(c.p2p_flags.p, 0, c.p2p_flags.bytes(), c.stream));
  ok = cudaIpcGetMemHandle(&mine.grad, c.gh_float.p) == cudaSuccess &&
       cudaIpcGetMemHandle(&mine.half, c.table_h.p) == cudaSuccess &&
       cudaIpcGetMemHandle(&mine.flags, c.p2p_flags.p) == cudaSuccess;
  cudaGetLastError();
  std::vector<Handles> all(c.world);
  DevBuf<uint8_t> buf;
  buf.alloc(sizeof(Handles) * c.world);
  CK(cudaMemcpyAsync(buf.p + sizeof(Handles) * c.rank, &mine, sizeof(Handles),
                     cudaMemcpyHostToDevice, c.stream));
  NK(ncclAllGather(buf.p + sizeof(Handles) * c.rank, buf.p, sizeof(Handles),
                   ncclChar, c.comm, c.stream));
  CK(cudaMemcpyAsync(all.data(), buf.p, buf.bytes(), cudaMemcpyDeviceToHost,
                     c.stream));
  CK(cudaStreamSynchronize(c.stream));
  PeerTable pt{};
  for (int r = 0; r < c.world && ok; ++r) {
    if (r == c.rank) {
      pt.grad[r] = c.gh_float.p;
      pt.table_h[r] = c.table_h.p;
      pt.flags[r] = c.p2p_flags.p;
      continue;
    }
    void *g = nullptr, *h = nullptr, *f = nullptr;
    ok = cudaIpcOpenMemHandle(&g, all[r].grad, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
    if (g) c.p2p_opened.push_back(g);
    ok = ok && cudaIpcOpenMemHandle(&h, all[r].half, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
    if (h) c.p2p_opened.push_back(h);
    ok = ok && cudaIpcOpenMemHandle(&f, all[r].flags, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
    if (f) c.p2p_opened.push_back(f);
    pt.grad[r] = g;
    pt.table_h[r] = static_cast<__half *>(h);
    pt.flags[r] = static_cast<uint32_t *>(f);
  }
  cudaGetLastError();
  if (!p2p_vote(c, ok ? 1 : 0)) {
    for (void *q : c.p2p_opened) cudaIpcCloseMemHandle(q);
    c.p2p_opened.clear();
    c.p2p_flags.release();
    return;
  }
  c.peers = pt;
  c.p2p_epoch = 0;
  c.p2p = true;
  // first, so that the plan's 128-character reason field keeps it
  c.plan_text = "peer-memory sharded update; " + c.plan_text;
}

// One data-parallel training pass of the Tiled family, pipelined per bucket
// of levels over two streams:
//
//   main:  encode, MLP | scatter b0 | scatter b1 | ... | Adam MLP |
//          Adam b0 | Adam b1 | ...
//   comm:  MLP + loss allreduce | reduce b0 | reduce b1 | ... |
//          all-gather b0 | all-gather b1 | ...
//
// Bucket g's reduction (a reduce-scatter with the sharded optimizer, else an
// allreduce) starts when its scatter is done and overlaps the later
// buckets' scatter; its Adam starts when its reduction is done, and (sharded)
// its all-gather when its Adam is done.  The main stream joins the comm
// stream at the end, so the next step sees a complete table.
void step_overlapped(tmnn_ctx &c, const float *pos, const float *tgt,
                     uint32_t N, float inv_N, bool shard, bool gate,
                     const std::vector<Bucket> &bs, bool prof) {
  const NetDims &nd = c.nd;
  const bool fixed = nd.grad_fixed != 0;
  const bool exch_touched = c.sparse && !c.implicit_touch;
  const uint64_t w = (uint64_t)c.entry_width;
  cudaStream_t cs = c.comm_stream;
  if (shard && !c.p2p_decided) {
    // only a process that asks for the peer path votes: without the
    // variable the step runs no extra collective
    c.p2p_decided = true;
    if (p2p_requested()) p2p_setup(c);
  }
  // peer path: bucket g's sum + Adam + fp16 copy to every rank in one
  // kernel on the comm stream right after its scatter, then the reset of
  // the bucket's gradients once every rank has read them
  const bool peer = shard && c.p2p;
  c.launches += tiled_encode(nd, c.params.p, c.gather_half(), pos, c.feat.p, N,
                             c.stream);
  c.launches += fused_mlp_train(c.fws, nd, c.mlp_w(), c.feat.p, tgt, nullptr,
                                inv_N, c.gm.p, c.loss_acc.p, c.dfeat.p, N,
                                c.num_sms, c.stream, 0);
  CK(cudaEventRecord(c.dp_ev[0], c.stream));
  CK(cudaStreamWaitEvent(cs, c.dp_ev[0], 0));
  NK(ncclGroupStart());
  NK(ncclAllReduce(c.gm.p, c.gm.p, c.mlp_count, ncclFloat32, ncclSum, c.comm, cs));
  NK(ncclAllReduce(c.loss_acc.p, c.loss_acc.p, 1, ncclFloat64, ncclSum, c.comm, cs));
  NK(ncclGroupEnd());
  CK(cudaEventRecord(c.ev_comm[kMaxLevels], cs));
  for (size_t g = 0; g < bs.size(); ++g) {
    const Bucket &b = bs[g];
    c.launches += tiled_scatter(nd, pos, c.dfeat.p, c.gh_fixed.p, c.gh_float.p,
                                c.touched.p, N, c.implicit_touch, c.stream,
                                b.l0, b.l1);
    CK(cudaEventRecord(c.dp_ev[1 + g], c.stream));
    CK(cudaStreamWaitEvent(cs, c.dp_ev[1 + g], 0));
    if (peer) {
      const uint64_t gs = b.n / c.world;
      AdamArgs ah = adam_args(c);
      ah.hash_count = gs;
      ah.slots = gs / w;
      ah.mlp_count = 0;
      c.launches += launch_peer_exchange(ah, c.peers, c.rank, c.world,
                                         b.e0 + gs * c.rank, c.params.p, c.m.p,
                                         c.v.p, c.p2p_epoch,
                                         &c.stats()->exchange_err, c.num_sms, cs);
      CK(cudaMemsetAsync(c.ghf(b.e0), 0, b.n * c.gh_elem(), cs));
      CK(cudaEventRecord(c.ev_comm[g], cs));
      continue;
    }
    NK(ncclGroupStart());
    if (shard) {
      const uint64_t gs = b.n / c.world, own = b.e0 + gs * c.rank;
      if (fixed)
        NK(ncclReduceScatter(c.gh_fixed.p + b.e0, c.gh_fixed.p + own, gs,
                             ncclInt32, ncclSum, c.comm, cs));
      else
        NK(ncclReduceScatter(c.ghf(b.e0), c.ghf(own), gs,
                             c.gh_type(), ncclSum, c.comm, cs));
      if (exch_touched)
        NK(ncclReduceScatter(c.touched.p + b.e0 / w, c.touched.p + own / w,
                             gs / w, ncclUint8, ncclMax, c.comm, cs));
    } else {
      if (fixed)
        NK(ncclAllReduce(c.gh_fixed.p + b.e0, c.gh_fixed.p + b.e0, b.n,
                         ncclInt32, ncclSum, c.comm, cs));
      else
        NK(ncclAllReduce(c.ghf(b.e0), c.ghf(b.e0), b.n,
                         c.gh_type(), ncclSum, c.comm, cs));
      if (exch_touched)
        NK(ncclAllReduce(c.touched.p + b.e0 / w, c.touched.p + b.e0 / w,
                         b.n / w, ncclUint8, ncclMax, c.comm, cs));
    }
    NK(ncclGroupEnd());
    CK(cudaEventRecord(c.ev_comm[g], cs));
  }
  if (prof) CK(cudaEventRecord(c.ev[2], c.stream));
  // MLP update (and, replicated, the unforced numerics check of the loss)
  CK(cudaStreamWaitEvent(c.stream, c.ev_comm[kMaxLevels], 0));
  AdamArgs a = adam_args(c);
  if (!shard) {
    probe_numerics(c, false, gate);
    a.guard = c.stats();
  }
  launch_adam_mlp(a, c.params.p, c.m.p, c.v.p, c.gm.p, c.num_sms, c.stream);
  c.launches++;
  const bool half = c.tensor_core_family() && c.table_h.p;
  const bool per_bucket_gather =
      bs[0].n * (half ? 2 : 4) >= (32ull << 20);  // bytes of a bucket's table
  for (size_t g = 0; g < bs.size() && !peer; ++g) {
    const Bucket &b = bs[g];
    CK(cudaStreamWaitEvent(c.stream, c.ev_comm[g], 0));
    if (prof && g + 1 == bs.size()) CK(cudaEventRecord(c.ev[3], c.stream));
    const uint64_t gs = shard ? b.n / c.world : b.n;
    const uint64_t off = shard ? b.e0 + gs * c.rank : b.e0;
    AdamArgs ah = a;
    ah.hash_count = gs;
    ah.slots = gs / w;
    ah.mlp_count = 0;
    launch_adam(ah, c.params.p + off, c.m.p + off, c.v.p + off,
                c.gh_fixed.p ? c.gh_fixed.p + off : nullptr,
                c.ghf(off), c.gm.p,
                c.touched.p + off / w, c.table_h.p ? c.table_h.p + off : nullptr,
                c.num_sms, c.stream);
    c.launches++;
    if (shard) {
      // the bucket's other ranks' partial sums (outside this rank's shard)
      if (c.gh_fixed.p)
        CK(cudaMemsetAsync(c.gh_fixed.p + b.e0, 0, b.n * 4, c.stream));
      if (c.gh_float.p)
        CK(cudaMemsetAsync(c.ghf(b.e0), 0, b.n * c.gh_elem(), c.stream));
      CK(cudaMemsetAsync(c.touched.p + b.e0 / w, 0, b.n / w, c.stream));
      // large buckets gather as soon as their Adam is done (overlapping the
      // next bucket's Adam); small ones in one grouped call at the end
      if (per_bucket_gather || g + 1 == bs.size()) {
        CK(cudaEventRecord(c.ev_adam[g], c.stream));
        CK(cudaStreamWaitEvent(cs, c.ev_adam[g], 0));
        NK(ncclGroupStart());
        for (size_t q = per_bucket_gather ? g : 0; q <= g; ++q) {
          const uint64_t qs = bs[q].n / c.world, qo = bs[q].e0 + qs * c.rank;
          if (half)
            NK(ncclAllGather(c.table_h.p + qo, c.table_h.p + bs[q].e0, qs,
                             ncclHalf, c.comm, cs));
          else
            NK(ncclAllGather(c.params.p + qo, c.params.p + bs[q].e0, qs,
                             ncclFloat32, c.comm, cs));
        }
        NK(ncclGroupEnd());
      }
    } else if (!c.sparse) {
      CK(cudaMemsetAsync(c.touched.p + b.e0 / w, 0, b.n / w, c.stream));
    }
  }
  if (shard) {
    CK(cudaEventRecord(c.dp_ev[kMaxLevels + 1], cs));
    CK(cudaStreamWaitEvent(c.stream, c.dp_ev[kMaxLevels + 1], 0));
    if (!half && c.table_h.p) {
      launch_to_half(c.params.p, c.table_h.p, c.hash_count, c.num_sms, c.stream);
      c.launches++;
    }
    c.stale = true;
    c.stale_layout.clear();
    for (const Bucket &b : bs) c.stale_layout.push_back({b.l0, b.l1});
  }
  fused_weights_changed(c.fws);
  c.step++;
}

// Sharded update after a bucketed reduce-scatter: Adam on this rank's
// shard of every bucket (and on the replicated MLP), reset of the whole
// local gradient buffer, all-gather of the updated table per bucket (the
// fp16 gather copy the tensor-core kernels read, else the fp32 table).
void dp_finish_sharded(tmnn_ctx &c, const std::vector<Bucket> &bs,
                       const StepStats *guard = nullptr) {
  AdamArgs a = adam_args(c);
  a.guard = guard;
  const uint64_t w = (uint64_t)c.entry_width;
  for (const Bucket &b : bs) {
    const uint64_t gs = b.n / c.world, off = b.e0 + gs * c.rank;
    AdamArgs ah = a;
    ah.hash_count = gs;
    ah.slots = gs / w;
    ah.mlp_count = 0;
    launch_adam(ah, c.params.p + off, c.m.p + off, c.v.p + off,
                c.gh_fixed.p ? c.gh_fixed.p + off : nullptr,
                c.ghf(off), c.gm.p,
                c.touched.p + off / w, c.table_h.p ? c.table_h.p + off : nullptr,
                c.num_sms, c.stream);
    c.launches++;
  }
  launch_adam_mlp(a, c.params.p, c.m.p, c.v.p, c.gm.p, c.num_sms, c.stream);
  c.launches++;
  if (c.gh_fixed.p)
    CK(cudaMemsetAsync(c.gh_fixed.p, 0, c.gh_fixed.bytes(), c.stream));
  if (c.gh_float.p)
    CK(cudaMemsetAsync(c.gh_float.p, 0, c.gh_float.bytes(), c.stream));
  CK(cudaMemsetAsync(c.touched.p, 0, c.touched.bytes(), c.stream));
  const bool half = c.tensor_core_family() && c.table_h.p;
  NK(ncclGroupStart());
  for (const Bucket &b : bs) {
    const uint64_t gs = b.n / c.world, off = b.e0 + gs * c.rank;
    if (half)
      NK(ncclAllGather(c.table_h.p + off, c.table_h.p + b.e0, gs, ncclHalf,
                       c.comm, c.stream));
    else
      NK(ncclAllGather(c.params.p + off, c.params.p + b.e0, gs, ncclFloat32,
                       c.comm, c.stream));
  }
  NK(ncclGroupEnd());
  if (!half && c.table_h.p) {
    launch_to_half(c.params.p, c.table_h.p, c.hash_count, c.num_sms, c.stream);
    c.launches++;
  }
  c.stale = true;
  c.stale_layout.clear();
  for (const Bucket &b : bs) c.stale_layout.push_back({b.l0, b.l1});
  fused_weights_changed(c.fws);
  c.step++;
}

// The shards of the sharded optimizer: per bucket of levels when the Tiled
// family exchanges bucket by bucket, else one range over the whole table.
std::vector<Bucket> shard_layout(const tmnn_ctx &c) {
  if (c.family == TMNN_FAMILY_TILED && c.dp_buckets > 1) {
    std::vector<Bucket> bs = dp_bucket_list(c);
    if (bs.size() > 1 && buckets_shardable(c, bs)) return bs;
  }
  return {Bucket{0, c.nd.L, 0, c.hash_count}};
}

bool layout_is(const tmnn_ctx &c, const std::vector<Bucket> &bs) {
  if (c.stale_layout.size() != bs.size()) return false;
  for (size_t i = 0; i < bs.size(); ++i)
    if (c.stale_layout[i].first != bs[i].l0 || c.stale_layout[i].second != bs[i].l1)
      return false;
  return true;
}

void dp_sync_state(tmnn_ctx &c);

// Data-parallel update with the optimizer sharded over the ranks (ZeRO-1
// style): reduce-scatter the hash gradients and touched map so each rank
// owns 1/world of every shard range, Adam on those shards only (MLP
// replicated after an allreduce), then all-gather the updated table.  Same
// bytes on NVLink as one allreduce, 1/world of the table's Adam work per
// rank.  With `probe` the numerics probe scans this rank's shards and the
// ranks combine its results, so every rank takes the same decision.
void dp_update(tmnn_ctx &c, bool with_loss, cudaEvent_t after_comm,
               bool probe = false, bool gate = false) {
  const std::vector<Bucket> bs = shard_layout(c);
  if (c.stale && !layout_is(c, bs)) dp_sync_state(c);
  const uint64_t w = (uint64_t)c.entry_width;
  NK(ncclGroupStart());
  for (const Bucket &b : bs) {
    const uint64_t gs = b.n / c.world, own = b.e0 + gs * c.rank;
    if (c.nd.grad_fixed)
      NK(ncclReduceScatter(c.gh_fixed.p + b.e0, c.gh_fixed.p + own, gs,
                           ncclInt32, ncclSum, c.comm, c.stream));
    else
      NK(ncclReduceScatter(c.ghf(b.e0), c.ghf(own), gs,
                           c.gh_type(), ncclSum, c.comm, c.stream));
    if (c.sparse && !c.implicit_touch)
      NK(ncclReduceScatter(c.touched.p + b.e0 / w, c.touched.p + own / w,
                           gs / w, ncclUint8, ncclMax, c.comm, c.stream));
  }
  NK(ncclAllReduce(c.gm.p, c.gm.p, c.mlp_count, ncclFloat32, ncclSum, c.comm,
                   c.stream));
  if (with_loss)
    NK(ncclAllReduce(c.loss_acc.p, c.loss_acc.p, 1, ncclFloat64, ncclSum,
                     c.comm, c.stream));
  NK(ncclGroupEnd());
  if (after_comm) CK(cudaEventRecord(after_comm, c.stream));
  const StepStats *guard = nullptr;
  if (probe) {
    AdamArgs a = adam_args(c);
    for (size_t i = 0; i < bs.size(); ++i) {
      const uint64_t gs = bs[i].n / c.world, off = bs[i].e0 + gs * c.rank;
      AdamArgs ap = a;
      ap.hash_count = gs;
      if (i > 0) ap.mlp_count = 0;  // the MLP is scanned once
      launch_numerics_probe(ap, c.params.p + off, c.m.p + off, c.v.p + off,
                            c.gh_fixed.p ? c.gh_fixed.p + off : nullptr,
                            c.ghf(off), c.gm.p,
                            c.hash_count - off, c.stats(), 1, gate ? 1 : 0,
                            c.num_sms, c.stream);
      c.launches++;
    }
    StepStats *st = c.stats();
    NK(ncclGroupStart());
    NK(ncclAllReduce(&st->grad_l2, &st->grad_l2, 1, ncclFloat64, ncclSum,
                     c.comm, c.stream));
    NK(ncclAllReduce(&st->max_abs_grad, &st->max_abs_grad, 4, ncclFloat32,
                     ncclMax, c.comm, c.stream));
    NK(ncclGroupEnd());
    guard = st;
  }
  dp_finish_sharded(c, bs, guard);
}

// Collective (every rank): gathers the shards of the fp32 table, m and v so
// every rank holds the full, current state again.
void dp_sync_state(tmnn_ctx &c) {
  if (!c.stale) return;
  const uint64_t per = (uint64_t)c.nd.T * c.nd.F;
  NK(ncclGroupStart());
  for (const auto &r : c.stale_layout) {
    const uint64_t e0 = per * r.first, n = per * (uint64_t)(r.second - r.first);
    const uint64_t gs = n / c.world, off = e0 + gs * c.rank;
    NK(ncclAllGather(c.params.p + off, c.params.p + e0, gs, ncclFloat32,
                     c.comm, c.stream));
    NK(ncclAllGather(c.m.p + off, c.m.p + e0, gs, ncclFloat32, c.comm,
                     c.stream));
    NK(ncclAllGather(c.v.p + off, c.v.p + e0, gs, ncclFloat32, c.comm,
                     c.stream));
  }
  NK(ncclGroupEnd());
  CK(cudaStreamSynchronize(c.stream));
  c.stale = false;
  c.stale_layout.clear();
}

void require_synced(const tmnn_ctx &c, const char *what) {
  if (c.stale)
    throw std::invalid_argument(
        std::string(what) +
        ": the data-parallel optimizer is sharded; call tmnn_cuda_dp_sync_state "
        "on every rank first");
}

void create(tmnn_ctx &c, int device, const tmnn_spec &spec,
            const tmnn_train_cfg &cfg) {
  validate(spec);
  if (cfg.hash_grad_format != TMNN_GRAD_FIXED16 &&
      cfg.hash_grad_format != TMNN_GRAD_F32 &&
      cfg.hash_grad_format != TMNN_GRAD_F16)
    throw std::invalid_argument("hash_grad_format must be FIXED16, F32 or F16");
  if (cfg.batch_size <= 0) throw std::invalid_argument("batch_size must be > 0");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
    throw std::runtime_error("no CUDA device available");
  if (device < 0 || device >= ndev)
    throw std::invalid_argument("device index out of range");
  c.device = device;
  CK(cudaSetDevice(device));
  CK(cudaDeviceGetAttribute(&c.num_sms, cudaDevAttrMultiProcessorCount, device));
  CK(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking));
  for (auto &e : c.ev) CK(cudaEventCreate(&e));
  CK(cudaMallocHost(&c.h_stats, sizeof(StepStats)));
  c.h_loss = &c.h_stats->loss;
  c.spec = spec;
  c.cfg = cfg;
  c.nd = make_dims(spec, cfg);
  c.hash_count = c.nd.hash_count;
  c.mlp_count = c.nd.mlp_count;
  c.entry_width = c.nd.F == 2 ? 2 : 1;
  c.slots = c.hash_count / c.entry_width;
  // use_sparse_hash_adam_path (default_trainer.cpp:1868-1876): sparse iff
  // l1_reg == 0, unless overridden.
  c.sparse = cfg.sparse_hash_adam < 0 ? cfg.l1_reg == 0.0f
                                      : cfg.sparse_hash_adam != 0;
  const uint64_t total = c.hash_count + c.mlp_count;
  c.params.alloc(total);
  c.m.alloc(total);
  c.v.alloc(total);
  if (spec.table_dtype == TMNN_DTYPE_F16) c.table_h.alloc(c.hash_count);
  plan_family(c);
  c.implicit_touch = c.tensor_core_family() && !c.nd.grad_fixed;
  if (c.nd.grad_fixed)
    c.gh_fixed.alloc(c.hash_count);
  else  // fp16 gradients share the float buffer (half its size)
    c.gh_float.alloc(c.nd.grad_half ? (c.hash_count + 1) / 2 : c.hash_count);
  c.gm.alloc(c.mlp_count);
  c.touched.alloc(c.slots);
  if (cfg.enable_probes)
    c.probe.alloc((sizeof(ProbeAcc) + sizeof(float) - 1) / sizeof(float));
  static_assert(sizeof(StepStats) % sizeof(double) == 0, "StepStats size");
  c.loss_acc.alloc(sizeof(StepStats) / sizeof(double));
  c.guard.mode = cfg.numerics_sampling_mode;
  c.guard.interval = cfg.numerics_sample_interval > 0
                         ? (uint32_t)cfg.numerics_sample_interval
                         : 128u;
  if (cfg.numerics_sampling_mode < 0 || cfg.numerics_sampling_mode > 3)
    throw std::invalid_argument("numerics_sampling_mode out of range");
  if (cfg.bad_step_recovery < 0 || cfg.bad_step_recovery > 4)
    throw std::invalid_argument("bad_step_recovery out of range");
  const size_t sf = exact_scratch_floats(c.nd, c.num_sms);
  if (sf) c.scratch.alloc(sf);
  init_weights(c);
  refresh_gather_copy(c);
  reset_optimizer(c);
  zero_grads(c);
  CK(cudaMemsetAsync(c.loss_acc.p, 0, sizeof(double), c.stream));
  CK(cudaStreamSynchronize(c.stream));
  CK(cudaGetLastError());
}

// activate_safe_family (default_trainer.cpp:1860-1866): from now on this
// context trains with the fp32 reference-order kernels.
void activate_safe_family(tmnn_ctx &c) {
  c.safe_family_active = true;
  c.family = TMNN_FAMILY_SAFE_DEBUG;
  c.implicit_touch = false;  // the fp32 kernels store touched bytes
  c.plan_text += " -> SafeDebug after a numerics anomaly";
}

// One forward/backward + update of an already staged (and sorted) batch,
// ending with the read-back of the step statistics.  `force` probes the
// gradients whatever the loss; `gate` lets an anomaly veto the update.
void enqueue_step(tmnn_ctx &c, const float *p, const float *t, uint32_t N,
                  float inv_N, bool prof, bool force, bool gate,
                  StepStats *host_stats) {
  CK(cudaMemsetAsync(c.loss_acc.p, 0, sizeof(StepStats), c.stream));
  // Bucketed exchange behind the level-major scatter (Tiled family, data
  // parallel).  Probed steps take the plain path below: their probe reads
  // the reduced gradients of every bucket before any update.
  const bool shard = can_shard(c);
  std::vector<Bucket> bs;
  if (can_overlap(c) && !force) {
    bs = shard ? shard_layout(c) : dp_bucket_list(c);
    if (bs.size() < 2) bs.clear();
  }
  if (!bs.empty()) {
    if (shard && c.stale && !layout_is(c, bs)) dp_sync_state(c);
    if (prof) CK(cudaEventRecord(c.ev[1], c.stream));
    step_overlapped(c, p, t, N, inv_N, shard, gate, bs, prof);
    if (prof) CK(cudaEventRecord(c.ev[4], c.stream));
    CK(cudaMemcpyAsync(host_stats, c.loss_acc.p, sizeof(StepStats),
                       cudaMemcpyDeviceToHost, c.stream));
    if (prof) CK(cudaEventRecord(c.ev[5], c.stream));
    return;
  }
  if (prof) CK(cudaEventRecord(c.ev[1], c.stream));
  fwd_bwd(c, p, t, nullptr, N, inv_N);
  if (prof) CK(cudaEventRecord(c.ev[2], c.stream));
  if (shard) {
    // sharded: the probe needs a cross-rank combine, so it runs only on
    // forced steps (sampled steps and every step of a recovery mode)
    dp_update(c, true, prof ? c.ev[3] : nullptr, force, gate);
  } else {
    allreduce_grads(c, true);
    if (prof) CK(cudaEventRecord(c.ev[3], c.stream));
    probe_numerics(c, force, gate);
    adam(c, c.stats());
  }
  if (prof) CK(cudaEventRecord(c.ev[4], c.stream));
  CK(cudaMemcpyAsync(host_stats, c.loss_acc.p, sizeof(StepStats),
                     cudaMemcpyDeviceToHost, c.stream));
  if (prof) CK(cudaEventRecord(c.ev[5], c.stream));
}

// One step's device work followed by the read-back of its statistics into
// c.h_stats and a host wait.
void run_step(tmnn_ctx &c, const float *p, const float *t, uint32_t N,
              float inv_N, bool prof, bool force, bool gate) {
  enqueue_step(c, p, t, N, inv_N, prof, force, gate, c.h_stats);
  CK(cudaStreamSynchronize(c.stream));
  CK(cudaGetLastError());
}

// NumericsReport of the last run_step (make_numerics_report,
// training_step_execution.cpp:409-456): finite_forward from the loss, the
// rest from the probe when it ran.
struct StepReport {
  float mean_loss = 0.0f, grad_norm = 0.0f, max_g = 0.0f, max_u = 0.0f;
  bool ff = true, fb = true, fu = true, probed = false;
  bool anomaly() const { return !ff || !fb || !fu; }
};

StepReport read_report(const StepStats &h, uint64_t global_n) {
  if (h.exchange_err)
    throw std::runtime_error(
        "data-parallel exchange: a rank did not reach the peer-memory "
        "barrier within its wait bound; the step's update is incomplete");
  StepReport r;
  // finalize_async_step: mean_loss = total / float(batch_N)
  // (parameter_store.cpp:303-322)
  r.mean_loss = global_n ? (float)h.loss / (float)global_n : 0.0f;
  r.ff = std::isfinite(r.mean_loss);
  r.probed = h.probed != 0;
  if (r.probed) {
    r.fb = h.nonfinite_bwd == 0.0f;
    r.max_g = h.max_abs_grad;
    r.grad_norm = (float)std::sqrt(std::max(0.0, h.grad_l2));
    r.fu = r.fb && h.nonfinite_upd == 0.0f;
    r.max_u = r.fb ? h.max_abs_update : 0.0f;
  }
  return r;
}

std::string describe(const StepReport &r) {
  return std::string("forward=") + (r.ff ? "finite" : "nonfinite") +
         ", backward=" + (r.fb ? "finite" : "nonfinite") +
         ", update=" + (r.fu ? "finite" : "nonfinite") +
         ", max_abs_gradient=" + std::to_string(r.max_g) +
         ", max_abs_update=" + std::to_string(r.max_u);
}

// The step driver with the numerics guard (finalize_training_step,
// training_step_execution.cpp:1080-1235): the probe is forced on sampled
// steps and on every step of a recovery mode; in a recovery mode an anomaly
// vetoes the update on the device (the gradients are still cleared), and
// the host then throws (Throw), reports Skipped / RolledBack, or switches
// to the SafeDebug family and re-runs the step (FallbackAndRetry).  The
// step counter advances as in the reference (default_trainer.cpp:1032),
// except when an error is thrown.
void train_step(tmnn_ctx &c, const float *pos, const float *tgt, uint32_t N,
                uint32_t flags, tmnn_step_result *res) {
  if (N > 0 && (!pos || !tgt))
    throw std::invalid_argument("training_step: null positions or targets");
  if (c.n_pending)
    throw std::invalid_argument(
        "training_step: enqueued steps are pending; finalize them first");
  CK(cudaSetDevice(c.device));
  ensure_batch(c, N);
  const bool prof = flags & TMNN_PROFILE;
  if (prof) CK(cudaEventRecord(c.ev[0], c.stream));
  const float *p = stage_in(c, pos, (size_t)N * c.nd.d, c.pos_in, flags);
  const float *t = stage_in(c, tgt, (size_t)N * c.nd.O, c.tgt_in, flags);
  if (c.cfg.morton_sort && N > 1) morton_sort(c, p, t, N, &p, &t);
  const uint64_t global_n = (uint64_t)N * (uint64_t)c.world;
  const float inv_N = global_n ? 1.0f / (float)global_n : 0.0f;
  const uint32_t done = c.step;
  const int mode = c.cfg.bad_step_recovery;
  const bool gate = mode != TMNN_BAD_STEP_SIGNAL_ONLY;
  const bool force = gate || c.guard.should_sample(done, false);
  run_step(c, p, t, N, inv_N, prof, force, gate);
  StepReport rep = read_report(*c.h_stats, global_n);
  bool anomaly = rep.anomaly();
  bool reported = c.guard.should_sample(done, anomaly);
  if (reported) c.guard.record(done, anomaly);
  int action = TMNN_RECOVERY_NONE;
  if (anomaly && gate) {
    if (mode == TMNN_BAD_STEP_THROW) {
      c.step = done;
      throw OperationFailed("training_step: numerics anomaly detected at step " +
                            std::to_string(done) + " (" + describe(rep) + ")");
    } else if (mode == TMNN_BAD_STEP_SKIP) {
      action = TMNN_RECOVERY_SKIPPED;
      ++c.n_skipped;
    } else if (mode == TMNN_BAD_STEP_ROLLBACK) {
      action = TMNN_RECOVERY_ROLLED_BACK;
      ++c.n_rolled_back;
    } else {
      if (c.safe_family_active || c.family == TMNN_FAMILY_SAFE_DEBUG) {
        c.step = done;
        throw OperationFailed(
            "training_step: numerics anomaly persisted while SafeDebug is "
            "already active at step " + std::to_string(done) + " (" +
            describe(rep) + ")");
      }
      activate_safe_family(c);
      c.step = done;  // the vetoed update is re-done with the same step
      // Under the sharded optimizer the fp32 master outside this rank's
      // shard is out of date (only the fp16 gather copy was all-gathered),
      // and the SafeDebug kernels read the fp32 master: gather it first.
      // Every rank reaches this point together (the anomaly decision is
      // combined over the ranks), so the collective is matched.
      if (c.stale) dp_sync_state(c);
      run_step(c, p, t, N, inv_N, prof, true, true);
      rep = read_report(*c.h_stats, global_n);
      anomaly = rep.anomaly();
      c.guard.record(done, anomaly);
      reported = true;
      if (anomaly) {
        c.step = done;
        throw OperationFailed(
            "training_step: SafeDebug retry still produced a numerics anomaly "
            "at step " + std::to_string(done) + " (" + describe(rep) + ")");
      }
      action = TMNN_RECOVERY_RETRIED_WITH_SAFE_FAMILY;
      ++c.n_safe_recoveries;
    }
  }
  if (res) {
    std::memset(res, 0, sizeof *res);
    res->loss = rep.mean_loss;
    res->step = done;
    res->batch_size = N;
    res->numerics_ok = anomaly ? 0 : 1;
    res->family = c.family;
    res->grad_norm = rep.grad_norm;
    res->finite_forward = rep.ff;
    res->finite_backward = rep.fb;
    res->finite_update = rep.fu;
    res->max_abs_gradient = rep.max_g;
    res->max_abs_update = rep.max_u;
    res->numerics_probed = rep.probed;
    res->numerics_reported = reported;
    res->has_numerics_anomaly = anomaly;
    res->recovery_action = action;
    if (prof) {
      CK(cudaEventElapsedTime(&res->gpu_ms, c.ev[0], c.ev[5]));
      CK(cudaEventElapsedTime(&res->sort_ms, c.ev[0], c.ev[1]));
      CK(cudaEventElapsedTime(&res->fwd_bwd_ms, c.ev[1], c.ev[2]));
      CK(cudaEventElapsedTime(&res->allreduce_ms, c.ev[2], c.ev[3]));
      CK(cudaEventElapsedTime(&res->adam_ms, c.ev[3], c.ev[4]));
    }
  }
}

// Pipelined training steps (enqueue_training_step / finalize_training_step,
// training_step_execution.cpp:887-1235, with the reference's two step lanes,
// default_trainer.cpp:41): enqueue uploads the batch into a free lane on a
// copy stream and queues the step's device work behind it without waiting;
// finalize waits for the oldest pending step and reports it.  With two steps
// in flight the host->device copy of one overlaps the other's kernels.  The
// numerics probe is sampled as in training_step; recovery modes other than
// SignalOnly need the host between steps and are refused here.
void train_step_enqueue(tmnn_ctx &c, const float *pos, const float *tgt,
                        uint32_t N, uint32_t flags) {
  if (N > 0 && (!pos || !tgt))
    throw std::invalid_argument("training_step_enqueue: null positions or targets");
  if (c.cfg.bad_step_recovery != TMNN_BAD_STEP_SIGNAL_ONLY)
    throw std::invalid_argument(
        "training_step_enqueue: bad-step recovery modes need training_step");
  if (c.n_pending >= 2)
    throw std::invalid_argument(
        "training_step_enqueue: two steps are pending; finalize one first");
  CK(cudaSetDevice(c.device));
  if (!c.copy_stream)
    CK(cudaStreamCreateWithFlags(&c.copy_stream, cudaStreamNonBlocking));
  auto &L = c.lanes[c.lane_next];
  if (!L.h_stats) {
    CK(cudaMallocHost(&L.h_stats, sizeof(StepStats)));
    for (cudaEvent_t *e : {&L.copied, &L.consumed, &L.done})
      CK(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
  }
  ensure_batch(c, N);
  const size_t np = (size_t)N * c.nd.d, nt = (size_t)N * c.nd.O;
  const float *p = pos, *t = tgt;
  if (!(flags & TMNN_PTR_DEVICE)) {
    L.pos.ensure(np);
    L.tgt.ensure(nt);
    // the lane's previous batch must have been read before it is overwritten
    if (L.used) CK(cudaStreamWaitEvent(c.copy_stream, L.consumed, 0));
    if (np)
      CK(cudaMemcpyAsync(L.pos.p, pos, np * sizeof(float),
                         cudaMemcpyHostToDevice, c.copy_stream));
    if (nt)
      CK(cudaMemcpyAsync(L.tgt.p, tgt, nt * sizeof(float),
                         cudaMemcpyHostToDevice, c.copy_stream));
    CK(cudaEventRecord(L.copied, c.copy_stream));
    CK(cudaStreamWaitEvent(c.stream, L.copied, 0));
    p = L.pos.p;
    t = L.tgt.p;
  }
  bool sorted = false;
  if (c.cfg.morton_sort && N > 1) {
    morton_sort(c, p, t, N, &p, &t);
    sorted = true;
    CK(cudaEventRecord(L.consumed, c.stream));
  }
  const uint64_t global_n = (uint64_t)N * (uint64_t)c.world;
  const float inv_N = global_n ? 1.0f / (float)global_n : 0.0f;
  L.step = c.step;
  L.N = N;
  const bool force = c.guard.should_sample(L.step, false);
  enqueue_step(c, p, t, N, inv_N, false, force, false, L.h_stats);
  if (!sorted) CK(cudaEventRecord(L.consumed, c.stream));
  CK(cudaEventRecord(L.done, c.stream));
  L.used = true;
  c.lane_next ^= 1;
  ++c.n_pending;
}

void train_step_finalize(tmnn_ctx &c, tmnn_step_result *res) {
  if (c.n_pending == 0)
    throw std::invalid_argument("training_step_finalize: no step is pending");
  CK(cudaSetDevice(c.device));
  auto &L = c.lanes[c.lane_oldest];
  CK(cudaEventSynchronize(L.done));
  CK(cudaGetLastError());
  c.lane_oldest ^= 1;
  --c.n_pending;
  const uint64_t global_n = (uint64_t)L.N * (uint64_t)c.world;
  const StepReport rep = read_report(*L.h_stats, global_n);
  const bool anomaly = rep.anomaly();
  const bool reported = c.guard.should_sample(L.step, anomaly);
  if (reported) c.guard.record(L.step, anomaly);
  if (res) {
    std::memset(res, 0, sizeof *res);
    res->loss = rep.mean_loss;
    res->step = L.step;
    res->batch_size = L.N;
    res->numerics_ok = anomaly ? 0 : 1;
    res->family = c.family;
    res->grad_norm = rep.grad_norm;
    res->finite_forward = rep.ff;
    res->finite_backward = rep.fb;
    res->finite_update = rep.fu;
    res->max_abs_gradient = rep.max_g;
    res->max_abs_update = rep.max_u;
    res->numerics_probed = rep.probed;
    res->numerics_reported = reported;
    res->has_numerics_anomaly = anomaly;
    res->recovery_action = TMNN_RECOVERY_NONE;
  }
}

void copy_out(tmnn_ctx &c, float *dst, const float *src, size_t count,
              uint32_t flags) {
  if (!count) return;
  CK(cudaMemcpyAsync(dst, src, count * sizeof(float),
                     (flags & TMNN_PTR_DEVICE) ? cudaMemcpyDeviceToDevice
                                               : cudaMemcpyDeviceToHost,
                     c.stream));
}

void forward_api(tmnn_ctx &c, const float *pos, float *out, uint32_t N,
                 uint32_t flags) {
  if (N > 0 && (!pos || !out))
    throw std::invalid_argument("forward: null positions or outputs");
  CK(cudaSetDevice(c.device));
  ensure_batch(c, N);
  const float *p = stage_in(c, pos, (size_t)N * c.nd.d, c.pos_in, flags);
  float *o = (flags & TMNN_PTR_DEVICE) ? out : c.out_buf.p;
  forward_dev(c, p, o, N);
  if (!(flags & TMNN_PTR_DEVICE)) copy_out(c, out, o, (size_t)N * c.nd.O, flags);
  CK(cudaStreamSynchronize(c.stream));
  CK(cudaGetLastError());
}

// FieldEvaluator::evaluate_with_gradient (default_trainer.cpp:467-622): the
// field value [N] and d(value)/d(pos) [N x d] of a single-output network, from
// the fp32 parameters (the reference compiles this kernel with fp16 off).
void evaluate_with_gradient(tmnn_ctx &c, const float *pos, float *out,
                            float *grad, uint32_t N, uint32_t flags) {
  if (c.nd.O != 1)
    throw std::invalid_argument(
        "evaluate_with_gradient: the network must have exactly one output "
        "(num_outputs = " + std::to_string(c.nd.O) + ")");
  if (N > 0 && (!pos || !out || !grad))
    throw std::invalid_argument(
        "evaluate_with_gradient: positions, output, and gradients must be "
        "non-null when N > 0");
  require_synced(c, "evaluate_with_gradient");
  if (N == 0) return;
  CK(cudaSetDevice(c.device));
  ensure_batch(c, N);
  const size_t d = c.nd.d;
  const float *p = stage_in(c, pos, (size_t)N * d, c.pos_in, flags);
  const bool dev = flags & TMNN_PTR_DEVICE;
  float *o = dev ? out : c.out_buf.p;
  float *g = grad;
  if (!dev) {
    c.grad_out.ensure((size_t)N * d);
    g = c.grad_out.p;
  }
  const size_t sf = eval_gradient_scratch_floats(c.nd, c.num_sms);
  if (sf) c.eg_scratch.ensure(sf);
  launch_eval_gradient(c.nd, c.hash_w(), c.mlp_w(), p, o, g, N,
                       c.eg_scratch.p, c.num_sms, c.stream);
  c.launches++;
  if (!dev) {
    copy_out(c, out, o, N, flags);
    copy_out(c, grad, g, (size_t)N * d, flags);
  }
  CK(cudaStreamSynchronize(c.stream));
  CK(cudaGetLastError());
}

void backward_accumulate(tmnn_ctx &c, const float *pos, const float *dout,
                         uint32_t N, uint32_t flags) {
  if (N > 0 && (!pos || !dout))
    throw std::invalid_argument("backward_accumulate: null arguments");
  CK(cudaSetDevice(c.device));
  ensure_batch(c, N);
  const float *p = stage_in(c, pos, (size_t)N * c.nd.d, c.pos_in, flags);
  const float *g = stage_in(c, dout, (size_t)N * c.nd.O, c.tgt_in, flags);
  if (c.cfg.morton_sort && N > 1) morton_sort(c, p, g, N, &p, &g);
  fwd_bwd(c, p, nullptr, g, N, 0.0f);
  CK(cudaStreamSynchronize(c.stream));
  CK(cudaGetLastError());
}

}  // namespace

// ====================================================================== ABI

namespace tmnn {
int ctx_world(const tmnn_ctx *c) { return c ? c->world : 1; }
void ctx_allreduce_sum(tmnn_ctx *c, float *f32, size_t n32, double *f64,
                       size_t n64) {
  if (!c || !c->comm || c->world <= 1) return;
  NK(ncclGroupStart());
  if (n32)
    NK(ncclAllReduce(f32, f32, n32, ncclFloat32, ncclSum, c->comm, c->stream));
  if (n64)
    NK(ncclAllReduce(f64, f64, n64, ncclFloat64, ncclSum, c->comm, c->stream));
  NK(ncclGroupEnd());
}
}  // namespace tmnn

extern "C" {

void tmnn_cuda_default_train_cfg(tmnn_train_cfg *c) {
  if (!c) return;
  std::memset(c, 0, sizeof *c);
  c->batch_size = 1024;
  c->lr_encoding = 1e-2f;
  c->lr_network = 1e-3f;
  c->beta1 = 0.9f;
  c->beta2 = 0.99f;
  c->epsilon = 1e-15f;
  c->hash_init = 0;
  c->hash_init_range = 1.0e-4f;
  c->mlp_init = 0;
  c->mlp_nonlinearity = 1;
  c->mlp_uniform_range = 1.0e-2f;
  c->mlp_normal_stddev = 1.0e-2f;
  c->seed = 42u;
  c->family = TMNN_FAMILY_AUTO;
  c->hash_grad_format = TMNN_GRAD_FIXED16;
  c->morton_sort = 1;
  c->sparse_hash_adam = -1;
  // load_runtime_policy (src/tiny_metal_nn/runtime/runtime_policy.h:144-175)
  c->numerics_sampling_mode = TMNN_NUMERICS_SAMPLED;
  c->numerics_sample_interval = 128;
  c->bad_step_recovery = TMNN_BAD_STEP_SIGNAL_ONLY;
  c->morton_key_bits = 12;
  apply_policy_env(*c);
}

tmnn_status tmnn_cuda_get_numerics_stats(tmnn_ctx *c, tmnn_numerics_stats *o) {
  REQUIRE_CTX(c);
  if (!o) {
    g_last_error = "null argument";
    return TMNN_ERR_NULL_OBJECT;
  }
  std::memset(o, 0, sizeof *o);
  o->reports = c->guard.report_count;
  o->anomalies = c->guard.anomaly_count;
  o->skipped = c->n_skipped;
  o->rolled_back = c->n_rolled_back;
  o->safe_family_recoveries = c->n_safe_recoveries;
  o->last_anomaly_step = c->guard.last_anomaly_step;
  o->safe_family_active = c->safe_family_active ? 1 : 0;
  return TMNN_OK;
}

tmnn_status tmnn_cuda_validate_spec(const tmnn_spec *spec) {
  if (!spec) {
    g_last_error = "null spec";
    return TMNN_ERR_NULL_OBJECT;
  }
  return guarded([&] { validate(*spec); });
}

tmnn_status tmnn_cuda_ctx_create(int device, const tmnn_spec *spec,
                                 const tmnn_train_cfg *cfg, tmnn_ctx **out) {
  if (!spec || !out) {
    g_last_error = "null argument";
    return TMNN_ERR_NULL_OBJECT;
  }
  *out = nullptr;
  tmnn_train_cfg dflt;
  tmnn_cuda_default_train_cfg(&dflt);
  std::unique_ptr<tmnn_ctx> c(new tmnn_ctx);
  tmnn_status st = guarded([&] { create(*c, device, *spec, cfg ? *cfg : dflt); });
  if (st == TMNN_OK) *out = c.release();
  return st;
}

tmnn_status tmnn_cuda_ctx_create_from_json(int device, uint32_t n_input,
                                           uint32_t n_output, const char *json,
                                           tmnn_ctx **out) {
  if (!out) {
    g_last_error = "null argument";
    return TMNN_ERR_NULL_OBJECT;
  }
  *out = nullptr;
  tmnn_spec spec;
  tmnn_train_cfg cfg;
  tmnn_status st =
      guarded([&] { config_from_json(n_input, n_output, json, &spec, &cfg); });
  if (st != TMNN_OK) return st;
  return tmnn_cuda_ctx_create(device, &spec, &cfg, out);
}

tmnn_status tmnn_cuda_ctx_destroy(tmnn_ctx *ctx) {
  REQUIRE_CTX(ctx);
  return guarded([&] {
    cudaSetDevice(ctx->device);
    delete ctx;
  });
}

tmnn_status tmnn_cuda_set_initial_weights(tmnn_ctx *c, const float *hash,
                                          size_t hash_count, const float *mlp,
                                          size_t mlp_count) {
  REQUIRE_CTX(c);
  return guarded([&] {
    BusyGuard g(c);
    if (hash && hash_count != c->hash_count)
      throw std::invalid_argument("set_initial_weights: hash count mismatch");
    if (mlp && mlp_count != c->mlp_count)
      throw std::invalid_argument("set_initial_weights: mlp count mismatch");
    CK(cudaSetDevice(c->device));
    if (hash)
      CK(cudaMemcpyAsync(c->hash_w(), hash, hash_count * 4,
                         cudaMemcpyHostToDevice, c->stream));
    if (mlp)
      CK(cudaMemcpyAsync(c->mlp_w(), mlp, mlp_count * 4,
                         cudaMemcpyHostToDevice, c->stream));
    refresh_gather_copy(*c);
    reset_optimizer(*c);
    zero_grads(*c);
    CK(cudaStreamSynchronize(c->stream));
    if (hash) c->stale = false;  // full table written, moments reset
  });
}

tmnn_status tmnn_cuda_get_weights(tmnn_ctx *c, float *hash, size_t hash_count,
                                  float *mlp, size_t mlp_count) {
  REQUIRE_CTX(c);
  return guarded([&] {
    BusyGuard g(c);
    if (hash && hash_count != c->hash_count)
      throw std::invalid_argument("get_weights: hash count mismatch");
    if (mlp && mlp_count != c->mlp_count)
      throw std::invalid_argument("get_weights: mlp count mismatch");
    require_synced(*c, "get_weights");
    CK(cudaSetDevice(c->device));
    if (hash)
      CK(cudaMemcpyAsync(hash, c->hash_w(), hash_count * 4,
                         cudaMemcpyDeviceToHost, c->stream));
    if (mlp)
      CK(cudaMemcpyAsync(mlp, c->mlp_w(), mlp_count * 4,
                         cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
  });
}

tmnn_status tmnn_cuda_train_step(tmnn_ctx *c, const float *positions,
                                 const float *targets, uint32_t n,
                                 uint32_t flags, tmnn_step_result *result) {
  REQUIRE_CTX(c);
  return guarded([&] {
    BusyGuard g(c);
    train_step(*c, positions, targets, n, flags, result);
  });
}

tmnn_status tmnn_cuda_train_step_enqueue(tmnn_ctx *c, const float *positions,
                                         const float *targets, uint32_t n,
                                         uint32_t flags) {
  REQUIRE_CTX(c);
  return guarded([&] {
    BusyGuard g(c);
    train_step_enqueue(*c, positions, targets, n, flags);
  });
}

tmnn_status tmnn_cuda_train_step_finalize(tmnn_ctx *c,
                                          tmnn_step_result *result) {
  REQUIRE_CTX(c);
  return guarded([&] {
    BusyGuard g(c);
    train_step_finalize(*c, result);
  });
}

tmnn_status tmnn_cuda_forward_backward(tmnn_ctx *c, const float *positions,
                                       const float *targets, uint32_t n,
                                       uint32_t flags, double *loss_sum) {
  REQUIRE_CTX(c);
  return guarded([&] {
    BusyGuard g(c);
    if (n > 0 && (!positions || !targets))
      throw std::invalid_argument("forward_backward: null arguments");
    CK(cudaSetDevice(c->device));
    ensure_batch(*c, n);
    const float *p = stage_in(*c, positions, (size_t)n * c->nd.d, c->pos_in, flags);
    const float *t = stage_in(*c, targets, (size_t)n * c->nd.O, c->tgt_in, flags);
    if (c->cfg.morton_sort && n > 1) morton_sort(*c, p, t, n, &p, &t);
    CK(cudaMemsetAsync(c->loss_acc.p, 0, sizeof(double), c->stream));
    const uint64_t global_n = (uint64_t)n * (uint64_t)c->world;
    fwd_bwd(*c, p, t, nullptr, n, global_n ? 1.0f / (float)global_n : 0.0f);
    CK(cudaMemcpyAsync(c->h_loss, c->loss_acc.p, sizeof(double),
                       cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaGetLastError());
    if (loss_sum) *loss_sum = *c->h_loss;
  });
}

// ---------------------------------------------------------------------------
// forward_backward without allocation.
//
// Some callers cannot call cudaMalloc at the point where they run a step:
// code running under a framework's memory pool or a fixed-footprint serving
// budget, real-time loops that must not stall on the allocator, or hosts that
// have forbidden device allocation after start-up.  The ordinary
// tmnn_cuda_forward_backward grows the context's batch staging buffers
// (Morton codes, permutation, sorted copies, radix-sort temporary) on demand,
// which allocates.  This variant keeps that scratch in one file-scope device
// array of fixed size instead, so a call allocates nothing.
namespace {

constexpr uint32_t kNoAllocMaxPoints = 65536;  // the reference's batch cap
constexpr uint32_t kNoAllocMaxOutputs = 16;
constexpr size_t kNoAllocSortTempBytes = 2u << 20;
constexpr size_t kNoAllocBytes =
    4 * (size_t)kNoAllocMaxPoints * 4 +                       // codes x2, idx, perm
    (size_t)kNoAllocMaxPoints * 4 * 4 +                       // sorted positions
    (size_t)kNoAllocMaxPoints * kNoAllocMaxOutputs * 4 +      // sorted targets
    kNoAllocSortTempBytes;                                    // radix-sort temp

// Shared by every call on a device; holds the last call's contents.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
uint8_t *g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of the scratch array for `device` (which must be current).
// The array's name is a host-side stand-in, so the address is looked up once
// per device with cudaGetSymbolAddress.
uint8_t *noalloc_scratch(int device) {
  if (device < 0 || device >= kNoAllocMaxDevices)
    throw std::invalid_argument("forward_backward_noalloc: device index too large");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[device]) {
    void *p = nullptr;
    CK(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    if (morton_temp_bytes(kNoAllocMaxPoints) > kNoAllocSortTempBytes)
      throw std::runtime_error(
          "forward_backward_noalloc: radix-sort temporary exceeds its reserve");
    g_noalloc_ptr[device] = static_cast<uint8_t *>(p);
  }
  return g_noalloc_ptr[device];
}

}  // namespace

tmnn_status tmnn_cuda_forward_backward_noalloc(tmnn_ctx *c,
                                               const float *positions,
                                               const float *targets,
                                               uint32_t n, double *loss_sum) {
  REQUIRE_CTX(c);
  return guarded([&] {
    BusyGuard g(c);
    if (n > 0 && (!positions || !targets))
      throw std::invalid_argument("forward_backward_noalloc: null arguments");
    if (n > kNoAllocMaxPoints)
      throw std::invalid_argument(
          "forward_backward_noalloc: batch of " + std::to_string(n) +
          " points exceeds the maximum of 65536 (use tmnn_cuda_forward_backward)");
    if (c->nd.O > (int)kNoAllocMaxOutputs)
      throw std::invalid_argument(
          "forward_backward_noalloc: more than 16 outputs are not supported");
    if (c->family == TMNN_FAMILY_TILED &&
        (c->feat.n < (size_t)n * c->nd.In || c->dfeat.n < (size_t)n * c->nd.In))
      throw std::invalid_argument(
          "forward_backward_noalloc: the Tiled family's feature buffers are "
          "smaller than this batch; run one ordinary training_step or "
          "forward_backward with at least this many points first");
    if (c->tensor_core_family() &&
        (!c->fws.err || !c->fws.wpack))
      throw std::invalid_argument(
          "forward_backward_noalloc: the fused kernel's weight image is not set "
          "up yet; run one ordinary training_step or forward_backward first");
    CK(cudaSetDevice(c->device));
    uint8_t *base = noalloc_scratch(c->device);
    const size_t N = kNoAllocMaxPoints;
    uint32_t *codes = reinterpret_cast<uint32_t *>(base);
    uint32_t *codes_alt = codes + N;
    uint32_t *idx = codes_alt + N;
    uint32_t *perm = idx + N;
    float *pos_s = reinterpret_cast<float *>(perm + N);
    float *tgt_s = pos_s + N * 4;
    uint8_t *sort_tmp = reinterpret_cast<uint8_t *>(tgt_s + N * kNoAllocMaxOutputs);
    const float *p = positions, *t = targets;
    if (c->cfg.morton_sort && n > 1) {
      launch_morton_order(p, c->nd.d, n, codes, codes_alt, idx, perm, sort_tmp,
                          kNoAllocSortTempBytes, c->stream,
                          c->cfg.morton_key_bits);
      launch_gather_rows(p, c->nd.d, perm, pos_s, n, c->stream);
      launch_gather_rows(t, c->nd.O, perm, tgt_s, n, c->stream);
      c->launches += 4;
      p = pos_s;
      t = tgt_s;
    }
    CK(cudaMemsetAsync(c->loss_acc.p, 0, sizeof(double), c->stream));
    const uint64_t global_n = (uint64_t)n * (uint64_t)c->world;
    fwd_bwd(*c, p, t, nullptr, n, global_n ? 1.0f / (float)global_n : 0.0f);
    CK(cudaMemcpyAsync(c->h_loss, c->loss_acc.p, sizeof(double),
                       cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaGetLastError());
    if (loss_sum) *loss_sum = *c->h_loss;
  });
}

tmnn_status tmnn_cuda_read_buffer(tmnn_ctx *c, int32_t role, void *host,
                                  size_t bytes) {
  REQUIRE_CTX(c);
  tmnn_buffer_view v;
  tmnn_status st = tmnn_cuda_get_buffer(c, role, &v);
  if (st != TMNN_OK) return st;
  return guarded([&] {
    BusyGuard g(c);
    if (!host || bytes != v.bytes)
      throw std::invalid_argument("read_buffer: size mismatch");
    if (role == TMNN_BUF_HASH_WEIGHTS || role == TMNN_BUF_FUSED_WEIGHTS ||
        role == TMNN_BUF_FUSED_M || role == TMNN_BUF_FUSED_V)
      require_synced(*c, "read_buffer");
    CK(cudaSetDevice(c->device));
    if (role == TMNN_BUF_TOUCHED && c->implicit_touch)
      launch_touched_from_grads(c->gh_float.p, c->touched.p, c->slots,
                                c->entry_width, c->grad_half(), c->num_sms,
                                c->stream);
    CK(cudaMemcpyAsync(host, v.device_ptr, bytes, cudaMemcpyDeviceToHost,
                       c->stream));
    CK(cudaStreamSynchronize(c->stream));
  });
}

tmnn_status tmnn_cuda_forward(tmnn_ctx *c, const float *positions,
                              float *outputs, uint32_t n, uint32_t flags) {
  REQUIRE_CTX(c);
  return guarded([&] {
    BusyGuard g(c);
    forward_api(*c, positions, outputs, n, flags);
  });
}

tmnn_status tmnn_cuda_zero_grads(tmnn_ctx *c) {
  REQUIRE_CTX(c);
  return guarded([&] {
    BusyGuard g(c);
    CK(cudaSetDevice(c->device));
    zero_grads(*c);
    CK(cudaStreamSynchronize(c->stream));
  });
}

tmnn_status tmnn_cuda_backward_accumulate(tmnn_ctx *c, const float *positions,
                                          const float *d_output, uint32_t n,
                                          uint32_t flags) {
  REQUIRE_CTX(c);
  return guarded([&] {
    BusyGuard g(c);
    backward_accumulate(*c, positions, d_output, n, flags);
  });
}

tmnn_status tmnn_cuda_adam_step(tmnn_ctx *c) {
  REQUIRE_CTX(c);
  return guarded([&] {
    BusyGuard g(c);
    CK(cudaSetDevice(c->device));
    if (can_shard(*c)) {
      dp_update(*c, false, nullptr);
    } else {
      allreduce_grads(*c, false);
      adam(*c);
    }
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaGetLastError());
  });
}

tmnn_status tmnn_cuda_evaluate(tmnn_ctx *c, const float *positions,
                               float *outputs, uint32_t n, uint32_t flags) {
  REQUIRE_CTX(c);
  return guarded([&] {
    BusyGuard g(c);
    forward_api(*c, positions, outputs, n, flags);
  });
}

tmnn_status tmnn_cuda_evaluate_with_gradient(tmnn_ctx *c,
                                             const float *positions,
                                             float *outputs, float *gradients,
                                             uint32_t n, uint32_t flags) {
  REQUIRE_CTX(c);
  return guarded([&] {
    BusyGuard g(c);
    evaluate_with_gradient(*c, positions, outputs, gradients, n, flags);
  });
}

tmnn_status tmnn_cuda_debug_morton_order(tmnn_ctx *c, const float *positions,
                                         uint32_t n, int32_t key_bits,
                                         uint32_t *perm) {
  REQUIRE_CTX(c);
  return guarded([&] {
    BusyGuard g(c);
    if (n > 0 && (!positions || !perm))
      throw std::invalid_argument("debug_morton_order: null arguments");
    if (n == 0) return;
    CK(cudaSetDevice(c->device));
    ensure_batch(*c, n);
    const float *p = stage_in(*c, positions, (size_t)n * c->nd.d, c->pos_in, 0);
    launch_morton_order(p, c->nd.d, n, c->codes.p, c->codes_alt.p, c->idx.p,
                        c->perm.p, c->sort_tmp.p, c->sort_tmp.n, c->stream,
                        key_bits);
    c->launches += 3;
    CK(cudaMemcpyAsync(perm, c->perm.p, (size_t)n * 4, cudaMemcpyDeviceToHost,
                       c->stream));
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaGetLastError());
  });
}

tmnn_status tmnn_cuda_debug_encode(tmnn_ctx *c, const float *positions,
                                   uint32_t n, float *features,
                                   uint32_t *corner_index, int32_t *cells) {
  REQUIRE_CTX(c);
  return guarded([&] {
    BusyGuard g(c);
    if (n > 0 && (!positions || !features))
      throw std::invalid_argument("debug_encode: null arguments");
    require_synced(*c, "debug_encode");
    CK(cudaSetDevice(c->device));
    ensure_batch(*c, n);
    const float *p = stage_in(*c, positions, (size_t)n * c->nd.d, c->pos_in, 0);
    DevBuf<float> feat;
    DevBuf<uint32_t> ci;
    DevBuf<int32_t> ce;
    const size_t nc = (size_t)1 << c->nd.d;
    feat.alloc((size_t)n * c->nd.In);
    if (corner_index) ci.alloc((size_t)n * c->nd.L * nc);
    if (cells) ce.alloc((size_t)n * c->nd.L * c->nd.d);
    launch_encode_debug(c->nd, c->hash_w(), p, feat.p, ci.p, ce.p, n, c->stream);
    c->launches++;
    if (n) {
      CK(cudaMemcpyAsync(features, feat.p, feat.bytes(), cudaMemcpyDeviceToHost,
                         c->stream));
      if (corner_index)
        CK(cudaMemcpyAsync(corner_index, ci.p, ci.bytes(),
                           cudaMemcpyDeviceToHost, c->stream));
      if (cells)
        CK(cudaMemcpyAsync(cells, ce.p, ce.bytes(), cudaMemcpyDeviceToHost,
                           c->stream));
    }
    CK(cudaStreamSynchronize(c->stream));
  });
}

tmnn_status tmnn_cuda_export_opt_state(tmnn_ctx *c, uint8_t *buf, size_t cap,
                                       size_t *len, uint32_t *step) {
  REQUIRE_CTX(c);
  return guarded([&] {
    BusyGuard g(c);
    if (!len) throw std::invalid_argument("export_opt_state: null len");
    require_synced(*c, "export_opt_state");
    const size_t hb = c->hash_count * 4, mb = (size_t)c->mlp_count * 4;
    if (hb > 0xFFFFFFFFull)
      throw CapacityError("export_opt_state: section exceeds u32 length");
    const size_t need = 4 * 4 + 2 * hb + 2 * mb;
    *len = need;
    if (step) *step = c->step;
    if (!buf) return;
    if (cap < need) throw CapacityError("export_opt_state: buffer too small");
    CK(cudaSetDevice(c->device));
    // sections [m_hash, v_hash, m_mlp, v_mlp] (default_trainer.cpp:83-100)
    struct Sec {
      const float *src;
      size_t bytes;
    } secs[4] = {{c->m.p, hb}, {c->v.p, hb}, {c->m.p + c->hash_count, mb},
                 {c->v.p + c->hash_count, mb}};
    size_t off = 0;
    for (auto &s : secs) {
      for (int i = 0; i < 4; ++i) buf[off + i] = (uint8_t)(s.bytes >> (8 * i));
      off += 4;
      CK(cudaMemcpyAsync(buf + off, s.src, s.bytes, cudaMemcpyDeviceToHost,
                         c->stream));
      off += s.bytes;
    }
    CK(cudaStreamSynchronize(c->stream));
  });
}

tmnn_status tmnn_cuda_import_opt_state(tmnn_ctx *c, const uint8_t *buf,
                                       size_t len, uint32_t step) {
  REQUIRE_CTX(c);
  return guarded([&] {
    BusyGuard g(c);
    if (!buf) throw std::invalid_argument("import_opt_state: null buffer");
    const size_t hb = c->hash_count * 4, mb = (size_t)c->mlp_count * 4;
    const size_t want[4] = {hb, hb, mb, mb};
    float *dst[4] = {c->m.p, c->v.p, c->m.p + c->hash_count,
                     c->v.p + c->hash_count};
    size_t off = 0;
    for (int s = 0; s < 4; ++s) {
      if (off + 4 > len)
        throw std::invalid_argument("import_opt_state: truncated payload");
      uint32_t n = 0;
      for (int i = 0; i < 4; ++i) n |= (uint32_t)buf[off + i] << (8 * i);
      off += 4;
      if (n != want[s])
        throw std::invalid_argument(
            "import_opt_state: section size mismatch (layout differs)");
      if (off + n > len)
        throw std::invalid_argument("import_opt_state: truncated payload");
      off += n;
    }
    if (off != len)
      throw std::invalid_argument("import_opt_state: trailing bytes");
    CK(cudaSetDevice(c->device));
    off = 0;
    for (int s = 0; s < 4; ++s) {
      off += 4;
      CK(cudaMemcpyAsync(dst[s], buf + off, want[s], cudaMemcpyHostToDevice,
                         c->stream));
      off += want[s];
    }
    CK(cudaStreamSynchronize(c->stream));
    c->step = step;
  });
}

tmnn_status tmnn_cuda_reset_optimizer(tmnn_ctx *c) {
  REQUIRE_CTX(c);
  return guarded([&] {
    BusyGuard g(c);
    CK(cudaSetDevice(c->device));
    reset_optimizer(*c);
    CK(cudaStreamSynchronize(c->stream));
  });
}

tmnn_status tmnn_cuda_get_step(tmnn_ctx *c, uint32_t *step) {
  REQUIRE_CTX(c);
  if (!step) return TMNN_ERR_INVALID_ARGUMENT;
  *step = c->step;
  return TMNN_OK;
}

tmnn_status tmnn_cuda_last_probe(tmnn_ctx *c, tmnn_probe_result *r) {
  REQUIRE_CTX(c);
  return guarded([&] {
    if (!r) throw std::invalid_argument("last_probe: null result");
    if (!c->cfg.enable_probes)
      throw std::invalid_argument("last_probe: enable_probes is off");
    if (!c->probe_ran)
      throw std::runtime_error("last_probe: no forward/backward pass has run");
    BusyGuard g(c);
    CK(cudaSetDevice(c->device));
    ProbeAcc a{};
    CK(cudaMemcpyAsync(&a, c->probe.p, sizeof a, cudaMemcpyDeviceToHost,
                       c->stream));
    CK(cudaStreamSynchronize(c->stream));
    // aggregate_probe_partials (training_step_execution.cpp:1326-1369)
    std::memset(r, 0, sizeof *r);
    r->num_hidden_layers = (uint32_t)c->nd.H;
    r->has_nan_forward = a.fwd_nan > 0.f;
    r->has_nan_backward = a.bwd_nan > 0.f;
    r->hash_grad_l2 = 0.f;
    r->output_abs_max = a.out_abs_max;
    r->output_min = -a.out_neg_min;
    for (int l = 0; l < c->nd.H && l < 8; ++l) {
      r->act_max[l] = a.act_max[l];
      r->grad_l2[l] = a.grad_l2[l];
    }
  });
}

tmnn_status tmnn_cuda_get_buffer(tmnn_ctx *c, int32_t role,
                                 tmnn_buffer_view *v) {
  REQUIRE_CTX(c);
  return guarded([&] {
    if (!v) throw std::invalid_argument("get_buffer: null view");
    std::memset(v, 0, sizeof *v);
    switch (role) {
      case TMNN_BUF_HASH_WEIGHTS:
        *v = {c->hash_w(), c->hash_count * 4, 0};
        break;
      case TMNN_BUF_MLP_WEIGHTS:
        *v = {c->mlp_w(), (size_t)c->mlp_count * 4, 0};
        break;
      case TMNN_BUF_GRAD_HASH:
        if (c->gh_fixed.p)
          *v = {c->gh_fixed.p, c->gh_fixed.bytes(), 2};
        else
          *v = {c->gh_float.p, c->hash_count * c->gh_elem(),
                c->grad_half() ? 1 : 0};
        break;
      case TMNN_BUF_GRAD_MLP:
        *v = {c->gm.p, c->gm.bytes(), 0};
        break;
      case TMNN_BUF_FUSED_WEIGHTS:
        *v = {c->params.p, c->params.bytes(), 0};
        break;
      case TMNN_BUF_FUSED_M:
        *v = {c->m.p, c->m.bytes(), 0};
        break;
      case TMNN_BUF_FUSED_V:
        *v = {c->v.p, c->v.bytes(), 0};
        break;
      case TMNN_BUF_HASH_GATHER:
        if (!c->table_h.p)
          throw std::invalid_argument("get_buffer: no fp16 gather copy");
        *v = {c->table_h.p, c->table_h.bytes(), 1};
        break;
      case TMNN_BUF_TOUCHED:
        *v = {c->touched.p, c->touched.bytes(), 3};
        break;
      default:
        throw std::invalid_argument("get_buffer: unknown role");
    }
  });
}

tmnn_status tmnn_cuda_get_plan(tmnn_ctx *c, tmnn_plan *p) {
  REQUIRE_CTX(c);
  return guarded([&] {
    if (!p) throw std::invalid_argument("get_plan: null plan");
    std::memset(p, 0, sizeof *p);
    p->family = c->family;
    p->fallback_reason = c->fallback_reason;
    p->mlp_weight_count = c->mlp_count;
    p->hash_grid_size = c->hash_count;
    p->device_bytes = c->params.bytes() + c->m.bytes() + c->v.bytes() +
                      c->table_h.bytes() + c->gh_fixed.bytes() +
                      c->gh_float.bytes() + c->gm.bytes() + c->touched.bytes() +
                      c->scratch.bytes();
    p->n_levels = c->nd.L;
    p->n_features_per_level = c->nd.F;
    p->spatial_dims = c->nd.d;
    p->num_outputs = c->nd.O;
    std::snprintf(p->reason, sizeof p->reason, "%s", c->plan_text.c_str());
  });
}

tmnn_status tmnn_cuda_get_stream(tmnn_ctx *c, void **stream) {
  REQUIRE_CTX(c);
  if (!stream) return TMNN_ERR_INVALID_ARGUMENT;
  *stream = (void *)c->stream;
  return TMNN_OK;
}

tmnn_status tmnn_cuda_synchronize(tmnn_ctx *c) {
  REQUIRE_CTX(c);
  return guarded([&] {
    CK(cudaSetDevice(c->device));
    CK(cudaStreamSynchronize(c->stream));
  });
}

tmnn_status tmnn_cuda_dp_unique_id(uint8_t out[128]) {
  return guarded([&] {
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
    ncclUniqueId id;
    NK(ncclGetUniqueId(&id));
    std::memcpy(out, &id, 128);
  });
}

tmnn_status tmnn_cuda_dp_sync_state(tmnn_ctx *c) {
  REQUIRE_CTX(c);
  return guarded([&] {
    BusyGuard g(c);
    CK(cudaSetDevice(c->device));
    dp_sync_state(*c);
  });
}

tmnn_status tmnn_cuda_dp_init(tmnn_ctx *c, const uint8_t unique_id[128],
                              int rank, int world) {
  REQUIRE_CTX(c);
  return guarded([&] {
    BusyGuard g(c);
    if (world < 1 || rank < 0 || rank >= world)
      throw std::invalid_argument("dp_init: bad rank/world");
    CK(cudaSetDevice(c->device));
    if (c->comm) {
      ncclCommDestroy(c->comm);
      c->comm = nullptr;
    }
    if (c->stale) throw std::invalid_argument(
        "dp_init: call tmnn_cuda_dp_sync_state before re-initialising");
    // a new communicator decides the peer-memory path afresh
    if (c->comm_stream) CK(cudaStreamSynchronize(c->comm_stream));
    for (void *q : c->p2p_opened) cudaIpcCloseMemHandle(q);
    c->p2p_opened.clear();
    if (c->p2p) c->plan_text.erase(0, c->plan_text.find("; ") + 2);
    c->p2p_decided = c->p2p = false;
    c->rank = rank;
    c->world = world;
    if (world > 1) {
      ncclUniqueId id;
      std::memcpy(&id, unique_id, 128);
      NK(ncclCommInitRank(&c->comm, world, id, rank));
      if (!c->comm_stream) {
        // highest priority: the collectives' blocks are scheduled ahead of
        // the pending blocks of the scatter they overlap
        int lo = 0, hi = 0;
        CK(cudaDeviceGetStreamPriorityRange(&lo, &hi));
        CK(cudaStreamCreateWithPriority(&c->comm_stream, cudaStreamNonBlocking, hi));
      }
      for (auto &e : c->dp_ev)
        if (!e) CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
      for (auto &e : c->ev_comm)
        if (!e) CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
      for (auto &e : c->ev_adam)
        if (!e) CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
      // buckets of at least 32 MiB of fp32 gradient, at most 4: more,
      // smaller ones pay more in per-collective latency and contention with
      // the scatter than their overlap wins (measured at 4 ranks, steps/s:
      // sdf3d, 64 MiB: 1 bucket 6312, 2 6618, 4 5189; field4d, 512 MiB:
      // 1 bucket 1732, 4 1893, 8 1714, 16 1662)
      {
        const uint64_t mib = (c->hash_count * 4) >> 20;
        int g = (int)(mib / 32);
        if (g < 1) g = 1;
        if (g > 4) g = 4;
        c->dp_buckets = g;
      }
      if (const char *e = std::getenv("TMNN_DP_BUCKETS")) {
        const int v = std::atoi(e);
        if (v >= 1) c->dp_buckets = v;
      }
      // Under data parallelism the Tiled family (same per-point arithmetic
      // as FullyFused) lets the gradient exchange overlap its level-major
      // scatter; Auto switches to it when it can run the shape.
      if (c->cfg.family == TMNN_FAMILY_AUTO &&
          c->family == TMNN_FAMILY_FULLY_FUSED && c->dp_buckets > 1 &&
          tiled_supported(c->nd, nullptr)) {
        c->family = TMNN_FAMILY_TILED;
        c->plan_text += "; data parallel: Tiled, so the gradient exchange "
                        "overlaps the level-major scatter";
      }
    }
  });
}

const char *tmnn_cuda_last_error(void) { return g_last_error.c_str(); }

tmnn_status tmnn_cuda_launch_count(tmnn_ctx *c, uint64_t *count) {
  REQUIRE_CTX(c);
  if (!count) return TMNN_ERR_INVALID_ARGUMENT;
  *count = c->launches;
  return TMNN_OK;
}

}  // extern "C"
