/*
 * tmnn_cuda.h -- C ABI of the B200 (sm_100a) implementation of
 * tiny-metal-nn's neural-field hot path: multiresolution HashGrid encoding,
 * FullyFusedMLP forward/backward and fused Adam, with the training-step
 * lifecycle around them.
 *
 * This ABI replaces tmnn's Metal device seam and runtime root:
 *   - src/tiny_metal_nn/runtime/metal_device.h:60-164 (probe, buffers,
 *     command buffers, compile_pipeline, encode_dispatch, blit fill/copy),
 *   - include/tiny-metal-nn/metal_context.h:105-149 (MetalContext) with its
 *     pipeline registry / prewarm and command-batch pool,
 * and is what tmnn's ITrainerRuntime implementation
 * (include/tiny-metal-nn/trainer.h:136-219, DefaultRuntime in
 * src/tiny_metal_nn/runtime/default_trainer.cpp:836-2414) calls instead.
 * Each entry point below cites the reference interface it replaces.
 *
 * Conventions
 *   - Every function returns tmnn_status (0 = OK) and never throws.  The
 *     message of the last failure on the calling thread is returned by
 *     tmnn_cuda_last_error().
 *   - Host arrays are float32, row-major: positions [N x spatial_dims],
 *     targets / outputs / d_output [N x num_outputs].  With TMNN_PTR_DEVICE
 *     in `flags` the same arguments are CUDA device pointers (zero copy).
 *   - One context = one GPU = one CUDA stream.  Calls on one context are
 *     serialised by the caller; a concurrent call fails with
 *     TMNN_ERR_CONCURRENT_CALL (the reference's in-flight guard,
 *     src/python/tmnn_pybind.cpp training_step).
 */
#ifndef TMNN_CUDA_H
#define TMNN_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TMNN_CUDA_ABI_VERSION 1

/* Status codes mirror tmnn::DiagnosticCode
 * (include/tiny-metal-nn/diagnostics.h:36-54). */
typedef enum tmnn_status {
  TMNN_OK = 0,
  TMNN_ERR_INVALID_ARGUMENT = 1,
  TMNN_ERR_NULL_OBJECT = 2,
  TMNN_ERR_GPU_UNAVAILABLE = 8,
  TMNN_ERR_KERNEL_UNAVAILABLE = 10,
  TMNN_ERR_UNSUPPORTED_OPERATION = 11,
  TMNN_ERR_CONFIGURATION_CONFLICT = 14,
  TMNN_ERR_SCHEMA_MISMATCH = 15,
  TMNN_ERR_OPERATION_FAILED = 16,
  TMNN_ERR_CONCURRENT_CALL = 17,
  TMNN_ERR_CAPACITY = 18
} tmnn_status;

typedef enum tmnn_loss { TMNN_LOSS_L2 = 0, TMNN_LOSS_L1 = 1,
                         TMNN_LOSS_HUBER = 2, TMNN_LOSS_COSINE = 3 } tmnn_loss;

/* Network families: tmnn::NetworkFamily
 * (include/tiny-metal-nn/detail/network_planning.h:29-33). */
typedef enum tmnn_family {
  TMNN_FAMILY_AUTO = -1,
  TMNN_FAMILY_FULLY_FUSED = 0, /* one persistent tcgen05 kernel per step */
  TMNN_FAMILY_TILED = 1,       /* encode / MLP / scatter as separate kernels */
  TMNN_FAMILY_SAFE_DEBUG = 2   /* fp32 CUDA-core kernels, reference order,
                                  bounds-checked table indices */
} tmnn_family;

/* Hash-table gradient format.  FIXED16 is the reference's int32 fixed point
 * (int(d*w*65536), truncation; mlp_kernel_emitter.cpp:20, :735-738).  F32 is
 * a float accumulator for batches where 2^-16 quantisation underflows.  F16
 * accumulates d*w*2^18 in fp16 with fp16x2 vector reductions (half the
 * scatter, clear and exchange bytes of F32); a slot's summed gradient must
 * stay below 65504 / 2^18 = 0.25 in magnitude (an overflow is an Inf that the
 * numerics guard reports).  F16 runs in the tensor-core families (FullyFused,
 * Tiled) and in SafeDebug; the buffer view of TMNN_BUF_GRAD_HASH is then
 * dtype 1 (fp16) holding the scaled values. */
typedef enum tmnn_grad_format {
  TMNN_GRAD_FIXED16 = 0,
  TMNN_GRAD_F32 = 1,
  TMNN_GRAD_F16 = 2
} tmnn_grad_format;

typedef enum tmnn_dtype { TMNN_DTYPE_F32 = 0, TMNN_DTYPE_F16 = 1 } tmnn_dtype;

/* KernelSpec fields the hot path needs (include/tiny-metal-nn/kernels/
 * kernel_spec.h:17-58), validated with kernel_spec.cpp:12-44's limits. */
typedef struct tmnn_spec {
  int32_t n_levels;             /* L, [1, 32] */
  int32_t n_features_per_level; /* F, {1, 2, 4} */
  int32_t log2_hashmap_size;    /* [10, 24] */
  int32_t spatial_dims;         /* 3 or 4 */
  float base_resolution;
  float per_level_scale;
  int32_t hidden_dim;           /* (0, 512] */
  int32_t num_hidden_layers;    /* [1, 8] */
  int32_t num_outputs;          /* >= 1 */
  int32_t loss;                 /* tmnn_loss */
  float huber_delta;
  int32_t table_dtype;          /* tmnn_dtype of the gather copy of the
                                   table; master weights are always fp32 */
} tmnn_spec;

/* TrainerConfig + WeightInitConfig (include/tiny-metal-nn/trainer.h:34-61,
 * include/tiny-metal-nn/weight_init.h:113-141) plus this build's knobs. */
typedef struct tmnn_train_cfg {
  int32_t batch_size;
  float lr_encoding, lr_network, beta1, beta2, epsilon, l1_reg, l2_reg;
  float grad_clip, weight_decay;
  /* weight init */
  int32_t hash_init;            /* 0 Uniform, 1 Zero */
  float hash_init_range;
  int32_t mlp_init;             /* 0 KaimingUniform 1 KaimingNormal
                                   2 XavierUniform 3 XavierNormal 4 Uniform
                                   5 Normal 6 Zero */
  int32_t mlp_nonlinearity;     /* 0 Linear 1 ReLU 2 LeakyReLU 3 Tanh 4 Sigmoid */
  float mlp_uniform_range, mlp_normal_stddev, mlp_kaiming_a;
  uint64_t seed;
  /* execution */
  int32_t family;               /* tmnn_family */
  int32_t hash_grad_format;     /* tmnn_grad_format */
  int32_t morton_sort;          /* 1: Morton-sort every training batch */
  int32_t sparse_hash_adam;     /* -1 auto (sparse iff l1_reg == 0), 0, 1 */
  int32_t active_levels;        /* <= 0: all levels receive gradients */
  int32_t dp_replicated_optimizer; /* 1: every rank runs the full Adam after
                                      one allreduce; 0 (default): from 4
                                      ranks on, Adam is sharded over the
                                      ranks (reduce-scatter, Adam on 1/world
                                      of the table, all-gather); -1: sharded
                                      from 2 ranks on */
  /* numerics guard (RuntimePolicy, include/tiny-metal-nn/runtime_policy.h:
   * 13-40; defaults from TMNN_NUMERICS_SAMPLING_MODE,
   * TMNN_NUMERICS_SAMPLE_INTERVAL, TMNN_BAD_STEP_MODE like
   * load_runtime_policy, src/tiny_metal_nn/runtime/runtime_policy.h:144-175) */
  int32_t numerics_sampling_mode; /* tmnn_numerics_sampling */
  int32_t numerics_sample_interval; /* steps between sampled probes (128) */
  int32_t bad_step_recovery;      /* tmnn_bad_step_recovery */
  int32_t morton_key_bits;        /* Morton sort key: the top k bits of the
                                     code (1..32); 0 = the whole code (30 bits
                                     in 3D, 32 in 4D, the reference's order up
                                     to ties).  Default 12. */
  int32_t enable_probes;          /* TrainerConfig::enable_probes
                                     (include/tiny-metal-nn/trainer.h:51-54):
                                     1 = per-step activation / gradient
                                     telemetry (tmnn_cuda_last_probe).  Like
                                     the reference, which then runs its scalar
                                     training kernel, training steps run the
                                     fp32 reference-order kernels. */
  int32_t reserved;
} tmnn_train_cfg;

/* NumericsSamplingMode (runtime_policy.h:13-18). */
typedef enum tmnn_numerics_sampling {
  TMNN_NUMERICS_SAMPLED = 0,   /* steps 0 and 1, every interval, after an anomaly */
  TMNN_NUMERICS_PERIODIC = 1,  /* every interval, after an anomaly */
  TMNN_NUMERICS_FULL = 2,      /* every step */
  TMNN_NUMERICS_DISABLED = 3   /* only when the loss is not finite */
} tmnn_numerics_sampling;

/* BadStepRecoveryMode (runtime_policy.h:20-26) and BadStepRecoveryAction
 * (include/tiny-metal-nn/common.h:71-76). */
typedef enum tmnn_bad_step_recovery {
  TMNN_BAD_STEP_SIGNAL_ONLY = 0,
  TMNN_BAD_STEP_THROW = 1,
  TMNN_BAD_STEP_SKIP = 2,
  TMNN_BAD_STEP_ROLLBACK = 3,
  TMNN_BAD_STEP_SAFE_FAMILY_RETRY = 4
} tmnn_bad_step_recovery;
typedef enum tmnn_recovery_action {
  TMNN_RECOVERY_NONE = 0,
  TMNN_RECOVERY_SKIPPED = 1,
  TMNN_RECOVERY_ROLLED_BACK = 2,
  TMNN_RECOVERY_RETRIED_WITH_SAFE_FAMILY = 3
} tmnn_recovery_action;

/* TrainingStepResult (include/tiny-metal-nn/common.h:97-110), reduced. */
typedef struct tmnn_step_result {
  float loss;          /* mean loss over the (global) batch */
  uint32_t step;       /* logical step that completed */
  uint32_t batch_size; /* points processed by this rank */
  int32_t numerics_ok; /* 1 when loss and update were finite */
  float gpu_ms;        /* device time of the step (TMNN_PROFILE) */
  int32_t family;      /* family that ran */
  float sort_ms;       /* device time of upload + Morton sort (TMNN_PROFILE) */
  float fwd_bwd_ms;    /* device time of forward/backward/scatter */
  float allreduce_ms;  /* device time of the gradient allreduce */
  float adam_ms;       /* device time of Adam + gradient reset */
  /* NumericsReport (include/tiny-metal-nn/detail/runtime_stats.h:32-40) of
   * the step, from the device probe; backward/update fields are meaningful
   * when numerics_probed is 1 */
  float grad_norm;            /* sqrt(sum g^2) over finite gradients */
  int32_t finite_forward;
  int32_t finite_backward;
  int32_t finite_update;
  float max_abs_gradient;
  float max_abs_update;
  int32_t numerics_probed;    /* the probe scanned this step's gradients */
  int32_t numerics_reported;  /* the guard recorded this step */
  int32_t has_numerics_anomaly;
  int32_t recovery_action;    /* tmnn_recovery_action */
} tmnn_step_result;

/* ProbeResult (include/tiny-metal-nn/common.h:78-94): statistics of the
 * last forward/backward pass with enable_probes set, over the points of this
 * rank.  act_max[l] = max |activation| of hidden layer l; grad_l2[l] = sum
 * over points of |dL/d(pre-activation of layer l)|^2; output_abs_max = max
 * |output|; output_min = min(0, min output) for one output and 0 otherwise
 * (the reference's TG reduction starts at 0); hash_grad_l2 stays 0 as in the
 * reference, whose kernel never accumulates it. */
typedef struct tmnn_probe_result {
  uint32_t num_hidden_layers;
  int32_t has_nan_forward, has_nan_backward;
  float hash_grad_l2;
  float act_max[8];
  float grad_l2[8];
  float output_abs_max, output_min;
} tmnn_probe_result;

/* Counters of the numerics guard (context_record_training_step,
 * training_step_execution.cpp:1047-1058). */
typedef struct tmnn_numerics_stats {
  uint64_t reports, anomalies, skipped, rolled_back, safe_family_recoveries;
  uint32_t last_anomaly_step;
  int32_t safe_family_active; /* 1 after a FallbackAndRetry switched family */
} tmnn_numerics_stats;

/* RuntimeBufferRole (include/tiny-metal-nn/detail/runtime_authority.h:68-79) */
typedef enum tmnn_buffer_role {
  TMNN_BUF_HASH_WEIGHTS = 1,
  TMNN_BUF_MLP_WEIGHTS = 2,
  TMNN_BUF_GRAD_HASH = 3,
  TMNN_BUF_GRAD_MLP = 4,
  TMNN_BUF_FUSED_WEIGHTS = 7,
  TMNN_BUF_FUSED_M = 8,
  TMNN_BUF_FUSED_V = 9,
  TMNN_BUF_HASH_GATHER = 20, /* fp16 gather copy (table_dtype == F16) */
  TMNN_BUF_TOUCHED = 21      /* u8 per tracked slot (pair when F == 2) */
} tmnn_buffer_role;

typedef struct tmnn_buffer_view {
  void *device_ptr;
  size_t bytes;
  int32_t dtype; /* 0 f32, 1 f16, 2 i32, 3 u8 */
} tmnn_buffer_view;

/* NetworkPlan (include/tiny-metal-nn/detail/network_planning.h:120-174). */
typedef struct tmnn_plan {
  int32_t family;          /* selected tmnn_family */
  int32_t fallback_reason; /* tmnn::PlannerFallbackReason value */
  uint32_t mlp_weight_count;
  uint64_t hash_grid_size;
  uint64_t device_bytes;   /* resident device memory of the context */
  int32_t n_levels, n_features_per_level, spatial_dims, num_outputs;
  char reason[128];
} tmnn_plan;

#define TMNN_PTR_DEVICE 1u  /* array arguments are device pointers */
#define TMNN_PROFILE 2u     /* time the step with CUDA events */

typedef struct tmnn_ctx tmnn_ctx;

/* Defaults of TrainerConfig / WeightInitConfig. */
void tmnn_cuda_default_train_cfg(tmnn_train_cfg *cfg);
/* KernelSpec::validate (kernel_spec.cpp:12-44).  Message via last_error. */
tmnn_status tmnn_cuda_validate_spec(const tmnn_spec *spec);

/* MetalContext::create + DefaultRuntime ctor (default_trainer.cpp:836-869):
 * allocates the parameter store, runs the Philox weight init, zeroes Adam. */
tmnn_status tmnn_cuda_ctx_create(int device, const tmnn_spec *spec,
                                 const tmnn_train_cfg *cfg, tmnn_ctx **out);
/* try_create_from_config (include/tiny-metal-nn/factory_json.h:284-361):
 * tcnn-style JSON {encoding, network, loss, optimizer, weight_init,
 * batch_size}; plus an optional "b200" object for this build's knobs. */
tmnn_status tmnn_cuda_ctx_create_from_json(int device, uint32_t n_input,
                                           uint32_t n_output, const char *json,
                                           tmnn_ctx **out);
/* ~DefaultRuntime (drains the stream, releases device memory). */
tmnn_status tmnn_cuda_ctx_destroy(tmnn_ctx *ctx);

/* ITrainerRuntime::set_initial_weights (trainer.h:186-196): also resets the
 * optimizer state and the step counter.  NULL/0 skips a buffer. */
tmnn_status tmnn_cuda_set_initial_weights(tmnn_ctx *ctx, const float *hash,
                                          size_t hash_count, const float *mlp,
                                          size_t mlp_count);
/* Host copy of the live weights (RuntimeAuthority buffer read-back). */
tmnn_status tmnn_cuda_get_weights(tmnn_ctx *ctx, float *hash, size_t hash_count,
                                  float *mlp, size_t mlp_count);

/* ITrainerRuntime::training_step (trainer.h:140-141,
 * default_trainer.cpp:883-1045): Morton sort, fused forward/backward/scatter,
 * [data-parallel gradient allreduce], Adam, gradient reset. */
tmnn_status tmnn_cuda_train_step(tmnn_ctx *ctx, const float *positions,
                                 const float *targets, uint32_t n,
                                 uint32_t flags, tmnn_step_result *result);

/* Pipelined training steps (enqueue_training_step / finalize_training_step,
 * src/tiny_metal_nn/runtime/training_step_execution.cpp:887-1235, over the
 * two step lanes of default_trainer.cpp:41).  _enqueue copies the batch into
 * one of two device lanes on a copy stream and queues the step behind it;
 * it returns without waiting.  _finalize waits for the oldest pending step
 * and fills *result (the same fields as tmnn_cuda_train_step).  At most two
 * steps may be pending; with two in flight the upload of one batch overlaps
 * the other's kernels.  Host arrays must stay unchanged until their step is
 * finalized; pinned host memory makes the copy asynchronous.  Numerics
 * recovery modes other than SignalOnly are refused (they need the host
 * between steps); tmnn_cuda_train_step refuses to run while steps are
 * pending. */
tmnn_status tmnn_cuda_train_step_enqueue(tmnn_ctx *ctx, const float *positions,
                                         const float *targets, uint32_t n,
                                         uint32_t flags);
tmnn_status tmnn_cuda_train_step_finalize(tmnn_ctx *ctx,
                                          tmnn_step_result *result);

/* The forward/backward half of training_step without the optimizer: Morton
 * sort, fused forward/backward/scatter with the internal loss, gradients
 * ACCUMULATED into the gradient buffers (the command batch that
 * submit_forward_backward_batch encodes, training_step_execution.cpp:458-508).
 * *loss_sum receives the summed (not averaged) loss of this batch. */
tmnn_status tmnn_cuda_forward_backward(tmnn_ctx *ctx, const float *positions,
                                       const float *targets, uint32_t n,
                                       uint32_t flags, double *loss_sum);

/* forward_backward for callers that cannot allocate device memory at call
 * time (a framework owning the memory pool, a fixed serving footprint, a
 * real-time loop that must not stall in the allocator).  No counterpart in
 * the reference: tmnn has no such entry point.
 * Same work and result as tmnn_cuda_forward_backward with device pointers
 * (positions and targets MUST be device pointers), but the scratch the batch
 * needs (Morton codes, permutation, sorted copies, radix-sort temporary)
 * lives in one fixed device array inside the library, about 8 MiB, that every
 * GPU which loads the library keeps until the process exits.  Nothing is
 * allocated: n is limited to 65536 points and num_outputs to 16; larger
 * requests fail with TMNN_ERR_INVALID_ARGUMENT.  The first call on a device
 * looks up the array's device address (cudaGetSymbolAddress), so make that
 * first call before any stream capture.  All calls on a device share the one
 * array, which keeps the last call's contents; calls that overlap on the GPU
 * (two contexts on one device driven from two threads) race on it.  With the
 * FullyFused family, one ordinary training_step or forward_backward must
 * have run on the context first (it sets up the fused weight image). */
tmnn_status tmnn_cuda_forward_backward_noalloc(tmnn_ctx *ctx,
                                               const float *positions,
                                               const float *targets,
                                               uint32_t n, double *loss_sum);

/* ITrainerRuntime::forward_for_training (trainer.h:145-149): outputs for an
 * external loss, in input order. */
tmnn_status tmnn_cuda_forward(tmnn_ctx *ctx, const float *positions,
                              float *outputs, uint32_t n, uint32_t flags);
/* ITrainerRuntime::zero_gradients / backward_accumulate / adam_step
 * (trainer.h:160-177; default_trainer.cpp:1300-1443). */
tmnn_status tmnn_cuda_zero_grads(tmnn_ctx *ctx);
tmnn_status tmnn_cuda_backward_accumulate(tmnn_ctx *ctx,
                                          const float *positions,
                                          const float *d_output, uint32_t n,
                                          uint32_t flags);
tmnn_status tmnn_cuda_adam_step(tmnn_ctx *ctx);

/* Trainer::evaluate -> DefaultEvaluator::evaluate
 * (default_trainer.cpp:321-465). */
tmnn_status tmnn_cuda_evaluate(tmnn_ctx *ctx, const float *positions,
                               float *outputs, uint32_t n, uint32_t flags);

/* Trainer::evaluate_with_gradient / inference_with_gradient
 * (trainer.h:378-386) -> FieldEvaluator::evaluate_with_gradient
 * (evaluator.h:45; default_trainer.cpp:467-622) and the EvalGradient kernel
 * (mlp_kernel_emitter.cpp:1716-2090).  For a single-output network
 * (num_outputs == 1, else TMNN_ERR_INVALID_ARGUMENT): outputs [n] = the field
 * value, gradients [n x spatial_dims] = d(value)/d(position), from the fp32
 * parameters.  The reference returns the two deinterleaved from one
 * [value, gx, gy, gz] buffer; here they are written separately.  n == 0 is a
 * no-op; NULL arrays with n > 0 fail like the reference.  Host pointers, or
 * device pointers with TMNN_PTR_DEVICE. */
tmnn_status tmnn_cuda_evaluate_with_gradient(tmnn_ctx *ctx,
                                             const float *positions,
                                             float *outputs, float *gradients,
                                             uint32_t n, uint32_t flags);

/* NeRF-style field (the benchmark's NeRF configuration; tmnn itself has no
 * SH encoding and no chained networks, so nothing here replaces a reference
 * entry point): a density network (the HashGrid + FullyFusedMLP of
 * `density`, 3D input, 16 outputs, sigma = exp(output 0)) and a colour
 * network on [SH degree 4 of the unit view direction (16) | density outputs
 * 1..15 | a zero pad] -> sigmoid RGB.  Loss per sample:
 * sum_c (rgb_c - rgb_t,c)^2 + (sigma - sigma_t)^2, averaged over the batch.
 * Adam (lr, beta 0.9/0.99, eps 1e-15) on both networks. */
typedef struct tmnn_nerf tmnn_nerf;
typedef struct tmnn_nerf_cfg {
  tmnn_spec density;           /* spatial_dims 3, num_outputs 16 */
  float lr;
  uint32_t color_width;        /* 64 or 128 */
  uint32_t color_hidden_layers;/* 1..4 */
  int32_t family;              /* density network family (tmnn_family) */
  uint64_t seed;
} tmnn_nerf_cfg;
tmnn_status tmnn_cuda_nerf_create(int device, const tmnn_nerf_cfg *cfg,
                                  tmnn_nerf **out);
tmnn_status tmnn_cuda_nerf_destroy(tmnn_nerf *nerf);
/* The density network's context (owned by the nerf object): weights,
 * buffers and plan through the tmnn_cuda_* context calls. */
tmnn_status tmnn_cuda_nerf_density(tmnn_nerf *nerf, tmnn_ctx **density);
/* Colour network weights in the reference MLP layout (fp32); writing them
 * resets its Adam state. */
tmnn_status tmnn_cuda_nerf_color_weights(tmnn_nerf *nerf, const float *host_in,
                                         float *host_out, size_t count);
/* One training step on n samples: positions [n x 3], unit directions
 * [n x 3], target RGB [n x 3], target density [n]; *loss = mean loss.  Host
 * pointers, or device pointers with TMNN_PTR_DEVICE. */
tmnn_status tmnn_cuda_nerf_train_step(tmnn_nerf *nerf, const float *positions,
                                      const float *directions,
                                      const float *rgb, const float *sigma,
                                      uint32_t n, uint32_t flags, float *loss);
/* Data-parallel training of the field (no reference counterpart): the same
 * unique id / rank / world as tmnn_cuda_dp_init.  Each rank trains on its
 * shard of every batch; the colour network's gradients and the losses are
 * summed over the ranks before its Adam step, the density network exchanges
 * its own gradients, and all means are over the global batch. */
tmnn_status tmnn_cuda_nerf_dp_init(tmnn_nerf *nerf, const uint8_t unique_id[128],
                                   int rank, int world);
/* rgb [n x 3] (after the sigmoid) and sigma [n] (after exp). */
tmnn_status tmnn_cuda_nerf_inference(tmnn_nerf *nerf, const float *positions,
                                     const float *directions, float *rgb,
                                     float *sigma, uint32_t n, uint32_t flags);
/* Device milliseconds of the phases of the last step run with TMNN_PROFILE
 * (phase_ms[4]: density forward + colour input; colour network train + Adam;
 * density backward_accumulate, Morton sort included; density Adam), and the
 * number of kernels this object and its density context launched. */
tmnn_status tmnn_cuda_nerf_profile(tmnn_nerf *nerf, float *phase_ms,
                                   uint64_t *launches);
const char *tmnn_cuda_nerf_last_error(void);

/* Numerics guard counters of this context. */
tmnn_status tmnn_cuda_get_numerics_stats(tmnn_ctx *ctx,
                                         tmnn_numerics_stats *out);

/* Encoding only (parity instrument): features [n x L*F] f32, and when
 * non-NULL the first table index of every corner [n x L x 2^d] (u32) and the
 * base grid cell [n x L x d] (i32). Host pointers. */
/* Morton order of a batch (parity instrument for morton_sort.h:60-110): perm
 * [n] = input index of the i-th point after the device's stable sort on the
 * top key_bits of the code (0: the whole code).  Host pointers. */
tmnn_status tmnn_cuda_debug_morton_order(tmnn_ctx *ctx, const float *positions,
                                         uint32_t n, int32_t key_bits,
                                         uint32_t *perm);

tmnn_status tmnn_cuda_debug_encode(tmnn_ctx *ctx, const float *positions,
                                   uint32_t n, float *features,
                                   uint32_t *corner_index, int32_t *cells);

/* OptimizerStateBlob v1 (default_trainer.cpp:83-100, :1645-1768;
 * docs/CHECKPOINT-CONTRACT.md:31-82): 4 sections [m_hash, v_hash, m_mlp,
 * v_mlp], each a little-endian u32 byte length then raw fp32 bytes. With
 * buf == NULL the required length is returned in *len. */
tmnn_status tmnn_cuda_export_opt_state(tmnn_ctx *ctx, uint8_t *buf, size_t cap,
                                       size_t *len, uint32_t *step);
tmnn_status tmnn_cuda_import_opt_state(tmnn_ctx *ctx, const uint8_t *buf,
                                       size_t len, uint32_t step);
/* ITrainerRuntime::reset_optimizer: zero m/v, step = 0. */
tmnn_status tmnn_cuda_reset_optimizer(tmnn_ctx *ctx);
tmnn_status tmnn_cuda_get_step(tmnn_ctx *ctx, uint32_t *step);

/* RuntimeAuthority::buffer (runtime_authority.h:110-121). */
tmnn_status tmnn_cuda_get_buffer(tmnn_ctx *ctx, int32_t role,
                                 tmnn_buffer_view *view);
/* Host copy of a whole buffer (RuntimeBufferView::cpu_data read-back);
 * bytes must equal the buffer's size. */
tmnn_status tmnn_cuda_read_buffer(tmnn_ctx *ctx, int32_t role, void *host,
                                  size_t bytes);
/* TrainingStepResult::probe / ITrainerRuntime::read_last_split_probe
 * (include/tiny-metal-nn/trainer.h:178-181, :363-366): the probe of the last
 * training_step or forward_backward.  TMNN_ERR_INVALID_ARGUMENT when
 * enable_probes is off, TMNN_ERR_OPERATION_FAILED when no pass ran yet (the
 * reference returns nullopt in both cases). */
tmnn_status tmnn_cuda_last_probe(tmnn_ctx *ctx, tmnn_probe_result *probe);
/* NetworkPlan of the context (network_planner.cpp:132-290). */
tmnn_status tmnn_cuda_get_plan(tmnn_ctx *ctx, tmnn_plan *plan);
/* The context's CUDA stream (cudaStream_t) for interop. */
tmnn_status tmnn_cuda_get_stream(tmnn_ctx *ctx, void **stream);
tmnn_status tmnn_cuda_synchronize(tmnn_ctx *ctx);

/* Data parallelism (no reference counterpart: tmnn is single-device).
 * unique_id: 128 bytes of an ncclUniqueId made by rank 0
 * (tmnn_cuda_dp_unique_id) and broadcast by the caller.  After this call
 * every train_step / adam_step sums gradients over the ranks with one NCCL
 * allreduce (and ORs the touched-slot map), and divides by the global batch. */
tmnn_status tmnn_cuda_dp_unique_id(uint8_t out[128]);
tmnn_status tmnn_cuda_dp_init(tmnn_ctx *ctx, const uint8_t unique_id[128],
                              int rank, int world);

/* From 4 ranks on the optimizer is sharded (dp_replicated_optimizer == 0):
 * each rank keeps the current fp32 table, m and v only for its 1/world shard
 * (the gather copy the kernels read is always complete).  This collective
 * call -- every rank must make it -- gathers the shards; until then
 * get_weights, export_opt_state, debug_encode and reading the weight or
 * moment buffers fail with TMNN_ERR_INVALID_ARGUMENT.  No reference
 * counterpart (tmnn is single-device). */
tmnn_status tmnn_cuda_dp_sync_state(tmnn_ctx *ctx);

/* Standalone FullyFusedMLP inference (include/tiny-metal-nn/fully_fused_mlp.h
 * evaluated without an input encoding): ReLU hidden layers, linear outputs,
 * weights in the reference layout (mlp_kernel_emitter.cpp:163-191),
 * Xavier-uniform Philox init.  Inputs are fp16 device arrays [n x n_input]
 * (16-byte aligned), outputs fp32 device arrays [n x n_output].
 * n_input a multiple of 16 up to 128; width 16/32/64/128; n_output <= 16. */
typedef struct tmnn_mlp tmnn_mlp;
tmnn_status tmnn_cuda_mlp_create(int device, uint32_t n_input, uint32_t width,
                                 uint32_t hidden_layers, uint32_t n_output,
                                 uint64_t seed, tmnn_mlp **out);
tmnn_status tmnn_cuda_mlp_destroy(tmnn_mlp *mlp);
/* Host weights in (set) and/or out (get); count = total weight count. */
tmnn_status tmnn_cuda_mlp_weights(tmnn_mlp *mlp, const float *host_in,
                                  float *host_out, size_t count);
tmnn_status tmnn_cuda_mlp_forward(tmnn_mlp *mlp, const void *input_f16,
                                  float *output, uint32_t n);
tmnn_status tmnn_cuda_mlp_stream(tmnn_mlp *mlp, void **stream);
const char *tmnn_cuda_mlp_last_error(void);

/* Message of the last failure on this thread ("" if none). */
const char *tmnn_cuda_last_error(void);
/* Kernels launched by this context since creation (instrumentation). */
tmnn_status tmnn_cuda_launch_count(tmnn_ctx *ctx, uint64_t *count);

#ifdef __cplusplus
}
#endif
#endif
