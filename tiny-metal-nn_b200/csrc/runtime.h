// runtime.h -- internal interfaces between the C ABI (runtime.cu), the JSON
// front end (json_config.cpp), the planner and the kernel families.
#pragma once
#include <stdint.h>

#include <string>

#include "../../include/tmnn_cuda.h"

namespace tmnn {

// json_config.cpp
void config_from_json(uint32_t n_input, uint32_t n_output, const char *text,
                      tmnn_spec *spec, tmnn_train_cfg *cfg);

// Data-parallel helpers for objects built on a context (nerf.cu): the
// context's rank count, and an in-place sum over its ranks on its stream
// (no-op with one rank).
int ctx_world(const tmnn_ctx *c);
void ctx_allreduce_sum(tmnn_ctx *c, float *f32, size_t n32, double *f64,
                       size_t n64);

// tmnn::PlannerFallbackReason values
// (include/tiny-metal-nn/detail/network_planning.h:45-59).
enum PlannerFallbackReason : int32_t {
  kReasonNone = 0,
  kReasonNoGPUContext = 1,
  kReasonUnsupportedInputDims = 6,
  kReasonUnsupportedOutputDims = 7,
  kReasonHiddenDimUnsupported = 9,
  kReasonForcedTiled = 10,
  kReasonForcedSafeDebug = 11,
  kReasonEncodingRequiresTiledFamily = 12,
};

}  // namespace tmnn
