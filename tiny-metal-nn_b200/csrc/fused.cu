// fused.cu -- FullyFused family (tcgen05).  Placeholder: not yet available.
#include "fused.h"

namespace tmnn {

bool fused_supported(const tmnn_spec &, const tmnn_train_cfg &,
                     std::string *why) {
  if (why) *why = "fused tcgen05 kernel not built";
  return false;
}
void fused_weights_changed(FusedWorkspace &ws) { ws.dirty = true; }
void fused_release(FusedWorkspace &ws) {
  if (ws.wpack) cudaFree(ws.wpack);
  ws.wpack = nullptr;
}
int fused_train(FusedWorkspace &, const NetDims &, const tmnn_spec &,
                const float *, const __half *, const float *, const float *,
                const float *, float, float *, int32_t *, float *, uint8_t *,
                double *, uint32_t, int, cudaStream_t) {
  return 0;
}
int fused_forward(FusedWorkspace &, const NetDims &, const tmnn_spec &,
                  const float *, const __half *, const float *, float *,
                  uint32_t, int, cudaStream_t) {
  return 0;
}

}  // namespace tmnn
