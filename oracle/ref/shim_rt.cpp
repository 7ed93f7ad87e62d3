// Per-thread barriers and simdgroup state used by metal_shim.h (test
// infrastructure).
#include "metal_shim.h"
thread_local std::barrier<> *metal::g_tg_barrier = nullptr;
thread_local std::barrier<> *metal::g_simd_barrier = nullptr;
thread_local unsigned metal::g_simd_lane = 0;
thread_local float *metal::g_simd_scratch = nullptr;
