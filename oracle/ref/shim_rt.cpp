// Per-thread threadgroup barrier used by metal_shim.h (test infrastructure).
#include "metal_shim.h"
thread_local std::barrier<> *metal::g_tg_barrier = nullptr;
