// Runs one emulated Metal threadgroup: `n` std::threads that share a
// std::barrier, each calling body(lid).  Threads 32k..32k+31 form simdgroup
// k, with their own barrier and reduction scratch.  Test infrastructure.
#pragma once
#include <memory>
#include <thread>
#include <vector>
#include "metal_shim.h"

template <class Body> void run_threadgroup(unsigned n, Body body) {
  std::barrier<> bar(n);
  const unsigned groups = (n + 31) / 32;
  std::vector<std::unique_ptr<std::barrier<>>> sbar;
  for (unsigned g = 0; g < groups; ++g)
    sbar.emplace_back(new std::barrier<>(g + 1 < groups ? 32 : n - 32 * g));
  std::vector<float> scratch(32 * groups, 0.0f);
  std::vector<std::thread> ts;
  ts.reserve(n);
  for (unsigned lid = 0; lid < n; ++lid)
    ts.emplace_back([&, lid] {
      metal::g_tg_barrier = &bar;
      metal::g_simd_barrier = sbar[lid / 32].get();
      metal::g_simd_lane = lid % 32;
      metal::g_simd_scratch = scratch.data() + 32 * (lid / 32);
      body(lid);
    });
  for (auto &t : ts) t.join();
}
