// Runs one emulated Metal threadgroup: `n` std::threads that share a
// std::barrier, each calling body(lid).  Test infrastructure.
#pragma once
#include <thread>
#include <vector>
#include "metal_shim.h"

template <class Body> void run_threadgroup(unsigned n, Body body) {
  std::barrier<> bar(n);
  std::vector<std::thread> ts;
  ts.reserve(n);
  for (unsigned lid = 0; lid < n; ++lid)
    ts.emplace_back([&, lid] {
      metal::g_tg_barrier = &bar;
      body(lid);
    });
  for (auto &t : ts) t.join();
}
