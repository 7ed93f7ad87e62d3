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

// Runs `tgs` threadgroups of `n` threads on `lanes` lanes at once.  A lane is
// a persistent set of n std::threads (one emulated threadgroup) that works
// through threadgroups lane, lane + lanes, ...; body(lane, tg, lid) must use
// threadgroup storage private to its lane (the caller compiles one copy of
// the kernel per lane).  The lane barrier after each threadgroup keeps a
// lane's next threadgroup from overwriting storage its previous one is still
// reading.  Threads are created once per call, not once per threadgroup.
template <class Body>
void run_threadgroups_lanes(unsigned lanes, unsigned n, unsigned tgs, Body body) {
  const unsigned groups = (n + 31) / 32;
  struct Lane {
    std::unique_ptr<std::barrier<>> bar;
    std::vector<std::unique_ptr<std::barrier<>>> sbar;
    std::vector<float> scratch;
  };
  std::vector<Lane> ls(lanes);
  for (auto &l : ls) {
    l.bar.reset(new std::barrier<>(n));
    for (unsigned g = 0; g < groups; ++g)
      l.sbar.emplace_back(new std::barrier<>(g + 1 < groups ? 32 : n - 32 * g));
    l.scratch.assign(32 * groups, 0.0f);
  }
  std::vector<std::thread> ts;
  ts.reserve(lanes * n);
  for (unsigned ln = 0; ln < lanes; ++ln)
    for (unsigned lid = 0; lid < n; ++lid)
      ts.emplace_back([&, ln, lid] {
        Lane &l = ls[ln];
        metal::g_tg_barrier = l.bar.get();
        metal::g_simd_barrier = l.sbar[lid / 32].get();
        metal::g_simd_lane = lid % 32;
        metal::g_simd_scratch = l.scratch.data() + 32 * (lid / 32);
        for (unsigned tg = ln; tg < tgs; tg += lanes) {
          body(ln, tg, lid);
          l.bar->arrive_and_wait();
        }
      });
  for (auto &t : ts) t.join();
}
