// tiled.cu -- the Tiled family (network_planning.h:29-33 TiledMetal: encode,
// MLP and scatter as separate dispatches), laid out for B200's L2.
//
// The FullyFused kernel maps threads to points and walks all L levels per
// point; when the tables overflow the 126 MB L2 (the 4D field: 268 MB fp16
// gather copy, 537 MB fp32 gradients) every fine-level corner is then a
// random HBM sector.  Here the two hash-grid kernels are level-major: block
// b of a launch works on level b / blocks_per_level, so the CTAs resident
// at any moment cover about one level, whose slice of the table (T * F
// entries) and of the gradients is all that is being touched.  The slices
// fit in L2, so the gathers and the reductions hit L2 after the first touch
// of each sector and HBM sees each slice about once.
//
//   k_tiled_encode   one point per thread: cell, 2^d corners, n-linear
//                    interpolation in the reference's order (the same
//                    arithmetic as the fused kernel's encode), fp16 out;
//   (MLP)            k_fused<D = 0> training: tcgen05 forward, loss,
//                    backward, weight gradients in TMEM, dL/d(features);
//   k_tiled_scatter  one point per thread: d_feature * corner weight into
//                    the level's gradients (warp-aggregated on coarse
//                    levels, where the Morton-sorted lanes of a warp share
//                    corners).
#include <cuda_fp16.h>

#include <cstdlib>
#include <stdexcept>
#include <string>

#include "hashgrid.cuh"
#include "tiled.h"

namespace tmnn {
namespace {

// TMNN_TILED_PREFETCH=0 turns the next-level L2 prefetch off (for
// measurements); default on.
int prefetch_enabled() {
  static const int on = [] {
    const char *e = std::getenv("TMNN_TILED_PREFETCH");
    return e && e[0] == '0' ? 0 : 1;
  }();
  return on;
}

constexpr int kThreads = 256;
// Levels whose resolution is at most this are scattered with warp
// aggregation (as in the fused kernel).
constexpr float kAggMaxRes = 24.0f;

struct TiledParams {
  NetDims nd;
  const float *pos;
  const float *table32;
  const __half *table16;
  __half *feat;
  const float *dfeat;
  float *gh_float;
  int32_t *gh_fixed;
  uint8_t *touched;
  uint32_t N;
  uint32_t blocks_per_level;
  int level0;  // level of the launch's first block (scatter of a level range)
  int implicit_touch;
  int prefetch;  // stage the next level's slice into L2 ahead of its blocks
};

// Bulk prefetch of a contiguous byte range into L2 (TMA unit, no data
// returned to the SM).  Address and size are multiples of 16 bytes.
__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p),
               "r"(bytes)
               : "memory");
}

// Block b of level l prefetches its 1/blocks_per_level share of level l+1's
// slice of `base` (slice_bytes per level), so the next level's first
// touches find their sectors in L2.
__device__ __forceinline__ void prefetch_next_level(const TiledParams &P,
                                                    const void *base,
                                                    uint64_t slice_bytes,
                                                    int l, int levels) {
  if (!P.prefetch || threadIdx.x != 0 || l + 1 >= levels) return;
  const uint64_t chunk =
      ((slice_bytes + P.blocks_per_level - 1) / P.blocks_per_level + 15) & ~15ull;
  const uint64_t start = (uint64_t)(blockIdx.x % P.blocks_per_level) * chunk;
  if (start >= slice_bytes) return;
  const uint64_t n = slice_bytes - start < chunk ? slice_bytes - start : chunk;
  prefetch_l2(reinterpret_cast<const uint8_t *>(base) +
                  (uint64_t)(l + 1) * slice_bytes + start,
              (uint32_t)n);
}

// Scalar loads: positions may be a caller's device array with 4-byte
// alignment only.
template <int D>
__device__ __forceinline__ void load_pos(const TiledParams &P, uint32_t i,
                                         float *p) {
#pragma unroll
  for (int a = 0; a < D; ++a) p[a] = __ldg(P.pos + (size_t)i * D + a);
}

template <int D, int F, bool HALF>
__global__ void __launch_bounds__(kThreads)
    k_tiled_encode(const __grid_constant__ TiledParams P) {
  const NetDims &nd = P.nd;
  const int l = (int)(blockIdx.x / P.blocks_per_level);
  if (HALF)
    prefetch_next_level(P, P.table16, (uint64_t)nd.T * F * 2, l, nd.L);
  else
    prefetch_next_level(P, P.table32, (uint64_t)nd.T * F * 4, l, nd.L);
  const uint32_t i =
      (blockIdx.x % P.blocks_per_level) * kThreads + threadIdx.x;
  if (i >= P.N) return;
  constexpr int NC = 1 << D;
  float p[4];
  load_pos<D>(P, i, p);
  Cell<D> c;
  cell_of<D>(p, nd.res[l], c);
  const uint64_t lb = (uint64_t)l * nd.T * F;
  uint32_t offs[NC];
  float ws[NC];
#pragma unroll
  for (int k = 0; k < NC; ++k) corner<D, F>(c, k, nd.T - 1u, lb, offs[k], ws[k]);
  float vals[NC][F];
#pragma unroll
  for (int k = 0; k < NC; ++k)
    load_table_entry<F, HALF>(P.table32, P.table16, offs[k], vals[k]);
  float f[F];
#pragma unroll
  for (int q = 0; q < F; ++q) {
    float a = 0.f;
#pragma unroll
    for (int k = 0; k < NC; ++k) a = __fadd_rn(a, __fmul_rn(ws[k], vals[k][q]));
    f[q] = a;
  }
  __half *dst = P.feat + (size_t)i * nd.In + l * F;
  if (F == 1) {
    *dst = __float2half_rn(f[0]);
  } else if (F == 2) {
    *reinterpret_cast<__half2 *>(dst) = __floats2half2_rn(f[0], f[F - 1]);
  } else {
    __half2 h[2] = {__floats2half2_rn(f[0], f[1 % F]),
                    __floats2half2_rn(f[2 % F], f[3 % F])};
    *reinterpret_cast<uint2 *>(dst) = *reinterpret_cast<uint2 *>(h);
  }
}

template <int D, int F>
__global__ void __launch_bounds__(kThreads)
    k_tiled_scatter(const __grid_constant__ TiledParams P) {
  __shared__ float stage[kThreads / 32][64];
  const NetDims &nd = P.nd;
  const int l = P.level0 + (int)(blockIdx.x / P.blocks_per_level);
  if (l >= nd.active_levels) return;  // uniform over the block
  if (nd.grad_fixed)
    prefetch_next_level(P, P.gh_fixed, (uint64_t)nd.T * F * 4, l, nd.active_levels);
  else
    prefetch_next_level(P, P.gh_float, (uint64_t)nd.T * F * (nd.grad_half ? 2 : 4),
                        l, nd.active_levels);
  const uint32_t i =
      (blockIdx.x % P.blocks_per_level) * kThreads + threadIdx.x;
  const bool valid = i < P.N;
  const unsigned vmask = __ballot_sync(0xffffffffu, valid);
  if (!valid) return;
  const int lane = threadIdx.x & 31;
  float *sa = stage[threadIdx.x >> 5];
  float p[4];
  load_pos<D>(P, i, p);
  float dfe[F];
  const float *src = P.dfeat + (size_t)i * nd.In + l * F;
  if (F == 2) {
    const float2 v = __ldg(reinterpret_cast<const float2 *>(src));
    dfe[0] = v.x;
    dfe[F - 1] = v.y;
  } else if (F == 4) {
    const float4 v = __ldg(reinterpret_cast<const float4 *>(src));
    dfe[0] = v.x;
    dfe[1 % F] = v.y;
    dfe[2 % F] = v.z;
    dfe[3 % F] = v.w;
  } else {
    dfe[0] = __ldg(src);
  }
  Cell<D> c;
  cell_of<D>(p, nd.res[l], c);
  const uint64_t lb = (uint64_t)l * nd.T * F;
  const bool aggregate = F == 2 && nd.res[l] <= kAggMaxRes;
#pragma unroll
  for (int k = 0; k < (1 << D); ++k) {
    uint32_t off;
    float w;
    corner<D, F>(c, k, nd.T - 1u, lb, off, w);
    if (nd.grad_fixed) {
#pragma unroll
      for (int q = 0; q < F; ++q)
        atomicAdd(P.gh_fixed + off + q,
                  fixed_trunc(__fmul_rn(__fmul_rn(dfe[q], w), kGradScale)));
    } else {
      float gv[F];
      bool zero = true;
#pragma unroll
      for (int q = 0; q < F; ++q) {
        gv[q] = dfe[q] * w;
        zero = zero && gv[q] == 0.f;
      }
      if (P.implicit_touch && zero) {
        // an all-zero contribution still touches its slot: it adds the
        // smallest normal float 2^-126 (reductions flush subnormals) so the
        // slot's sum is nonzero; the value is below any weight's ulp
#pragma unroll
        for (int q = 0; q < F; ++q)
          gv[q] = (F == 2 && q == 1) ? 0.f : touch_mark(nd.grad_half);
      }
      if (aggregate) {
        // lanes with the same corner hand their contributions to the lowest
        // such lane, which issues one reduction for the group
        const unsigned peers = __match_any_sync(vmask, off);
        sa[2 * lane] = gv[0];
        sa[2 * lane + 1] = gv[F - 1];
        __syncwarp(vmask);
        if (lane == __ffs(peers) - 1) {
          float a = 0.f, b = 0.f;
          for (unsigned m = peers; m; m &= m - 1) {
            const int s = __ffs(m) - 1;
            a += sa[2 * s];
            b += sa[2 * s + 1];
          }
          const float ab[2] = {a, b};
          red_grad<2>(P.gh_float, nd.grad_half, off, ab);
        }
        __syncwarp(vmask);
      } else {
        red_grad<F>(P.gh_float, nd.grad_half, off, gv);
      }
      if (P.implicit_touch) continue;
    }
    if (F == 2)
      P.touched[off >> 1] = 1;
    else if (F == 4)
      *reinterpret_cast<uint32_t *>(P.touched + off) = 0x01010101u;
    else
      P.touched[off] = 1;
  }
}

using TiledFn = void (*)(TiledParams);

TiledFn pick_encode(int d, int F, bool half) {
#define TMNN_ENC(DD, FF)                                                     \
  if (d == DD && F == FF)                                                    \
    return half ? (TiledFn)k_tiled_encode<DD, FF, true>                      \
                : (TiledFn)k_tiled_encode<DD, FF, false>;
  TMNN_ENC(3, 1) TMNN_ENC(3, 2) TMNN_ENC(3, 4)
  TMNN_ENC(4, 1) TMNN_ENC(4, 2) TMNN_ENC(4, 4)
#undef TMNN_ENC
  return nullptr;
}

TiledFn pick_scatter(int d, int F) {
#define TMNN_SC(DD, FF) \
  if (d == DD && F == FF) return (TiledFn)k_tiled_scatter<DD, FF>;
  TMNN_SC(3, 1) TMNN_SC(3, 2) TMNN_SC(3, 4)
  TMNN_SC(4, 1) TMNN_SC(4, 2) TMNN_SC(4, 4)
#undef TMNN_SC
  return nullptr;
}

NetDims mlp_dims(const NetDims &nd) {
  NetDims n0 = nd;
  n0.d = 0;
  n0.hash_count = 0;
  return n0;
}

}  // namespace

bool tiled_supported(const NetDims &nd, std::string *why) {
  if (nd.d != 3 && nd.d != 4) {
    if (why) *why = "spatial dims must be 3 or 4";
    return false;
  }
  return fused_mlp_train_supported(mlp_dims(nd), why) &&
         fused_mlp_supported(mlp_dims(nd), why);
}

int tiled_encode(const NetDims &nd, const float *table32,
                 const __half *table16, const float *pos, __half *feat,
                 uint32_t N, cudaStream_t st) {
  if (N == 0) return 0;
  TiledFn fn = pick_encode(nd.d, nd.F, table16 != nullptr);
  if (!fn) throw std::runtime_error("tiled: no encode kernel for this shape");
  TiledParams P{};
  P.nd = nd;
  P.pos = pos;
  P.table32 = table32;
  P.table16 = table16;
  P.feat = feat;
  P.N = N;
  P.prefetch = prefetch_enabled();
  P.blocks_per_level = (N + kThreads - 1) / kThreads;
  fn<<<P.blocks_per_level * (uint32_t)nd.L, kThreads, 0, st>>>(P);
  return 1;
}

int tiled_scatter(const NetDims &nd, const float *pos, const float *dfeat,
                  int32_t *gh_fixed, float *gh_float, uint8_t *touched,
                  uint32_t N, bool implicit_touch, cudaStream_t st, int l0,
                  int l1) {
  const int active = nd.active_levels < nd.L ? nd.active_levels : nd.L;
  if (l1 < 0 || l1 > active) l1 = active;
  if (l0 < 0) l0 = 0;
  if (N == 0 || l1 <= l0) return 0;
  TiledFn fn = pick_scatter(nd.d, nd.F);
  if (!fn) throw std::runtime_error("tiled: no scatter kernel for this shape");
  TiledParams P{};
  P.nd = nd;
  P.pos = pos;
  P.dfeat = dfeat;
  P.gh_fixed = gh_fixed;
  P.gh_float = gh_float;
  P.touched = touched;
  P.N = N;
  P.implicit_touch = implicit_touch ? 1 : 0;
  P.prefetch = prefetch_enabled();
  P.blocks_per_level = (N + kThreads - 1) / kThreads;
  P.level0 = l0;
  fn<<<P.blocks_per_level * (uint32_t)(l1 - l0), kThreads, 0, st>>>(P);
  return 1;
}

int tiled_train(FusedWorkspace &ws, const NetDims &nd, const float *params,
                const __half *table_h, const float *pos, const float *tgt,
                const float *dext, float inv_N, float *gm, int32_t *gh_fixed,
                float *gh_float, uint8_t *touched, double *loss_acc,
                __half *feat, float *dfeat, uint32_t N, int num_sms,
                cudaStream_t st, bool implicit_touch) {
  if (N == 0) return 0;
  int launches = tiled_encode(nd, params, table_h, pos, feat, N, st);
  launches += fused_mlp_train(ws, nd, params + nd.hash_count, feat, tgt, dext,
                              inv_N, gm, loss_acc, dfeat, N, num_sms, st, 0);
  launches += tiled_scatter(nd, pos, dfeat, gh_fixed, gh_float, touched, N,
                            implicit_touch, st);
  return launches;
}

int tiled_forward(FusedWorkspace &ws, const NetDims &nd, const float *params,
                  const __half *table_h, const float *pos, float *out,
                  __half *feat, uint32_t N, int num_sms, cudaStream_t st) {
  if (N == 0) return 0;
  int launches = tiled_encode(nd, params, table_h, pos, feat, N, st);
  launches += fused_mlp_forward(ws, nd, params + nd.hash_count, feat, out, N,
                                num_sms, st, 0);
  return launches;
}

}  // namespace tmnn
