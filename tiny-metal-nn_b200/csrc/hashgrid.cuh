// hashgrid.cuh -- device helpers of the multiresolution hash-grid kernels
// shared by the FullyFused and Tiled families: grid cell and fraction of a
// point at one level, the corners' table offsets and interpolation weights,
// table-entry loads (fp16 or fp32 tables) and vector float reductions.
//
// Arithmetic follows the reference's generated kernels
// (mlp_kernel_emitter.cpp:224-255 cell/frac, :144-161 hash, :264-317 corner
// order dz -> dy -> dx with dw outermost and weight ((wx*wy)*wz)*wt), with
// every product rounded separately so the fp32 results match the CPU
// restatement bit for bit.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "common.cuh"

namespace tmnn {

template <int D>
struct Cell {
  int32_t bc[D];
  float frac[D];
};

template <int D>
__device__ __forceinline__ void cell_of(const float *p, float res, Cell<D> &c) {
#pragma unroll
  for (int a = 0; a < D; ++a) {
    const float s = __fmul_rn(p[a], res);
    const float fl = floorf(s);
    c.bc[a] = (int32_t)fl;
    c.frac[a] = __fsub_rn(s, fl);
  }
}

// corner k (dx fastest, then dy, dz, dw): table element offset of feature 0
// and the weight product ((wx*wy)*wz)*wt.
template <int D, int F>
__device__ __forceinline__ void corner(const Cell<D> &c, int k, uint32_t mask,
                                       uint64_t level_base, uint32_t &off,
                                       float &w) {
  const int dx = k & 1, dy = (k >> 1) & 1, dz = (k >> 2) & 1, dw = (k >> 3) & 1;
  uint32_t h;
  if (D == 4)
    h = hash4(c.bc[0] + dx, c.bc[1] + dy, c.bc[2] + dz, c.bc[D - 1] + dw, mask);
  else
    h = hash3(c.bc[0] + dx, c.bc[1] + dy, c.bc[2] + dz, mask);
  off = (uint32_t)(level_base + (uint64_t)h * F);
  const float wx = dx ? c.frac[0] : 1.0f - c.frac[0];
  const float wy = dy ? c.frac[1] : 1.0f - c.frac[1];
  const float wz = dz ? c.frac[2] : 1.0f - c.frac[2];
  w = __fmul_rn(__fmul_rn(wx, wy), wz);
  if (D == 4) {
    const float wt = dw ? c.frac[D - 1] : 1.0f - c.frac[D - 1];
    w = __fmul_rn(w, wt);
  }
}

template <int F, bool HALF>
__device__ __forceinline__ void load_table_entry(const float *table32,
                                                 const __half *table16,
                                                 uint32_t off, float *v) {
  if (HALF) {
    const __half *t = table16 + off;
    if (F == 1) {
      v[0] = __half2float(__ldg(t));
    } else if (F == 2) {
      const __half2 h = __ldg(reinterpret_cast<const __half2 *>(t));
      v[0] = __low2float(h);
      v[1] = __high2float(h);
    } else {
      const uint2 u = __ldg(reinterpret_cast<const uint2 *>(t));
      const __half2 a = *reinterpret_cast<const __half2 *>(&u.x);
      const __half2 b = *reinterpret_cast<const __half2 *>(&u.y);
      v[0] = __low2float(a);
      v[1] = __high2float(a);
      v[2] = __low2float(b);
      v[3] = __high2float(b);
    }
  } else {
    const float *t = table32 + off;
    if (F == 1) {
      v[0] = __ldg(t);
    } else if (F == 2) {
      const float2 f = __ldg(reinterpret_cast<const float2 *>(t));
      v[0] = f.x;
      v[1] = f.y;
    } else {
      const float4 f = __ldg(reinterpret_cast<const float4 *>(t));
      v[0] = f.x;
      v[1] = f.y;
      v[2] = f.z;
      v[3] = f.w;
    }
  }
}

__device__ __forceinline__ void red_add_f32x2(float *addr, float a, float b) {
  asm volatile("red.relaxed.gpu.global.add.v2.f32 [%0], {%1, %2};" ::"l"(addr),
               "f"(a), "f"(b)
               : "memory");
}
__device__ __forceinline__ void red_add_f32x4(float *addr, float a, float b,
                                              float c, float d) {
  asm volatile(
      "red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr),
      "f"(a), "f"(b), "f"(c), "f"(d)
      : "memory");
}

// fp16 hash-gradient reductions of values already scaled by
// kHalfGradScale (noftz keeps subnormal sums).  A contribution whose fp16
// rounding is all zero adds the smallest subnormal 2^-24 instead (true
// scale 2^-42), so every slot that received a contribution holds a nonzero
// sum: the implicit touch mark of the float formats, which Adam reads as
// "touched", and below any weight's ulp.
__device__ __forceinline__ uint32_t half2_bits_marked(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  uint32_t u = *reinterpret_cast<const uint32_t *>(&h);
  if ((u & 0x7fff7fffu) == 0u) u = 0x00000001u;
  return u;
}
__device__ __forceinline__ void red_add_f16x2(__half *addr, float a, float b) {
  asm volatile("red.relaxed.gpu.global.add.noftz.f16x2 [%0], %1;" ::"l"(addr),
               "r"(half2_bits_marked(a, b))
               : "memory");
}
__device__ __forceinline__ void red_add_f16x4(__half *addr, float a, float b,
                                              float c, float d) {
  const __half2 h0 = __floats2half2_rn(a, b), h1 = __floats2half2_rn(c, d);
  uint32_t u0 = *reinterpret_cast<const uint32_t *>(&h0);
  const uint32_t u1 = *reinterpret_cast<const uint32_t *>(&h1);
  if (((u0 | u1) & 0x7fff7fffu) == 0u) u0 = 0x00000001u;
  asm volatile("red.relaxed.gpu.global.add.noftz.v2.f16x2 [%0], {%1, %2};" ::"l"(addr),
               "r"(u0), "r"(u1)
               : "memory");
}
__device__ __forceinline__ void red_add_f16(__half *addr, float a) {
  const __half h = __float2half_rn(a);
  uint16_t u = *reinterpret_cast<const uint16_t *>(&h);
  if ((u & 0x7fffu) == 0u) u = 0x0001u;
  asm volatile("red.relaxed.gpu.global.add.noftz.f16 [%0], %1;" ::"l"(addr),
               "h"(u)
               : "memory");
}

// Implicit touch mark of an all-zero contribution to the fp32 format: the
// smallest normal float (float reductions flush subnormals).  The fp16
// format marks inside its reductions (above), so it needs none here.
__device__ __forceinline__ float touch_mark(int half) {
  return half ? 0.0f : __int_as_float(0x00800000);
}

// One corner's float contribution gv[F] (true scale) into the hash
// gradients at element off: fp32 vector reductions, or fp16 ones of the
// values times kHalfGradScale when half is set (gh then holds __half).
template <int F>
__device__ __forceinline__ void red_grad(float *gh, bool half, uint32_t off,
                                         const float *gv) {
  if (half) {
    __half *hp = reinterpret_cast<__half *>(gh) + off;
    if (F == 2)
      red_add_f16x2(hp, gv[0] * kHalfGradScale, gv[F - 1] * kHalfGradScale);
    else if (F == 4)
      red_add_f16x4(hp, gv[0] * kHalfGradScale, gv[1 % F] * kHalfGradScale,
                    gv[2 % F] * kHalfGradScale, gv[3 % F] * kHalfGradScale);
    else
      red_add_f16(hp, gv[0] * kHalfGradScale);
    return;
  }
  if (F == 2)
    red_add_f32x2(gh + off, gv[0], gv[F - 1]);
  else if (F == 4)
    red_add_f32x4(gh + off, gv[0], gv[1 % F], gv[2 % F], gv[3 % F]);
  else
    atomicAdd(gh + off, gv[0]);
}

}  // namespace tmnn
