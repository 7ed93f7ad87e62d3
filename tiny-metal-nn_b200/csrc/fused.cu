// fused.cu -- the FullyFused family: one persistent sm_100a kernel per
// training step.  Each CTA (128 threads, one point per thread) loops over
// 128-point tiles:
//
//   encode     thread t gathers the 2^d corners of every level for point t
//              from the (fp16 or fp32) table and interpolates in fp32
//              (mlp_kernel_emitter.cpp:205-360), writing fp16 features into
//              a core-blocked shared tile X[128 x In];
//   forward    D = X.W0, H_k = relu(D + b) ..., Y = H.Wout + bout on tcgen05
//              (fp16 operands from shared memory, fp32 accumulators in TMEM;
//              thread t reads TMEM lane t = point t in the epilogues);
//   loss       L1/L2/Huber/Cosine per point (mlp_kernel_emitter.cpp:562-670);
//              dY is scaled by a power of two so fp16 keeps its precision;
//   backward   dH = (dY.Wout^T) o relu', ..., dX = dH0.W0^T on tcgen05; the
//              weight gradients dW^T = dH^T.[H | 1] (the ones column yields
//              the bias gradient) accumulate in TMEM across all tiles of the
//              CTA and are flushed once with fp32 atomics;
//   scatter    thread t recomputes its corners and adds d_feature * weight
//              into the hash-gradient buffer with vector reductions
//              (red.global.add.v2.f32 for two features) or the reference's
//              int32 fixed point, and marks the touched slots.
//
// The same kernel without the backward half is the inference path.
#include <cuda_fp16.h>

#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>

#include "fused.h"
#include "hashgrid.cuh"
#include "tc.cuh"

namespace tmnn {
namespace {

constexpr int kTile = 128;
constexpr int kThreads = 256;
constexpr int kMaxTrainHidden = 8;
constexpr int kOutCols = 16;  // output layer padded to N = 16
// Levels whose resolution is at most this are scattered with warp
// aggregation (coarse grids: many points of a Morton-sorted warp share
// corners there).
constexpr float kAggMaxRes = 24.0f;
constexpr uint32_t kAggBytes = 16 * 32 * 2 * 4;  // 16 warps x 32 lanes x 2 floats
constexpr uint32_t kWaitBound = 1u << 26;

struct Layout {
  // weight image (same bytes in global and shared memory)
  uint32_t w[kMaxHidden + 1];  // W0, W1..W(H-1), Wout (core-blocked fp16)
  uint32_t b[kMaxHidden + 1];  // fp32 biases (bout padded to 16)
  uint32_t image_bytes;
  // shared-memory homes of the weights and biases; with stream_w the hidden
  // weight matrices are copied per layer into two alternating slots
  uint32_t sw[kMaxHidden + 1], sb[kMaxHidden + 1];
  uint32_t tail_src, tail_dst, tail_bytes;
  int stream_w;
  // activation tiles
  uint32_t x, h[kMaxHidden], dy, agg, misc;
  uint32_t total;
  int xc, hc;                  // stored columns of X and H tiles
  int n_h_tiles;
  // TMEM columns
  uint32_t t_scratch, t_dw0, t_dwk[kMaxHidden], t_dwout, tmem_cols;
};

inline uint32_t align128(uint32_t v) { return (v + 127u) & ~127u; }

Layout make_layout(const NetDims &nd, bool train, bool stream = false) {
  Layout L{};
  const int In = nd.In, W = nd.W, H = nd.H;
  uint32_t off = 0;
  L.w[0] = off;
  off = align128(off + In * W * 2);
  for (int k = 1; k < H; ++k) {
    L.w[k] = off;
    off = align128(off + W * W * 2);
  }
  L.w[H] = off;
  off = align128(off + W * kOutCols * 2);
  for (int k = 0; k < H; ++k) {
    L.b[k] = off;
    off = align128(off + W * 4);
  }
  L.b[H] = off;
  off = align128(off + kOutCols * 4);
  L.image_bytes = off;
  L.stream_w = stream ? 1 : 0;
  if (!stream) {
    for (int k = 0; k <= H; ++k) {
      L.sw[k] = L.w[k];
      L.sb[k] = L.b[k];
    }
    L.tail_src = L.tail_dst = 0;
    L.tail_bytes = L.image_bytes;
  } else {
    const uint32_t slot = align128((uint32_t)(In > W ? In : W) * W * 2);
    for (int k = 0; k < H; ++k) L.sw[k] = (uint32_t)(k & 1) * slot;
    L.tail_src = L.w[H];
    L.tail_dst = 2 * slot;
    L.tail_bytes = L.image_bytes - L.w[H];
    L.sw[H] = L.tail_dst;
    for (int k = 0; k <= H; ++k) L.sb[k] = L.tail_dst + (L.b[k] - L.w[H]);
    off = L.tail_dst + L.tail_bytes;
  }
  L.xc = train ? In + 16 : In;
  // training tiles: W activation columns, a ones column block (bias
  // gradients), and at least 64 columns in all, since the weight-gradient
  // MMAs read dH^T as an M = 64 operand when W < 64
  L.hc = train ? (W + 16 > 64 ? W + 16 : 64) : W;
  L.x = off;
  off = align128(off + kTile * L.xc * 2);
  L.n_h_tiles = train ? H : (H > 1 ? 2 : 1);
  for (int k = 0; k < L.n_h_tiles; ++k) {
    L.h[k] = off;
    off = align128(off + kTile * L.hc * 2);
  }
  if (train) {
    // the pre-activation gradients of layer k overwrite H_k in place
    L.dy = off;
    off = align128(off + kTile * kOutCols * 2);
    L.agg = off;  // per-warp staging of the warp-aggregated scatter
    off = align128(off + kAggBytes);
  }
  L.misc = off;
  off = align128(off + 256);
  L.total = off;
  // TMEM
  uint32_t col = 0;
  L.t_scratch = col;
  col += (uint32_t)(W > In ? W : In);
  if (train) {
    L.t_dw0 = col;
    col += In + 16;
    for (int k = 1; k < H; ++k) {
      L.t_dwk[k] = col;
      col += W + 16;
    }
    L.t_dwout = col;
    col += kOutCols;
  }
  uint32_t alloc = 32;
  while (alloc < col) alloc <<= 1;
  L.tmem_cols = alloc;
  if (!train && !stream && L.total > 200 * 1024) return make_layout(nd, train, true);
  return L;
}

struct FusedParams {
  NetDims nd;
  Layout lay;
  const float *pos;
  const __half *xin;  // D == 0: fp16 input features [N x In] (no encoding)
  const float *tgt;
  const float *dext;
  float *out;
  const float *table32;
  const __half *table16;
  const uint8_t *wimage;
  float *gm;
  int32_t *gh_fixed;
  float *gh_float;
  uint8_t *touched;
  double *loss_acc;
  int *err;
  float inv_N;
  float dscale;      // dY scale (power of two)
  float inv_dscale;
  uint32_t N;
  uint32_t ntiles;
  int mode;          // 0 internal loss, 1 external dL/dy
  int implicit_touch; // float gradients: a slot with a nonzero sum is touched
                      // (no touched-byte stores)
  int out_act;        // output activation: 0 none, 1 sigmoid
  float *dxout;       // D == 0 training: dL/dx [N x In] fp32 (may be null)
};

// ------------------------------------------------------------- device parts

template <int F, bool HALF>
__device__ __forceinline__ void load_entry(const FusedParams &P, uint32_t off,
                                           float *v) {
  load_table_entry<F, HALF>(P.table32, P.table16, off, v);
}

// Point loss and dL/dy (reference order, fp32).
__device__ __forceinline__ float loss_and_grad(const NetDims &nd, const float *y,
                                               const float *t, float inv_N,
                                               float *d) {
  const int O = nd.O;
  if (nd.loss == 3) {
    float dot = 0.f, pn = 0.f, tn = 0.f;
    for (int m = 0; m < O; ++m) {
      dot += y[m] * t[m];
      pn += y[m] * y[m];
      tn += t[m] * t[m];
    }
    const float pred_norm = sqrtf(pn + 1e-8f), target_norm = sqrtf(tn + 1e-8f);
    const float denom = pred_norm * target_norm, cosine = dot / denom;
    for (int m = 0; m < O; ++m)
      d[m] = ((cosine * y[m]) / (pn + 1e-8f) - t[m] / denom) * inv_N;
    return 1.0f - cosine;
  }
  float loss = 0.f;
  for (int m = 0; m < O; ++m) {
    const float r = y[m] - t[m];
    if (nd.loss == 0) {
      loss += r * r;
      d[m] = (2.0f * r) * inv_N;
    } else if (nd.loss == 1) {
      loss += fabsf(r);
      d[m] = (r > 0.f ? 1.f : (r < 0.f ? -1.f : 0.f)) * inv_N;
    } else {
      const float ar = fabsf(r), delta = nd.huber_delta;
      if (ar <= delta) {
        loss += (0.5f * r) * r;
        d[m] = r * inv_N;
      } else {
        loss += delta * (ar - 0.5f * delta);
        d[m] = (delta * (r > 0.f ? 1.f : -1.f)) * inv_N;
      }
    }
  }
  return loss;
}

// Writes 16 fp32 values as fp16 into row r, columns c0..c0+15 of a
// core-blocked tile (two 16-byte stores).
__device__ __forceinline__ void store_row16(__half *tile, int cols, int r,
                                            int c0, const float *v) {
  uint4 u[2];
  __half2 *h = reinterpret_cast<__half2 *>(u);
#pragma unroll
  for (int i = 0; i < 8; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4 *>(tile + tc::cb(r, c0, cols)) = u[0];
  *reinterpret_cast<uint4 *>(tile + tc::cb(r, c0 + 8, cols)) = u[1];
}

__device__ __forceinline__ void load_row16(const __half *tile, int cols, int r,
                                           int c0, float *v) {
  uint4 u[2];
  u[0] = *reinterpret_cast<const uint4 *>(tile + tc::cb(r, c0, cols));
  u[1] = *reinterpret_cast<const uint4 *>(tile + tc::cb(r, c0 + 8, cols));
  const __half2 *h = reinterpret_cast<const __half2 *>(u);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// 8 fp32 values -> one 16-byte fp16 row segment of a core-blocked tile.
__device__ __forceinline__ void store_row8(__half *tile, int cols, int r, int c0,
                                           const float *v) {
  uint4 u;
  __half2 *h = reinterpret_cast<__half2 *>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4 *>(tile + tc::cb(r, c0, cols)) = u;
}

// Interpolated features of NL consecutive levels starting at l0, with all
// NL * 2^D table loads issued before any is consumed.
template <int D, int F, bool HALF, int NL>
__device__ __forceinline__ void encode_levels(const FusedParams &P,
                                              const float *p, int l0,
                                              float *out /* [NL*F] */) {
  const NetDims &nd = P.nd;
  constexpr int NC = 1 << D;
  uint32_t offs[NL][NC];
  float ws[NL][NC];
#pragma unroll
  for (int j = 0; j < NL; ++j) {
    Cell<D> c;
    cell_of<D>(p, nd.res[l0 + j], c);
    const uint64_t lb = (uint64_t)(l0 + j) * nd.T * F;
#pragma unroll
    for (int k = 0; k < NC; ++k) corner<D, F>(c, k, nd.T - 1u, lb, offs[j][k], ws[j][k]);
  }
  float vals[NL][NC][F];
#pragma unroll
  for (int j = 0; j < NL; ++j)
#pragma unroll
    for (int k = 0; k < NC; ++k) load_entry<F, HALF>(P, offs[j][k], vals[j][k]);
#pragma unroll
  for (int j = 0; j < NL; ++j)
#pragma unroll
    for (int q = 0; q < F; ++q) {
      float f = 0.f;
#pragma unroll
      for (int k = 0; k < NC; ++k) f = __fadd_rn(f, __fmul_rn(ws[j][k], vals[j][k][q]));
      out[j * F + q] = f;
    }
}

// 8 consecutive fp32 TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float *v) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
        "=r"(r[6]), "=r"(r[7])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// The CTA has 128 * Q threads (Q = 2 or 4): threads t, t + 128, ... share
// point (row) t % 128.  Encode and scatter split the point's levels among the
// Q in 8-column chunks; epilogues split the columns; TMEM lane quarter =
// warp % 4.  Q = 4 serves shapes whose TMEM budget allows only two CTAs per
// SM, so that an SM still holds 32 warps to keep table accesses in flight.
template <int D, int F, int W, bool HALF, bool TRAIN, int Q = 2>
__global__ void __launch_bounds__(128 * Q, 8 / Q)
    k_fused(const __grid_constant__ FusedParams P) {
  extern __shared__ __align__(128) uint8_t sm[];
  const NetDims &nd = P.nd;
  const Layout &Ly = P.lay;
  const int t = threadIdx.x;
  const int warp = t >> 5;
  const int r = t & (kTile - 1);   // point row in the tile
  const int half = t >> 7;         // which part of the work on that row
  const int In = nd.In, H = nd.H, O = nd.O;
  constexpr int LPC = 8 / F;       // levels per 8-column chunk
  // rows of the weight-gradient MMAs (M = W, padded to the smallest M of
  // a one-CTA tcgen05.mma, 64; the padding rows are never flushed)
  constexpr int MW = W < 64 ? 64 : W;
  constexpr int NL = D == 4 ? 1 : (LPC < 2 ? LPC : 2);  // levels per load batch
  const int n_chunks = In / 8;
  uint64_t *mbar = reinterpret_cast<uint64_t *>(sm + Ly.misc);
  uint32_t *tslot = reinterpret_cast<uint32_t *>(sm + Ly.misc + 8);
  float *s_red = reinterpret_cast<float *>(sm + Ly.misc + 64);  // 16 + 4
  __half *X = reinterpret_cast<__half *>(sm + Ly.x);

  // ---- prologue: weights to shared, ones columns, barrier, TMEM
  {
    const uint4 *src = reinterpret_cast<const uint4 *>(P.wimage + Ly.tail_src);
    uint4 *dst = reinterpret_cast<uint4 *>(sm + Ly.tail_dst);
    for (uint32_t i = t; i < Ly.tail_bytes / 16; i += 128 * Q) dst[i] = src[i];
    if (TRAIN && half == 0) {
      float ones[16] = {1.f};
      store_row16(X, Ly.xc, r, In, ones);
      const float zeros[16] = {0.f};
      for (int k = 0; k < H; ++k) {
        store_row16(reinterpret_cast<__half *>(sm + Ly.h[k]), Ly.hc, r, W, ones);
        for (int c0 = W + 16; c0 < Ly.hc; c0 += 16)  // M = 64 padding (W < 64)
          store_row16(reinterpret_cast<__half *>(sm + Ly.h[k]), Ly.hc, r, c0, zeros);
      }
    }
    if (t < 20) s_red[t] = 0.f;
    if (t == 0) tc::mbar_init(tc::smem_u32(mbar), 1);
    if (warp == 0) tc::tmem_alloc(tc::smem_u32(tslot), Ly.tmem_cols);
  }
  tc::fence_proxy_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tslot;
  const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
  const uint32_t T_s = tmem + Ly.t_scratch;
  const uint32_t mbar_a = tc::smem_u32(mbar);
  const uint32_t sbase = tc::smem_u32(sm);
  uint32_t phase = 0;
  bool ok = true;
  bool first = true;
  float loss_sum = 0.f;
  float db_out[kOutCols];
#pragma unroll
  for (int m = 0; m < kOutCols; ++m) db_out[m] = 0.f;

  auto sync_mma = [&]() {
    if (!tc::mbar_wait(mbar_a, phase, kWaitBound)) {
      ok = false;
      if (t == 0) atomicExch(P.err, 1);
    }
    phase ^= 1u;
    tc::fence_after_sync();
  };
  auto publish = [&]() {
    tc::fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
  };

  for (uint32_t tile = blockIdx.x; tile < P.ntiles && ok; tile += gridDim.x) {
    const uint32_t row = tile * kTile + r;
    const bool valid = row < P.N;
    float p[4] = {0.f, 0.f, 0.f, 0.f};
    if (valid) {
#pragma unroll
      for (int a = 0; a < D; ++a) p[a] = __ldg(P.pos + (size_t)row * D + a);
    }
    if constexpr (D == 0) {
      // plain MLP: the input features come from memory (fp16)
      for (int ch = half; ch < n_chunks; ch += Q) {
        uint4 u = make_uint4(0u, 0u, 0u, 0u);
        if (valid)
          u = __ldg(reinterpret_cast<const uint4 *>(P.xin + (size_t)row * In) + ch);
        *reinterpret_cast<uint4 *>(X + tc::cb(r, ch * 8, Ly.xc)) = u;
      }
    } else {
      // ---- encode: chunks of 8 feature columns, alternating between halves
      for (int ch = half; ch < n_chunks; ch += Q) {
        float acc[8];
#pragma unroll
        for (int j = 0; j < LPC; j += NL)
          encode_levels<D, F, HALF, NL>(P, p, ch * LPC + j, acc + j * F);
        store_row8(X, Ly.xc, r, ch * 8, acc);
      }
    }
    publish();
    // ---- forward
    for (int k = 0; k < H; ++k) {
      const int hk = TRAIN ? k : (k & 1);
      const int hp = TRAIN ? k - 1 : ((k - 1) & 1);
      if (!TRAIN && Ly.stream_w) {
        const uint32_t bytes = (uint32_t)(k == 0 ? In : W) * W * 2;
        const uint4 *src = reinterpret_cast<const uint4 *>(P.wimage + Ly.w[k]);
        uint4 *dst = reinterpret_cast<uint4 *>(sm + Ly.sw[k]);
        for (uint32_t i = t; i < bytes / 16; i += 128 * Q) dst[i] = src[i];
        publish();
      }
      if (t == 0) {
        tc::fence_after_sync();
        tc::Operand A = k == 0 ? tc::Operand{sbase + Ly.x, Ly.xc, 0}
                               : tc::Operand{sbase + Ly.h[hp], Ly.hc, 0};
        tc::Operand B{sbase + Ly.sw[k], W, 1};
        tc::gemm(T_s, A, B, kTile, W, k == 0 ? In : W, 0);
        tc::commit(mbar_a);
      }
      sync_mma();
      if (!ok) break;
      const float *bk = reinterpret_cast<const float *>(sm + Ly.sb[k]);
      __half *Hk = reinterpret_cast<__half *>(sm + Ly.h[hk]);
      for (int c0 = half * 16; c0 < W; c0 += 16 * Q) {
        float v[16];
        tc::tmem_ld16(T_s + lane_base + c0, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = fmaxf(v[i] + bk[c0 + i], 0.f);
        store_row16(Hk, Ly.hc, r, c0, v);
      }
      publish();
    }
    if (!ok) break;
    const int hl = TRAIN ? H - 1 : ((H - 1) & 1);
    // ---- output layer
    if (t == 0) {
      tc::fence_after_sync();
      tc::gemm(T_s, tc::Operand{sbase + Ly.h[hl], Ly.hc, 0},
               tc::Operand{sbase + Ly.sw[H], kOutCols, 1}, kTile, kOutCols, W, 0);
      tc::commit(mbar_a);
    }
    sync_mma();
    if (!ok) break;
    if (half == 0) {
      float y[kOutCols];
      tc::tmem_ld16(T_s + lane_base, y);
      const float *bo = reinterpret_cast<const float *>(sm + Ly.sb[H]);
#pragma unroll
      for (int m = 0; m < kOutCols; ++m) y[m] += bo[m];
      if (P.out_act == 1) {
#pragma unroll
        for (int m = 0; m < kOutCols; ++m) y[m] = 1.0f / (1.0f + expf(-y[m]));
      }
      if (!TRAIN) {
        if (valid)
          for (int m = 0; m < O; ++m) P.out[(size_t)row * O + m] = y[m];
      } else {
        // loss / external gradient -> scaled dY in shared memory
        float d[kOutCols];
#pragma unroll
        for (int m = 0; m < kOutCols; ++m) d[m] = 0.f;
        if (valid) {
          if (P.mode == 0) {
            float tg[kOutCols];
            for (int m = 0; m < O; ++m) tg[m] = __ldg(P.tgt + (size_t)row * O + m);
            loss_sum += loss_and_grad(nd, y, tg, P.inv_N, d);
          } else {
            for (int m = 0; m < O; ++m) d[m] = __ldg(P.dext + (size_t)row * O + m);
          }
        }
        if (P.out_act == 1) {
          // d/dz of sigmoid(z) = y (1 - y): the loss (or the caller's
          // gradient) is w.r.t. the activated output
#pragma unroll
          for (int m = 0; m < kOutCols; ++m) d[m] *= y[m] * (1.0f - y[m]);
        }
#pragma unroll
        for (int m = 0; m < kOutCols; ++m) {
          db_out[m] += d[m];
          d[m] *= P.dscale;
        }
        store_row16(reinterpret_cast<__half *>(sm + Ly.dy), kOutCols, r, 0, d);
      }
    }
    if (!TRAIN) {
      tc::fence_before_sync();
      __syncthreads();
      continue;
    }
    publish();
    // ---- backward through the output layer
    if (t == 0) {
      tc::fence_after_sync();
      // dH = dY . Wout^T   (B = Wout stored [W x 16] as K-major rows N = j)
      tc::gemm(T_s, tc::Operand{sbase + Ly.dy, kOutCols, 0},
               tc::Operand{sbase + Ly.sw[H], kOutCols, 0}, kTile, W, kOutCols, 0);
      // dWout += H^T . dY
      tc::gemm(tmem + Ly.t_dwout, tc::Operand{sbase + Ly.h[hl], Ly.hc, 1},
               tc::Operand{sbase + Ly.dy, kOutCols, 1}, MW, kOutCols, kTile,
               first ? 0u : 1u);
      tc::commit(mbar_a);
    }
    sync_mma();
    if (!ok) break;
    for (int k = H - 1; k >= 0; --k) {
      // dpre_k = D * relu'(H_k), written over H_k (each thread rewrites
      // the elements it read; the MMAs that read H_k have completed, and its
      // ones column is left alone)
      {
        __half *Hk = reinterpret_cast<__half *>(sm + Ly.h[k]);
        for (int c0 = half * 16; c0 < W; c0 += 16 * Q) {
          float v[16], hv[16];
          tc::tmem_ld16(T_s + lane_base + c0, v);
          load_row16(Hk, Ly.hc, r, c0, hv);
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = hv[i] > 0.f ? v[i] : 0.f;
          store_row16(Hk, Ly.hc, r, c0, v);
        }
      }
      publish();
      if (t == 0) {
        tc::fence_after_sync();
        const tc::Operand dHk{sbase + Ly.h[k], Ly.hc, 0};
        const tc::Operand dHkT{sbase + Ly.h[k], Ly.hc, 1};
        if (k > 0) {
          tc::gemm(T_s, dHk, tc::Operand{sbase + Ly.sw[k], W, 0}, kTile, W, W, 0);
          tc::gemm(tmem + Ly.t_dwk[k], dHkT,
                   tc::Operand{sbase + Ly.h[k - 1], Ly.hc, 1}, MW, W + 16, kTile,
                   first ? 0u : 1u);
        } else {
          tc::gemm(T_s, dHk, tc::Operand{sbase + Ly.sw[0], W, 0}, kTile, In, W, 0);
          tc::gemm(tmem + Ly.t_dw0, dHkT, tc::Operand{sbase + Ly.x, Ly.xc, 1}, MW,
                   In + 16, kTile, first ? 0u : 1u);
        }
        tc::commit(mbar_a);
      }
      sync_mma();
      if (!ok) break;

    }
    if (!ok) break;
    first = false;
    // ---- scatter d_feature * corner weight into the hash gradients
    if constexpr (D > 0) {
      const int levels = nd.active_levels;
      const int lane = t & 31;
      float *sa = reinterpret_cast<float *>(sm + Ly.agg) + warp * 64;
      for (int ch = half; ch < n_chunks; ch += Q) {
        float df[8];
        tmem_ld8(T_s + lane_base + ch * 8, df);
        const unsigned vmask = __ballot_sync(0xffffffffu, valid);
        if (!valid) continue;
#pragma unroll
        for (int j = 0; j < LPC; ++j) {
          const int l = ch * LPC + j;
          if (l >= levels) break;
          float dfe[F];
#pragma unroll
          for (int q = 0; q < F; ++q) dfe[q] = df[j * F + q] * P.inv_dscale;
          Cell<D> c;
          cell_of<D>(p, nd.res[l], c);
          const uint64_t lb = (uint64_t)l * nd.T * F;
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
                // an all-zero contribution still touches its slot: it adds
                // the smallest normal float 2^-126 (float reductions flush
                // subnormals; the fp16 reductions mark by themselves), so
                // the slot's sum is nonzero and Adam treats it as touched;
                // the value is below any weight's ulp
#pragma unroll
                for (int q = 0; q < F; ++q)
                  gv[q] = (F == 2 && q == 1) ? 0.f : touch_mark(nd.grad_half);
              }
              if (F == 2 && nd.res[l] <= kAggMaxRes) {
                // warp aggregation: lanes with the same corner hand their
                // contributions to the lowest such lane, which issues one
                // reduction for the group
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
      }
    } else {
      // plain MLP: dL/dx to memory (unscaled fp32), for a caller that
      // back-propagates further (e.g. into the features of another network)
      if (P.dxout) {
        for (int ch = half; ch < n_chunks; ch += Q) {
          float df[8];
          tmem_ld8(T_s + lane_base + ch * 8, df);
          if (!valid) continue;
          float4 *dst = reinterpret_cast<float4 *>(P.dxout + (size_t)row * In + ch * 8);
          dst[0] = make_float4(df[0] * P.inv_dscale, df[1] * P.inv_dscale,
                               df[2] * P.inv_dscale, df[3] * P.inv_dscale);
          dst[1] = make_float4(df[4] * P.inv_dscale, df[5] * P.inv_dscale,
                               df[6] * P.inv_dscale, df[7] * P.inv_dscale);
        }
      }
    }
    tc::fence_before_sync();
    __syncthreads();
  }

  // ---- epilogue: weight gradients, bias of the output layer, loss
  if (TRAIN && !first && ok) {
    tc::fence_after_sync();
    // M = W: row rr of an accumulator lives in lane rr (W == 128) or in lane
    // (rr / 16) * 32 + rr % 16 (W == 64).
    const int lane = t & 31;
    const int rr = W == 128 ? r : (warp & 3) * 16 + lane;
    const bool has_row = (W == 128 || lane < 16) && rr < W;
    const float s = P.inv_dscale;
    auto flush = [&](uint32_t tcol, int ncols, auto &&dest) {
      for (int c0 = half * 16; c0 < ncols; c0 += 16 * Q) {
        float v[16];
        tc::tmem_ld16(tmem + lane_base + tcol + c0, v);
        if (!has_row) continue;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float *dst = dest(c0 + i);
          if (dst && v[i] != 0.f) atomicAdd(dst, v[i] * s);
        }
      }
    };
    flush(Ly.t_dw0, In + 16, [&](int c) -> float * {
      if (c < In) return P.gm + nd.w_off[0] + (int64_t)c * W + rr;
      if (c == In) return P.gm + nd.b_off[0] + rr;
      return nullptr;
    });
    for (int k = 1; k < H; ++k)
      flush(Ly.t_dwk[k], W + 16, [&](int c) -> float * {
        if (c < W) return P.gm + nd.w_off[k] + (int64_t)c * W + rr;
        if (c == W) return P.gm + nd.b_off[k] + rr;
        return nullptr;
      });
    flush(Ly.t_dwout, kOutCols, [&](int c) -> float * {
      return c < O ? P.gm + nd.w_off[H] + (int64_t)rr * O + c : nullptr;
    });
  }
  if (TRAIN && half == 0) {
#pragma unroll
    for (int m = 0; m < kOutCols; ++m) {
      float v = db_out[m];
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if ((t & 31) == 0 && m < O) atomicAdd(s_red + m, v);
    }
    float ls = loss_sum;
    for (int o = 16; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
    if ((t & 31) == 0) atomicAdd(s_red + 16, ls);
  }
  tc::fence_before_sync();
  __syncthreads();
  if (TRAIN && t == 0) {
    for (int m = 0; m < O; ++m)
      if (s_red[m] != 0.f) atomicAdd(P.gm + nd.b_off[H] + m, s_red[m]);
    if (P.mode == 0) atomicAdd(P.loss_acc, (double)s_red[16]);
  }
  if (warp == 0) tc::tmem_dealloc(tmem, Ly.tmem_cols);
}

// Packs the fp32 MLP weights into the fp16 core-blocked image.
__global__ void k_pack(NetDims nd, Layout Ly, const float *__restrict__ mlp,
                       uint8_t *img) {
  const int W = nd.W, In = nd.In, H = nd.H, O = nd.O;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  // W0 [In x W]
  if (i < In * W) {
    const int r = i / W, c = i % W;
    reinterpret_cast<__half *>(img + Ly.w[0])[tc::cb(r, c, W)] =
        __float2half_rn(mlp[nd.w_off[0] + i]);
  }
  for (int k = 1; k < H; ++k)
    if (i < W * W) {
      const int r = i / W, c = i % W;
      reinterpret_cast<__half *>(img + Ly.w[k])[tc::cb(r, c, W)] =
          __float2half_rn(mlp[nd.w_off[k] + i]);
    }
  if (i < W * kOutCols) {
    const int r = i / kOutCols, c = i % kOutCols;
    reinterpret_cast<__half *>(img + Ly.w[H])[tc::cb(r, c, kOutCols)] =
        __float2half_rn(c < O ? mlp[nd.w_off[H] + (int64_t)r * O + c] : 0.f);
  }
  for (int k = 0; k < H; ++k)
    if (i < W) reinterpret_cast<float *>(img + Ly.b[k])[i] = mlp[nd.b_off[k] + i];
  if (i < kOutCols)
    reinterpret_cast<float *>(img + Ly.b[H])[i] = i < O ? mlp[nd.b_off[H] + i] : 0.f;
}

// ------------------------------------------------ pipelined MLP inference
//
// Plain FullyFusedMLP inference with NG 128-row tiles in flight per CTA.
// The activations never touch shared memory: each tile keeps, in its own
// TMEM columns, an fp32 accumulator (W columns) and the fp16 activations
// that feed the next layer as the MMA's A operand (two per 32-bit column,
// max(In, W) / 2 columns); only the weights (the B operand) are read from
// shared memory, so a layer moves W*W*2 bytes of shared memory for
// 2*128*W*W flops.
//   warp 0 (one thread)   issues every layer's tcgen05.mma for the NG tiles
//                         in turn and commits to that tile's mma_done barrier;
//   warps 4 .. 4+4NG-1    NG epilogue groups of 128 threads, one row each
//                         (TMEM lane quarter = warp % 4): write the input row
//                         into the A columns (tcgen05.st), then per layer wait
//                         mma_done, read the accumulator, add the bias, ReLU,
//                         store fp16 into the A columns and arrive on
//                         act_ready; the output layer goes to memory.
// All weights stay in shared memory (one copy per CTA, one CTA per SM).
// Every barrier wait is bounded; on a timeout the kernel sets the error word
// and stops issuing work.
struct PipeParams {
  NetDims nd;
  Layout lay;           // weight image offsets (inference layout)
  const uint8_t *wimage;
  const __half *xin;
  float *out;
  int *err;
  uint32_t N, ntiles;
  uint32_t bar_off;
  uint32_t bias_off;    // bias slabs (per layer) and the ones operand
  uint32_t gcols;       // TMEM columns per tile (accumulator + A operand)
  uint32_t tcols;       // allocated TMEM columns
  int out_act;
};

__device__ __forceinline__ void mbar_arrive(uint32_t mbar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(mbar)
               : "memory");
}

// D = A . B with A [128 x K] fp16 in TMEM (K/2 columns from a_tmem) and B a
// core-blocked MN-major shared-memory operand; one thread issues.
__device__ __forceinline__ void gemm_ta(uint32_t tmem_d, uint32_t a_tmem,
                                        uint32_t b_base, int b_cols, int N,
                                        int K, bool accumulate = false) {
  const uint32_t id = tc::idesc(kTile, N, 0, 1);
  const uint32_t b_l = (uint32_t)b_cols * 16u, b_s = 128u;
  for (int s = 0; s < K / 16; ++s) {
    const uint64_t bd = tc::sdesc(b_base + s * 2u * b_l, b_l, b_s);
    const uint32_t acc = (s > 0 || accumulate) ? 1u : 0u;
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(
            tmem_d),
        "r"(a_tmem + 8u * s), "l"(bd), "r"(id), "r"(acc));
  }
}

// 16 / 8 packed fp16 pairs into consecutive TMEM columns of this lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t *v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,"
      "%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]),
      "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]),
      "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t *v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::
          "r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]),
      "r"(v[6]), "r"(v[7])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t *>(&h);
}
// fp16 pair {relu(a) low, relu(b) high}, round to nearest: one instruction
__device__ __forceinline__ uint32_t pack_relu_h2(float a, float b) {
  uint32_t u;
  asm("cvt.rn.relu.f16x2.f32 %0, %1, %2;" : "=r"(u) : "f"(b), "f"(a));
  return u;
}

// Bias slabs of the pipelined kernel: per layer a K = 16 MN-major operand
// [16 x N] whose row 0 holds the fp16 rounding of the bias and row 1 the
// fp16 rounding of the remainder (bias = hi + lo to ~2^-22 relative), and a
// K-major ones operand [128 x 16] with ones in columns 0 and 1: the MMA
// ones . slab starts every accumulator at the bias, so the epilogue only
// applies ReLU and packs.
__device__ __forceinline__ uint32_t pipe_slab_bytes(int W) {
  return 16u * (uint32_t)(W > kOutCols ? W : kOutCols) * 2u;
}

// S = 2 splits each tile's epilogue over two warpgroups (one half of the
// columns each), halving the epilogue's share of the per-layer chain.
template <int W, int NG, int S>
__global__ void __launch_bounds__(128 + 128 * NG * S)
    k_mlp_pipe(const __grid_constant__ PipeParams P) {
  extern __shared__ __align__(128) uint8_t sm[];
  const NetDims &nd = P.nd;
  const Layout &Ly = P.lay;
  const int t = threadIdx.x, warp = t >> 5;
  const int In = nd.In, H = nd.H, O = nd.O;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + P.bar_off);
  uint32_t *tslot = reinterpret_cast<uint32_t *>(sm + P.bar_off + 16 * NG);
  {
    const uint4 *src = reinterpret_cast<const uint4 *>(P.wimage);
    uint4 *dst = reinterpret_cast<uint4 *>(sm);
    for (uint32_t i = t; i < Ly.image_bytes / 16; i += blockDim.x) dst[i] = src[i];
    // bias slabs from the biases in global memory (the image copy above
    // may still be in flight), then the ones operand
    const uint32_t slab = pipe_slab_bytes(W);
    const float *gimg = reinterpret_cast<const float *>(P.wimage);
    for (int k = 0; k <= H; ++k) {
      const int n = k < H ? W : kOutCols;
      __half *sl = reinterpret_cast<__half *>(sm + P.bias_off + (uint32_t)k * slab);
      for (int i = t; i < 16 * n; i += blockDim.x) {
        const int kr = i / n, c = i % n;
        float v = 0.f;
        if (kr < 2) {
          const float b = gimg[Ly.b[k] / 4 + c];
          const __half hi = __float2half_rn(b);
          v = kr == 0 ? __half2float(hi) : b - __half2float(hi);
        }
        sl[tc::cb(kr, c, n)] = __float2half_rn(v);
      }
    }
    {
      __half *ones = reinterpret_cast<__half *>(sm + P.bias_off + (uint32_t)(H + 1) * slab);
      for (int i = t; i < kTile * 16; i += blockDim.x) {
        const int r = i / 16, c = i % 16;
        ones[tc::cb(r, c, 16)] = __float2half_rn(c < 2 ? 1.f : 0.f);
      }
    }
    if (t < NG) {
      tc::mbar_init(tc::smem_u32(bars + t), 1);         // mma_done[g]
      tc::mbar_init(tc::smem_u32(bars + NG + t), 128 * S);  // act_ready[g]
    }
    if (warp == 0) tc::tmem_alloc(tc::smem_u32(tslot), P.tcols);
  }
  tc::fence_proxy_async();
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tslot;
  const uint32_t sbase = tc::smem_u32(sm);
  const uint32_t stride = gridDim.x * NG;
  bool ok = true;

  if (warp == 0) {
    if ((t & 31) == 0) {
      // MMA issuer: round robin over the groups, one layer at a time
      uint32_t tile[NG], ph[NG];
      int layer[NG];
      bool live[NG];
      int n_live = 0;
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        tile[g] = blockIdx.x * NG + g;
        ph[g] = 0;
        layer[g] = 0;
        live[g] = tile[g] < P.ntiles;
        n_live += live[g];
      }
      while (n_live > 0 && ok) {
#pragma unroll
        for (int g = 0; g < NG; ++g) {
          if (!live[g] || !ok) continue;
          if (!tc::mbar_wait(tc::smem_u32(bars + NG + g), ph[g], kWaitBound)) {
            ok = false;
            atomicExch(P.err, 1);
            break;
          }
          ph[g] ^= 1u;
          tc::fence_after_sync();
          const int k = layer[g];
          const uint32_t acc = tmem + (uint32_t)g * P.gcols;
          const uint32_t a = acc + (uint32_t)W;
          const int n = k < H ? W : kOutCols;
          const uint32_t slab = sbase + P.bias_off + (uint32_t)k * pipe_slab_bytes(W);
          const uint32_t ones = sbase + P.bias_off + (uint32_t)(H + 1) * pipe_slab_bytes(W);
          tc::gemm(acc, tc::Operand{ones, 16, 0}, tc::Operand{slab, n, 1}, kTile,
                   n, 16, 0);
          if (k < H)
            gemm_ta(acc, a, sbase + Ly.w[k], W, W, k == 0 ? In : W, true);
          else
            gemm_ta(acc, a, sbase + Ly.w[H], kOutCols, kOutCols, W, true);
          tc::commit(tc::smem_u32(bars + g));
          if (k == H) {
            layer[g] = 0;
            tile[g] += stride;
            if (tile[g] >= P.ntiles) {
              live[g] = false;
              --n_live;
            }
          } else {
            layer[g] = k + 1;
          }
        }
      }
    }
  } else if (warp >= 4) {
    const int g = (warp - 4) / (4 * S);
    const int part = ((warp - 4) >> 2) % S;  // column part of the epilogue
    const int r = (t - 128) & 127;           // row of the tile = TMEM lane
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t acc = tmem + (uint32_t)g * P.gcols + lane_base;
    const uint32_t a_cols = acc + (uint32_t)W;
    const uint32_t done_bar = tc::smem_u32(bars + g);
    const uint32_t ready_bar = tc::smem_u32(bars + NG + g);
    uint32_t ph = 0;
    // The input row of the group's next tile is loaded into registers while
    // the current tile's layers run (parts of at most 64 columns: 8 x 16 B),
    // so staging a tile does not wait on global memory.
    const int cbeg = part * (In / S), cend = (part + 1) * (In / S);
    constexpr int PB = (W / S) / 8 < 8 ? (W / S) / 8 : 8;  // 16-byte chunks
    const bool pre = cend - cbeg <= 8 * PB;
    uint4 nxt[PB];
#define TMNN_FETCH_NEXT(TL)                                                   \
  {                                                                           \
    const uint32_t tl_ = (TL), rw_ = tl_ * kTile + r;                          \
    const bool v_ = tl_ < P.ntiles && rw_ < P.N;                               \
    const uint4 *src_ = reinterpret_cast<const uint4 *>(P.xin + (size_t)rw_ * In + cbeg); \
    _Pragma("unroll") for (int j = 0; j < PB; ++j) {                          \
      nxt[j] = make_uint4(0u, 0u, 0u, 0u);                                    \
      if (v_ && cbeg + 8 * j < cend) nxt[j] = __ldg(src_ + j);                \
    }                                                                         \
  }
    if (pre) TMNN_FETCH_NEXT(blockIdx.x * NG + g)
    for (uint32_t tile = blockIdx.x * NG + g; tile < P.ntiles && ok;
         tile += stride) {
      const uint32_t row = tile * kTile + r;
      const bool valid = row < P.N;
      // input row -> A columns (8 fp16 = 4 columns per 16-byte load)
      if (pre) {
#pragma unroll
        for (int j = 0; j + 1 < PB; j += 2) {
          if (cbeg + 8 * j >= cend) continue;  // uniform over the warp
          const uint32_t u[8] = {nxt[j].x,     nxt[j].y,     nxt[j].z,
                                 nxt[j].w,     nxt[j + 1].x, nxt[j + 1].y,
                                 nxt[j + 1].z, nxt[j + 1].w};
          tmem_st8(a_cols + (uint32_t)((cbeg + 8 * j) / 2), u);
        }
      } else {
        for (int c0 = cbeg; c0 < cend; c0 += 16) {
          uint32_t u[8];
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            uint4 x = make_uint4(0u, 0u, 0u, 0u);
            if (valid)
              x = __ldg(reinterpret_cast<const uint4 *>(P.xin + (size_t)row * In + c0) + q);
            u[4 * q] = x.x;
            u[4 * q + 1] = x.y;
            u[4 * q + 2] = x.z;
            u[4 * q + 3] = x.w;
          }
          tmem_st8(a_cols + (uint32_t)(c0 / 2), u);
        }
      }
      tmem_st_wait();
      if (pre) TMNN_FETCH_NEXT(tile + stride)
#undef TMNN_FETCH_NEXT
      tc::fence_before_sync();
      mbar_arrive(ready_bar);
      for (int k = 0; k <= H && ok; ++k) {
        if (!tc::mbar_wait(done_bar, ph, kWaitBound)) {
          ok = false;
          atomicExch(P.err, 1);
          break;
        }
        ph ^= 1u;
        tc::fence_after_sync();
        if (k < H) {
          constexpr int WP = W / S;               // this part's columns
          constexpr int CHM = 32;  // register budget (the prefetched input row)
          constexpr int CH = WP < CHM ? WP : CHM; // columns per TMEM load wait
#pragma unroll
          for (int cc = 0; cc < WP; cc += CH) {
            const int c0 = part * WP + cc;
            float v[CH];
            if (CH == 64)
              tc::tmem_ld64(acc + c0, v);
            else if (CH == 32)
              tc::tmem_ld32(acc + c0, v);
            else
              tc::tmem_ld16(acc + c0, v);
            uint32_t hpk[CH / 2];
#pragma unroll
            for (int i = 0; i < CH; i += 2) hpk[i / 2] = pack_relu_h2(v[i], v[i + 1]);
#pragma unroll
            for (int q = 0; q < CH / 2; q += 8)
              tmem_st8(a_cols + (uint32_t)(c0 / 2 + q), hpk + q);
          }
          tmem_st_wait();
          tc::fence_before_sync();
          mbar_arrive(ready_bar);
        } else if (part == 0) {
          float y[kOutCols];
          tc::tmem_ld16(acc, y);
          tc::fence_before_sync();
          if (P.out_act == 1) {
#pragma unroll
            for (int m = 0; m < kOutCols; ++m) y[m] = 1.0f / (1.0f + expf(-y[m]));
          }
          if (valid) {
            float *o = P.out + (size_t)row * O;
            if (O == 16) {
#pragma unroll
              for (int q = 0; q < 4; ++q)
                reinterpret_cast<float4 *>(o)[q] =
                    make_float4(y[4 * q], y[4 * q + 1], y[4 * q + 2], y[4 * q + 3]);
            } else {
              for (int m = 0; m < O; ++m) o[m] = y[m];
            }
          }
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, P.tcols);
  }
}

constexpr uint32_t kPipeSmemMax = 220 * 1024;

int ensure_packed(FusedWorkspace &ws, const NetDims &nd, const float *params,
                  cudaStream_t st, bool train);

// TMEM columns per tile: W fp32 accumulator columns + max(In, W)/2 columns
// of fp16 pairs, rounded up to 32.
uint32_t pipe_gcols(const NetDims &nd) {
  const uint32_t c = (uint32_t)nd.W + (uint32_t)(nd.In > nd.W ? nd.In : nd.W) / 2;
  return (c + 31u) & ~31u;
}

// Tiles in flight: as many as TMEM holds, 2..6; 0 when the weights do not
// fit in shared memory.
// Shared memory past the weight image: barriers and TMEM slot (128 bytes),
// one bias slab per layer and the ones operand.
uint32_t pipe_extra(const NetDims &nd) {
  const uint32_t slab = 16u * (uint32_t)(nd.W > kOutCols ? nd.W : kOutCols) * 2u;
  return 128u + (uint32_t)(nd.H + 1) * slab + kTile * 16u * 2u;
}

int pipe_groups(const NetDims &nd) {
  const Layout L = make_layout(nd, false);
  if (align128(L.image_bytes) + pipe_extra(nd) > kPipeSmemMax) return 0;
  int ng = (int)(512 / pipe_gcols(nd));
  if (ng > 6) ng = 6;
  if (nd.W >= 64 && ng > 4) ng = 4;  // measured: more tiles do not help there
  return ng >= 2 ? ng : 0;
}

uint32_t pipe_smem(const NetDims &nd) {
  if (!pipe_groups(nd)) return 0;
  return align128(make_layout(nd, false).image_bytes) + pipe_extra(nd);
}

int launch_mlp_pipe(FusedWorkspace &ws, const NetDims &nd, const float *mlp,
                    const __half *x, float *out, uint32_t N, int num_sms,
                    cudaStream_t st, int out_act) {
  int launches = ensure_packed(ws, nd, mlp, st, false);
  PipeParams P{};
  P.nd = nd;
  P.lay = make_layout(nd, false);
  P.wimage = (const uint8_t *)ws.wpack + make_layout(nd, true).image_bytes;
  P.xin = x;
  P.out = out;
  P.err = ws.err;
  P.N = N;
  P.ntiles = (N + kTile - 1) / kTile;
  // epilogue split over two warpgroups per tile (W = 128: 419 against 376
  // TFLOP/s at H = 2, 578 against 543 at H = 4, N = 2^22; no gain at
  // W <= 64), with at most three tiles in flight to stay within 1024
  // threads; TMNN_PIPE_SPLIT=1 or 2 forces a choice (2 needs W >= 32 and
  // In a multiple of 32)
  // each part's input and hidden columns must be whole 16-column chunks
  const bool can_split = nd.W >= 32 && nd.In % 32 == 0;
  int split = nd.W >= 128 && can_split ? 2 : 1;  // measured: no gain at W <= 64
  if (const char *e = std::getenv("TMNN_PIPE_SPLIT"))
    split = (e[0] == '2' && can_split) ? 2 : 1;
  int NG = pipe_groups(nd);
  if (split == 2 && NG > 3) NG = 3;
  P.bar_off = align128(P.lay.image_bytes);
  P.bias_off = P.bar_off + 128u;
  P.gcols = pipe_gcols(nd);
  P.tcols = 32;
  while (P.tcols < (uint32_t)NG * P.gcols) P.tcols <<= 1;
  P.out_act = out_act;
  const uint32_t smem = pipe_smem(nd);
  using PipeFn = void (*)(PipeParams);
  PipeFn fn = nullptr;
#define TMNN_PIPE(WW)                                                       \
  case WW:                                                                  \
    if (split == 2)                                                         \
      fn = NG == 2 ? k_mlp_pipe<WW, 2, 2> : k_mlp_pipe<WW, 3, 2>;           \
    else                                                                    \
      fn = NG == 2 ? k_mlp_pipe<WW, 2, 1>                                   \
           : NG == 3 ? k_mlp_pipe<WW, 3, 1> : NG == 4 ? k_mlp_pipe<WW, 4, 1> \
           : NG == 5 ? k_mlp_pipe<WW, 5, 1> : k_mlp_pipe<WW, 6, 1>;         \
    break;
  switch (nd.W) { TMNN_PIPE(16) TMNN_PIPE(32) TMNN_PIPE(64) TMNN_PIPE(128) }
#undef TMNN_PIPE
  if (!fn || !smem) throw std::runtime_error("mlp pipe: unsupported shape");
  cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       (int)smem);
  uint32_t grid = (P.ntiles + NG - 1) / NG;
  if (grid > (uint32_t)num_sms) grid = (uint32_t)num_sms;
  if (grid == 0) return launches;
  fn<<<grid, 128 + 128 * NG * split, smem, st>>>(P);
  return launches + 1;
}

using KernelFn = void (*)(FusedParams);

template <int D, int F, bool HALF, bool TRAIN>
KernelFn pick_w(int W) {
  switch (W) {
    case 16: return (KernelFn)k_fused<D, F, 16, HALF, TRAIN>;
    case 32: return (KernelFn)k_fused<D, F, 32, HALF, TRAIN>;
    case 64: return (KernelFn)k_fused<D, F, 64, HALF, TRAIN>;
    case 128: return (KernelFn)k_fused<D, F, 128, HALF, TRAIN>;
  }
  return nullptr;
}

// Training kernels with four threads per point (Q = 4), for the common
// width 64 with two features per level.
KernelFn pick_train_q4(int d, int F, int W, bool half) {
  if (d == 0 && W == 64) return (KernelFn)k_fused<0, 2, 64, false, true, 4>;
  if (F != 2 || W != 64) return nullptr;
  if (d == 3) return half ? (KernelFn)k_fused<3, 2, 64, true, true, 4>
                          : (KernelFn)k_fused<3, 2, 64, false, true, 4>;
  if (d == 4) return half ? (KernelFn)k_fused<4, 2, 64, true, true, 4>
                          : (KernelFn)k_fused<4, 2, 64, false, true, 4>;
  return nullptr;
}

template <bool TRAIN>
KernelFn pick(int d, int F, int W, bool half) {
#define TMNN_PICK(DD, FF)                                                       \
  if (d == DD && F == FF)                                                       \
    return half ? pick_w<DD, FF, true, TRAIN>(W) : pick_w<DD, FF, false, TRAIN>(W);
  TMNN_PICK(3, 1) TMNN_PICK(3, 2) TMNN_PICK(3, 4)
  TMNN_PICK(4, 1) TMNN_PICK(4, 2) TMNN_PICK(4, 4)
#undef TMNN_PICK
  if (d == 0) return pick_w<0, 2, false, TRAIN>(W);
  return nullptr;
}

bool shape_ok(const NetDims &nd, bool train, std::string *why) {
  auto no = [&](const char *m) {
    if (why) *why = m;
    return false;
  };
  if (nd.In % 16 != 0 || nd.In > 128)
    return no("encoding width (levels x features) must be a multiple of 16, <= 128");
  if (nd.O > kOutCols) return no("more than 16 outputs");
  if (train) {
    if (nd.W != 16 && nd.W != 32 && nd.W != 64 && nd.W != 128)
      return no("hidden width must be 16, 32, 64 or 128");
    if (nd.H > kMaxTrainHidden) return no("more than 8 hidden layers");
  } else if (nd.W != 16 && nd.W != 32 && nd.W != 64 && nd.W != 128) {
    return no("hidden width must be 16, 32, 64 or 128");
  }
  const Layout L = make_layout(nd, train);
  if (L.total > 200 * 1024) return no("shared memory tile exceeds 200 KB");
  if (L.tmem_cols > 512) return no("TMEM columns exceed 512");
  return true;
}

NetDims dims_of(const tmnn_spec &s) {
  NetDims nd{};
  nd.L = s.n_levels;
  nd.F = s.n_features_per_level;
  nd.d = s.spatial_dims;
  nd.W = s.hidden_dim;
  nd.H = s.num_hidden_layers;
  nd.O = s.num_outputs;
  nd.In = nd.L * nd.F;
  return nd;
}

// (Re)packs the training and inference weight images when the weights
// changed; returns the kernels launched.
// (Re)packs the training or the inference weight image (whichever the
// caller is about to use) if the weights changed since it was last packed;
// returns the kernels launched.
int ensure_packed(FusedWorkspace &ws, const NetDims &nd, const float *params,
                  cudaStream_t st, bool train) {
  int launches = 0;
  if (!ws.err) {
    if (cudaMalloc(&ws.err, sizeof(int)) != cudaSuccess)
      throw std::runtime_error("fused: cudaMalloc failed");
    cudaMemsetAsync(ws.err, 0, sizeof(int), st);
  }
  const Layout Lt = make_layout(nd, true), Lf = make_layout(nd, false);
  const size_t need = (size_t)Lt.image_bytes + Lf.image_bytes;
  if (ws.wpack_bytes < need) {
    if (ws.wpack) cudaFree(ws.wpack);
    if (cudaMalloc(&ws.wpack, need) != cudaSuccess)
      throw std::runtime_error("fused: cudaMalloc failed");
    ws.wpack_bytes = need;
    cudaMemsetAsync(ws.wpack, 0, need, st);  // alignment gaps stay zero
    ws.dirty = ws.dirty_infer = true;
  }
  bool &dirty = train ? ws.dirty : ws.dirty_infer;
  if (dirty) {
    const float *mlp = params + nd.hash_count;
    const int n = nd.W * nd.W > nd.In * nd.W ? nd.W * nd.W : nd.In * nd.W;
    const int grid = (n + 255) / 256 + 1;
    if (train)
      k_pack<<<grid, 256, 0, st>>>(nd, Lt, mlp, (uint8_t *)ws.wpack);
    else
      k_pack<<<grid, 256, 0, st>>>(nd, Lf, mlp,
                                   (uint8_t *)ws.wpack + Lt.image_bytes);
    launches += 1;
    dirty = false;
  }
  return launches;
}

int launch(FusedWorkspace &ws, const NetDims &nd, const tmnn_spec &spec,
           const float *params, const __half *table_h, bool train,
           FusedParams &P, int num_sms, cudaStream_t st) {
  const Layout Ly = make_layout(nd, train);
  int launches = ensure_packed(ws, nd, params, st, train);
  P.nd = nd;
  P.lay = Ly;
  P.wimage = (const uint8_t *)ws.wpack +
             (train ? 0 : make_layout(nd, true).image_bytes);
  P.table32 = params;
  P.table16 = table_h;
  P.err = ws.err;
  P.ntiles = (P.N + kTile - 1) / kTile;
  const bool half = spec.table_dtype == TMNN_DTYPE_F16 && table_h;
  KernelFn fn = train ? pick<true>(nd.d, nd.F, nd.W, half)
                      : pick<false>(nd.d, nd.F, nd.W, half);
  int threads = kThreads;
  if (train && 512 / Ly.tmem_cols <= 2) {
    if (KernelFn f4 = pick_train_q4(nd.d, nd.F, nd.W, half)) {
      fn = f4;
      threads = 512;
    }
  }
  if (!fn) throw std::runtime_error("fused: no kernel for this shape");
  cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       (int)Ly.total);
  // CTAs per SM: the tighter of shared memory (1 KB reserved per CTA),
  // threads and TMEM columns.
  int dev = 0, smem_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor,
                         dev);
  int per_sm = smem_sm / (int)(Ly.total + 1024);
  if (per_sm > 2048 / threads) per_sm = 2048 / threads;
  const int tmem_fit = (int)(512 / Ly.tmem_cols);
  if (per_sm > tmem_fit) per_sm = tmem_fit;
  if (per_sm < 1) per_sm = 1;
  ws.ctas_per_sm = per_sm;
  uint32_t grid = (uint32_t)num_sms * per_sm;
  if (grid > P.ntiles) grid = P.ntiles;
  if (grid == 0) return launches;
  fn<<<grid, threads, Ly.total, st>>>(P);
  return launches + 1;
}

}  // namespace

bool fused_supported(const tmnn_spec &spec, const tmnn_train_cfg &cfg,
                     std::string *why) {
  (void)cfg;
  NetDims nd = dims_of(spec);
  return shape_ok(nd, true, why) && shape_ok(nd, false, why);
}

void fused_weights_changed(FusedWorkspace &ws) {
  ws.dirty = ws.dirty_infer = true;
}

void fused_release(FusedWorkspace &ws) {
  if (ws.wpack) cudaFree(ws.wpack);
  if (ws.err) cudaFree(ws.err);
  ws.wpack = nullptr;
  ws.err = nullptr;
  ws.wpack_bytes = 0;
}

int fused_train(FusedWorkspace &ws, const NetDims &nd, const tmnn_spec &spec,
                const float *params, const __half *table_h, const float *pos,
                const float *tgt, const float *dext, float inv_N, float *gm,
                int32_t *gh_fixed, float *gh_float, uint8_t *touched,
                double *loss_acc, uint32_t N, int num_sms, cudaStream_t st,
                bool implicit_touch) {
  FusedParams P{};
  P.implicit_touch = implicit_touch ? 1 : 0;
  P.pos = pos;
  P.tgt = tgt;
  P.dext = dext;
  P.gm = gm;
  P.gh_fixed = gh_fixed;
  P.gh_float = gh_float;
  P.touched = touched;
  P.loss_acc = loss_acc;
  P.inv_N = inv_N;
  // dY scale: a power of two near 1/inv_N (the batch), so fp16 dY ~ O(1)
  // (external gradients of a mean loss have the same 1/batch magnitude).
  int e = 0;
  frexpf(dext ? (float)(N > 0 ? N : 1) : (inv_N > 0.f ? 1.0f / inv_N : 1.0f), &e);
  P.dscale = ldexpf(1.0f, e - 1);
  P.inv_dscale = 1.0f / P.dscale;
  P.N = N;
  P.mode = dext ? 1 : 0;
  return launch(ws, nd, spec, params, table_h, true, P, num_sms, st);
}

int fused_forward(FusedWorkspace &ws, const NetDims &nd, const tmnn_spec &spec,
                  const float *params, const __half *table_h, const float *pos,
                  float *out, uint32_t N, int num_sms, cudaStream_t st) {
  FusedParams P{};
  P.pos = pos;
  P.out = out;
  P.N = N;
  P.dscale = P.inv_dscale = 1.0f;
  return launch(ws, nd, spec, params, table_h, false, P, num_sms, st);
}

int fused_mlp_forward(FusedWorkspace &ws, const NetDims &nd,
                      const float *mlp, const __half *x, float *out,
                      uint32_t N, int num_sms, cudaStream_t st, int out_act) {
  FusedParams P{};
  P.xin = x;
  P.out = out;
  P.N = N;
  P.out_act = out_act;
  P.dscale = P.inv_dscale = 1.0f;
  tmnn_spec spec{};
  spec.table_dtype = TMNN_DTYPE_F32;
  NetDims n0 = nd;
  n0.d = 0;
  n0.hash_count = 0;
  if (!ws.no_pipe && pipe_smem(n0))
    return launch_mlp_pipe(ws, n0, mlp, x, out, N, num_sms, st, out_act);
  return launch(ws, n0, spec, mlp, nullptr, false, P, num_sms, st);
}

int fused_mlp_train(FusedWorkspace &ws, const NetDims &nd, const float *mlp,
                    const __half *x, const float *tgt, const float *dext,
                    float inv_N, float *gm, double *loss_acc, float *dx,
                    uint32_t N, int num_sms, cudaStream_t st, int out_act) {
  FusedParams P{};
  P.xin = x;
  P.tgt = tgt;
  P.dext = dext;
  P.gm = gm;
  P.loss_acc = loss_acc;
  P.dxout = dx;
  P.inv_N = inv_N;
  P.out_act = out_act;
  int e = 0;
  frexpf(dext ? (float)(N > 0 ? N : 1) : (inv_N > 0.f ? 1.0f / inv_N : 1.0f), &e);
  P.dscale = ldexpf(1.0f, e - 1);
  P.inv_dscale = 1.0f / P.dscale;
  P.N = N;
  P.mode = dext ? 1 : 0;
  tmnn_spec spec{};
  spec.table_dtype = TMNN_DTYPE_F32;
  NetDims n0 = nd;
  n0.d = 0;
  n0.hash_count = 0;
  return launch(ws, n0, spec, mlp, nullptr, true, P, num_sms, st);
}

bool fused_mlp_supported(const NetDims &nd, std::string *why) {
  return shape_ok(nd, false, why);
}

bool fused_mlp_train_supported(const NetDims &nd, std::string *why) {
  return shape_ok(nd, true, why);
}

int fused_error(FusedWorkspace &ws, cudaStream_t st) {
  if (!ws.err) return 0;
  int h = 0;
  cudaMemcpyAsync(&h, ws.err, sizeof(int), cudaMemcpyDeviceToHost, st);
  cudaStreamSynchronize(st);
  return h;
}

}  // namespace tmnn
