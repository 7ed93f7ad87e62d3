// tc.cuh -- thin inline-PTX helpers for sm_100a tensor-core (tcgen05) work:
// shared-memory matrix descriptors, the instruction descriptor of
// kind::f16, MMA issue/commit, mbarrier waits with an iteration bound, and
// tensor-memory (TMEM) allocation and loads.
//
// Shared-memory operand layout used throughout ("core-blocked"): a matrix
// stored as rows x cols (cols contiguous) is cut into 8x8 fp16 core
// matrices of 128 contiguous bytes (8 rows of 16 bytes); core matrix
// (row/8, col/8) sits at byte ((row/8) * (cols/8) + col/8) * 128.  The same
// bytes serve as a K-major operand (rows = M or N, cols = K; LBO = 128,
// SBO = cols*16) and as an MN-major operand (rows = K, cols = M or N;
// SBO = 128, LBO = cols*16), with no swizzle.
#pragma once
#include <stdint.h>

namespace tmnn {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// element offset (in fp16 elements) of (r, c) in a core-blocked tile
__device__ __forceinline__ uint32_t cb(int r, int c, int cols) {
  return (uint32_t)(((r >> 3) * (cols >> 3) + (c >> 3)) * 64 + (r & 7) * 8 +
                    (c & 7));
}

// tcgen05 shared memory descriptor, SWIZZLE_NONE, version 1.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo,
                                          uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) |
         ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46);
}

// kind::f16 instruction descriptor: fp16 A/B, fp32 D.
__host__ __device__ constexpr uint32_t idesc(int M, int N, int a_mn_major,
                                             int b_mn_major) {
  return (1u << 4) | ((uint32_t)a_mn_major << 15) |
         ((uint32_t)b_mn_major << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t a, uint64_t b,
                                    uint32_t id, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "l"(a), "l"(b), "r"(id), "r"(accumulate));
}

// Operand view of a core-blocked tile.
struct Operand {
  uint32_t base;  // shared address of element (0, 0)
  int cols;       // stored columns
  int mn_major;   // 0: rows = M/N, cols = K; 1: rows = K, cols = M/N
};

// D[M x N] (+)= A[M x K] . B[K x N]; issued by one thread.
__device__ __forceinline__ void gemm(uint32_t tmem_d, const Operand &A,
                                     const Operand &B, int M, int N, int K,
                                     uint32_t accumulate) {
  const uint32_t id = idesc(M, N, A.mn_major, B.mn_major);
  const uint32_t a_l = A.mn_major ? (uint32_t)A.cols * 16u : 128u;
  const uint32_t a_s = A.mn_major ? 128u : (uint32_t)A.cols * 16u;
  const uint32_t b_l = B.mn_major ? (uint32_t)B.cols * 16u : 128u;
  const uint32_t b_s = B.mn_major ? 128u : (uint32_t)B.cols * 16u;
  const uint32_t a_step = A.mn_major ? 2u * a_l : 256u;
  const uint32_t b_step = B.mn_major ? 2u * b_l : 256u;
  for (int s = 0; s < K / 16; ++s) {
    mma(tmem_d, sdesc(A.base + s * a_step, a_l, a_s),
        sdesc(B.base + s * b_step, b_l, b_s), id,
        (s > 0 || accumulate) ? 1u : 0u);
  }
}

__device__ __forceinline__ void commit(uint32_t mbar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
      "[%0];" ::"r"(mbar)
      : "memory");
}

__device__ __forceinline__ void mbar_init(uint32_t mbar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(mbar), "r"(count));
}

// Waits for the phase with the given parity; returns false after `bound`
// unsuccessful polls (the caller records an error and stops issuing work).
__device__ __forceinline__ bool mbar_wait(uint32_t mbar, uint32_t parity,
                                          uint32_t bound) {
  uint32_t done = 0;
  for (uint32_t it = 0; it < bound; ++it) {
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], "
        "%2;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(mbar), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Warp-collective TMEM allocation; the address lands in *slot (shared).
__device__ __forceinline__ void tmem_alloc(uint32_t slot, uint32_t ncols) {
  asm volatile(
      "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          slot),
      "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(
                   taddr),
               "r"(ncols));
}

// 16 consecutive fp32 columns of this thread's TMEM lane (32x32b shape: warp
// w of a warpgroup reads lanes 32w..32w+31).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float *v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,"
      "%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]),
        "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 consecutive fp32 columns of this thread's lane, one wait.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float *v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,"
      "%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,"
      "%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]),
        "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Two 32-column loads in flight, one wait (64 columns).
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float *v) {
  uint32_t r[64];
#pragma unroll
  for (int h = 0; h < 2; ++h)
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,"
        "%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,"
        "%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[32 * h + 0]), "=r"(r[32 * h + 1]), "=r"(r[32 * h + 2]),
          "=r"(r[32 * h + 3]), "=r"(r[32 * h + 4]), "=r"(r[32 * h + 5]),
          "=r"(r[32 * h + 6]), "=r"(r[32 * h + 7]), "=r"(r[32 * h + 8]),
          "=r"(r[32 * h + 9]), "=r"(r[32 * h + 10]), "=r"(r[32 * h + 11]),
          "=r"(r[32 * h + 12]), "=r"(r[32 * h + 13]), "=r"(r[32 * h + 14]),
          "=r"(r[32 * h + 15]), "=r"(r[32 * h + 16]), "=r"(r[32 * h + 17]),
          "=r"(r[32 * h + 18]), "=r"(r[32 * h + 19]), "=r"(r[32 * h + 20]),
          "=r"(r[32 * h + 21]), "=r"(r[32 * h + 22]), "=r"(r[32 * h + 23]),
          "=r"(r[32 * h + 24]), "=r"(r[32 * h + 25]), "=r"(r[32 * h + 26]),
          "=r"(r[32 * h + 27]), "=r"(r[32 * h + 28]), "=r"(r[32 * h + 29]),
          "=r"(r[32 * h + 30]), "=r"(r[32 * h + 31])
        : "r"(taddr + 32u * h));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

}  // namespace tc
}  // namespace tmnn
