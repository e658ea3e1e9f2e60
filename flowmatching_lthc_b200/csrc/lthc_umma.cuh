// 5th-generation tensor-core (tcgen05) building blocks for sm_100a: shared-memory
// matrix descriptors, the instruction descriptor of a bf16 x bf16 -> fp32 MMA,
// the MMA issue / commit, tensor-memory (TMEM) allocation and loads.
//
// Operand layout used throughout: "K-major, 128-byte swizzle" — a matrix of R
// rows x 64 bf16 (128 bytes per row) stored as 8-row atoms of 1024 bytes; in row
// r of an atom, 16-byte chunk j sits at chunk position j ^ (r % 8).  Atoms are
// stacked along the rows at 1024-byte stride (the descriptor's stride byte
// offset).  Wider K is stored as separate 64-column blocks.  The descriptor of a
// K step of 16 elements inside a row starts 32 bytes further; atoms must start
// on 1024-byte boundaries.  (Bit positions follow the sm_100 descriptor formats
// of the PTX ISA; the CUTLASS/CuTe `UMMA::SmemDescriptor` and
// `UMMA::InstrDescriptor` unions document the same fields.)
#pragma once

#include <stdint.h>

#include "lthc_tma.cuh"

namespace lthc {

// Byte offset of element (row, k) of a K-major, 128-byte-swizzled bf16 block
// whose rows hold 64 elements.
__host__ __device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t k) {
  return (row >> 3) * 1024u + (row & 7u) * 128u + ((((k >> 3) ^ row) & 7u) << 4) + (k & 7u) * 2u;
}

// Shared-memory matrix descriptor: K-major, SWIZZLE_128B, 1024-byte stride between
// 8-row atoms.  `addr` is the shared-space byte address of the K step's first
// element (atom-aligned base + 32 * step within the row).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);          // start address  [0,14)
  d |= static_cast<uint64_t>(1u) << 16;                        // leading byte offset (unused for swizzled K-major) [16,30)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;                // stride byte offset [32,46)
  d |= static_cast<uint64_t>(1u) << 46;                        // descriptor version (sm_100) [46,48)
  d |= static_cast<uint64_t>(2u) << 61;                        // layout: SWIZZLE_128B [61,64)
  return d;
}

// Instruction descriptor, kind::f16: A, B bf16 (K-major), D fp32, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_bf16_f32(int M, int N) {
  return (1u << 4)                                   // D format: f32   [4,6)
         | (1u << 7)                                 // A format: bf16  [7,10)
         | (1u << 10)                                // B format: bf16  [10,13)
         | (static_cast<uint32_t>(N >> 3) << 17)     // N / 8           [17,23)
         | (static_cast<uint32_t>(M >> 4) << 24);    // M / 16          [24,29)
}

// D[tmem] (+)= A[desc] * B[desc]^T, issued by one thread.
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          bool accumulate) {
  const uint32_t acc = accumulate ? 1u : 0u;
  const uint32_t z = 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc), "r"(z), "r"(z), "r"(z), "r"(z)
      : "memory");
}

// Arrives once on the mbarrier when every MMA issued so far by this thread completes.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// TMEM allocation by one whole warp; the base address is written to *dst_smem.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// As tmem_ld32, without the wait: the registers are valid only after
// tmem_wait_ld(), so several loads can be in flight together.
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane (warp w reads lanes
// 32 * (w % 4) .. + 31; `taddr` carries that lane base in bits [16, 32)).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// ---------------------------------------------------------------------------
// Self-test: D[128 x N] = A[128 x K] * B[N x K]^T (bf16 in, fp32 out), one CTA of
// 4 warps.  Exercises the descriptors, the instruction descriptor, the commit
// and the TMEM load exactly as the fused kernels use them.  A and B are
// row-major [rows][K] bf16 in global memory, K a multiple of 64, N in {64, 128,
// 256}.  `status` receives 0, or 1 if the MMA completion wait gave up.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128, 1)
    umma_selftest_kernel(const __nv_bfloat16* A, const __nv_bfloat16* B, float* D, int N, int K, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int kblocks = K / 64;
  uint8_t* sa = smem;                                  // kblocks x [128 rows x 128 B]
  uint8_t* sb = sa + kblocks * 128 * 128;              // kblocks x [N rows x 128 B]
  uint64_t* bar = reinterpret_cast<uint64_t*>(sb + kblocks * N * 128);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5;

  for (int i = tid; i < 128 * K; i += blockDim.x) {
    const int r = i / K, k = i % K;
    *reinterpret_cast<__nv_bfloat16*>(sa + (k / 64) * 128 * 128 + sw128_offset(r, k % 64)) = A[i];
  }
  for (int i = tid; i < N * K; i += blockDim.x) {
    const int r = i / K, k = i % K;
    *reinterpret_cast<__nv_bfloat16*>(sb + (k / 64) * N * 128 + sw128_offset(r, k % 64)) = B[i];
  }
  fence_proxy_async_smem();
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tslot, 256);
  tmem_fence_before_sync();
  __syncthreads();
  tmem_fence_after_sync();
  const uint32_t tmem = *tslot;

  if (tid == 0) {
    const uint32_t idesc = umma_idesc_bf16_f32(128, N);
    for (int s = 0; s < K / 16; ++s) {
      const uint32_t a = smem_u32(sa + (s / 4) * 128 * 128) + (s % 4) * 32;
      const uint32_t b = smem_u32(sb + (s / 4) * N * 128) + (s % 4) * 32;
      umma_bf16(tmem, umma_desc_sw128(a), umma_desc_sw128(b), idesc, s > 0);
    }
    umma_commit(bar);
  }
  const bool ok = mbar_wait(bar, 0);
  tmem_fence_after_sync();
  if (ok) {
    const int row = 32 * warp + (tid & 31);
    for (int c0 = 0; c0 < N; c0 += 32) {
      float v[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(32 * warp) << 16) + c0, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) D[row * N + c0 + i] = v[i];
    }
  }
  const int bad = __syncthreads_or(!ok);
  if (tid == 0) *status = bad ? 1 : 0;
  tmem_fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// ---------------------------------------------------------------------------
// Raw-descriptor self-test: the host supplies byte images of an A and a B operand
// region (each at most kUmmaProbeRegion bytes, copied verbatim into shared
// memory), the shared-memory descriptors of each MMA step with start addresses
// relative to their region, and the instruction descriptor (M = 128).  The
// kernel adds the regions' shared addresses, issues the steps (accumulating after
// the first) and writes D[128 x N] fp32.  This pins the no-swizzle K-major and
// MN-major operand layouts the materialisation backward relies on.  The
// dynamic allocation is larger than the two regions, so that a descriptor whose
// strides reach past them still reads allocated shared memory.
// ---------------------------------------------------------------------------
constexpr int kUmmaProbeRegion = 65536;
constexpr int kUmmaProbeMaxSteps = 8;
constexpr int kUmmaProbeSmem = 200 * 1024;

struct UmmaProbeParams {
  uint64_t a_desc[kUmmaProbeMaxSteps];
  uint64_t b_desc[kUmmaProbeMaxSteps];
  int steps;
  uint32_t idesc;
  int N;
  int a_bytes, b_bytes;
};

__global__ void __launch_bounds__(128, 1)
    umma_probe_kernel(const uint4* a_img, const uint4* b_img, const __grid_constant__ UmmaProbeParams p, float* D,
                      int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + kUmmaProbeRegion;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 2 * kUmmaProbeRegion);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5;
  for (int i = tid; i < 2 * kUmmaProbeRegion / 16; i += blockDim.x) reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  __syncthreads();
  for (int i = tid; i < p.a_bytes / 16; i += blockDim.x) reinterpret_cast<uint4*>(sa)[i] = a_img[i];
  for (int i = tid; i < p.b_bytes / 16; i += blockDim.x) reinterpret_cast<uint4*>(sb)[i] = b_img[i];
  fence_proxy_async_smem();
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tslot, 256);
  tmem_fence_before_sync();
  __syncthreads();
  tmem_fence_after_sync();
  const uint32_t tmem = *tslot;
  if (tid == 0) {
    const uint64_t abase = smem_u32(sa) >> 4, bbase = smem_u32(sb) >> 4;
    for (int s = 0; s < p.steps; ++s) umma_bf16(tmem, p.a_desc[s] + abase, p.b_desc[s] + bbase, p.idesc, s > 0);
    umma_commit(bar);
  }
  const bool ok = mbar_wait(bar, 0);
  tmem_fence_after_sync();
  if (ok) {
    const int row = 32 * warp + (tid & 31);
    for (int c0 = 0; c0 < p.N; c0 += 32) {
      float v[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(32 * warp) << 16) + c0, v);
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (c0 + i < p.N) D[row * p.N + c0 + i] = v[i];
    }
  }
  const int bad = __syncthreads_or(!ok);
  if (tid == 0) *status = bad ? 1 : 0;
  tmem_fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

}  // namespace lthc
