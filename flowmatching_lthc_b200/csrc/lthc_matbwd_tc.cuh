// Materialisation backward on the 5th-generation tensor cores (16-bit
// activations, 2 <= L <= LTHC_MAX_LAYERS):
//   grad_dz_l[cell, c] = sum_r beta_l[c, r] * gX[cell, r, c]         (GEMM 1)
//   grad_beta_l[c, r]  = sum_cells gX[cell, r, c] * dz_l[cell, c]     (GEMM 2)
// for gX = grad X_L [B, 4G, 4G, C] (r = 4 * row + col inside a 4x4 cell), the
// backward of X_L = X_0 + sum_l P_l(dz_l) (local_thc_triton_kernels.py:1897-1912,
// K12 :512-595, K13 :598-680).  The weights differ per channel, so the channel
// is a batch index of both contractions, and it is the contiguous dimension in
// HBM.  One CTA per SM walks tiles of 128 cells x 16 channels (one 32-byte
// sector of every row).  CTA b owns slice b % S and cell range b / S, so the
// CTAs that run together read every slice of the same cell rows (whole rows of
// the residual; slice-major order left each DRAM page touched 32 bytes at a
// time and ran at half the speed).  Each tile arrives as four stages of 32
// cells: grad X_L by TMA into a ring that the transposers release, dz by
// cp.async into a ring that GEMM 2 releases (measured faster than 32-byte-row
// TMA boxes for dz, and it keeps the TMA engine for grad X_L).  The host sizes
// the rings per call: with the weight gradient 3 dz slots and what shared memory
// leaves for grad X_L (2 slots at L = 12), without it grad X_L alone (4 slots).
// grad X_L is transposed in shared memory (ldmatrix.trans + stmatrix) into one
// of two buffers (tile parity)
//   T[channel half][position half][8 channels][cell][8 positions]   (16-bit, no swizzle)
// which is a K-major operand for GEMM 1 (per channel: M = 128 cells, K = 16
// positions, N = 16 layer slots, one MMA per weight part) and an MN-major
// operand for GEMM 2 (M = 8 channels x 16 positions, K = cells, N = layers x 8
// channels, of which the block diagonal is kept: 8x the useful products, still
// a small fraction of the tensor pipe).  Accumulators live in TMEM:
//   D1 [128 cells][16 channels x 16 layer slots]   columns   0..255
//   D2 [128 (position half, channel, position)][L x 8] per channel half   columns 256..
// The fp32 weights enter GEMM 1 as two 16-bit parts (hi = rn(beta),
// lo = rn(beta - hi)), so the products carry 16 (bf16) or 22 (fp16) bits of
// each weight; GEMM 2's products are exact.  grad_beta is summed per tile in
// the tensor core, across a CTA's tiles in fp32 in tile order (in its partial
// buffer), and across CTAs by a fixed-order finalize: bitwise reproducible.
//
// grad_dz leaves through TMA tile stores: the epilogue packs a tile's rows into
// that tile's T buffer (free once its MMAs completed) and hands the buffer back
// to the transposers when the stores have read it.
//
// Warp roles (256 threads): 0 producer (TMA + cp.async), 1 MMA issuer + TMEM
// owner, 2-3 transposers (and the weight operands when the channel slice
// changes), 4-7 epilogue (TMEM -> staged grad_dz rows -> TMA stores; grad_beta
// accumulation).  Every wait is bounded; a role that gives up records the
// error and leaves its loop, the MMA issuer drains its MMAs before TMEM is
// released, the producer waits for its copies in flight and the storing thread
// for its stores.
#pragma once

#include "lthc_common.cuh"
#include "lthc_tma.cuh"
#include "lthc_umma.cuh"

namespace lthc {

constexpr int kMbTileCells = 128;                 // GEMM-1 M
constexpr int kMbQuarterCells = 32;               // cells per TMA stage
constexpr int kMbSliceCh = 16;                    // channels per tile
constexpr uint32_t kMbTChan = 2064;               // bytes between the channels of T (128 cells x 16 B + 16: the
                                                  // stmatrix rows of 8 channels fall in 8 distinct bank groups)
constexpr uint32_t kMbTHalf = 8 * kMbTChan;       // bytes between the position halves of a channel half
constexpr uint32_t kMbTGroup = 2 * kMbTHalf;      // bytes between the two channel halves (8 channels each)
static_assert(2 * kMbTGroup <= 66560, "T region");
constexpr uint32_t kMbTRegion = 66560;            // 2 x kMbTGroup, rounded up to 1 KB
constexpr uint32_t kMbGxBytes = kMbQuarterCells * kPos * kMbSliceCh * 2;   // 16 KB per stage
constexpr uint32_t kMbDzLayerBytes = kMbQuarterCells * kMbSliceCh * 2;     // 1 KB per layer per stage
constexpr uint32_t kMbBetaBytes = kMbSliceCh * 2 * 512;                    // 16 channels x 2 parts x [16 x 16]
constexpr int kMbThreads = 256;                    // 8 warps: at most 2 per SM sub-partition, so
                                                  // the epilogue may use up to 255 registers
constexpr int kMbMaxStages = 6;
constexpr uint32_t kMbSmemAlign = 128;
constexpr int kMbTransposeWarps = 2;
constexpr uint32_t kMbTmemCols = 512;
constexpr uint32_t kMbD2Col = 256;
constexpr int kMbQready = 8;                      // quarter hand-offs in flight (transposers run at most 7 ahead)
constexpr int kMbBarriers = 4 * kMbMaxStages + kMbQready + 8;

struct MatBwdTcParams {
  CUtensorMap tm_gx;               // 4D (C, 4G, 4G, B), box (16, 4 Gq, 4 Rq, 1)
  const void* dz[kMaxLayers];      // [B*G*G, C]
  const void* beta[kMaxLayers];    // [C, 16]
  CUtensorMap tm_gdz[kMaxLayers];  // grad_dz as 2D (C, B*G*G), box (16, 128): one tile's rows of a layer
  float* partial;                  // [grid][visits][L][16 channels][16 positions]
  int beta_dtype;
  int L, Lp;                       // layers, rounded up to even (GEMM-2 N = 8 Lp)
  int G, Gq, Rq;                   // cells per side; cells per box row (<= 32); cell rows per stage
  int gstages, dstages;             // grad X_L ring (TMA) and dz ring (cp.async) depths
  int need_pool, need_wgrad;
  int visits;                      // channel slices per CTA (at most)
  int64_t C;
  int64_t S;                       // 16-channel slices
  int64_t Tc;                      // 128-cell tiles (of every slice)
  int64_t parts;                   // cell ranges per slice
};

// Shared-memory descriptor of a no-swizzle operand: LBO steps between 8 x 16 B
// core matrices along K, SBO along M / N.
__device__ __forceinline__ uint64_t umma_desc_nosw(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (static_cast<uint64_t>(1u) << 46);
}

// Instruction descriptor, kind::f16 with fp32 accumulation; A and B both T
// (bf16 or fp16), each K-major or MN-major.
template <typename T>
__host__ __device__ constexpr uint32_t umma_idesc_16(int M, int N, bool a_mn, bool b_mn) {
  constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// Four 8x8 16-bit matrices: row i of matrix j at the address of lane 8 j + i.
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&v)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void stsm_x4(uint32_t addr, const uint32_t (&v)[4]) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v[0]), "r"(v[1]),
               "r"(v[2]), "r"(v[3])
               : "memory");
}

template <typename T>
__device__ __forceinline__ uint16_t to16(float x) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
  } else {
    return __half_as_ushort(__float2half_rn(x));
  }
}
template <typename T>
__device__ __forceinline__ float from16(uint16_t x) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    return __bfloat162float(__ushort_as_bfloat16(x));
  } else {
    return __half2float(__ushort_as_half(x));
  }
}

// Work of CTA b: the slices b % S, b % S + grid, ... (< S), each over its cell
// range part b / S of `parts` ([part * Tc / parts, (part + 1) * Tc / parts)).
// With grid = parts * S (S <= SMs) every CTA owns one slice and CTAs b, b + S,
// ... split its cells; the CTAs that run at the same time read every slice of
// the same cell rows together (whole 1536-byte rows of a C = 768 residual,
// rather than 32-byte pieces scattered over DRAM pages).
struct MbWork {
  int64_t s0, c0, ncell;
  int nslices;
  __host__ __device__ MbWork(int64_t b, int64_t grid, int64_t S, int64_t Tc, int64_t parts) {
    s0 = b % S;
    const int64_t part = b / S;
    c0 = part * Tc / parts;
    ncell = (part + 1) * Tc / parts - c0;
    nslices = static_cast<int>((S - 1 - s0) / grid + 1);
  }
  __host__ __device__ int64_t items() const { return nslices * ncell; }
  __host__ __device__ int64_t slice(int64_t i, int64_t grid) const { return s0 + (i / ncell) * grid; }
  __host__ __device__ int64_t ctile(int64_t i) const { return c0 + i % ncell; }
};

// grad_beta of lane m = 32 lq + lane of a D2 half, i.e. channel c' = 4 (lq & 1) +
// lane / 8 of the half: the block-diagonal entry of 32 accumulator columns
// (4 layers x 8 channels).
template <int ODD>
__device__ __forceinline__ float mb_diag(const float (&v)[32], int j, int q8) {
  const float a = q8 & 1 ? v[8 * j + 4 * ODD + 1] : v[8 * j + 4 * ODD];
  const float b = q8 & 1 ? v[8 * j + 4 * ODD + 3] : v[8 * j + 4 * ODD + 2];
  return q8 & 2 ? b : a;
}

// 16-byte asynchronous copy global -> shared through the load/store unit
// (bypassing L1); completion is tracked per thread.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
// The barrier receives one arrival when all of this thread's earlier cp.async
// copies have landed (the arrival is part of its expected count).
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ void red_add_f32(float* p, float v) {
  asm volatile("red.relaxed.gpu.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

template <typename T>
__global__ void __launch_bounds__(kMbThreads, 1) matbwd_tc_kernel(const __grid_constant__ MatBwdTcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // no-swizzle TMA boxes and descriptors need 128-byte (16-byte) alignment only
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + (kMbSmemAlign - 1)) &
                                             ~uintptr_t(kMbSmemAlign - 1));
  const int L = p.L;
  const uint32_t dz_bytes = static_cast<uint32_t>(L) * kMbDzLayerBytes;
  uint8_t* sT = smem;                                  // two T buffers (tile parity)
  uint8_t* sGx = smem + 2 * kMbTRegion;                // grad X_L ring (TMA)
  uint8_t* sDz = sGx + p.gstages * kMbGxBytes;         // dz ring (cp.async): [l][octet][cell][8 ch]
  uint8_t* sBeta = sDz + p.dstages * dz_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sBeta + kMbBetaBytes);
  uint64_t* gfull = bars;                              // grad X_L landed (TMA transaction)
  uint64_t* gempty = bars + kMbMaxStages;              // grad X_L transposed (transposer warps)
  uint64_t* dfull = bars + 2 * kMbMaxStages;           // dz landed (32 lanes' copies)
  uint64_t* dempty = bars + 3 * kMbMaxStages;          // dz consumed by GEMM 2 (MMA commit)
  uint64_t* qready = bars + 4 * kMbMaxStages;          // [kMbQready] quarter transposed into T
  uint64_t* tfree = qready + kMbQready;                // [2]: T buffer free again (its tile's MMAs completed)
  uint64_t* d1full = tfree + 2;
  uint64_t* d1empty = tfree + 3;
  uint64_t* d2full = tfree + 4;
  uint64_t* d2empty = tfree + 5;
  uint64_t* drain = tfree + 6;
  uint64_t* staged = tfree + 7;                        // grad_dz rows of a tile staged (epilogue warps)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + kMbBarriers);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t grid = gridDim.x;
  const MbWork work(blockIdx.x, grid, p.S, p.Tc, p.parts);
  const int n_tiles = static_cast<int>(work.items());
  const int n_q = 4 * n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.gstages; ++s) {
      mbar_init(&gfull[s], 1);
      mbar_init(&gempty[s], kMbTransposeWarps);
    }
    for (int s = 0; s < p.dstages; ++s) {
      mbar_init(&dfull[s], 32);
      mbar_init(&dempty[s], 1);
    }
    for (int s = 0; s < kMbQready; ++s) mbar_init(&qready[s], kMbTransposeWarps);
    mbar_init(&tfree[0], 1);
    mbar_init(&tfree[1], 1);
    mbar_init(d1full, 1);
    mbar_init(d1empty, 4);
    mbar_init(d2full, 1);
    mbar_init(d2empty, 4);
    mbar_init(drain, 1);
    mbar_init(staged, 4);
    fence_barrier_init();
  }
  // weight operands of the first slice, by every thread (independent loads):
  // [c][part][layer group][position half][8 layers][8 positions]
  auto build_beta = [&](int64_t slice, int t, int nthreads) {
#pragma unroll 8
    for (int idx = t; idx < kMbSliceCh * 16 * 16; idx += nthreads) {
      const int c = idx >> 8, l = (idx >> 4) & 15, rr = idx & 15;
      uint16_t hi = 0, lo = 0;
      if (l < L) {
        const float bv = load_weight(p.beta[l], p.beta_dtype, (slice * kMbSliceCh + c) * kPos + rr);
        hi = to16<T>(bv);
        lo = to16<T>(bv - from16<T>(hi));
      }
      const int off = c * 1024 + (l >> 3) * 256 + (rr >> 3) * 128 + (l & 7) * 16 + (rr & 7) * 2;
      *reinterpret_cast<uint16_t*>(sBeta + off) = hi;
      *reinterpret_cast<uint16_t*>(sBeta + off + 512) = lo;
    }
  };
  if (p.need_pool && n_tiles > 0) build_beta(work.s0, threadIdx.x, kMbThreads);
  fence_proxy_async_smem();
  if (warp == 1) tmem_alloc(tslot, kMbTmemCols);
  tmem_fence_before_sync();
  __syncthreads();
  tmem_fence_after_sync();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    // ---------------- producer: one grad X_L box (lane 0, TMA) and one set of dz
    // pieces (every lane, cp.async; [layer][channel octet][cell][8 channels], the
    // GEMM-2 B operand) per quarter of 32 cells
    if (n_q > 0) {
      if (lane == 0) prefetch_tmap(&p.tm_gx);
      const uint64_t pol = policy_evict_first();
      const int64_t GG = static_cast<int64_t>(p.G) * p.G;
      const int pc = lane & 15, half = lane >> 4;  // cell (of 16) and channel octet of this lane's copies
      int g_issued = 0;
      for (int Q = 0; Q < n_q; ++Q) {
        const int sg = Q % p.gstages, sd = Q % p.dstages;
        bool ok = true;
        if (lane == 0 && Q >= p.gstages) ok = mbar_wait(&gempty[sg], ((Q / p.gstages) & 1) ^ 1);
        if (!__all_sync(0xffffffffu, ok)) break;
        const int64_t slice = work.slice(Q / 4, grid);
        const int64_t cell0 = work.ctile(Q / 4) * kMbTileCells + kMbQuarterCells * (Q % 4);
        if (lane == 0) {
          const int64_t b = cell0 / GG;
          const int64_t rem = cell0 - b * GG;
          const int cy = static_cast<int>(rem / p.G), cx = static_cast<int>(rem % p.G);
          mbar_arrive_expect_tx(&gfull[sg], kMbGxBytes);
          tma_load_4d(sGx + sg * kMbGxBytes, &p.tm_gx, &gfull[sg], static_cast<int32_t>(slice * kMbSliceCh), 4 * cx,
                      4 * cy, static_cast<int32_t>(b), pol);
        }
        g_issued = Q + 1;
        if (p.need_wgrad) {
          if (Q >= p.dstages) ok = mbar_wait(&dempty[sd], ((Q / p.dstages) & 1) ^ 1);
          if (!__all_sync(0xffffffffu, ok)) break;
          const uint32_t dst0 = smem_u32(sDz + sd * dz_bytes) + half * 512 + pc * 16;
          const int64_t src0 = (cell0 + pc) * p.C + slice * kMbSliceCh + 8 * half;
          for (int l = 0; l < L; ++l) {
            const T* src = static_cast<const T*>(p.dz[l]) + src0;
            cp_async16(dst0 + l * kMbDzLayerBytes, src);
            cp_async16(dst0 + l * kMbDzLayerBytes + 16 * 16, src + 16 * p.C);
          }
          cp_async_arrive(&dfull[sd]);
        }
      }
      // copies still in flight land before the CTA's shared memory is released
      cp_async_wait_all();
      if (lane == 0)
        for (int Q = max(0, g_issued - p.gstages); Q < g_issued; ++Q)
          if (!mbar_wait(&gfull[Q % p.gstages], (Q / p.gstages) & 1)) break;
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer --------------------------------------------------
    if (lane == 0 && n_q > 0) {
      const uint32_t aT = smem_u32(sT), aDz = smem_u32(sDz), aB = smem_u32(sBeta);
      const uint32_t idesc1 = umma_idesc_16<T>(128, 16, false, false);
      const uint32_t idesc2 = umma_idesc_16<T>(128, 8 * p.Lp, true, true);
      const uint32_t d2 = tmem + kMbD2Col;
      bool ok = true;
      for (int tt = 0; ok && tt < n_tiles; ++tt) {
        const uint32_t aTt = aT + (tt & 1) * kMbTRegion;
        for (int q = 0; q < 4; ++q) {
          const int Q = 4 * tt + q, sd = Q % p.dstages;
          if (!mbar_wait(&qready[Q % kMbQready], (Q / kMbQready) & 1)) {
            ok = false;
            break;
          }
          if (p.need_wgrad) {
            if (!mbar_wait(&dfull[sd], (Q / p.dstages) & 1)) {
              ok = false;
              break;
            }
            if (q == 0 && tt > 0 && !mbar_wait(d2empty, (tt - 1) & 1)) {
              ok = false;
              break;
            }
            tmem_fence_after_sync();
            // GEMM 2: D2[h] += T[(position half, c, r) of channel half h][32 cells] x dz[32 cells][(l, c)]
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int ks = 0; ks < 2; ++ks) {
                const uint64_t a = umma_desc_nosw(aTt + h * kMbTGroup + (4 * q + 2 * ks) * 128, 128, kMbTChan);
                const uint64_t bd = umma_desc_nosw(aDz + sd * dz_bytes + h * 512 + ks * 256, 128, 1024);
                umma_bf16(d2 + h * 8 * p.Lp, a, bd, idesc2, q > 0 || ks > 0);
              }
            umma_commit(&dempty[sd]);  // the dz slot is free once these MMAs are done with it
          }
          if (q == 3) {
            if (p.need_wgrad) umma_commit(d2full);
            if (p.need_pool) {
              if (tt > 0 && !mbar_wait(d1empty, (tt - 1) & 1)) {
                ok = false;
                break;
              }
              tmem_fence_after_sync();
              // GEMM 1 per channel: D1[cells][c, 16 layer slots] = T_c[cells][16 positions] x beta_c parts
#pragma unroll 4
              for (int c = 0; c < kMbSliceCh; ++c)
#pragma unroll
                for (int part = 0; part < 2; ++part) {
                  const uint64_t a = umma_desc_nosw(aTt + (c >> 3) * kMbTGroup + (c & 7) * kMbTChan, kMbTHalf, 128);
                  const uint64_t bd = umma_desc_nosw(aB + c * 1024 + part * 512, 128, 256);
                  umma_bf16(tmem + c * 16, a, bd, idesc1, part > 0);
                }
              umma_commit(d1full);
            }
            // with grad_dz the epilogue releases T after its stores have read the rows
            // it staged there; without, T is free when these MMAs complete
            if (!p.need_pool) umma_commit(&tfree[tt & 1]);
          }
        }
      }
      umma_commit(drain);
      mbar_wait(drain, 0);  // every MMA issued has completed before TMEM is released
    }
  } else if (warp < 2 + kMbTransposeWarps) {
    // ---------------- transposers: stage [rows][columns][16 ch] -> T ---------------
    const int w = warp - 2;
    const int mi = lane >> 3, row = lane & 7;
    const int rhalf = mi >> 1, octet = mi & 1;
    const int r = 8 * rhalf + row;
    const uint32_t aT = smem_u32(sT);
    const uint32_t src_lane = static_cast<uint32_t>(((r >> 2) * 4 * p.Gq + (r & 3)) * 32 + octet * 16);
    const uint32_t dst_lane = static_cast<uint32_t>(octet * kMbTGroup + rhalf * kMbTHalf + row * kMbTChan);
    const int tid_t = threadIdx.x - 64;  // 0 .. 32 * kMbTransposeWarps - 1
    int64_t cur_slice = work.s0;  // its weight operands were built at the start
    bool ok = true;
    for (int tt = 0; ok && tt < n_tiles; ++tt) {
      const int64_t slice = work.slice(tt, grid);
      const uint32_t aTt = aT + (tt & 1) * kMbTRegion;
      for (int q = 0; q < 4; ++q) {
        const int Q = 4 * tt + q, sg = Q % p.gstages;
        if (!mbar_wait(&gfull[sg], (Q / p.gstages) & 1)) {
          ok = false;
          break;
        }
        if (q == 0) {
          // this T buffer is rewritten only after the MMAs of its previous tile (tt - 2) completed
          if (tt >= 2 && !mbar_wait(&tfree[tt & 1], ((tt >> 1) - 1) & 1)) {
            ok = false;
            break;
          }
          if (p.need_pool && slice != cur_slice) {
            // a new slice's weight operands replace the old ones once the last tile
            // of the old slice (tt - 1, the other buffer) has completed too
            if (!mbar_wait(&tfree[(tt - 1) & 1], ((tt - 1) >> 1) & 1)) {
              ok = false;
              break;
            }
            build_beta(slice, tid_t, 32 * kMbTransposeWarps);
            cur_slice = slice;
          }
        }
        const uint32_t st = smem_u32(sGx + sg * kMbGxBytes) + src_lane;
        // all loads of this warp's cells first, then all stores: the loads overlap
        // instead of each store waiting for its own load
        constexpr int kCells = kMbQuarterCells / kMbTransposeWarps;
        uint32_t v[kCells][4];
#pragma unroll
        for (int k = 0; k < kCells; ++k) {
          const int i = kCells * w + k;  // cell of this quarter
          const int cyl = i / p.Gq, cx = i - cyl * p.Gq;
          ldsm_x4_trans(st + static_cast<uint32_t>((4 * cyl * 4 * p.Gq + 4 * cx) * 32), v[k]);
        }
#pragma unroll
        for (int k = 0; k < kCells; ++k)
          stsm_x4(aTt + dst_lane + static_cast<uint32_t>((kMbQuarterCells * q + kCells * w + k) * 16), v[k]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&gempty[sg]);  // the grad X_L slot has been read
          mbar_arrive(&qready[Q % kMbQready]);
        }
      }
    }
  } else {
    // ---------------- epilogue: D1 -> grad_dz, D2 diagonal -> grad_beta --------------
    const int lq = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(32 * lq) << 16;
    // D2 lane m = 32 lq + lane holds position half lq / 2, channel c' = 4 (lq & 1) +
    // lane / 8 of its channel half, position 8 (lq / 2) + lane % 8
    const int q8 = lane >> 3;
    const int cprime = 4 * (lq & 1) + q8, rpos = 8 * (lq >> 1) + (lane & 7);
    // this lane's grad_beta sums live in the CTA's partial buffer (one fp32 per
    // half and layer): the first tile of a slice stores, later tiles add with a
    // fire-and-forget reduction.  Only this thread touches these words, and one
    // thread's operations on one address take effect in program order, so the
    // sum runs in tile order and is bitwise reproducible; the registers stay
    // free for the grad_dz rows and no load latency sits in the drain.
    float* const Pcta = p.partial + static_cast<int64_t>(blockIdx.x) * p.visits * L * 256 + cprime * 16 + rpos;
    bool ok = true;
    for (int tt = 0; tt < n_tiles; ++tt) {
      const int64_t slice = work.slice(tt, grid);
      const int64_t ctile = work.ctile(tt);
      if (p.need_wgrad) {
        const bool first = tt % work.ncell == 0;  // first tile of this slice: store instead of add
        float* const P = Pcta + (tt / work.ncell) * L * 256;
        if (!mbar_wait(d2full, tt & 1)) {
          ok = false;
          break;
        }
        tmem_fence_after_sync();
        float d[2][kMaxLayers];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int chunk = 0; chunk < (kMaxLayers + 3) / 4; ++chunk) {
            if (4 * chunk < L) {
              float v[32];
              tmem_ld32(tmem + lane_base + kMbD2Col + h * 8 * p.Lp + 32 * chunk, v);
#pragma unroll
              for (int j = 0; j < 4; ++j)
                if (4 * chunk + j < kMaxLayers) d[h][4 * chunk + j] = lq & 1 ? mb_diag<1>(v, j, q8) : mb_diag<0>(v, j, q8);
            }
          }
        // D2 may be overwritten as soon as it is in registers
        tmem_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(d2empty);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int l = 0; l < kMaxLayers; ++l)
            if (l < L) {
              float* const e = P + l * 256 + 8 * h * 16;
              if (first) {
                *e = d[h][l];
              } else {
                red_add_f32(e, d[h][l]);
              }
            }
      }
      if (p.need_pool) {
        if (!mbar_wait(d1full, tt & 1)) {
          ok = false;
          break;
        }
        tmem_fence_after_sync();
        // the tile's T buffer (free: GEMM 1 and 2 of this tile have completed) stages
        // the packed rows as [layer][cell][16 channels] for the TMA tile stores
        uint8_t* const stg = sT + (tt & 1) * kMbTRegion;
        const uint32_t row_lane = smem_u32(stg) + (32 * lq + lane) * (kMbSliceCh * 2);
        // two passes of half the layers each (the packed rows of all layers at once
        // would not fit in registers)
        constexpr int kHalfL = (kMaxLayers + 1) / 2;
#pragma unroll
        for (int lh = 0; lh < 2; ++lh) {
          if (lh * kHalfL < L) {
            uint32_t o[kHalfL][8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              float v[32];
              tmem_ld32(tmem + lane_base + 32 * k, v);  // channels 2k (layer slots 0..15) and 2k + 1 (16..31)
#pragma unroll
              for (int j = 0; j < kHalfL; ++j) {
                const int l = lh * kHalfL + j;
                if constexpr (std::is_same<T, __nv_bfloat16>::value) {
                  const __nv_bfloat162 pr = __floats2bfloat162_rn(v[l], v[16 + l]);
                  o[j][k] = *reinterpret_cast<const uint32_t*>(&pr);
                } else {
                  const __half2 pr = __floats2half2_rn(v[l], v[16 + l]);
                  o[j][k] = *reinterpret_cast<const uint32_t*>(&pr);
                }
              }
            }
#pragma unroll
            for (int j = 0; j < kHalfL; ++j) {
              const int l = lh * kHalfL + j;
              if (l < L) {
                const uint32_t a = row_lane + l * (kMbTileCells * kMbSliceCh * 2);
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(o[j][0]), "r"(o[j][1]),
                             "r"(o[j][2]), "r"(o[j][3])
                             : "memory");
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a + 16), "r"(o[j][4]), "r"(o[j][5]),
                             "r"(o[j][6]), "r"(o[j][7])
                             : "memory");
              }
            }
          }
        }
        tmem_fence_before_sync();
        fence_proxy_async_smem();  // the staged rows are read by the TMA engine
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(d1empty);
          mbar_arrive(staged);
        }
        if (warp == 4 && lane == 0) {
          // one thread stores the tile's L row blocks and, once they have been read
          // from shared memory, hands the T buffer back to the transposers
          if (!mbar_wait(staged, tt & 1)) {
            ok = false;
            break;
          }
#pragma unroll 1
          for (int l = 0; l < L; ++l)
            tma_store_2d(&p.tm_gdz[l], stg + l * (kMbTileCells * kMbSliceCh * 2), static_cast<int32_t>(slice * kMbSliceCh),
                         static_cast<int32_t>(ctile * kMbTileCells));
          bulk_commit();
          bulk_wait_read<0>();
          mbar_arrive(&tfree[tt & 1]);
        }
      }
    }
    if (warp == 4 && lane == 0) bulk_wait_all();  // the stores have completed before the CTA exits
  }
  tmem_fence_before_sync();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, kMbTmemCols);
}

// grad_beta[l][c][r] = sum over the cell ranges of c's slice, in order, of their
// CTAs' partial sums.
__global__ void matbwd_tc_finalize_kernel(const float* __restrict__ partial, float* __restrict__ grad_beta, int L,
                                          int64_t C, int64_t S, int64_t parts, int64_t grid, int visits) {
  const int64_t n = static_cast<int64_t>(L) * C * kPos;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < n;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t l = idx / (C * kPos);
    const int64_t c = (idx / kPos) % C;
    const int64_t rr = idx % kPos;
    const int64_t slice = c / kMbSliceCh;
    const int64_t visit = slice / grid;
    float acc = 0.f;
    for (int64_t part = 0; part < parts; ++part) {
      const int64_t b = part * S + slice % grid;
      acc += partial[((b * visits + visit) * L + l) * 256 + (c % kMbSliceCh) * kPos + rr];
    }
    grad_beta[idx] = acc;
  }
}

}  // namespace lthc
