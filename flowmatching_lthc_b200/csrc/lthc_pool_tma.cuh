// Read family on the TMA pipeline, one pass over a residual-sized tensor H:
//   pool   : out_l[cell, c]        = sum_r w_l[c, r] * H[cell, r, c]        (POOL)
//   wgrad  : partial_l[blk][c, r] += sum_cells H[cell, r, c] * low_l[cell, c] (WGRAD)
// The read forward is POOL with L = 1 (w = alpha); the weight gradient of the
// read is WGRAD with L = 1 (low = grad_z); the write backward is both with L = 1
// and the materialisation backward is both with L = 12 (H = grad X_L, w = beta_l,
// low = dz_l), so grad X_L is read from HBM exactly once.
//
// CTA roles (one 64-channel slice, lane = channel pair):
//   WGRAD warps             4 cell rows x layer groups; each lane keeps 4 columns x
//                           its layers x 2 channels of fp32 accumulators in registers
//   next POOL_WARPS warps   POOL: each owns CELLS_PER_POOL cells of the strip and
//                           reads the weights from a shared-memory copy laid out
//                           [r][layer pair][lane] as float4 (one 16-byte load
//                           feeds two layers, conflict-free)
//   last warp               producer (one elected lane issues the TMA loads)
// A strip is kStripCells horizontally adjacent cells; stages hold the H tile
// [4 rows][4*kStripCells columns][64 channels] and, for WGRAD, the L low tiles
// [L][4 cells][64 channels].  Sums run in fp32 in position order r = 0..15
// (POOL) and strip order (WGRAD); WGRAD partials are per CTA and reduced later
// in CTA order, so the result is bitwise reproducible.
#pragma once

#include "lthc_broadcast_tma.cuh"
#include "lthc_common.cuh"
#include "lthc_tma.cuh"

namespace lthc {

// Weight-gradient warps: 4 cell rows x WGRAD layer groups (the accumulators of
// a deep update stack are split across warps so that every warp of the CTA
// stays near 80 registers).
#ifndef LTHC_WGRAD_LAYERS_PER_WARP
#define LTHC_WGRAD_LAYERS_PER_WARP 12
#endif

template <int LMAX>
constexpr int wgrad_layer_groups() {
  return LMAX <= 2 ? 1 : (LMAX + LTHC_WGRAD_LAYERS_PER_WARP - 1) / LTHC_WGRAD_LAYERS_PER_WARP;
}

// Layers per pooling warp for the deep (L = 12) variants; the pooling work of a
// strip is split across warps by layer group so that no warp is the critical path.
#ifndef LTHC_POOL_LAYERS_PER_WARP
#define LTHC_POOL_LAYERS_PER_WARP 4
#endif

// Positions of the pooling loop that are unrolled together (loads of the next
// position overlap the FMAs of the current one).
#ifndef LTHC_POOL_UNROLL
#define LTHC_POOL_UNROLL 4
#endif
constexpr int kPoolUnroll = LTHC_POOL_UNROLL;

template <int LMAX>
constexpr int pool_layer_groups() {
  return LMAX <= 2 ? 1 : (LMAX + LTHC_POOL_LAYERS_PER_WARP - 1) / LTHC_POOL_LAYERS_PER_WARP;
}

// Stage count (16-bit activations; fp32 half as many) per role set.  The
// single-layer passes (read forward: pooling; read backward: weight gradient)
// move one residual tile per strip with little arithmetic per byte and take a
// deeper ring (measured on B200: read forward 5110 -> 5800 GB/s with 6 stages
// instead of 3; 12 stages 5480; 16 or more, one CTA per SM, 3280).
#ifndef LTHC_READ1_STAGES_16BIT
#define LTHC_READ1_STAGES_16BIT 6
#endif
#ifndef LTHC_WGRAD1_STAGES_16BIT
#define LTHC_WGRAD1_STAGES_16BIT 6
#endif
template <int LMAX, bool POOL, bool WGRAD>
constexpr int pool_stages16() {
  return LMAX == 1 && POOL && !WGRAD ? LTHC_READ1_STAGES_16BIT
         : LMAX == 1 && WGRAD && !POOL ? LTHC_WGRAD1_STAGES_16BIT
                                       : LTHC_STAGES_16BIT;
}

template <typename T, int LMAX, bool POOL, bool WGRAD, int CELLS_PER_POOL>
struct PoolLayout {
  static constexpr int kLayerGroups = pool_layer_groups<LMAX>();
  static constexpr int kGroupPairs = ((LMAX + 1) / 2 + kLayerGroups - 1) / kLayerGroups;  // layer pairs per warp
  static constexpr int kPoolWarps = POOL ? (kStripCells / CELLS_PER_POOL) * kLayerGroups : 0;
  static constexpr int kWgradGroups = wgrad_layer_groups<LMAX>();
  static constexpr int kWgradLayers = (LMAX + kWgradGroups - 1) / kWgradGroups;  // layers per WGRAD warp
  static constexpr int kWgradWarps = WGRAD ? 4 * kWgradGroups : 0;
  static constexpr int kConsumerWarps = kWgradWarps + kPoolWarps;
  static constexpr int kThreads = 32 * (kConsumerWarps + 1);
  static constexpr int kHBytes = 4 * kBoxCols * kSliceCh * static_cast<int>(sizeof(T));
  static constexpr int kLowTileBytes = kStripCells * kSliceCh * static_cast<int>(sizeof(T));
  static constexpr int kStageBytes = kHBytes + (WGRAD ? LMAX * kLowTileBytes : 0);
  static constexpr int kStages16 = pool_stages16<LMAX, POOL, WGRAD>();
  static constexpr int kStages = sizeof(T) == 2 ? kStages16 : (kStages16 + 1) / 2;
  static constexpr int kLayerPairs = (LMAX + 1) / 2;
  static constexpr int kWBytes = POOL ? kPos * kLayerPairs * 32 * 16 : 0;  // [r][lp][lane] float4
  static constexpr int kWOffset = kStages * kStageBytes;
  static constexpr int kBarrierOffset = kWOffset + kWBytes;
  static constexpr int kSmemBytes = kBarrierOffset + 2 * kStages * 8 + 128;
  static_assert(kSmemBytes <= 227 * 1024, "read-family stages exceed the shared memory of a CTA");
};

struct PoolTmaParams {
  CUtensorMap tm_h;                  // 4D (C, 4G, 4G, B) box (64, 16, 4, 1)
  CUtensorMap tm_low[kMaxLayers];    // 2D (C, B*G*G) box (64, 4)        (WGRAD)
  const void* w[kMaxLayers];         // [C, 16] weights, dtype w_dtype   (POOL)
  void* out[kMaxLayers];             // T[B, G*G, C]                     (POOL)
  float* partial;                    // [gridDim.x][L][C][16]            (WGRAD)
  int w_dtype;
  int L;
  int G;
  int strips_per_row;
  int64_t C;
  int64_t strips;
  int64_t strips_per_cta;
};

__device__ __forceinline__ float4 lds128f(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

// Resident CTAs per SM the register allocation is sized for.
#ifndef LTHC_READ_MIN_BLOCKS
#define LTHC_READ_MIN_BLOCKS 2
#endif
// Cells per pooling warp for deep (L > 1) stacks.
#ifndef LTHC_POOL_CELLS_DEEP
#define LTHC_POOL_CELLS_DEEP 4
#endif

template <typename T, int LT, bool POOL, bool WGRAD, int CELLS_PER_POOL>
__global__ void __launch_bounds__(PoolLayout<T, (LT > 0 ? LT : kMaxLayers), POOL, WGRAD, CELLS_PER_POOL>::kThreads,
                                  LTHC_READ_MIN_BLOCKS)
    pool_tma_kernel(const __grid_constant__ PoolTmaParams p) {
  constexpr int LMAX = LT > 0 ? LT : kMaxLayers;
  using Lay = PoolLayout<T, LMAX, POOL, WGRAD, CELLS_PER_POOL>;
  constexpr int kProducerWarp = Lay::kConsumerWarps;
  constexpr int kPoolWarp0 = Lay::kWgradWarps;
  constexpr uint32_t kEs = sizeof(T);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Lay::kBarrierOffset);
  uint64_t* empty = full + Lay::kStages;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int L = LT > 0 ? LT : p.L;
  const int64_t c0 = static_cast<int64_t>(blockIdx.y) * kSliceCh;
  const int64_t s_begin = static_cast<int64_t>(blockIdx.x) * p.strips_per_cta;
  const int64_t s_end = min(s_begin + p.strips_per_cta, p.strips);
  const int n_it = s_end > s_begin ? static_cast<int>(s_end - s_begin) : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Lay::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], Lay::kConsumerWarps);
    }
    fence_barrier_init();
  }
  if constexpr (POOL) {
    // Weights of this slice as [r][layer pair][lane] float4 = (w_2lp[c], w_2lp[c+1], w_2lp+1[c], w_2lp+1[c+1]).
    float4* ws = reinterpret_cast<float4*>(smem + Lay::kWOffset);
    for (int i = threadIdx.x; i < kPos * Lay::kLayerPairs * 32; i += blockDim.x) {
      const int pl = i & 31;
      const int lp = (i >> 5) % Lay::kLayerPairs;
      const int r = (i >> 5) / Lay::kLayerPairs;
      const int64_t cc = c0 + 2 * pl;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (cc < p.C) {
        const int l0 = 2 * lp, l1 = 2 * lp + 1;
        if (l0 < L) {
          v.x = load_weight(p.w[l0], p.w_dtype, cc * kPos + r);
          v.y = load_weight(p.w[l0], p.w_dtype, (cc + 1) * kPos + r);
        }
        if (l1 < L) {
          v.z = load_weight(p.w[l1], p.w_dtype, cc * kPos + r);
          v.w = load_weight(p.w[l1], p.w_dtype, (cc + 1) * kPos + r);
        }
      }
      ws[i] = v;
    }
  }
  __syncthreads();

  if (warp == kProducerWarp) {
    // ---------------- producer ----------------------------------------------------
    if (lane == 0) {
      prefetch_tmap(&p.tm_h);
      if constexpr (WGRAD) {
        for (int l = 0; l < LMAX; ++l)
          if (l < L) prefetch_tmap(&p.tm_low[l]);
      }
      const uint64_t pol = policy_evict_first();
      const uint32_t tx = Lay::kHBytes + (WGRAD ? static_cast<uint32_t>(L) * Lay::kLowTileBytes : 0u);
      const int64_t GG = static_cast<int64_t>(p.G) * p.G;
      int issued = 0;
      StripCursor cur(s_begin, p.G, p.strips_per_row);
      for (int it = 0; it < n_it; ++it, cur.next()) {
        const int s = it % Lay::kStages;
        const uint32_t ph = (it / Lay::kStages) & 1;
        if (it >= Lay::kStages && !mbar_wait(&empty[s], ph ^ 1)) break;
        const int64_t b = cur.b;
        const int wy = cur.wy, wx0 = cur.wx0();
        uint8_t* st = smem + s * Lay::kStageBytes;
        mbar_arrive_expect_tx(&full[s], tx);
        tma_load_4d(st, &p.tm_h, &full[s], static_cast<int32_t>(c0), 4 * wx0, 4 * wy, static_cast<int32_t>(b), pol);
        if constexpr (WGRAD) {
          const int32_t row0 = static_cast<int32_t>(b * GG + static_cast<int64_t>(wy) * p.G + wx0);
#pragma unroll
          for (int l = 0; l < LMAX; ++l)
            if (l < L)
              tma_load_2d(st + Lay::kHBytes + l * Lay::kLowTileBytes, &p.tm_low[l], &full[s],
                          static_cast<int32_t>(c0), row0, pol);
        }
        issued = it + 1;
      }
      for (int it = max(0, issued - Lay::kStages); it < issued; ++it)
        if (!mbar_wait(&full[it % Lay::kStages], (it / Lay::kStages) & 1)) break;
    }
    return;
  }

  const int64_t c = c0 + 2 * lane;
  const bool cvalid = c < p.C;
  const uint32_t smem_base = smem_u32(smem);

  if (WGRAD && warp < Lay::kWgradWarps) {
    // ---------------- weight-gradient consumers (cell row x layer group) ------------
    constexpr int LW = Lay::kWgradLayers;
    const int row = warp & 3;
    const int l0 = (warp >> 2) * LW;
    float2 acc[LW][4];
#pragma unroll
    for (int j = 0; j < LW; ++j)
#pragma unroll
      for (int col = 0; col < 4; ++col) acc[j][col] = make_float2(0.f, 0.f);
    StripCursor cur(s_begin, p.G, p.strips_per_row);
    for (int it = 0; it < n_it; ++it, cur.next()) {
      const int s = it % Lay::kStages;
      if (!mbar_wait(&full[s], (it / Lay::kStages) & 1)) break;
      const int ncell = min(kStripCells, p.G - cur.wx0());
      const uint32_t sb = smem_base + s * Lay::kStageBytes;
#pragma unroll
      for (int k = 0; k < kStripCells; ++k) {
        if (k < ncell) {
          float2 h[4];
#pragma unroll
          for (int col = 0; col < 4; ++col)
            h[col] = lds_pair<T>(sb + ((row * kBoxCols + 4 * k + col) * kSliceCh + 2 * lane) * kEs);
#pragma unroll
          for (int j = 0; j < LW; ++j) {
            if (l0 + j < L) {
              const float2 d =
                  lds_pair<T>(sb + Lay::kHBytes + (((l0 + j) * kStripCells + k) * kSliceCh + 2 * lane) * kEs);
#pragma unroll
              for (int col = 0; col < 4; ++col) acc[j][col] = ffma2(h[col], d, acc[j][col]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (cvalid) {
      float* P = p.partial + static_cast<int64_t>(blockIdx.x) * L * p.C * kPos;
#pragma unroll
      for (int j = 0; j < LW; ++j) {
        const int l = l0 + j;
        if (l < L) {
          *reinterpret_cast<float4*>(P + (l * p.C + c) * kPos + row * 4) =
              make_float4(acc[j][0].x, acc[j][1].x, acc[j][2].x, acc[j][3].x);
          *reinterpret_cast<float4*>(P + (l * p.C + c + 1) * kPos + row * 4) =
              make_float4(acc[j][0].y, acc[j][1].y, acc[j][2].y, acc[j][3].y);
        }
      }
    }
    return;
  }

  if constexpr (POOL) {
    // ---------------- pooling consumers (CELLS_PER_POOL cells x one layer group) ----
    constexpr int GP = Lay::kGroupPairs;
    const int pw = warp - kPoolWarp0;
    const int k0 = (pw / Lay::kLayerGroups) * CELLS_PER_POOL;
    const int lp0 = (pw % Lay::kLayerGroups) * GP;  // first layer pair of this warp
    const uint32_t wbase = smem_base + Lay::kWOffset + lane * 16;
    const int64_t GG = static_cast<int64_t>(p.G) * p.G;
    StripCursor cur(s_begin, p.G, p.strips_per_row);
    for (int it = 0; it < n_it; ++it, cur.next()) {
      const int s = it % Lay::kStages;
      if (!mbar_wait(&full[s], (it / Lay::kStages) & 1)) break;
      const int64_t b = cur.b;
      const int wy = cur.wy, wx0 = cur.wx0();
      const int ncell = min(kStripCells, p.G - wx0);
      const uint32_t sb = smem_base + s * Lay::kStageBytes;
      float2 acc[2 * GP][CELLS_PER_POOL];
#pragma unroll
      for (int l = 0; l < 2 * GP; ++l)
#pragma unroll
        for (int k = 0; k < CELLS_PER_POOL; ++k) acc[l][k] = make_float2(0.f, 0.f);
#pragma unroll kPoolUnroll
      for (int r = 0; r < kPos; ++r) {
        float2 h[CELLS_PER_POOL];
#pragma unroll
        for (int k = 0; k < CELLS_PER_POOL; ++k)
          h[k] = lds_pair<T>(sb + (((r >> 2) * kBoxCols + 4 * (k0 + k) + (r & 3)) * kSliceCh + 2 * lane) * kEs);
#pragma unroll
        for (int j = 0; j < GP; ++j) {
          if (lp0 + j < Lay::kLayerPairs) {
            const float4 wv = lds128f(wbase + (r * Lay::kLayerPairs + lp0 + j) * 32 * 16);
#pragma unroll
            for (int k = 0; k < CELLS_PER_POOL; ++k) {
              acc[2 * j][k] = ffma2(make_float2(wv.x, wv.y), h[k], acc[2 * j][k]);
              acc[2 * j + 1][k] = ffma2(make_float2(wv.z, wv.w), h[k], acc[2 * j + 1][k]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (cvalid) {
        const int64_t m0 = b * GG + static_cast<int64_t>(wy) * p.G + wx0;
#pragma unroll
        for (int k = 0; k < CELLS_PER_POOL; ++k) {
          if (k0 + k < ncell) {
#pragma unroll
            for (int j = 0; j < 2 * GP; ++j) {
              const int l = 2 * lp0 + j;
              if (l < L) Act<T>::st(static_cast<T*>(p.out[l]) + (m0 + k0 + k) * p.C + c, acc[j][k]);
            }
          }
        }
      }
    }
  }
}

}  // namespace lthc
