// Write family on the TMA pipeline: out = base + sum_{l<L} w_l (.) dz_l broadcast
// over each 4x4 cell (write, write_add, the fused materialisation and the read
// backward's grad_x).
//
// CTA = 4 consumer warps + 1 producer warp, owning one 64-channel slice of the
// residual.  The producer's elected lane streams "strips" of 4 horizontally
// adjacent cells into a ring of shared-memory stages with TMA:
//   base tile  [4 rows][16 columns][64 channels]   (box of the NHWC residual)
//   dz tiles   [L][4 cells][64 channels]           (box of each workspace update)
// Consumer warp `row` owns cell row `row`; lane l owns channel pair (2l, 2l+1)
// and keeps w_l[c, 4*row + col] for all L layers and 4 columns in registers, so
// each weight is loaded once per CTA.  Per cell a lane reads 4 base pairs and
// L update pairs from shared memory (128 contiguous bytes per warp access, no
// bank conflicts), accumulates in fp32 with packed fp32x2 FMAs in the order
// base, l = 0, 1, ... and stores 4 pairs with streaming stores.
// Full/empty mbarriers hand stages between producer and consumers; every wait
// is bounded (lthc_tma.cuh).
#pragma once

#include "lthc_common.cuh"
#include "lthc_tma.cuh"

namespace lthc {

constexpr int kStripCells = 4;
constexpr int kBcastConsumerWarps = 4;
constexpr int kBcastThreads = 32 * (kBcastConsumerWarps + 1);

template <typename T, int LMAX>
struct BcastLayout {
  static constexpr int kBaseBytes = 4 * 16 * kSliceCh * static_cast<int>(sizeof(T));
  static constexpr int kDzTileBytes = kStripCells * kSliceCh * static_cast<int>(sizeof(T));
  static constexpr int kStageBytes = kBaseBytes + LMAX * kDzTileBytes;
  static constexpr int kStages = sizeof(T) == 2 ? 4 : 2;
  static constexpr int kBarrierOffset = kStages * kStageBytes;
  static constexpr int kSmemBytes = kBarrierOffset + 2 * kStages * 8 + 128;  // + alignment slack
};

struct BcastTmaParams {
  CUtensorMap tm_base;                 // 4D (C, 4G, 4G, B) box (64, 16, 4, 1); unused without a base
  CUtensorMap tm_dz[kMaxLayers];       // 2D (C, B*G*G) box (64, 4)
  const void* w[kMaxLayers];           // [C, 16] weights, dtype w_dtype
  void* out;                           // T[B, 4G, 4G, C]
  int w_dtype;
  int L;
  int G;
  int strips_per_row;                  // ceil(G / 4)
  int64_t C;
  int64_t strips;                      // B * G * strips_per_row
  int64_t strips_per_cta;
};

__device__ __forceinline__ void strip_coords(int64_t strip, int G, int spr, int64_t& b, int& wy, int& wx0) {
  const int64_t per_img = static_cast<int64_t>(G) * spr;
  b = strip / per_img;
  const int rem = static_cast<int>(strip - b * per_img);
  wy = rem / spr;
  wx0 = (rem - wy * spr) * kStripCells;
}

template <typename T, int LT, bool HAS_BASE>
__global__ void __launch_bounds__(kBcastThreads, 3) broadcast_tma_kernel(const __grid_constant__ BcastTmaParams p) {
  constexpr int LMAX = LT > 0 ? LT : kMaxLayers;
  using Lay = BcastLayout<T, LMAX>;
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
      mbar_init(&empty[s], kBcastConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kBcastConsumerWarps) {
    // ---------------- producer: one elected lane issues every TMA load ----------
    if (lane == 0) {
      if constexpr (HAS_BASE) prefetch_tmap(&p.tm_base);
      for (int l = 0; l < LMAX; ++l)
        if (l < L) prefetch_tmap(&p.tm_dz[l]);
      const uint64_t pol = policy_evict_first();
      const uint32_t tx = (HAS_BASE ? Lay::kBaseBytes : 0) + static_cast<uint32_t>(L) * Lay::kDzTileBytes;
      const int64_t GG = static_cast<int64_t>(p.G) * p.G;
      int issued = 0;
      for (int it = 0; it < n_it; ++it) {
        const int s = it % Lay::kStages;
        const uint32_t ph = (it / Lay::kStages) & 1;
        if (it >= Lay::kStages && !mbar_wait(&empty[s], ph ^ 1)) break;
        int64_t b;
        int wy, wx0;
        strip_coords(s_begin + it, p.G, p.strips_per_row, b, wy, wx0);
        uint8_t* st = smem + s * Lay::kStageBytes;
        mbar_arrive_expect_tx(&full[s], tx);
        if constexpr (HAS_BASE)
          tma_load_4d(st, &p.tm_base, &full[s], static_cast<int32_t>(c0), 4 * wx0, 4 * wy, static_cast<int32_t>(b),
                      pol);
        const int32_t row0 = static_cast<int32_t>(b * GG + static_cast<int64_t>(wy) * p.G + wx0);
#pragma unroll
        for (int l = 0; l < LMAX; ++l)
          if (l < L)
            tma_load_2d(st + Lay::kBaseBytes + l * Lay::kDzTileBytes, &p.tm_dz[l], &full[s], static_cast<int32_t>(c0),
                        row0, pol);
        issued = it + 1;
      }
      // Do not leave while copies into this CTA's shared memory are in flight.
      for (int it = max(0, issued - Lay::kStages); it < issued; ++it)
        if (!mbar_wait(&full[it % Lay::kStages], (it / Lay::kStages) & 1)) break;
    }
    return;
  }

  // ---------------- consumers ---------------------------------------------------
  const int row = warp;
  const int64_t c = c0 + 2 * lane;
  const bool cvalid = c < p.C;
  float2 w[LMAX][4];
#pragma unroll
  for (int l = 0; l < LMAX; ++l) {
#pragma unroll
    for (int col = 0; col < 4; ++col) {
      if (cvalid && l < L) {
        w[l][col].x = load_weight(p.w[l], p.w_dtype, c * kPos + row * 4 + col);
        w[l][col].y = load_weight(p.w[l], p.w_dtype, (c + 1) * kPos + row * 4 + col);
      } else {
        w[l][col] = make_float2(0.f, 0.f);
      }
    }
  }
  T* out = static_cast<T*>(p.out);
  const int64_t H = 4 * static_cast<int64_t>(p.G);
  const uint32_t smem_base = smem_u32(smem);
  constexpr uint32_t kEs = sizeof(T);

  for (int it = 0; it < n_it; ++it) {
    const int s = it % Lay::kStages;
    if (!mbar_wait(&full[s], (it / Lay::kStages) & 1)) break;
    int64_t b;
    int wy, wx0;
    strip_coords(s_begin + it, p.G, p.strips_per_row, b, wy, wx0);
    const uint32_t sb = smem_base + s * Lay::kStageBytes;
    const int ncell = min(kStripCells, p.G - wx0);
    if (cvalid) {
      const int64_t tok_row = ((b * H + 4 * wy + row) * H + 4 * wx0) * p.C + c;
#pragma unroll
      for (int k = 0; k < kStripCells; ++k) {
        if (k < ncell) {
          float2 acc[4];
#pragma unroll
          for (int col = 0; col < 4; ++col) {
            if constexpr (HAS_BASE)
              acc[col] = lds_pair<T>(sb + ((row * 16 + 4 * k + col) * kSliceCh + 2 * lane) * kEs);
            else
              acc[col] = make_float2(0.f, 0.f);
          }
#pragma unroll
          for (int l = 0; l < LMAX; ++l) {
            if (l < L) {
              const float2 d = lds_pair<T>(sb + Lay::kBaseBytes + ((l * kStripCells + k) * kSliceCh + 2 * lane) * kEs);
#pragma unroll
              for (int col = 0; col < 4; ++col) acc[col] = ffma2(w[l][col], d, acc[col]);
            }
          }
          T* dst = out + tok_row + static_cast<int64_t>(4 * k) * p.C;
#pragma unroll
          for (int col = 0; col < 4; ++col) Act<T>::st_stream(dst + col * p.C, acc[col]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
}

}  // namespace lthc
