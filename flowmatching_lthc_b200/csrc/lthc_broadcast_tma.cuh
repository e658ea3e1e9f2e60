// Write family on the TMA pipeline: out = base + sum_{l<L} w_l (.) dz_l broadcast
// over each 4x4 cell (write, write_add, the fused materialisation and the read
// backward's grad_x).  The WGRAD variant is the whole read backward in one pass:
// its stages also carry the x tile, and the consumers add x (.) grad_z into
// per-lane sums that become one partial block per CTA (the read's grad_alpha,
// reduced in CTA order by reduce_partials_kernel), so x and grad_z are each read
// once.
//
// CTA = consumer warps + 1 producer warp, owning one 64-channel slice of the
// residual.  The producer's elected lane streams "strips" of kStripCells
// horizontally adjacent cells into a ring of shared-memory stages with TMA:
//   base tile  [4 rows][4*strip columns][64 channels] (box of the NHWC residual)
//   dz tiles   [L][4 cells][64 channels]           (box of each workspace update)
// A consumer warp owns one cell row (or, for L = 1 with a base, one position of
// the row: BcastShape); lane l owns channel pair (2l, 2l+1) and keeps
// w_l[c, 4*row + col] for all L layers and its columns in registers, so each
// weight is loaded once per CTA.  Per cell a lane reads 4 base pairs and
// L update pairs from shared memory (128 contiguous bytes per warp access, no
// bank conflicts), accumulates in fp32 with packed fp32x2 FMAs in the order
// base, l = 0, 1, ... and writes the rounded result back over the base tile,
// which one TMA store per strip then writes to the output.
// Full/empty mbarriers hand stages between producer and consumers; every wait
// is bounded (lthc_tma.cuh).
#pragma once

#include "lthc_common.cuh"
#include "lthc_tma.cuh"

namespace lthc {

// Pipeline shape.  A strip is kStripCells horizontally adjacent cells (its
// residual box spans 4 * kStripCells token columns); 16-bit activations use
// LTHC_BCAST_STAGES_16BIT (write family) / LTHC_STAGES_16BIT (read family)
// shared-memory stages per CTA, fp32 half as many.
#ifndef LTHC_STRIP_CELLS
#define LTHC_STRIP_CELLS 4
#endif
#ifndef LTHC_STAGES_16BIT
#define LTHC_STAGES_16BIT 3   // read family (lthc_pool_tma.cuh)
#endif
#ifndef LTHC_BCAST_STAGES_16BIT
#define LTHC_BCAST_STAGES_16BIT 6   // write family (this file), L != 1
#endif

constexpr int kStripCells = LTHC_STRIP_CELLS;
constexpr int kBoxCols = 4 * kStripCells;

// Consumer shape of the write-family kernel for a layer count and base.  Deep
// stacks (L = 12) keep one warp per cell row holding the weights of all 4
// columns in registers (each update pair loaded from shared memory feeds 4
// FMAs), two CTAs per SM.  A single update with a base (write_add) has almost
// no arithmetic and is bound by bytes in flight: one warp per cell (row,
// column) and a single CTA per SM with a deep ring.  Without a base (write, the
// read backward's grad_x) the loads are small and the output stores dominate:
// several CTAs per SM, each with several tile stores in flight (kStoreLag).
#ifndef LTHC_BCAST1_COLS
#define LTHC_BCAST1_COLS 1
#endif
#ifndef LTHC_BCAST1_MIN_BLOCKS
#define LTHC_BCAST1_MIN_BLOCKS 1
#endif
#ifndef LTHC_BCAST1_STAGES_16BIT
#define LTHC_BCAST1_STAGES_16BIT 15
#endif
#ifndef LTHC_BCAST_COLS
#define LTHC_BCAST_COLS 4
#endif
#ifndef LTHC_BCAST_MIN_BLOCKS
#define LTHC_BCAST_MIN_BLOCKS 3
#endif
#ifndef LTHC_BCAST_NOBASE_STORE_LAG
#define LTHC_BCAST_NOBASE_STORE_LAG 1
#endif
// With a base (materialisation, write_add) a CTA keeps two output tile stores
// in flight before it recycles a stage (measured on B200: materialisation
// +3.5 % at the bench's buffer placement, +8 % over a sweep of placements).
#ifndef LTHC_BCAST_BASE_STORE_LAG
#define LTHC_BCAST_BASE_STORE_LAG 2
#endif
// The read backward in one pass (WGRAD): grad_x = (grad_x_in +) alpha (.) grad_z and
// grad_alpha partials from x; its stages also carry the x tile.  Measured on B200
// at B = 64 bf16: without grad_x_in one CTA per SM with 12 stages (139 us against
// 171 us for two CTAs with 6); with grad_x_in (three residual streams) two CTAs
// with 6 (225 us against 244 us).
#ifndef LTHC_READBWD_STAGES_16BIT
#define LTHC_READBWD_STAGES_16BIT 12
#endif
#ifndef LTHC_READBWD_CTAS_PER_SM
#define LTHC_READBWD_CTAS_PER_SM 1
#endif
#ifndef LTHC_READBWD_BASE_STAGES_16BIT
#define LTHC_READBWD_BASE_STAGES_16BIT 6
#endif
#ifndef LTHC_READBWD_BASE_CTAS_PER_SM
#define LTHC_READBWD_BASE_CTAS_PER_SM 2
#endif
template <int LT, bool HAS_BASE, bool WGRAD = false>
struct BcastShape {
  static constexpr bool kSingle = LT == 1 && HAS_BASE && !WGRAD;
  static constexpr int kCols = kSingle ? LTHC_BCAST1_COLS : LTHC_BCAST_COLS;  // cell columns per consumer warp
  static constexpr int kWarpsPerRow = 4 / kCols;
  static_assert(kCols * kWarpsPerRow == 4, "columns per warp must divide 4");
  static constexpr int kConsumerWarps = 4 * kWarpsPerRow;
  static constexpr int kThreads = 32 * (kConsumerWarps + 1);
  static constexpr int kMinBlocks =
      WGRAD ? (HAS_BASE ? LTHC_READBWD_BASE_CTAS_PER_SM : LTHC_READBWD_CTAS_PER_SM)
            : (kSingle ? LTHC_BCAST1_MIN_BLOCKS : LTHC_BCAST_MIN_BLOCKS);
  static constexpr int kStages16 =
      WGRAD ? (HAS_BASE ? LTHC_READBWD_BASE_STAGES_16BIT : LTHC_READBWD_STAGES_16BIT)
            : (kSingle ? LTHC_BCAST1_STAGES_16BIT : LTHC_BCAST_STAGES_16BIT);
  // Output tile stores a CTA keeps in flight before it recycles a stage.
  static constexpr int kStoreLag = HAS_BASE ? LTHC_BCAST_BASE_STORE_LAG : LTHC_BCAST_NOBASE_STORE_LAG;
};

template <typename T, int LT, bool HAS_BASE, bool WGRAD = false>
struct BcastLayout {
  using Shape = BcastShape<LT, HAS_BASE, WGRAD>;
  static constexpr int LMAX = LT > 0 ? LT : kMaxLayers;
  static constexpr int kBaseBytes = 4 * kBoxCols * kSliceCh * static_cast<int>(sizeof(T));
  static constexpr int kDzTileBytes = kStripCells * kSliceCh * static_cast<int>(sizeof(T));
  static constexpr int kXOffset = kBaseBytes + LMAX * kDzTileBytes;  // x tile (WGRAD)
  static constexpr int kStageBytes = kXOffset + (WGRAD ? kBaseBytes : 0);
  static constexpr int kStages = sizeof(T) == 2 ? Shape::kStages16 : (Shape::kStages16 + 1) / 2;
  static_assert(Shape::kStoreLag >= 1 && Shape::kStoreLag < kStages, "store lag must be below the stage count");
  static constexpr int kBarrierOffset = kStages * kStageBytes;
  static constexpr int kSmemBytes = kBarrierOffset + 2 * kStages * 8 + 128;  // + alignment slack
  static_assert(kSmemBytes <= 227 * 1024, "write-family stages exceed the shared memory of a CTA");
};

struct BcastTmaParams {
  CUtensorMap tm_base;                 // 4D (C, 4G, 4G, B) box (64, 16, 4, 1); unused without a base
  CUtensorMap tm_out;                  // 4D map of the output, same box
  CUtensorMap tm_dz[kMaxLayers];       // 2D (C, B*G*G) box (64, 4)
  CUtensorMap tm_x;                    // WGRAD: 4D map of x, same box
  const void* w[kMaxLayers];           // [C, 16] weights, dtype w_dtype
  float* partial;                      // WGRAD: [gridDim.x][C][16] per-CTA sums of x (.) grad_z
  void* out;                           // T[B, 4G, 4G, C]
  int w_dtype;
  int L;
  int G;
  int strips_per_row;                  // ceil(G / 4)
  int64_t C;
  int64_t strips;                      // B * G * strips_per_row
  int64_t strips_per_cta;
};

// Position of a strip: image b, cell row wy, first cell column wx0.  A CTA walks
// consecutive strips, so the cursor advances with adds and compares only (the
// 64-bit division happens once, when the cursor is created).
struct StripCursor {
  int64_t b;
  int wy;
  int sx;   // strip index inside the cell row
  int G;
  int spr;  // strips per cell row
  __device__ __forceinline__ StripCursor(int64_t strip, int G_, int spr_) : G(G_), spr(spr_) {
    const int64_t per_img = static_cast<int64_t>(G_) * spr_;
    b = strip / per_img;
    const int rem = static_cast<int>(strip - b * per_img);
    wy = rem / spr_;
    sx = rem - wy * spr_;
  }
  __device__ __forceinline__ int wx0() const { return sx * kStripCells; }
  __device__ __forceinline__ void next() {
    if (++sx == spr) {
      sx = 0;
      if (++wy == G) {
        wy = 0;
        ++b;
      }
    }
  }
};

template <typename T, int LT, bool HAS_BASE, bool WGRAD = false>
__global__ void __launch_bounds__(BcastShape<LT, HAS_BASE, WGRAD>::kThreads,
                                  BcastShape<LT, HAS_BASE, WGRAD>::kMinBlocks)
    broadcast_tma_kernel(const __grid_constant__ BcastTmaParams p) {
  constexpr int LMAX = LT > 0 ? LT : kMaxLayers;
  static_assert(!WGRAD || LT == 1, "the fused read backward has one update (grad_z)");
  using Lay = BcastLayout<T, LT, HAS_BASE, WGRAD>;
  using Shape = typename Lay::Shape;
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
      mbar_init(&empty[s], 1);  // released by the thread that stores the stage's output tile
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == Shape::kConsumerWarps) {
    // ---------------- producer: one elected lane issues every TMA load ----------
    if (lane == 0) {
      if constexpr (HAS_BASE) prefetch_tmap(&p.tm_base);
      if constexpr (WGRAD) prefetch_tmap(&p.tm_x);
      for (int l = 0; l < LMAX; ++l)
        if (l < L) prefetch_tmap(&p.tm_dz[l]);
      const uint64_t pol = policy_evict_first();
      const uint32_t tx = (HAS_BASE ? Lay::kBaseBytes : 0) + static_cast<uint32_t>(L) * Lay::kDzTileBytes +
                          (WGRAD ? Lay::kBaseBytes : 0);
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
        if constexpr (HAS_BASE)
          tma_load_4d(st, &p.tm_base, &full[s], static_cast<int32_t>(c0), 4 * wx0, 4 * wy, static_cast<int32_t>(b),
                      pol);
        if constexpr (WGRAD)
          tma_load_4d(st + Lay::kXOffset, &p.tm_x, &full[s], static_cast<int32_t>(c0), 4 * wx0, 4 * wy,
                      static_cast<int32_t>(b), pol);
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
  // Each lane computes its 4 columns x cells of the strip in place over the staged
  // base tile; then one elected thread writes the whole tile with a TMA store
  // (which clips columns past the residual edge and channels past C) and hands
  // the stage back to the producer once the store has read it.
  constexpr int kCols = Shape::kCols;
  const int row = warp / Shape::kWarpsPerRow;
  const int col0 = (warp % Shape::kWarpsPerRow) * kCols;
  const int64_t c = c0 + 2 * lane;
  const bool cvalid = c < p.C;
  float2 w[LMAX][kCols];
#pragma unroll
  for (int l = 0; l < LMAX; ++l) {
#pragma unroll
    for (int col = 0; col < kCols; ++col) {
      if (cvalid && l < L) {
        w[l][col].x = load_weight(p.w[l], p.w_dtype, c * kPos + row * 4 + col0 + col);
        w[l][col].y = load_weight(p.w[l], p.w_dtype, (c + 1) * kPos + row * 4 + col0 + col);
      } else {
        w[l][col] = make_float2(0.f, 0.f);
      }
    }
  }
  const uint32_t smem_base = smem_u32(smem);
  constexpr uint32_t kEs = sizeof(T);
  const bool storer = warp == 0 && lane == 0;
  float2 accw[kCols];  // WGRAD: sum over cells of x (.) grad_z for this lane's columns, in strip order
#pragma unroll
  for (int col = 0; col < kCols; ++col) accw[col] = make_float2(0.f, 0.f);
  StripCursor cur(s_begin, p.G, p.strips_per_row);

  for (int it = 0; it < n_it; ++it, cur.next()) {
    const int s = it % Lay::kStages;
    if (!mbar_wait(&full[s], (it / Lay::kStages) & 1)) break;
    const uint32_t sb = smem_base + s * Lay::kStageBytes;
#pragma unroll
    for (int k = 0; k < kStripCells; ++k) {
      float2 acc[kCols];
      const uint32_t xa = sb + ((row * kBoxCols + 4 * k + col0) * kSliceCh + 2 * lane) * kEs;
#pragma unroll
      for (int col = 0; col < kCols; ++col) {
        if constexpr (HAS_BASE)
          acc[col] = lds_pair<T>(xa + col * kSliceCh * kEs);
        else
          acc[col] = make_float2(0.f, 0.f);
      }
#pragma unroll
      for (int l = 0; l < LMAX; ++l) {
        if (l < L) {
          const float2 d = lds_pair<T>(sb + Lay::kBaseBytes + ((l * kStripCells + k) * kSliceCh + 2 * lane) * kEs);
#pragma unroll
          for (int col = 0; col < kCols; ++col) acc[col] = ffma2(w[l][col], d, acc[col]);
          if constexpr (WGRAD) {
            // cells past the grid edge are zero in both tiles (TMA fill), so they add nothing
#pragma unroll
            for (int col = 0; col < kCols; ++col)
              accw[col] = ffma2(lds_pair<T>(xa + Lay::kXOffset + col * kSliceCh * kEs), d, accw[col]);
          }
        }
      }
#pragma unroll
      for (int col = 0; col < kCols; ++col) sts_pair<T>(xa + col * kSliceCh * kEs, acc[col]);
    }
    fence_proxy_async_smem();
    // All consumer warps wait on the same stage transaction, with 2-second limits
    // that start within microseconds of each other: a warp leaves the loop when that
    // transaction has not completed for 2 s, and the others give up with it unless
    // the transaction completes inside those microseconds (the producer stops
    // issuing once its own bounded wait fails, so a stalled pipeline does not
    // recover).  A bounded mbarrier hand-off here, or bar.red.and, would close that
    // window but measured 6-14 % slower on the single-layer shapes (write_add,
    // read backward).
    named_barrier(1, 32 * Shape::kConsumerWarps);
    if (storer) {
      tma_store_4d(&p.tm_out, smem + s * Lay::kStageBytes, static_cast<int32_t>(c0), 4 * cur.wx0(), 4 * cur.wy,
                   static_cast<int32_t>(cur.b));
      bulk_commit();
      // The store issued kStoreLag strips ago has read its tile: recycle that stage.
      bulk_wait_read<Shape::kStoreLag>();
      if (it >= Shape::kStoreLag) mbar_arrive(&empty[(it - Shape::kStoreLag) % Lay::kStages]);
    }
  }
  if constexpr (WGRAD) {
    if (cvalid) {
      float* P = p.partial + static_cast<int64_t>(blockIdx.x) * p.C * kPos;
#pragma unroll
      for (int col = 0; col < kCols; ++col) {
        P[c * kPos + row * 4 + col0 + col] = accw[col].x;
        P[(c + 1) * kPos + row * 4 + col0 + col] = accw[col].y;
      }
    }
  }
  if (storer) bulk_wait_all();
}

}  // namespace lthc
