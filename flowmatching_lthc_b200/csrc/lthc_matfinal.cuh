// The materialisation fused with the final layer's RMSNorm + shared-AdaLN
// modulate (inference):
//   X_L = X_0 + sum_l beta_l (.) dZ_l                 final_accumulate_reference
//                                                     (local_thc.py:1368-1372, 1416-1420)
//   m   = modulate(RMSNorm(X_L), shift, scale)        FinalLayerSharedAdaLN.forward without
//                                                     its Linear (:865-873, :37-38;
//                                                     RMSNorm jit_shared_adaln.py:20-30)
// X_L never leaves the chip: the kernel writes m only.
//
// The write-family pipeline (lthc_broadcast_tma.cuh) owns 64-channel slices, but
// the norm needs each token's sum of squares over all C channels.  The CTAs of
// the ceil(C/64) slices of one strip range form a thread-block cluster and walk
// the same strips in the same order.  Per strip each consumer warp (one residual
// row of the strip, 16 tokens) rounds X_L to the activation dtype, forms its
// slice's partial sum of squares per token and pushes the 16 sums into a slot of
// every cluster peer's shared memory (st.async, completion counted in bytes on the
// peer's mbarrier).  Once a CTA holds the partials of every slice it adds them in
// slice order (so every CTA derives the same rstd), applies the norm and the
// modulation to its 64 channels, stores the m tile with TMA and releases the
// slot to all senders with one remote mbarrier arrival each.  Every wait is a bounded
// mbarrier wait (2 s, then the device error word is set and the kernel returns).
#pragma once

#include "lthc_broadcast_tma.cuh"
#include "lthc_final.cuh"

namespace lthc {

// ---- cluster / distributed shared memory ----------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of every CTA of the cluster arrives and waits (used once, after
// the mbarriers are initialised and before any peer touches them).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The address of this CTA's shared-memory location `addr` in the CTA of cluster
// rank `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// 16-byte store into a peer's shared memory; its bytes count toward the peer's
// mbarrier transaction count.
__device__ __forceinline__ void st_async_v4(uint32_t raddr, float4 v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   raddr),
               "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(rbar)
               : "memory");
}

__device__ __forceinline__ void mbar_remote_arrive(uint32_t rbar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(rbar) : "memory");
}

// ---- kernel ----------------------------------------------------------------------
constexpr int kMatFinalMaxSlices = 16;      // C <= 1024: a cluster of at most 16 CTAs
constexpr int kStripTokens = 4 * kBoxCols;  // tokens of one strip (4 rows x 16 columns)

// Pipeline.  The load ring (kStages stages of X_0 + L update tiles) only feeds
// phase A, which rounds X_L into a separate ring of kRing output tiles and hands
// the load stage straight back, so every load stage stays available for
// prefetching.  Phase B of a strip runs kLook iterations after its phase A (its
// partials cross the cluster meanwhile); its output tile is stored by TMA and
// reused once at most kStoreLag newer stores are still reading it, which needs
// kRing >= kLook + kStoreLag + 2.  kXSlots exchange slots hold the partials of
// the strips between their phase A and their phase B.
#ifndef LTHC_MATFINAL_STAGES_16BIT
#define LTHC_MATFINAL_STAGES_16BIT 4
#endif
#ifndef LTHC_MATFINAL_LOOK_16BIT
#define LTHC_MATFINAL_LOOK_16BIT 2
#endif
template <typename T, int LT>
struct MatFinalPipe {
  static constexpr bool k16 = sizeof(T) == 2;
  static constexpr int kStages = k16 ? LTHC_MATFINAL_STAGES_16BIT : 2;
  static constexpr int kLook = k16 ? LTHC_MATFINAL_LOOK_16BIT : 1;
  static constexpr int kStoreLag = 1;
  static constexpr int kRing = kLook + kStoreLag + 2;
  static constexpr int kXSlots = kLook + 1;
  static constexpr int kMinBlocks = k16 ? 2 : 1;
};

struct MatFinalParams {
  BcastTmaParams m;       // tm_base = X_0, tm_dz / w = the updates and betas, tm_out = m
  const void* norm_w;     // [C] RMSNorm weight, dtype norm_w_dtype
  const void* shift;      // [B] rows of C (row stride mod_stride), activation dtype
  const void* scale;
  int norm_w_dtype;
  float eps;
  float inv_c;            // 1.0f / C
  int64_t mod_stride;
};

template <typename T, int LT>
struct MatFinalLayout {
  using Base = BcastLayout<T, LT, true>;
  using Pipe = MatFinalPipe<T, LT>;
  static constexpr int kStages = Pipe::kStages;
  static constexpr int kRing = Pipe::kRing;
  static constexpr int kXSlots = Pipe::kXSlots;
  static constexpr int kStageBytes = Base::kStageBytes;  // X_0 tile + L update tiles
  static constexpr int kTileBytes = Base::kBaseBytes;    // one X_L / m tile
  static constexpr int kRingOffset = kStages * kStageBytes;
  static constexpr int kRecvOffset = kRingOffset + kRing * kTileBytes;
  static constexpr int kRecvBytes = kXSlots * kMatFinalMaxSlices * kStripTokens * 4;
  static constexpr int kBarrierOffset = kRecvOffset + kRecvBytes;
  static constexpr int kSmemBytes = kBarrierOffset + (2 * kStages + 2 * kXSlots) * 8 + 128;
  static_assert(kStageBytes % 128 == 0 && kTileBytes % 128 == 0, "128-byte aligned tiles");
  static_assert(Pipe::kMinBlocks * (kSmemBytes + 1024) <= 228 * 1024, "shared memory of the resident CTAs");
};

// Sum of v[0..15] over the 32 lanes, scattered: afterwards lanes 2t and 2t + 1
// hold the total of value t (four halving exchange steps, then one add).
__device__ __forceinline__ float reduce_scatter16(float (&v)[16], int lane) {
#pragma unroll
  for (int n = 16, o = 16; n > 1; n >>= 1, o >>= 1) {
    const bool hi = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = hi ? v[i] : v[i + n / 2];
      const float keep = hi ? v[i + n / 2] : v[i];
      v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, o));
    }
  }
  return __fadd_rn(v[0], __shfl_xor_sync(0xffffffffu, v[0], 1));
}

// Named barrier over `count` threads that also returns whether `pred` held in all
// of them (every thread sees the same answer).
__device__ __forceinline__ bool named_barrier_and(int id, int count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.and.pred p, %2, %3, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

template <typename T>
__device__ __forceinline__ void sts_raw(uint32_t addr, typename Pair<T>::R v) {
  if constexpr (sizeof(T) == 4)
    sts64f(addr, v);
  else
    sts32(addr, v);
}

template <typename T, int LT>
__global__ void __launch_bounds__(BcastShape<LT, true>::kThreads, MatFinalPipe<T, LT>::kMinBlocks)
    materialise_final_kernel(const __grid_constant__ MatFinalParams q) {
  constexpr int LMAX = LT > 0 ? LT : kMaxLayers;
  using Lay = MatFinalLayout<T, LT>;
  using Shape = BcastShape<LT, true>;
  static_assert(Shape::kCols == 4 && Shape::kConsumerWarps == 4, "one consumer warp per residual row of a strip");
  using P2 = Pair<T>;
  using R = typename P2::R;
  const BcastTmaParams& p = q.m;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Lay::kBarrierOffset);
  uint64_t* empty = full + Lay::kStages;
  uint64_t* xfull = empty + Lay::kStages;
  uint64_t* xempty = xfull + Lay::kXSlots;
  float* recv = reinterpret_cast<float*>(smem + Lay::kRecvOffset);  // [slot][slice][token]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int L = LT > 0 ? LT : p.L;
  const int nsl = static_cast<int>(gridDim.y);  // cluster = the slices of one strip range
  const uint32_t rank = cluster_ctarank();
  const int64_t c0 = static_cast<int64_t>(blockIdx.y) * kSliceCh;
  const int64_t s_begin = static_cast<int64_t>(blockIdx.x) * p.strips_per_cta;
  const int64_t s_end = min(s_begin + p.strips_per_cta, p.strips);
  const int n_it = s_end > s_begin ? static_cast<int>(s_end - s_begin) : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Lay::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], Shape::kConsumerWarps);  // each consumer warp, once phase A has read the stage
    }
    for (int x = 0; x < Lay::kXSlots; ++x) {
      mbar_init(&xfull[x], 1);                             // + the peers' bytes
      mbar_init(&xempty[x], nsl);  // one release from every CTA of the cluster
    }
    fence_barrier_init();
  }
  __syncthreads();
  cluster_sync_all();  // no peer touches this CTA's barriers before they exist

  if (warp == Shape::kConsumerWarps) {
    // ---------------- producer: as the write family (base + L update tiles) ------
    if (lane == 0) {
      prefetch_tmap(&p.tm_base);
      for (int l = 0; l < LMAX; ++l)
        if (l < L) prefetch_tmap(&p.tm_dz[l]);
      const uint64_t pol = policy_evict_first();
      const uint32_t tx = Lay::Base::kBaseBytes + static_cast<uint32_t>(L) * Lay::Base::kDzTileBytes;
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
        tma_load_4d(st, &p.tm_base, &full[s], static_cast<int32_t>(c0), 4 * wx0, 4 * wy, static_cast<int32_t>(b), pol);
        const int32_t row0 = static_cast<int32_t>(b * GG + static_cast<int64_t>(wy) * p.G + wx0);
#pragma unroll
        for (int l = 0; l < LMAX; ++l)
          if (l < L)
            tma_load_2d(st + Lay::Base::kBaseBytes + l * Lay::Base::kDzTileBytes, &p.tm_dz[l], &full[s],
                        static_cast<int32_t>(c0), row0, pol);
        issued = it + 1;
      }
      // Do not leave while copies into this CTA's shared memory are in flight.
      for (int it = max(0, issued - Lay::kStages); it < issued; ++it)
        if (!mbar_wait(&full[it % Lay::kStages], (it / Lay::kStages) & 1)) break;
    }
    return;
  }

  // ---------------- consumers: warp `row` owns residual row `row` of the strip ------
  // Software pipeline: iteration it runs phase A of strip it (X_L, rounded, into
  // the staged tile; partial sums pushed to the cluster) and phase B of strip
  // it - kLook (totals, rstd, m over the tile, TMA store), so the exchange of a
  // strip overlaps the next strips' arithmetic.
  constexpr int kLook = MatFinalPipe<T, LT>::kLook;
  constexpr int kLag = MatFinalPipe<T, LT>::kStoreLag;
  constexpr int kXS = MatFinalPipe<T, LT>::kXSlots;
  constexpr int kRing = MatFinalPipe<T, LT>::kRing;
  static_assert(kRing >= kLook + kLag + 2, "an output tile is rewritten only after its store has read it");
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
  const float2 nw = cvalid ? make_float2(load_weight(q.norm_w, q.norm_w_dtype, c),
                                         load_weight(q.norm_w, q.norm_w_dtype, c + 1))
                           : make_float2(0.f, 0.f);
  int64_t mod_b = -1;
  float2 shv = make_float2(0.f, 0.f);
  R s1r = P2::rn(make_float2(0.f, 0.f));

  const uint32_t smem_base = smem_u32(smem);
  const uint32_t recv_base = smem_u32(recv);
  constexpr uint32_t kEs = sizeof(T);
  const bool storer = warp == 0 && lane == 0;
  const int grp = lane >> 3;  // 16-byte chunk (4 tokens) this lane sends
  int sent = 0;               // strips whose partials this warp has pushed to the cluster
  bool ok = true;             // this warp's waits so far succeeded
  StripCursor curB(s_begin, p.G, p.strips_per_row);

  for (int it = 0; it < n_it + kLook; ++it) {
    // ---------------- phase A: strip it ----------------------------------------
    if (it < n_it && ok) {
      const int s = it % Lay::kStages;
      const int x = it % kXS;
      if (storer) mbar_arrive_expect_tx(&xfull[x], static_cast<uint32_t>(nsl * kStripTokens * 4));
      ok = __all_sync(0xffffffffu, mbar_wait(&full[s], (it / Lay::kStages) & 1));
      if (ok) {
        const uint32_t sb = smem_base + s * Lay::kStageBytes;
        const uint32_t ob = smem_base + Lay::kRingOffset + (it % kRing) * Lay::kTileBytes;
        float sq[16];
#pragma unroll
        for (int k = 0; k < kStripCells; ++k) {
          const uint32_t tok = ((row * kBoxCols + 4 * k) * kSliceCh + 2 * lane) * kEs;
          const uint32_t xa = sb + tok;
          float2 acc[4];
#pragma unroll
          for (int col = 0; col < 4; ++col) acc[col] = lds_pair<T>(xa + col * kSliceCh * kEs);
#pragma unroll
          for (int l = 0; l < LMAX; ++l) {
            if (l < L) {
              const float2 d =
                  lds_pair<T>(sb + Lay::Base::kBaseBytes + ((l * kStripCells + k) * kSliceCh + 2 * lane) * kEs);
#pragma unroll
              for (int col = 0; col < 4; ++col) acc[col] = ffma2(w[l][col], d, acc[col]);
            }
          }
#pragma unroll
          for (int col = 0; col < 4; ++col) {
            const R rr = P2::rn(acc[col]);  // X_L as the materialisation stores it
            sts_raw<T>(ob + tok + col * kSliceCh * kEs, rr);
            const float2 v = P2::f(rr);
            sq[4 * k + col] = __fadd_rn(__fmul_rn(v.x, v.x), __fmul_rn(v.y, v.y));
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);  // the load stage is free for the next strips
        const float part = reduce_scatter16(sq, lane);  // lanes 2t, 2t + 1: token t of this row
        float4 chunk;
        chunk.x = __shfl_sync(0xffffffffu, part, 8 * grp + 0);
        chunk.y = __shfl_sync(0xffffffffu, part, 8 * grp + 2);
        chunk.z = __shfl_sync(0xffffffffu, part, 8 * grp + 4);
        chunk.w = __shfl_sync(0xffffffffu, part, 8 * grp + 6);
        // The slot's previous strip must be released by every receiver.
        if (it >= kXS) ok = __all_sync(0xffffffffu, mbar_wait(&xempty[x], ((it / kXS) - 1) & 1));
        if (ok) {
          const uint32_t off = ((x * kMatFinalMaxSlices + rank) * kStripTokens + row * 16 + 4 * grp) * 4;
          const uint32_t bar = smem_u32(&xfull[x]);
          for (int pr = lane & 7; pr < nsl; pr += 8)
            st_async_v4(mapa_shared(recv_base + off, pr), chunk, mapa_shared(bar, pr));
          sent = it + 1;
        }
      }
    }
    // ---------------- phase B: strip j = it - kLook ------------------------------
    const int j = it - kLook;
    if (j < 0) continue;
    const int x = j % kXS;
    const uint32_t sb = smem_base + Lay::kRingOffset + (j % kRing) * Lay::kTileBytes;
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&xfull[x], (j / kXS) & 1));
    if (ok) {
      // Token totals in slice order (identical in every CTA of the cluster), rstd.
      float r = 0.f;
      if (lane < 16) {
        const float* rv = recv + (x * kMatFinalMaxSlices) * kStripTokens + row * 16 + lane;
        float tot = 0.f;
        for (int k = 0; k < nsl; ++k) tot = __fadd_rn(tot, rv[k * kStripTokens]);
        r = rsqrtf(__fadd_rn(__fmul_rn(tot, q.inv_c), q.eps));
      }
      if (curB.b != mod_b) {  // the image's modulation rows (a strip lies in one image)
        mod_b = curB.b;
        if (cvalid) {
          const T* shp = static_cast<const T*>(q.shift) + mod_b * q.mod_stride;
          const T* scp = static_cast<const T*>(q.scale) + mod_b * q.mod_stride;
          shv = make_float2(act_load(shp, c), act_load(shp, c + 1));
          s1r = P2::rn(make_float2(__fadd_rn(1.f, act_load(scp, c)), __fadd_rn(1.f, act_load(scp, c + 1))));
        }
      }
      // m = modulate(norm(X_L)) over the staged tile.
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const float rt = __shfl_sync(0xffffffffu, r, t);
        const uint32_t a = sb + ((row * kBoxCols + t) * kSliceCh + 2 * lane) * kEs;
        const float2 tt = fmul2(lds_pair<T>(a), make_float2(rt, rt));
        const R nr = P2::rn(fmul2(tt, nw));
        sts_raw<T>(a, P2::rn(fadd2(P2::f(P2::mul(nr, s1r)), shv)));
      }
      fence_proxy_async_smem();
    }
    // A failed wait in any consumer warp ends the loop for all of them together.
    if (!named_barrier_and(1, 32 * Shape::kConsumerWarps, ok)) break;
    // Every consumer warp has read slot x: release it to every sender (once per CTA).
    if (warp == 0 && lane < nsl) mbar_remote_arrive(mapa_shared(smem_u32(&xempty[x]), lane));
    if (storer) {
      tma_store_4d(&p.tm_out, smem + Lay::kRingOffset + (j % kRing) * Lay::kTileBytes, static_cast<int32_t>(c0),
                   4 * curB.wx0(), 4 * curB.wy, static_cast<int32_t>(curB.b));
      bulk_commit();
      // Before the next consumer barrier: at most kLag stores still read their tiles,
      // so phase A may overwrite the tile of strip (next) - kRing.
      bulk_wait_read<kLag>();
    }
    curB.next();
  }
  if (storer) {
    bulk_wait_all();
    // Do not leave while peers may still arrive on this CTA's slot barriers: the
    // receivers release each strip this CTA sent to every sender, so wait for the
    // releases of the last strips sent.
    for (int k = max(0, sent - kXS); k < sent; ++k)
      if (!mbar_wait(&xempty[k % kXS], (k / kXS) & 1)) break;
  }
}

}  // namespace lthc
