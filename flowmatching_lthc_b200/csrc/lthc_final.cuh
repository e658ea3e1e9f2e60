// Final-layer prologue over the materialised residual, forward and backward:
//   n = (x.float() * rsqrt(mean_c(x.float()^2) + eps) * w).to(dtype)    RMSNorm
//   m = n * (1 + scale[b]) + shift[b]                                    modulate
// (FinalLayerSharedAdaLN.forward, local_thc.py:865-873; RMSNorm,
// jit_shared_adaln.py:20-30; modulate, local_thc.py:37-38).  The reference runs
// this as ~10 eager passes over the [B, T, C] residual; here it is one read of
// x and one write of m (forward) and one read of x and grad m plus one write of
// grad x (backward).
//
// Rounding follows the reference op by op: the norm in fp32 with one rounding
// to the activation dtype; 1 + scale, the product and the sum each rounded to
// the activation dtype (torch evaluates 16-bit elementwise ops in fp32 and
// rounds once per op).  Products and sums use explicit round-to-nearest
// intrinsics so that no FMA contraction changes a rounding.  Only the sums
// differ from torch: the two sums over channels (mean of squares; the
// backward's dot product) run in another order, and the backward's dot product
// and its grad-weight sum over tokens are fused multiply-adds.
//
// Mapping: a CTA owns a contiguous token range of one image (so the image's
// shift / scale / weight rows are read once per CTA) and walks it in tiles of
// `tile` tokens.  One elected thread streams the tiles (x, and grad m in the
// backward) into a ring of shared-memory stages with untiled bulk copies (the
// tokens of a tile are contiguous in memory).  Per tile:
//   phase 1  one warp per token: the token's sums over channels (mean of
//            squares -> r; backward: the dot product of grad t and x), lane l
//            owning the pairs 256 j + 64 e + 2 l (e < 4);
//   phase 2  one thread per channel pair: the elementwise outputs, written
//            over the staged x tile and sent out with one bulk store per tile,
//            and the backward's per-channel sums over tokens in registers.
// Phase 2 needs no per-channel state beyond a few registers.  Phase 1 of the
// next tile overlaps phase 2 of the current one (one CTA barrier per tile).
#pragma once

#include "lthc_common.cuh"
#include "lthc_kernels.cuh"
#include "lthc_tma.cuh"

namespace lthc {

constexpr int kFinalChunk = 256;       // channels of one 8-wide sweep of a warp (phase 1)
constexpr int kFinalMaxChunks = 4;     // C <= 1024
constexpr int kFinalMaxThreads = 512;  // one thread per channel pair in phase 2

// Channel pairs in the activation dtype.  R is the raw pair (two 16-bit values
// in one word, or a float2); mul() is the product of two pairs rounded once to
// the dtype.  For 16-bit types the fp32 product of two such values is exact, so
// the paired 16-bit multiply (round-to-nearest) gives the same result as torch's
// fp32 multiply followed by a rounding to the dtype.
template <typename T>
struct Pair;
template <>
struct Pair<float> {
  using R = float2;
  static __device__ __forceinline__ float2 f(R v) { return v; }
  static __device__ __forceinline__ R rn(float2 v) { return v; }
  static __device__ __forceinline__ R mul(R a, R b) { return fmul2(a, b); }
};
template <>
struct Pair<__nv_bfloat16> {
  using R = uint32_t;
  static __device__ __forceinline__ float2 f(R v) { return Act<__nv_bfloat16>::cvt(v); }
  static __device__ __forceinline__ R rn(float2 v) { return Act<__nv_bfloat16>::pack(v); }
  static __device__ __forceinline__ R mul(R a, R b) {
    const __nv_bfloat162 p =
        __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&a), *reinterpret_cast<const __nv_bfloat162*>(&b));
    return *reinterpret_cast<const uint32_t*>(&p);
  }
};
template <>
struct Pair<__half> {
  using R = uint32_t;
  static __device__ __forceinline__ float2 f(R v) { return Act<__half>::cvt(v); }
  static __device__ __forceinline__ R rn(float2 v) { return Act<__half>::pack(v); }
  static __device__ __forceinline__ R mul(R a, R b) {
    const __half2 p = __hmul2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    return *reinterpret_cast<const uint32_t*>(&p);
  }
};

template <typename T>
__device__ __forceinline__ typename Pair<T>::R ld_pair(const T* p) {
  return *reinterpret_cast<const typename Pair<T>::R*>(p);
}

template <typename T>
__device__ __forceinline__ float act_load(const T* p, int64_t i) {
  if constexpr (sizeof(T) == 4)
    return p[i];
  else if constexpr (Act<T>::kDtype == LTHC_DTYPE_BF16)
    return __bfloat162float(p[i]);
  else
    return __half2float(p[i]);
}

struct FinalParams {
  const void* x;          // [B, T, C] activations
  const void* w;          // [C] RMSNorm weight, dtype w_dtype
  const void* shift;      // [B, C] (row stride mod_stride), activation dtype (forward)
  const void* scale;      // [B, C] (row stride mod_stride), activation dtype
  const void* grad_out;   // backward: [B, T, C]
  void* out;              // forward: m [B, T, C]; backward: grad x [B, T, C]
  float* partial;         // backward: [B * ctas_per_image][3][C] fp32
  int w_dtype;
  int tile;               // tokens per tile (<= warps per CTA)
  int stages;             // tiles in flight
  float eps;
  float inv_c;            // 1.0f / C (torch's mean factor)
  float c_f;              // (float)C (torch's mean-backward divisor)
  int64_t T, C, mod_stride;
  int64_t tokens_per_cta;
};

// Shared-memory plan, identical on host and device.
struct FinalSmem {
  size_t tile_bytes, consts, r, bars, total;
  __host__ __device__ FinalSmem(int64_t C, int es, int tile, int stages, bool bwd) {
    tile_bytes = static_cast<size_t>(tile) * C * es;
    const size_t tiles = static_cast<size_t>(stages) * (bwd ? 2 : 1) * tile_bytes;
    consts = tiles;                                    // w, 1 + scale, shift: fp32 [C] each
    r = consts + 3 * static_cast<size_t>(C) * 4;       // r, 2 x grad of the squares: fp32 [2][tile] each
    bars = (r + 4 * static_cast<size_t>(tile) * 4 + 7) & ~static_cast<size_t>(7);
    total = bars + static_cast<size_t>(stages) * 8;
  }
};

// Phase-1 channel of lane `lane`, sub-pair e of 256-channel chunk j: the lanes of
// a warp read 32 consecutive pairs (conflict-free shared-memory accesses).
__device__ __forceinline__ int64_t final_channel(int j, int e, int lane) {
  return static_cast<int64_t>(j) * kFinalChunk + 64 * e + 2 * lane;
}

// rsqrt(mean of squares + eps) of one token from the lane's channel pairs: two
// running sums (even / odd channel of each pair) in (chunk, sub-pair) order,
// added, then summed over lanes by butterfly.  The forward and the backward
// share this code, so both see the same r.
template <int NV>
__device__ __forceinline__ float token_rstd(const float2 (&v)[NV][4], const FinalParams& p) {
  float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < NV; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) s2 = fadd2(s2, fmul2(v[j][e], v[j][e]));
  float ss = __fadd_rn(s2.x, s2.y);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  return rsqrtf(__fadd_rn(__fmul_rn(ss, p.inv_c), p.eps));
}

template <typename T, bool BWD, int NV>
__global__ void __launch_bounds__(kFinalMaxThreads) final_norm_modulate_kernel(const FinalParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int NT = BWD ? 2 : 1;
  constexpr int kEs = sizeof(T);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int64_t C = p.C;
  const FinalSmem plan(C, kEs, p.tile, p.stages, BWD);
  using P2 = Pair<T>;
  using R = typename P2::R;
  float* w_s = reinterpret_cast<float*>(smem + plan.consts);
  float* sh_s = w_s + C;
  T* s1_s = reinterpret_cast<T*>(sh_s + C);  // 1 + scale, rounded to the dtype
  float* r_s = reinterpret_cast<float*>(smem + plan.r);
  float* gsq_s = r_s + 2 * p.tile;  // backward: 2 x grad of the squares
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + plan.bars);

  const int64_t b = blockIdx.y;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * p.tokens_per_cta;
  const int64_t t_end = t0 + p.tokens_per_cta < p.T ? t0 + p.tokens_per_cta : p.T;
  const int64_t ntok = t_end > t0 ? t_end - t0 : 0;
  const int n_tiles = static_cast<int>((ntok + p.tile - 1) / p.tile);
  const T* xg = static_cast<const T*>(p.x) + (b * p.T + t0) * C;
  const T* gg = BWD ? static_cast<const T*>(p.grad_out) + (b * p.T + t0) * C : nullptr;
  T* og = static_cast<T*>(p.out) + (b * p.T + t0) * C;

  if (tid == 0) {
    for (int s = 0; s < p.stages; ++s) mbar_init(&full[s], 1);
    fence_barrier_init();
  }
  for (int64_t c = tid; c < C; c += blockDim.x) {
    w_s[c] = load_weight(p.w, p.w_dtype, c);
    sh_s[c] = BWD ? 0.f : act_load(static_cast<const T*>(p.shift), b * p.mod_stride + c);
    const float s1 = __fadd_rn(1.f, act_load(static_cast<const T*>(p.scale), b * p.mod_stride + c));
    if constexpr (sizeof(T) == 4)
      s1_s[c] = s1;
    else if constexpr (Act<T>::kDtype == LTHC_DTYPE_BF16)
      s1_s[c] = __float2bfloat16_rn(s1);
    else
      s1_s[c] = __float2half_rn(s1);
  }
  __syncthreads();

  auto issue = [&](int i) {  // thread 0: tile i into stage i % stages
    const int s = i % p.stages;
    const int64_t left = ntok - static_cast<int64_t>(i) * p.tile;
    const int64_t n = left < p.tile ? left : p.tile;
    const uint32_t bytes = static_cast<uint32_t>(n * C * kEs);
    mbar_arrive_expect_tx(&full[s], NT * bytes);
    const int64_t off = static_cast<int64_t>(i) * p.tile * C;
    bulk_load_1d(smem + (s * NT) * plan.tile_bytes, xg + off, bytes, &full[s]);
    if constexpr (BWD) bulk_load_1d(smem + (s * NT + 1) * plan.tile_bytes, gg + off, bytes, &full[s]);
  };
  int issued = 0;  // thread 0: tiles whose copies have been started
  if (tid == 0)
    for (; issued < min(p.stages, n_tiles); ++issued) issue(issued);

  // Phase-2 ownership: channel pair (c, c + 1), c = 2 * tid.
  const int64_t c = 2 * static_cast<int64_t>(tid);
  const bool own = c < C;
  const float2 wv = own ? *reinterpret_cast<const float2*>(w_s + c) : make_float2(0.f, 0.f);
  const float2 shv = own ? *reinterpret_cast<const float2*>(sh_s + c) : make_float2(0.f, 0.f);
  const R s1r = own ? ld_pair<T>(s1_s + c) : P2::rn(make_float2(0.f, 0.f));
  float2 aw = make_float2(0.f, 0.f), ash = aw, asc = aw;

  auto tile_rows = [&](int i) -> int {
    const int64_t left = ntok - static_cast<int64_t>(i) * p.tile;
    return static_cast<int>(left < p.tile ? left : p.tile);
  };
  auto stage_x = [&](int i) { return reinterpret_cast<const T*>(smem + ((i % p.stages) * NT) * plan.tile_bytes); };
  auto stage_g = [&](int i) { return reinterpret_cast<const T*>(smem + ((i % p.stages) * NT + 1) * plan.tile_bytes); };

  // Phase 1 of tile i: per-token sums (warp per token) into r / grad-of-squares
  // buffer i & 1.
  auto phase1 = [&](int i) {
    const int n = tile_rows(i);
    const T* xs = stage_x(i);
    const T* gs = stage_g(i);
    float* rb = r_s + (i & 1) * p.tile;
    float* qb = gsq_s + (i & 1) * p.tile;
    for (int k = warp; k < n; k += nwarps) {
      float2 v[NV][4];
#pragma unroll
      for (int j = 0; j < NV; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int64_t cc = final_channel(j, e, lane);
          v[j][e] = cc < C ? P2::f(ld_pair<T>(xs + k * C + cc)) : make_float2(0.f, 0.f);
        }
      const float r = token_rstd<NV>(v, p);
      float gsq = 0.f;
      if constexpr (BWD) {
        float2 d2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < NV; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int64_t cc = final_channel(j, e, lane);
            if (cc < C) {
              const float2 gn = P2::f(P2::mul(ld_pair<T>(gs + k * C + cc), ld_pair<T>(s1_s + cc)));
              const float2 gt = fmul2(gn, *reinterpret_cast<const float2*>(w_s + cc));
              d2 = ffma2(gt, v[j][e], d2);
            }
          }
        float dot = __fadd_rn(d2.x, d2.y);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dot = __fadd_rn(dot, __shfl_xor_sync(0xffffffffu, dot, o));
        // d/dr of rsqrt: -0.5 * g * r^3; mean backward: / C; square backward: * 2 here
        // (exact) and * x in phase 2, since (2 gsq) x equals gsq (2 x) in one rounding
        const float gv = __fmul_rn(__fmul_rn(-0.5f, dot), __fmul_rn(__fmul_rn(r, r), r));
        gsq = 2.f * __fdiv_rn(gv, p.c_f);
      }
      if (lane == 0) {
        rb[k] = r;
        qb[k] = gsq;
      }
    }
  };

  // Phase 2 of tile i: elementwise outputs (thread per channel pair).
  auto phase2 = [&](int i) {
    if (!own) return;
    const int n = tile_rows(i);
    const T* xs = stage_x(i);
    const T* gs = stage_g(i);
    const float* rb = r_s + (i & 1) * p.tile;
    const float* qb = gsq_s + (i & 1) * p.tile;
#pragma unroll 2
    for (int k = 0; k < n; ++k) {
      const float2 xv = P2::f(ld_pair<T>(xs + k * C + c));
      const float r = rb[k];
      const float2 tt = fmul2(xv, make_float2(r, r));
      const R nr = P2::rn(fmul2(tt, wv));  // n, rounded to the dtype
      R* dst = reinterpret_cast<R*>(const_cast<T*>(xs) + k * C + c);  // result over x, stored by bulk copy
      if constexpr (!BWD) {
        *dst = P2::rn(fadd2(P2::f(P2::mul(nr, s1r)), shv));
      } else {
        const R gr = ld_pair<T>(gs + k * C + c);
        const float2 gm = P2::f(gr);
        const float gsq = qb[k];
        const float2 gn = P2::f(P2::mul(gr, s1r));
        ash = fadd2(ash, gm);
        asc = fadd2(asc, P2::f(P2::mul(gr, nr)));
        aw = ffma2(gn, tt, aw);
        const float2 gt = fmul2(gn, wv);
        *dst = P2::rn(fadd2(fmul2(gt, make_float2(r, r)), fmul2(make_float2(gsq, gsq), xv)));
      }
    }
    fence_proxy_async_smem();  // the tile's bulk store reads these writes
  };

  // Software pipeline, one CTA barrier per tile: phase 2 of tile i runs while
  // other warps already do phase 1 of tile i + 1; the barrier then publishes
  // tile i's results (stored by thread 0) and tile i + 1's sums.
  bool alive = n_tiles > 0;
  int done = 0;  // tiles whose copies every thread has waited for
  if (alive) {
    alive = __syncthreads_and(mbar_wait(&full[0], 0));
    if (alive) {
      done = 1;
      phase1(0);
    }
    __syncthreads();
  }
  for (int i = 0; alive && i < n_tiles; ++i) {
    phase2(i);
    bool ok = true;
    if (i + 1 < n_tiles) {
      ok = mbar_wait(&full[(i + 1) % p.stages], ((i + 1) / p.stages) & 1);
      if (ok) phase1(i + 1);
    }
    alive = __syncthreads_and(ok);
    if (alive && i + 1 < n_tiles) done = i + 2;
    if (tid == 0 && alive) {
      // Tile i's results leave with one bulk store; the stage of tile i - 1 is
      // refilled once its store has read it (one store of lag).
      bulk_store_1d(og + static_cast<int64_t>(i) * p.tile * C, stage_x(i),
                    static_cast<uint32_t>(tile_rows(i) * C * kEs));
      bulk_commit();
      bulk_wait_read<1>();
      if (i >= 1 && i - 1 + p.stages < n_tiles) issue(issued++);
    }
  }
  if (tid == 0) {
    // a wait gave up: do not leave while copies into this CTA's memory are in flight
    for (int i = done; i < issued; ++i)
      if (!mbar_wait(&full[i % p.stages], (i / p.stages) & 1)) break;
    bulk_wait_all();
  }
  if constexpr (BWD) {
    if (own) {
      const int64_t cta = b * gridDim.x + blockIdx.x;
      float* P = p.partial + cta * 3 * C;
      P[c] = aw.x;
      P[c + 1] = aw.y;
      P[C + c] = ash.x;
      P[C + c + 1] = ash.y;
      P[2 * C + c] = asc.x;
      P[2 * C + c + 1] = asc.y;
    }
  }
}

// Sums the per-CTA partials in a fixed order: blocks [0, ceil(C/32)) form grad w
// over every CTA (column_sum32), the remaining blocks grad shift and grad scale
// over the CTAs of each image (CTA order), one thread per output element.
__global__ void __launch_bounds__(32 * kGammaFinalizeWarps) final_bwd_finalize_kernel(
    const float* __restrict__ partial, float* grad_w, float* grad_shift, float* grad_scale, int64_t B,
    int64_t per_image, int64_t C) {
  const int64_t w_blocks = (C + 31) / 32;
  if (blockIdx.x < w_blocks) {
    if (grad_w) {
      __shared__ float tot[32];
      const int64_t c0 = static_cast<int64_t>(blockIdx.x) * 32;
      column_sum32(partial, B * per_image, 3 * C, C, c0, tot);
      if (threadIdx.x < 32 && c0 + threadIdx.x < C) grad_w[c0 + threadIdx.x] = tot[threadIdx.x];
    }
    return;
  }
  if (!grad_shift && !grad_scale) return;
  const int64_t n_img = B * C;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x - w_blocks) * blockDim.x;
  for (int64_t e = static_cast<int64_t>(blockIdx.x - w_blocks) * blockDim.x + threadIdx.x; e < 2 * n_img;
       e += nthreads) {
    const int q = e < n_img ? 1 : 2;
    const int64_t be = e < n_img ? e : e - n_img;
    const int64_t b = be / C, c = be - b * C;
    float s = 0.f;
    for (int64_t k = 0; k < per_image; ++k) s = __fadd_rn(s, partial[((b * per_image + k) * 3 + q) * C + c]);
    float* dst = q == 1 ? grad_shift : grad_scale;
    if (dst) dst[be] = s;
  }
}

}  // namespace lthc
