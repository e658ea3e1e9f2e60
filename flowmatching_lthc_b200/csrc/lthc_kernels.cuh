// Streaming LTHC kernels (plain vectorised loads).
//
// Thread geometry shared by all kernels: a CTA owns a 64-channel slice of the
// residual (blockIdx.y), lane l of a warp owns the channel pair (2l, 2l+1) of the
// slice, so one warp-wide access touches 64 contiguous channels of one token.
// Cell weights live in registers for the whole CTA lifetime; the CTA then walks
// a contiguous range of cells.  Every kernel accumulates in fp32 and rounds once.
#pragma once

#include "lthc_common.cuh"

namespace lthc {

// ---------------------------------------------------------------------------
// read (single weight set): z[cell, c] = sum_r w[c, r] * x[cell, r, c]
// Thread (lane, warp) = (channel pair, cell stream); 16 weights per channel in
// registers, 16 independent loads per cell, sum in position order r = 0..15.
// ---------------------------------------------------------------------------
struct PoolParams {
  const void* x;      // T[B,4G,4G,C]
  const void* w;      // [C,16]
  void* z;            // T[B,G*G,C]
  int w_dtype;
  int G;
  int64_t C;
  int64_t cells;
};

constexpr int kPoolWarps = 8;

template <typename T>
__global__ void __launch_bounds__(256) pool1_kernel(const __grid_constant__ PoolParams p) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t c = static_cast<int64_t>(blockIdx.y) * kSliceCh + 2 * lane;
  if (c >= p.C) return;
  float2 w[kPos];
#pragma unroll
  for (int r = 0; r < kPos; ++r) {
    w[r].x = load_weight(p.w, p.w_dtype, c * kPos + r);
    w[r].y = load_weight(p.w, p.w_dtype, (c + 1) * kPos + r);
  }
  const T* x = static_cast<const T*>(p.x);
  T* z = static_cast<T*>(p.z);
  const int64_t rowstride = 4 * static_cast<int64_t>(p.G) * p.C;
  for (int64_t m = static_cast<int64_t>(blockIdx.x) * kPoolWarps + warp; m < p.cells;
       m += static_cast<int64_t>(gridDim.x) * kPoolWarps) {
    const int64_t tok = cell_token_offset(m, p.G, p.C, 0, 0) + c;
    typename Act<T>::Raw v[kPos];
#pragma unroll
    for (int r = 0; r < kPos; ++r) v[r] = Act<T>::ld_stream(x + tok + (r >> 2) * rowstride + (r & 3) * p.C);
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kPos; ++r) acc = ffma2(w[r], Act<T>::cvt(v[r]), acc);
    Act<T>::st(z + m * p.C + c, acc);
  }
}

// ---------------------------------------------------------------------------
// read with L weight sets (materialise backward, grad_dz):
//   out_l[cell, c] = sum_r w_l[c, r] * x[cell, r, c]
// The CTA stages its slice of all L weight sets in shared memory as
// [r][l][lane] float2 (conflict-free 8-byte reads); x is read once per cell.
// ---------------------------------------------------------------------------
struct PoolMultiParams {
  const void* x;
  const void* w[kMaxLayers];
  void* out[kMaxLayers];
  int w_dtype;
  int L;
  int G;
  int64_t C;
  int64_t cells;
};

template <typename T, int LT>
__global__ void __launch_bounds__(256) pool_multi_kernel(const __grid_constant__ PoolMultiParams p) {
  constexpr int LMAX = LT > 0 ? LT : kMaxLayers;
  const int L = LT > 0 ? LT : p.L;
  extern __shared__ float2 sw[];  // [kPos][LMAX][32]
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t cbase = static_cast<int64_t>(blockIdx.y) * kSliceCh;
  for (int i = threadIdx.x; i < kPos * LMAX * 32; i += blockDim.x) {
    const int pl = i & 31;
    const int l = (i >> 5) % LMAX;
    const int r = (i >> 5) / LMAX;
    const int64_t cc = cbase + 2 * pl;
    float2 v = make_float2(0.f, 0.f);
    if (l < L && cc < p.C) {
      v.x = load_weight(p.w[l], p.w_dtype, cc * kPos + r);
      v.y = load_weight(p.w[l], p.w_dtype, (cc + 1) * kPos + r);
    }
    sw[i] = v;
  }
  __syncthreads();
  const int64_t c = cbase + 2 * lane;
  if (c >= p.C) return;
  const T* x = static_cast<const T*>(p.x);
  const int64_t rowstride = 4 * static_cast<int64_t>(p.G) * p.C;
  for (int64_t m = static_cast<int64_t>(blockIdx.x) * kPoolWarps + warp; m < p.cells;
       m += static_cast<int64_t>(gridDim.x) * kPoolWarps) {
    const int64_t tok = cell_token_offset(m, p.G, p.C, 0, 0) + c;
    float2 acc[LMAX];
#pragma unroll
    for (int l = 0; l < LMAX; ++l) acc[l] = make_float2(0.f, 0.f);
#pragma unroll 4
    for (int r = 0; r < kPos; ++r) {
      const float2 xv = Act<T>::cvt(Act<T>::ld_stream(x + tok + (r >> 2) * rowstride + (r & 3) * p.C));
#pragma unroll
      for (int l = 0; l < LMAX; ++l) acc[l] = ffma2(sw[(r * LMAX + l) * 32 + lane], xv, acc[l]);
    }
#pragma unroll
    for (int l = 0; l < LMAX; ++l)
      if (l < L) Act<T>::st(static_cast<T*>(p.out[l]) + m * p.C + c, acc[l]);
  }
}

// ---------------------------------------------------------------------------
// weight gradient, stage 1:  partial[blk][l][c][r] = sum_{cells of blk} high[cell,r,c]*low_l[cell,c]
// Thread (lane, warp) = (channel pair, cell row) owns 4 positions x L layers x 2
// channels of fp32 accumulators; every output has exactly one owner, so no
// atomics: stage 2 sums the per-CTA partials in CTA order (deterministic).
// ---------------------------------------------------------------------------
struct WgradParams {
  const void* high;                 // T[B,4G,4G,C]
  const void* low[kMaxLayers];      // T[B,G*G,C]
  float* partial;                   // [nblk][L][C][16]
  int L;
  int G;
  int64_t C;
  int64_t cells;
  int64_t cells_per_block;
};

template <typename T, int LT>
__global__ void __launch_bounds__(128) wgrad_kernel(const __grid_constant__ WgradParams p) {
  constexpr int LMAX = LT > 0 ? LT : kMaxLayers;
  const int L = LT > 0 ? LT : p.L;
  const int lane = threadIdx.x & 31;
  const int row = threadIdx.x >> 5;
  const int64_t c = static_cast<int64_t>(blockIdx.y) * kSliceCh + 2 * lane;
  if (c >= p.C) return;
  float2 acc[LMAX][4];
#pragma unroll
  for (int l = 0; l < LMAX; ++l)
#pragma unroll
    for (int col = 0; col < 4; ++col) acc[l][col] = make_float2(0.f, 0.f);

  const T* high = static_cast<const T*>(p.high);
  const int64_t m0 = static_cast<int64_t>(blockIdx.x) * p.cells_per_block;
  const int64_t m1 = min(m0 + p.cells_per_block, p.cells);
#pragma unroll 2
  for (int64_t m = m0; m < m1; ++m) {
    const int64_t tok = cell_token_offset(m, p.G, p.C, row, 0) + c;
    typename Act<T>::Raw raw[4];
#pragma unroll
    for (int col = 0; col < 4; ++col) raw[col] = Act<T>::ld_stream(high + tok + col * p.C);
    float2 h[4];
#pragma unroll
    for (int col = 0; col < 4; ++col) h[col] = Act<T>::cvt(raw[col]);
    const int64_t zoff = m * p.C + c;
#pragma unroll
    for (int l = 0; l < LMAX; ++l) {
      if (l < L) {
        const float2 d = Act<T>::cvt(Act<T>::ld(static_cast<const T*>(p.low[l]) + zoff));
#pragma unroll
        for (int col = 0; col < 4; ++col) acc[l][col] = ffma2(h[col], d, acc[l][col]);
      }
    }
  }
  float* P = p.partial + static_cast<int64_t>(blockIdx.x) * L * p.C * kPos;
#pragma unroll
  for (int l = 0; l < LMAX; ++l) {
    if (l < L) {
      float4 a = make_float4(acc[l][0].x, acc[l][1].x, acc[l][2].x, acc[l][3].x);
      float4 b = make_float4(acc[l][0].y, acc[l][1].y, acc[l][2].y, acc[l][3].y);
      *reinterpret_cast<float4*>(P + (l * p.C + c) * kPos + row * 4) = a;
      *reinterpret_cast<float4*>(P + (l * p.C + c + 1) * kPos + row * 4) = b;
    }
  }
}

// Stage 2 of every two-stage reduction: out[i] = sum_{k < nblk} partial[k*n + i]
// in increasing k (fixed order, bitwise reproducible).
__global__ void __launch_bounds__(256) reduce_partials_kernel(const float* __restrict__ partial,
                                                              float* __restrict__ out, int64_t n,
                                                              int nblk) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < nblk; ++k) s += partial[static_cast<int64_t>(k) * n + i];
    out[i] = s;
  }
}

// ---------------------------------------------------------------------------
// lazy workspace recurrence: z_out = z + gamma (.) dz, gamma[c] = sum_r a[c,r] b[c,r]
// gamma is recomputed per thread from the two weight rows (32 fp32 FMAs).
// ---------------------------------------------------------------------------
struct LazyParams {
  const void* z;        // fwd: z ; bwd: grad_z_out
  const void* dz;
  const void* a;        // alpha [C,16]
  const void* b;        // beta  [C,16]
  void* out;            // fwd: z_out ; bwd: grad_dz
  float* partial;       // bwd: [nblk][C]
  int a_dtype;
  int b_dtype;
  int64_t N;
  int64_t C;
};

constexpr int kLazyWarps = 8;

__device__ __forceinline__ float2 gamma_pair(const LazyParams& p, int64_t c) {
  float2 g = make_float2(0.f, 0.f);
#pragma unroll
  for (int r = 0; r < kPos; ++r) {
    g.x = fmaf(load_weight(p.a, p.a_dtype, c * kPos + r), load_weight(p.b, p.b_dtype, c * kPos + r), g.x);
    g.y = fmaf(load_weight(p.a, p.a_dtype, (c + 1) * kPos + r), load_weight(p.b, p.b_dtype, (c + 1) * kPos + r),
               g.y);
  }
  return g;
}

template <typename T>
__global__ void __launch_bounds__(256) lazy_fwd_kernel(const __grid_constant__ LazyParams p) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t c = static_cast<int64_t>(blockIdx.y) * kSliceCh + 2 * lane;
  if (c >= p.C) return;
  const float2 g = gamma_pair(p, c);
  const T* z = static_cast<const T*>(p.z);
  const T* dz = static_cast<const T*>(p.dz);
  T* out = static_cast<T*>(p.out);
#pragma unroll 4
  for (int64_t n = static_cast<int64_t>(blockIdx.x) * kLazyWarps + warp; n < p.N;
       n += static_cast<int64_t>(gridDim.x) * kLazyWarps) {
    const int64_t off = n * p.C + c;
    const float2 zv = Act<T>::cvt(Act<T>::ld(z + off));
    const float2 dv = Act<T>::cvt(Act<T>::ld(dz + off));
    Act<T>::st(out + off, ffma2(g, dv, zv));
  }
}

template <typename T>
__global__ void __launch_bounds__(256) lazy_bwd_kernel(const __grid_constant__ LazyParams p) {
  __shared__ float2 red[kLazyWarps][32];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t c = static_cast<int64_t>(blockIdx.y) * kSliceCh + 2 * lane;
  const bool valid = c < p.C;
  float2 acc = make_float2(0.f, 0.f);
  if (valid) {
    const float2 g = gamma_pair(p, c);
    const T* gz = static_cast<const T*>(p.z);
    const T* dz = static_cast<const T*>(p.dz);
    T* gdz = static_cast<T*>(p.out);
#pragma unroll 4
    for (int64_t n = static_cast<int64_t>(blockIdx.x) * kLazyWarps + warp; n < p.N;
         n += static_cast<int64_t>(gridDim.x) * kLazyWarps) {
      const int64_t off = n * p.C + c;
      const float2 gv = Act<T>::cvt(Act<T>::ld(gz + off));
      const float2 dv = Act<T>::cvt(Act<T>::ld(dz + off));
      Act<T>::st(gdz + off, fmul2(g, gv));
      acc = ffma2(gv, dv, acc);
    }
  }
  red[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && valid) {
    float2 s = red[0][lane];
#pragma unroll
    for (int w = 1; w < kLazyWarps; ++w) s = fadd2(s, red[w][lane]);
    float* P = p.partial + static_cast<int64_t>(blockIdx.x) * p.C;
    P[c] = s.x;
    P[c + 1] = s.y;
  }
}

// ggamma[c] = sum_k partial[k][c];  grad_a[c,r] = ggamma*b[c,r];  grad_b[c,r] = ggamma*a[c,r]
__global__ void __launch_bounds__(256) lazy_bwd_finalize_kernel(const __grid_constant__ LazyParams p, int nblk,
                                                                float* __restrict__ grad_a,
                                                                float* __restrict__ grad_b) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // (c, r)
  if (i >= p.C * kPos) return;
  const int64_t c = i / kPos;
  float s = 0.f;
  for (int k = 0; k < nblk; ++k) s += p.partial[static_cast<int64_t>(k) * p.C + c];
  if (grad_a) grad_a[i] = s * load_weight(p.b, p.b_dtype, i);
  if (grad_b) grad_b[i] = s * load_weight(p.a, p.a_dtype, i);
}

}  // namespace lthc
