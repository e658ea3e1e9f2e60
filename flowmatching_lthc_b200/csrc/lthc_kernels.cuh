// Workspace-sized LTHC kernels (plain vectorised loads): the lazy recurrence and
// its backward, and the fixed-order second stage of the weight-gradient
// reductions.  A CTA owns a 64-channel slice (blockIdx.y); lane l of a warp owns
// the channel pair (2l, 2l+1), so a warp access covers 64 contiguous channels.
// Every kernel accumulates in fp32 and rounds once.
#pragma once

#include "lthc_common.cuh"

namespace lthc {

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
// Lane = one 16-byte vector of V = 16/sizeof(T) channels; a warp covers a slice
// of 32*V channels of one workspace row (blockIdx.y = slice), the 8 warps of a
// CTA walk rows.  gamma of the slice is computed once per CTA (fp32 FMAs in
// position order) into shared memory.
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

template <typename T>
struct Vec16 {
  static constexpr int V = 16 / sizeof(T);   // channels per 16-byte vector
  static constexpr int kSlice = 32 * V;      // channels per warp
};

template <typename T>
__device__ __forceinline__ void lazy_gamma_slice(const LazyParams& p, int64_t cbase, float* g_s) {
  for (int i = threadIdx.x; i < Vec16<T>::kSlice; i += blockDim.x) {
    const int64_t c = cbase + i;
    float g = 0.f;
    if (c < p.C) {
#pragma unroll
      for (int r = 0; r < kPos; ++r)
        g = fmaf(load_weight(p.a, p.a_dtype, c * kPos + r), load_weight(p.b, p.b_dtype, c * kPos + r), g);
    }
    g_s[i] = g;
  }
  __syncthreads();
}

// 16-byte vector of T as V floats
template <typename T>
__device__ __forceinline__ void ld_vec(const T* p, float (&v)[Vec16<T>::V]) {
  const uint4 raw = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(w[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = Act<T>::cvt(w[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
}

template <typename T>
__device__ __forceinline__ void st_vec(T* p, const float (&v)[Vec16<T>::V]) {
  uint4 raw;
  uint32_t* w = reinterpret_cast<uint32_t*>(&raw);
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = __float_as_uint(v[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = Act<T>::pack(make_float2(v[2 * i], v[2 * i + 1]));
  }
  *reinterpret_cast<uint4*>(p) = raw;
}

// Rows handled per batch by one lane: all their loads are issued before any
// store, so a lane keeps 2 * kLazyBatch 16-byte loads in flight even though the
// output may alias an input (in-place update).
constexpr int kLazyBatch = 4;

template <typename T>
__global__ void __launch_bounds__(256) lazy_fwd_kernel(const __grid_constant__ LazyParams p) {
  constexpr int V = Vec16<T>::V;
  __shared__ float g_s[Vec16<T>::kSlice];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t cbase = static_cast<int64_t>(blockIdx.y) * Vec16<T>::kSlice;
  lazy_gamma_slice<T>(p, cbase, g_s);
  const int64_t c = cbase + lane * V;
  if (c >= p.C) return;
  float g[V];
#pragma unroll
  for (int i = 0; i < V; ++i) g[i] = g_s[lane * V + i];
  const T* z = static_cast<const T*>(p.z);
  const T* dz = static_cast<const T*>(p.dz);
  T* out = static_cast<T*>(p.out);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kLazyWarps;
  for (int64_t n0 = static_cast<int64_t>(blockIdx.x) * kLazyWarps + warp; n0 < p.N; n0 += stride * kLazyBatch) {
    float zv[kLazyBatch][V], dv[kLazyBatch][V];
#pragma unroll
    for (int j = 0; j < kLazyBatch; ++j) {
      const int64_t n = n0 + j * stride;
      if (n < p.N) {
        ld_vec<T>(z + n * p.C + c, zv[j]);
        ld_vec<T>(dz + n * p.C + c, dv[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < kLazyBatch; ++j) {
      const int64_t n = n0 + j * stride;
      if (n < p.N) {
#pragma unroll
        for (int i = 0; i < V; i += 2) {
          const float2 r = ffma2(make_float2(g[i], g[i + 1]), make_float2(dv[j][i], dv[j][i + 1]),
                                 make_float2(zv[j][i], zv[j][i + 1]));
          zv[j][i] = r.x;
          zv[j][i + 1] = r.y;
        }
        st_vec<T>(out + n * p.C + c, zv[j]);
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) lazy_bwd_kernel(const __grid_constant__ LazyParams p) {
  constexpr int V = Vec16<T>::V;
  __shared__ float g_s[Vec16<T>::kSlice];
  __shared__ float red[kLazyWarps][Vec16<T>::kSlice];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t cbase = static_cast<int64_t>(blockIdx.y) * Vec16<T>::kSlice;
  lazy_gamma_slice<T>(p, cbase, g_s);
  const int64_t c = cbase + lane * V;
  const bool valid = c < p.C;
  float acc[V];
#pragma unroll
  for (int i = 0; i < V; ++i) acc[i] = 0.f;
  if (valid) {
    float g[V];
#pragma unroll
    for (int i = 0; i < V; ++i) g[i] = g_s[lane * V + i];
    const T* gz = static_cast<const T*>(p.z);
    const T* dz = static_cast<const T*>(p.dz);
    T* gdz = static_cast<T*>(p.out);
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kLazyWarps;
    for (int64_t n0 = static_cast<int64_t>(blockIdx.x) * kLazyWarps + warp; n0 < p.N; n0 += stride * kLazyBatch) {
      float gv[kLazyBatch][V], dv[kLazyBatch][V];
#pragma unroll
      for (int j = 0; j < kLazyBatch; ++j) {
        const int64_t n = n0 + j * stride;
        if (n < p.N) {
          ld_vec<T>(gz + n * p.C + c, gv[j]);
          ld_vec<T>(dz + n * p.C + c, dv[j]);
        }
      }
#pragma unroll
      for (int j = 0; j < kLazyBatch; ++j) {
        const int64_t n = n0 + j * stride;
        if (n < p.N) {
          float o[V];
#pragma unroll
          for (int i = 0; i < V; i += 2) {
            const float2 m = fmul2(make_float2(g[i], g[i + 1]), make_float2(gv[j][i], gv[j][i + 1]));
            o[i] = m.x;
            o[i + 1] = m.y;
            const float2 a2 = ffma2(make_float2(gv[j][i], gv[j][i + 1]), make_float2(dv[j][i], dv[j][i + 1]),
                                    make_float2(acc[i], acc[i + 1]));
            acc[i] = a2.x;
            acc[i + 1] = a2.y;
          }
          st_vec<T>(gdz + n * p.C + c, o);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < V; ++i) red[warp][lane * V + i] = acc[i];
  __syncthreads();
  for (int i = threadIdx.x; i < Vec16<T>::kSlice; i += blockDim.x) {
    const int64_t cc = cbase + i;
    if (cc < p.C) {
      float s = red[0][i];
#pragma unroll
      for (int w = 1; w < kLazyWarps; ++w) s += red[w][i];
      p.partial[static_cast<int64_t>(blockIdx.x) * p.C + cc] = s;
    }
  }
}

// ggamma[c] = sum_k partial[k * kstride + c];  grad_a[c,r] = ggamma*b[c,r];
// grad_b[c,r] = ggamma*a[c,r].  One block per 32 channels: warp w sums the
// partials k = w, w + 16, ... (coalesced over the channels, sixteen chains of
// eight loads in flight instead of one chain of nblk dependent adds), the warp
// sums are added in warp order, then the block writes its 32 x 16 outputs.
// Fixed order: bitwise reproducible.
constexpr int kGammaFinalizeWarps = 16;
constexpr int kColumnBatch = 8;  // independent partial loads in flight per warp

// Fixed-order column sums of 32 channels c0 .. c0+31 over nblk partial rows
// (row k at partial + k * kstride) by a block of kGammaFinalizeWarps warps; the
// result lands in tot[0..31] (shared), visible to the whole block on return.
__device__ __forceinline__ void column_sum32(const float* __restrict__ partial, int64_t nblk, int64_t kstride,
                                             int64_t C, int64_t c0, float* tot) {
  __shared__ float red[kGammaFinalizeWarps][32];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t c = c0 + lane;
  float s = 0.f;
  if (c < C) {
    int64_t k = warp;
    for (; k + (kColumnBatch - 1) * kGammaFinalizeWarps < nblk; k += kColumnBatch * kGammaFinalizeWarps) {
      float v[kColumnBatch];
#pragma unroll
      for (int j = 0; j < kColumnBatch; ++j) v[j] = partial[(k + j * kGammaFinalizeWarps) * kstride + c];
#pragma unroll
      for (int j = 0; j < kColumnBatch; ++j) s = __fadd_rn(s, v[j]);
    }
    for (; k < nblk; k += kGammaFinalizeWarps) s = __fadd_rn(s, partial[k * kstride + c]);
  }
  red[warp][lane] = s;
  __syncthreads();
  if (warp == 0) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kGammaFinalizeWarps; ++w) t = __fadd_rn(t, red[w][lane]);
    tot[lane] = t;
  }
  __syncthreads();
}

__device__ __forceinline__ void gamma_grad_block(const float* __restrict__ partial, int64_t nblk, int64_t kstride,
                                                 int64_t C, int64_t c0, const void* a, int a_dtype, const void* b,
                                                 int b_dtype, float* grad_a, float* grad_b) {
  __shared__ float tot[32];
  column_sum32(partial, nblk, kstride, C, c0, tot);
  for (int i = threadIdx.x; i < 32 * kPos; i += blockDim.x) {
    const int64_t cc = c0 + i / kPos;
    if (cc < C) {
      const int64_t idx = cc * kPos + i % kPos;
      const float g = tot[i / kPos];
      if (grad_a) grad_a[idx] = g * load_weight(b, b_dtype, idx);
      if (grad_b) grad_b[idx] = g * load_weight(a, a_dtype, idx);
    }
  }
}

// grid: ceil(C / 32) blocks of 32 * kGammaFinalizeWarps threads
__global__ void __launch_bounds__(32 * kGammaFinalizeWarps) lazy_bwd_finalize_kernel(
    const __grid_constant__ LazyParams p, int nblk, float* __restrict__ grad_a, float* __restrict__ grad_b) {
  gamma_grad_block(p.partial, nblk, p.C, p.C, static_cast<int64_t>(blockIdx.x) * 32, p.a, p.a_dtype, p.b, p.b_dtype,
                   grad_a, grad_b);
}

}  // namespace lthc
