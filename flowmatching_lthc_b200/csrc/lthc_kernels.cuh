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
