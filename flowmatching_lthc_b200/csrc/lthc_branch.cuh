// The workspace branch's output epilogue fused with the lazy workspace update
// (row (f)3 of the LTHC path):
//   dz = dz_attn + gate (.) mlp_out        WorkspaceSharedAdaLNBranch.forward
//                                          (local_thc.py:318-323; the gate product
//                                          and the sum each rounded to the dtype)
//   z' = z + gamma (.) dz                  lazy_workspace_update (:1325-1328),
//   gamma[c] = sum_r alpha[c,r] beta[c,r]  gamma_from_alpha (:1278-1283)
// One pass reads dz_attn, mlp_out and z and writes dz (kept for the
// materialisation) and z'.  The reference runs three elementwise kernels (gate
// product, sum, lazy update).  gate rows (one per image) have stride gstride.
//
// Backward (given grad dz from the materialisation, may be absent, and grad z'):
//   g_tot   = grad_dz + round(gamma * grad_z')   (the two uses of dz)
//   grad dz_attn = g_tot;  grad mlp_out = round(gate * g_tot)
//   grad gate[b] = sum over the image's rows of round(g_tot * mlp_out)   (fp32)
//   grad gamma   = sum over rows of grad_z' * dz (fp32) -> grad alpha / beta
// CTAs of the backward own contiguous row ranges of one image, so the per-image
// gate gradient is a fixed-order two-stage sum like every other reduction here.
#pragma once

#include "lthc_common.cuh"
#include "lthc_kernels.cuh"

namespace lthc {

struct BranchLazyParams {
  const void* z;         // fwd: z
  const void* attn;      // fwd: dz_attn
  const void* mlp;       // mlp_out (fwd and bwd)
  const void* gate;      // [B] rows of C, stride gstride
  const void* a;         // alpha [C,16]
  const void* b;         // beta  [C,16]
  const void* dz;        // bwd: the forward's dz
  const void* g_dz;      // bwd: grad dz (may be null)
  const void* g_zo;      // bwd: grad z'
  void* out0;            // fwd: dz          bwd: grad dz_attn
  void* out1;            // fwd: z'          bwd: grad mlp_out
  float* partial;        // bwd: [B * per_image][2][C]  (grad gate part, grad gamma part)
  int a_dtype, b_dtype;
  int64_t N, C, T, gstride;
  int64_t rows_per_cta;  // bwd
};

// gamma of the warp's 16-byte channel vector slice, like lazy_gamma_slice
template <typename T>
__device__ __forceinline__ void branch_gamma_slice(const BranchLazyParams& p, int64_t cbase, float* g_s) {
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

// A batch of rows is held as raw 16-byte vectors (4 registers each) and
// converted to fp32 at use, so a deep batch stays within the register budget of
// two 256-thread CTAs per SM.
__device__ __forceinline__ uint4 ld_raw(const void* p) { return *static_cast<const uint4*>(p); }

template <typename T>
__device__ __forceinline__ void unpack_vec(const uint4& raw, float (&v)[Vec16<T>::V]) {
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
__device__ __forceinline__ float rnd(float v) {
  if constexpr (sizeof(T) == 4)
    return v;
  else if constexpr (Act<T>::kDtype == LTHC_DTYPE_BF16)
    return __bfloat162float(__float2bfloat16_rn(v));
  else
    return __half2float(__float2half_rn(v));
}

template <typename T>
__global__ void __launch_bounds__(256, 2) branch_lazy_fwd_kernel(const __grid_constant__ BranchLazyParams p) {
  constexpr int V = Vec16<T>::V;
  __shared__ float g_s[Vec16<T>::kSlice];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t cbase = static_cast<int64_t>(blockIdx.y) * Vec16<T>::kSlice;
  branch_gamma_slice<T>(p, cbase, g_s);
  const int64_t c = cbase + lane * V;
  if (c >= p.C) return;
  float g[V];
#pragma unroll
  for (int i = 0; i < V; ++i) g[i] = g_s[lane * V + i];
  const T* z = static_cast<const T*>(p.z);
  const T* attn = static_cast<const T*>(p.attn);
  const T* mlp = static_cast<const T*>(p.mlp);
  const T* gate = static_cast<const T*>(p.gate);
  T* dz_out = static_cast<T*>(p.out0);
  T* z_out = static_cast<T*>(p.out1);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kLazyWarps;
  // kLazyBatch rows per warp in flight: every load of the batch is issued before
  // the first use
  for (int64_t n0 = static_cast<int64_t>(blockIdx.x) * kLazyWarps + warp; n0 < p.N; n0 += stride * kLazyBatch) {
    uint4 zr[kLazyBatch], ar[kLazyBatch], mr[kLazyBatch], gr[kLazyBatch];
#pragma unroll
    for (int j = 0; j < kLazyBatch; ++j) {
      const int64_t n = n0 + j * stride;
      if (n < p.N) {
        zr[j] = ld_raw(z + n * p.C + c);
        ar[j] = ld_raw(attn + n * p.C + c);
        mr[j] = ld_raw(mlp + n * p.C + c);
        gr[j] = ld_raw(gate + (n / p.T) * p.gstride + c);
      }
    }
#pragma unroll
    for (int j = 0; j < kLazyBatch; ++j) {
      const int64_t n = n0 + j * stride;
      if (n < p.N) {
        float zv[V], av[V], mv[V], gv[V], dz[V];
        unpack_vec<T>(zr[j], zv);
        unpack_vec<T>(ar[j], av);
        unpack_vec<T>(mr[j], mv);
        unpack_vec<T>(gr[j], gv);
#pragma unroll
        for (int i = 0; i < V; ++i) {
          dz[i] = rnd<T>(__fadd_rn(av[i], rnd<T>(__fmul_rn(gv[i], mv[i]))));
          zv[i] = fmaf(g[i], dz[i], zv[i]);
        }
        st_vec<T>(dz_out + n * p.C + c, dz);
        st_vec<T>(z_out + n * p.C + c, zv);
      }
    }
  }
}

// rows per warp in flight in the backward (four inputs per row)
constexpr int kBranchBwdBatch = 2;

template <typename T>
__global__ void __launch_bounds__(256, 2) branch_lazy_bwd_kernel(const __grid_constant__ BranchLazyParams p) {
  constexpr int V = Vec16<T>::V;
  constexpr int kS = Vec16<T>::kSlice;
  __shared__ float g_s[kS];
  __shared__ float red[kLazyWarps][2][kS];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t cbase = static_cast<int64_t>(blockIdx.y) * kS;
  branch_gamma_slice<T>(p, cbase, g_s);
  const int64_t per_image = (p.T + p.rows_per_cta - 1) / p.rows_per_cta;
  const int64_t img = blockIdx.x / per_image;
  const int64_t r0 = img * p.T + (blockIdx.x % per_image) * p.rows_per_cta;
  const int64_t r1 = min(r0 + p.rows_per_cta, (img + 1) * p.T);
  const int64_t c = cbase + lane * V;
  const bool valid = c < p.C;
  float acc_gate[V], acc_gam[V];
#pragma unroll
  for (int i = 0; i < V; ++i) acc_gate[i] = acc_gam[i] = 0.f;
  if (valid) {
    float g[V], gt[V];
#pragma unroll
    for (int i = 0; i < V; ++i) g[i] = g_s[lane * V + i];
    ld_vec<T>(static_cast<const T*>(p.gate) + img * p.gstride + c, gt);
    const T* g_dz = static_cast<const T*>(p.g_dz);
    const T* g_zo = static_cast<const T*>(p.g_zo);
    const T* dzp = static_cast<const T*>(p.dz);
    const T* mlp = static_cast<const T*>(p.mlp);
    T* g_attn = static_cast<T*>(p.out0);
    T* g_mlp = static_cast<T*>(p.out1);
    for (int64_t n0 = r0 + warp; n0 < r1; n0 += kLazyWarps * kBranchBwdBatch) {
      uint4 zr[kBranchBwdBatch], dr[kBranchBwdBatch], mr[kBranchBwdBatch], gr[kBranchBwdBatch];
#pragma unroll
      for (int j = 0; j < kBranchBwdBatch; ++j) {
        const int64_t n = n0 + j * kLazyWarps;
        gr[j] = make_uint4(0u, 0u, 0u, 0u);
        if (n < r1) {
          zr[j] = ld_raw(g_zo + n * p.C + c);
          dr[j] = ld_raw(dzp + n * p.C + c);
          mr[j] = ld_raw(mlp + n * p.C + c);
          if (g_dz) gr[j] = ld_raw(g_dz + n * p.C + c);
        }
      }
#pragma unroll
      for (int j = 0; j < kBranchBwdBatch; ++j) {
        const int64_t n = n0 + j * kLazyWarps;
        if (n < r1) {
          float zo[V], dzv[V], mv[V], gd[V], tot[V], gm[V];
          unpack_vec<T>(zr[j], zo);
          unpack_vec<T>(dr[j], dzv);
          unpack_vec<T>(mr[j], mv);
          unpack_vec<T>(gr[j], gd);
#pragma unroll
          for (int i = 0; i < V; ++i) {
            const float from_lazy = rnd<T>(__fmul_rn(g[i], zo[i]));
            tot[i] = g_dz ? rnd<T>(__fadd_rn(gd[i], from_lazy)) : from_lazy;
            gm[i] = rnd<T>(__fmul_rn(gt[i], tot[i]));
            acc_gate[i] = __fadd_rn(acc_gate[i], rnd<T>(__fmul_rn(tot[i], mv[i])));
            acc_gam[i] = fmaf(zo[i], dzv[i], acc_gam[i]);
          }
          st_vec<T>(g_attn + n * p.C + c, tot);
          st_vec<T>(g_mlp + n * p.C + c, gm);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < V; ++i) {
    red[warp][0][lane * V + i] = acc_gate[i];
    red[warp][1][lane * V + i] = acc_gam[i];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * kS; i += blockDim.x) {
    const int q = i / kS, j = i % kS;
    const int64_t cc = cbase + j;
    if (cc < p.C) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kLazyWarps; ++w) s = __fadd_rn(s, red[w][q][j]);
      p.partial[(static_cast<int64_t>(blockIdx.x) * 2 + q) * p.C + cc] = s;
    }
  }
}

// Blocks [0, ceil(C/32)) reduce grad gamma over every CTA's partial and form
// grad alpha / beta (gamma_grad_block); the remaining blocks form grad gate[b][c]
// = sum over the image's CTAs in CTA order.
__global__ void __launch_bounds__(32 * kGammaFinalizeWarps) branch_lazy_bwd_finalize_kernel(
    const __grid_constant__ BranchLazyParams p, int64_t B, int64_t per_image, float* grad_gate, float* grad_a,
    float* grad_b) {
  const int64_t gamma_blocks = (p.C + 31) / 32;
  if (blockIdx.x < gamma_blocks) {
    if (grad_a || grad_b)
      gamma_grad_block(p.partial + p.C, B * per_image, 2 * p.C, p.C, static_cast<int64_t>(blockIdx.x) * 32, p.a,
                       p.a_dtype, p.b, p.b_dtype, grad_a, grad_b);
    return;
  }
  if (!grad_gate) return;
  const int64_t n_gate = B * p.C;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x - gamma_blocks) * blockDim.x;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x - gamma_blocks) * blockDim.x + threadIdx.x; idx < n_gate;
       idx += nthreads) {
    const int64_t b = idx / p.C, c = idx - b * p.C;
    float s = 0.f;
    for (int64_t k = 0; k < per_image; ++k) s = __fadd_rn(s, p.partial[((b * per_image + k) * 2 + 0) * p.C + c]);
    grad_gate[idx] = s;
  }
}

}  // namespace lthc
