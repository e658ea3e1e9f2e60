// Device-side helpers shared by every LTHC kernel: geometry constants, packed
// fp32x2 arithmetic, channel-pair loads/stores for each activation dtype and
// runtime-dtype weight loads.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "lthc_b200.h"

namespace lthc {

// A workspace cell covers a 4x4 block of residual tokens (B/4 geometry of the
// reference: 64x64 residual grid over a 16x16 workspace grid).
constexpr int kCellSide = 4;
constexpr int kPos = 16;          // positions per cell, r = 4*row + col
constexpr int kSliceCh = 64;      // channels per CTA slice: 32 channel pairs = one warp
constexpr int kMaxLayers = LTHC_MAX_LAYERS;

// ---------------------------------------------------------------------------
// Packed fp32x2 arithmetic (sm_100: one instruction, two IEEE fp32 results,
// round-to-nearest-even per lane, no fused reassociation across lanes).
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned long long pack2(float2 v) {
  return (static_cast<unsigned long long>(__float_as_uint(v.y)) << 32) |
         static_cast<unsigned long long>(__float_as_uint(v.x));
}
__device__ __forceinline__ float2 unpack2(unsigned long long v) {
  return make_float2(__uint_as_float(static_cast<unsigned>(v & 0xffffffffull)),
                     __uint_as_float(static_cast<unsigned>(v >> 32)));
}
// d = a * b + c (per lane, single rounding)
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(pack2(a)), "l"(pack2(b)), "l"(pack2(c)));
  return unpack2(d);
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pack2(a)), "l"(pack2(b)));
  return unpack2(d);
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pack2(a)), "l"(pack2(b)));
  return unpack2(d);
}

// ---------------------------------------------------------------------------
// Channel-pair access: every thread owns two adjacent channels (c, c+1) so that
// a warp covers 64 contiguous channels of one token (128 B for 16-bit types).
// ---------------------------------------------------------------------------
template <typename T>
struct Act;

template <>
struct Act<float> {
  static constexpr int kDtype = LTHC_DTYPE_F32;
  using Raw = float2;
  static __device__ __forceinline__ Raw ld(const float* p) { return *reinterpret_cast<const float2*>(p); }
  static __device__ __forceinline__ Raw ld_stream(const float* p) {
    return __ldcs(reinterpret_cast<const float2*>(p));
  }
  static __device__ __forceinline__ float2 cvt(Raw v) { return v; }
  static __device__ __forceinline__ Raw pack(float2 v) { return v; }
  static __device__ __forceinline__ void st(float* p, float2 v) { *reinterpret_cast<float2*>(p) = v; }
  static __device__ __forceinline__ void st_stream(float* p, float2 v) {
    __stcs(reinterpret_cast<float2*>(p), v);
  }
};

template <>
struct Act<__nv_bfloat16> {
  static constexpr int kDtype = LTHC_DTYPE_BF16;
  using Raw = uint32_t;
  static __device__ __forceinline__ Raw ld(const __nv_bfloat16* p) {
    return *reinterpret_cast<const uint32_t*>(p);
  }
  static __device__ __forceinline__ Raw ld_stream(const __nv_bfloat16* p) {
    return __ldcs(reinterpret_cast<const unsigned int*>(p));
  }
  // bf16 -> fp32 is exact: the bf16 bits are the high half of the fp32 word.
  static __device__ __forceinline__ float2 cvt(Raw v) {
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
  }
  static __device__ __forceinline__ Raw pack(float2 v) {
    __nv_bfloat162 h = __float22bfloat162_rn(v);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ void st(__nv_bfloat16* p, float2 v) {
    *reinterpret_cast<uint32_t*>(p) = pack(v);
  }
  static __device__ __forceinline__ void st_stream(__nv_bfloat16* p, float2 v) {
    __stcs(reinterpret_cast<unsigned int*>(p), pack(v));
  }
};

template <>
struct Act<__half> {
  static constexpr int kDtype = LTHC_DTYPE_F16;
  using Raw = uint32_t;
  static __device__ __forceinline__ Raw ld(const __half* p) { return *reinterpret_cast<const uint32_t*>(p); }
  static __device__ __forceinline__ Raw ld_stream(const __half* p) {
    return __ldcs(reinterpret_cast<const unsigned int*>(p));
  }
  static __device__ __forceinline__ float2 cvt(Raw v) {
    __half2 h = *reinterpret_cast<__half2*>(&v);
    return __half22float2(h);
  }
  static __device__ __forceinline__ Raw pack(float2 v) {
    __half2 h = __float22half2_rn(v);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ void st(__half* p, float2 v) { *reinterpret_cast<uint32_t*>(p) = pack(v); }
  static __device__ __forceinline__ void st_stream(__half* p, float2 v) {
    __stcs(reinterpret_cast<unsigned int*>(p), pack(v));
  }
};

// Weight element load with the dtype chosen at run time (weights are tiny and
// loaded once per thread, so the switch costs nothing on the streaming path).
__device__ __forceinline__ float load_weight(const void* p, int dtype, int64_t idx) {
  switch (dtype) {
    case LTHC_DTYPE_BF16:
      return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[idx]);
    case LTHC_DTYPE_F16:
      return __half2float(reinterpret_cast<const __half*>(p)[idx]);
    default:
      return reinterpret_cast<const float*>(p)[idx];
  }
}

// Token offset (in elements) of channel c at position (row, col) of cell m in an
// NHWC residual [B, 4G, 4G, C].
__device__ __forceinline__ int64_t cell_token_offset(int64_t m, int G, int64_t C, int row, int col) {
  const int64_t GG = static_cast<int64_t>(G) * G;
  const int64_t b = m / GG;
  const int64_t rem = m - b * GG;
  const int64_t wy = rem / G;
  const int64_t wx = rem - wy * G;
  const int64_t H = 4 * static_cast<int64_t>(G);
  return ((b * H + 4 * wy + row) * H + 4 * wx + col) * C;
}

}  // namespace lthc
