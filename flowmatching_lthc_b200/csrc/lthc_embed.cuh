// Patch embedding fused with the shared read, on the tensor cores (row (f)2 of
// the LTHC path):
//   h1 = conv4x4/4(img; W1)        [tokens, 128]   (BottleneckPatchEmbedNHWC.proj1)
//   X0 = conv1x1(h1; W2) + b2      [tokens, C]     (proj2, then NHWC)
//   Z  = R(X0)                     [cells, C]      (SharedLocalRead.read)
// (local_thc.py:64-89 and 1211-1223).  Under bf16 autocast the reference runs
// both convolutions in bf16 with fp32 accumulation (h1 and the second product
// rounded to bf16, the bias then added as a separate bf16 op), writes X0 in NCHW,
// permutes it to NHWC and reads X0 back for Z.  This kernel rounds the same way
// (measured on B200: h1 identical to cuDNN's, X0 more than 99.99 %).  Here
// one pass computes both GEMMs per tile of 128 tokens with tcgen05 MMAs
// (accumulators in TMEM), writes X0 once (TMA tile stores) and pools Z from the
// staged X0 tile, in the same fp32 fused-multiply-add order as lthc_read_fwd, so
// Z equals the read of the X0 this kernel writes bit for bit.
//
// Tile: one image, one cell row, 8 cells = 4 token rows x 32 token columns; MMA
// row m = 16 * cell + 4 * row + col (a cell's 16 tokens are consecutive TMEM
// lanes).  A CTA owns one 256-channel chunk of X0 (its W2 rows stay in shared
// memory) and walks tiles; h1 is recomputed for each chunk (K = 48, cheap).
//
//   GEMM 1: D1[128 x 128] = A1[128 x 48(+16 zero)] * W1[128 x 48]^T     (3 K steps)
//   GEMM 2: D2[128 x 256] = A2[128 x 128] * W2chunk[256 x 128]^T      (8 K steps)
// Operands are K-major, 128-byte-swizzled bf16 (lthc_umma.cuh).
#pragma once

#include "lthc_common.cuh"
#include "lthc_tma.cuh"
#include "lthc_umma.cuh"

namespace lthc {

// (a, b) rounded to bf16 and widened back to fp32.
__device__ __forceinline__ float2 bf16_round2(float a, float b) {
  const __nv_bfloat162 t = __floats2bfloat162_rn(a, b);
  return __bfloat1622float2(t);
}

constexpr int kEmbedThreads = 256;     // 8 warps; two per TMEM lane quarter
constexpr int kEmbedTileTokens = 128;  // MMA M
constexpr int kEmbedBottleneck = 128;  // GEMM-1 N = GEMM-2 K
constexpr int kEmbedChunk = 256;       // GEMM-2 N: X0 channels per CTA
constexpr int kEmbedTileCols = 32;     // token columns per tile (8 cells)
constexpr int kEmbedMaxLoads = 8;      // 4-pixel loads per thread per tile (in_ch <= 4)

struct EmbedParams {
  CUtensorMap tm_x0;        // 4D (C, W, H, B) bf16, box (64, 32, 4, 1), 128-byte swizzle (store)
  const void* img;          // [B, in_ch, 4H, 4W] fp32 or bf16
  const __nv_bfloat16* w1;  // [128, in_ch * 16]
  const __nv_bfloat16* w2;  // [C, 128]
  const __nv_bfloat16* b2;  // [C]
  const __nv_bfloat16* alpha;  // [C, 16] read weights (activation dtype)
  __nv_bfloat16* z;         // [B, (H/4)*(W/4), C]
  int img_f32;
  int in_ch;
  int H;                    // token grid side (64 at B/4)
  int C;
  int64_t B;
  int64_t tiles;            // B * (H/4) * (W/32)
};

// Shared-memory plan (offsets from a 1024-byte aligned base).
struct EmbedSmem {
  static constexpr uint32_t kW1 = 0;                                      // 128 x 64  : 16 KB
  static constexpr uint32_t kW2 = kW1 + 16384;                            // 2 x 256 x 64 : 64 KB
  static constexpr uint32_t kA1 = kW2 + 65536;                            // 128 x 64 : 16 KB
  static constexpr uint32_t kA2 = kA1 + 16384;                            // 2 x 128 x 64 : 32 KB
  static constexpr uint32_t kX = kA2 + 32768;                             // 4 x 128 x 64 : 64 KB
  static constexpr uint32_t kAlpha = kX + 65536;                          // fp32 [16][256] : 16 KB
  static constexpr uint32_t kBias = kAlpha + 16384;                       // fp32 [256]
  static constexpr uint32_t kBars = kBias + 1024;                         // 2 mbarriers + TMEM slot
  static constexpr uint32_t kTotal = kBars + 64 + 1024;                   // + alignment slack
};
constexpr uint32_t kEmbedTmemCols = 512;  // D1: columns [0, 128); D2: [128, 384)

__global__ void __launch_bounds__(kEmbedThreads, 1) patch_embed_read_kernel(const __grid_constant__ EmbedParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar1 = reinterpret_cast<uint64_t*>(smem + EmbedSmem::kBars);
  uint64_t* bar2 = bar1 + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar1 + 2);
  float* alpha_s = reinterpret_cast<float*>(smem + EmbedSmem::kAlpha);
  float* bias_s = reinterpret_cast<float*>(smem + EmbedSmem::kBias);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nchunks = p.C / kEmbedChunk;
  const int chunk = blockIdx.x % nchunks;
  const int cta_in_chunk = blockIdx.x / nchunks;
  const int ctas_per_chunk = gridDim.x / nchunks;
  const int n0 = chunk * kEmbedChunk;
  const int K1 = p.in_ch * 16;

  // ---- one-time set-up: weights, read weights, bias; zero the GEMM-1 K padding
  for (int i = tid; i < 128 * 64; i += kEmbedThreads) {
    const int r = i >> 6, k = i & 63;
    const __nv_bfloat16 v = k < K1 ? p.w1[r * K1 + k] : __float2bfloat16_rn(0.f);
    *reinterpret_cast<__nv_bfloat16*>(smem + EmbedSmem::kW1 + sw128_offset(r, k)) = v;
    *reinterpret_cast<__nv_bfloat16*>(smem + EmbedSmem::kA1 + sw128_offset(r, k)) = __float2bfloat16_rn(0.f);
  }
  for (int i = tid; i < kEmbedChunk * kEmbedBottleneck / 8; i += kEmbedThreads) {
    const int r = i / (kEmbedBottleneck / 8), k8 = (i % (kEmbedBottleneck / 8)) * 8;
    const uint4 v = *reinterpret_cast<const uint4*>(p.w2 + static_cast<int64_t>(n0 + r) * kEmbedBottleneck + k8);
    *reinterpret_cast<uint4*>(smem + EmbedSmem::kW2 + (k8 >> 6) * 32768 + sw128_offset(r, k8 & 63)) = v;
  }
  for (int i = tid; i < kEmbedChunk * 16; i += kEmbedThreads) {
    const int n = i >> 4, r = i & 15;
    alpha_s[r * kEmbedChunk + n] = __bfloat162float(p.alpha[static_cast<int64_t>(n0 + n) * 16 + r]);
  }
  for (int n = tid; n < kEmbedChunk; n += kEmbedThreads) bias_s[n] = __bfloat162float(p.b2[n0 + n]);
  if (tid == 0) {
    mbar_init(bar1, 1);
    mbar_init(bar2, 1);
    fence_barrier_init();
    prefetch_tmap(&p.tm_x0);
  }
  if (warp == 0) tmem_alloc(tslot, kEmbedTmemCols);
  fence_proxy_async_smem();
  tmem_fence_before_sync();
  __syncthreads();
  tmem_fence_after_sync();
  const uint32_t tmem = *tslot;
  // Z pooling: this thread's channel pair and its 16 read weights (fixed for the kernel)
  const int zn = 2 * (tid % (kEmbedChunk / 2));
  float2 za[16];
#pragma unroll
  for (int r = 0; r < 16; ++r) za[r] = *reinterpret_cast<const float2*>(alpha_s + r * kEmbedChunk + zn);
  const uint32_t tmem_d1 = tmem;
  const uint32_t tmem_d2 = tmem + kEmbedBottleneck;
  const uint32_t idesc1 = umma_idesc_bf16_f32(kEmbedTileTokens, kEmbedBottleneck);
  const uint32_t idesc2 = umma_idesc_bf16_f32(kEmbedTileTokens, kEmbedChunk);
  const uint32_t sbase = smem_u32(smem);

  const int cell_rows = p.H / 4;
  const int halves = p.H / kEmbedTileCols;
  const int lq = warp & 3;            // TMEM lane quarter of this warp
  const int hf = warp >> 2;           // column half handled by this warp
  const int m = 32 * lq + lane;       // this thread's MMA row (token of the tile)
  const int m_cell = m >> 4, m_r = m & 15;
  const int m_R = (m_r >> 2) * kEmbedTileCols + 4 * m_cell + (m_r & 3);  // row of the staged X0 box
  const int64_t img_w = 4 * static_cast<int64_t>(p.H);
  bool alive = true;
  int it = 0;

  // Patch gather: 4 pixels (one token, one channel, one kernel row) per load;
  // load i of this thread covers pixel-row group i * kEmbedThreads + tid.  The
  // loaded words stay raw (fp32 pixels as 16 bytes, bf16 as 8) until they are
  // stored into A1 a tile later: converting them at load time would make every
  // thread wait there for its global loads.
  const int per_tile = p.in_ch * 16 * kEmbedTileCols;
  uint4 pre[kEmbedMaxLoads];  // next tile's pixels, as loaded
  auto gather_load = [&](int64_t t) {
    const int64_t bb = t / (cell_rows * halves);
    const int rr = static_cast<int>(t - bb * cell_rows * halves);
    const int wy_ = rr / halves, hx_ = rr % halves;
#pragma unroll
    for (int j = 0; j < kEmbedMaxLoads; ++j) {
      const int i = j * kEmbedThreads + tid;
      if (i < per_tile) {
        const int tx = i % kEmbedTileCols;
        const int py = (i / kEmbedTileCols) % 16;
        const int c = i / (kEmbedTileCols * 16);
        const int64_t gy = 16 * static_cast<int64_t>(wy_) + py;
        const int64_t gx = 4 * (static_cast<int64_t>(kEmbedTileCols) * hx_ + tx);
        const int64_t off = ((bb * p.in_ch + c) * img_w + gy) * img_w + gx;
        if (p.img_f32) {
          pre[j] = __ldcs(reinterpret_cast<const uint4*>(static_cast<const float*>(p.img) + off));
        } else {
          const uint2 v = __ldcs(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(p.img) + off));
          pre[j] = make_uint4(v.x, v.y, 0u, 0u);
        }
      }
    }
  };
  auto gather_store = [&](const uint4 (&v)[kEmbedMaxLoads]) {
#pragma unroll
    for (int j = 0; j < kEmbedMaxLoads; ++j) {
      const int i = j * kEmbedThreads + tid;
      if (i < per_tile) {
        const int tx = i % kEmbedTileCols;
        const int py = (i / kEmbedTileCols) % 16;
        const int c = i / (kEmbedTileCols * 16);
        const int mm = 16 * (tx >> 2) + 4 * (py >> 2) + (tx & 3);
        uint2 b;
        if (p.img_f32) {
          const __nv_bfloat162 lo = __floats2bfloat162_rn(__uint_as_float(v[j].x), __uint_as_float(v[j].y));
          const __nv_bfloat162 hi = __floats2bfloat162_rn(__uint_as_float(v[j].z), __uint_as_float(v[j].w));
          b.x = *reinterpret_cast<const uint32_t*>(&lo);
          b.y = *reinterpret_cast<const uint32_t*>(&hi);
        } else {
          b = make_uint2(v[j].x, v[j].y);
        }
        *reinterpret_cast<uint2*>(smem + EmbedSmem::kA1 + sw128_offset(mm, c * 16 + (py & 3) * 4)) = b;
      }
    }
  };
  // Tile pipeline: the next tile's patches are staged while this tile's GEMM 2
  // runs, and its GEMM 1 is issued before this tile's Z pooling, so both overlap
  // work of the current tile.
  auto issue_gemm1 = [&]() {
    if (tid == 0) {
      tmem_fence_after_sync();
      for (int s = 0; s < p.in_ch; ++s)
        umma_bf16(tmem_d1, umma_desc_sw128(sbase + EmbedSmem::kA1 + 32 * s),
                  umma_desc_sw128(sbase + EmbedSmem::kW1 + 32 * s), idesc1, s > 0);
      umma_commit(bar1);
    }
  };
  if (cta_in_chunk < p.tiles) {
    gather_load(cta_in_chunk);
    gather_store(pre);
    fence_proxy_async_smem();
    tmem_fence_before_sync();
    __syncthreads();
    issue_gemm1();
    if (cta_in_chunk + ctas_per_chunk < p.tiles) gather_load(cta_in_chunk + ctas_per_chunk);
  }

  for (int64_t tile = cta_in_chunk; alive && tile < p.tiles; tile += ctas_per_chunk, ++it) {
    const int64_t b = tile / (cell_rows * halves);
    const int rem = static_cast<int>(tile - b * cell_rows * halves);
    const int wy = rem / halves, hx = rem % halves;
    const bool has_next = tile + ctas_per_chunk < p.tiles;

    // ---- GEMM 1 of this tile (issued before the previous tile's Z pooling)
    bool ok = mbar_wait(bar1, it & 1);
    tmem_fence_after_sync();

    // ---- epilogue 1: h1 = bf16(D1) into A2 (row m, columns 64 * hf .. + 64)
    if (ok) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float v[32];
        tmem_ld32(tmem_d1 + (static_cast<uint32_t>(32 * lq) << 16) + 64 * hf + 32 * half, v);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 w;
          __nv_bfloat162 t0 = __floats2bfloat162_rn(v[8 * q + 0], v[8 * q + 1]);
          __nv_bfloat162 t1 = __floats2bfloat162_rn(v[8 * q + 2], v[8 * q + 3]);
          __nv_bfloat162 t2 = __floats2bfloat162_rn(v[8 * q + 4], v[8 * q + 5]);
          __nv_bfloat162 t3 = __floats2bfloat162_rn(v[8 * q + 6], v[8 * q + 7]);
          w.x = *reinterpret_cast<uint32_t*>(&t0);
          w.y = *reinterpret_cast<uint32_t*>(&t1);
          w.z = *reinterpret_cast<uint32_t*>(&t2);
          w.w = *reinterpret_cast<uint32_t*>(&t3);
          *reinterpret_cast<uint4*>(smem + EmbedSmem::kA2 + hf * 16384 + sw128_offset(m, 32 * half + 8 * q)) = w;
        }
      }
    }
    fence_proxy_async_smem();
    tmem_fence_before_sync();
    if (tid == 0) bulk_wait_read<0>();  // the previous tile's X0 stores have read the staging buffer
    alive = __syncthreads_and(ok);
    if (!alive) break;

    // ---- GEMM 2
    if (tid == 0) {
      tmem_fence_after_sync();
      for (int s = 0; s < kEmbedBottleneck / 16; ++s)
        umma_bf16(tmem_d2, umma_desc_sw128(sbase + EmbedSmem::kA2 + (s >> 2) * 16384 + 32 * (s & 3)),
                  umma_desc_sw128(sbase + EmbedSmem::kW2 + (s >> 2) * 32768 + 32 * (s & 3)), idesc2, s > 0);
      umma_commit(bar2);
    }
    // the next tile's patches into A1 (GEMM 1 of this tile has completed) while GEMM 2
    // runs, and at once the loads of the tile after it: a whole iteration to land
    if (has_next) gather_store(pre);
    if (tile + 2 * ctas_per_chunk < p.tiles) gather_load(tile + 2 * ctas_per_chunk);
    ok = mbar_wait(bar2, it & 1);
    tmem_fence_after_sync();

    // ---- epilogue 2: X0 = bf16(D2 + b2) into the staging boxes (row m_R, channels 128 * hf .. + 128)
    if (ok) {
      // two 32-column loads in flight per wait (the TMEM load latency is paid twice
      // per tile instead of four times)
#pragma unroll
      for (int q64 = 0; q64 < 2; ++q64) {
        uint32_t raw[2][32];
        tmem_ld32_async(tmem_d2 + (static_cast<uint32_t>(32 * lq) << 16) + 128 * hf + 64 * q64, raw[0]);
        tmem_ld32_async(tmem_d2 + (static_cast<uint32_t>(32 * lq) << 16) + 128 * hf + 64 * q64 + 32, raw[1]);
        tmem_wait_ld();
#pragma unroll
        for (int qq = 0; qq < 8; ++qq) {
          const int n = 128 * hf + 64 * q64 + 8 * qq;  // first of these 8 channels within the chunk
          float v8[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) v8[i] = __uint_as_float(raw[qq >> 2][8 * (qq & 3) + i]);
          // the convolution output is rounded to bf16, then the bias is added and
          // the sum rounded again (the reference adds the bias as a separate op)
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 conv = bf16_round2(v8[2 * e], v8[2 * e + 1]);
            const float2 bb = *reinterpret_cast<const float2*>(bias_s + n + 2 * e);
            const __nv_bfloat162 t = __floats2bfloat162_rn(__fadd_rn(conv.x, bb.x), __fadd_rn(conv.y, bb.y));
            o[e] = *reinterpret_cast<const uint32_t*>(&t);
          }
          uint4 w;
          w.x = o[0];
          w.y = o[1];
          w.z = o[2];
          w.w = o[3];
          *reinterpret_cast<uint4*>(smem + EmbedSmem::kX + (n >> 6) * 16384 + sw128_offset(m_R, n & 63)) = w;
        }
      }
    }
    fence_proxy_async_smem();
    tmem_fence_before_sync();
    alive = __syncthreads_and(ok);
    if (!alive) break;

    // ---- GEMM 1 of the next tile (its patches are staged, D1 was read by epilogue 1)
    if (has_next) issue_gemm1();

    // ---- X0 out: four TMA tile stores of 64 channels x 32 columns x 4 rows
    if (tid == 0) {
#pragma unroll
      for (int bx = 0; bx < kEmbedChunk / 64; ++bx)
        tma_store_4d(&p.tm_x0, smem + EmbedSmem::kX + bx * 16384, n0 + 64 * bx, kEmbedTileCols * hx, 4 * wy,
                     static_cast<int32_t>(b));
      bulk_commit();
    }

    // ---- Z: pool the staged X0 over each cell's 16 positions (r = 0..15 in order, fp32 FMA)
    const int64_t zrow0 = b * static_cast<int64_t>(cell_rows) * (p.H / 4) + static_cast<int64_t>(wy) * (p.H / 4) +
                          (kEmbedTileCols / 4) * hx;
    static_assert(kEmbedThreads % (kEmbedChunk / 2) == 0, "each thread pools one fixed channel pair");
    for (int pi = tid; pi < 8 * (kEmbedChunk / 2); pi += kEmbedThreads) {
      const int cell = pi / (kEmbedChunk / 2);
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        const int R = (r >> 2) * kEmbedTileCols + 4 * cell + (r & 3);
        const uint32_t raw = *reinterpret_cast<const uint32_t*>(smem + EmbedSmem::kX + (zn >> 6) * 16384 +
                                                                sw128_offset(R, zn & 63));
        acc = ffma2(za[r], Act<__nv_bfloat16>::cvt(raw), acc);
      }
      Act<__nv_bfloat16>::st(p.z + (zrow0 + cell) * p.C + n0 + zn, acc);
    }
  }
  if (tid == 0) bulk_wait_all();
  tmem_fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kEmbedTmemCols);
}

}  // namespace lthc
