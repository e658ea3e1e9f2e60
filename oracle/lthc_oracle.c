/*
 * lthc_oracle.c — CPU restatement of the reference's LTHC interface math.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA kernels and
 * the timed CPU baseline; it is never part of the product path.  Only tests/,
 * __graft_entry__.smoke() and bench.py (cpu_baseline leg and the reference arm)
 * may load it.
 *
 * Every function restates one piece of tongtongliang/flowmatching_lthc:
 *   oracle_read            SharedLocalRead.read              local_thc.py:1211-1223
 *   oracle_write           LayerLocalWrite.write             local_thc.py:1261-1273
 *   oracle_write_add       LayerLocalWrite.write_add         local_thc.py:1275-1276
 *   oracle_materialise     final_accumulate_reference loop   local_thc.py:1368-1372,
 *                          and the fused Triton op           local_thc_triton_kernels.py:317-405
 *   oracle_materialise_bwd _backward_final_accumulate_12     local_thc_triton_kernels.py:1897-1912
 *                          (grad_dz kernel :512-595, grad_beta kernel :598-680)
 *   oracle_weight_grad     _cell_weight_grad_kernel          local_thc_triton_kernels.py:167-199
 *   oracle_lazy_fwd        lazy_workspace_update + gamma     local_thc.py:1278-1283, 1325-1328
 *   oracle_lazy_bwd        autograd of the two lines above
 *   oracle_final_fwd       FinalLayerSharedAdaLN.forward     local_thc.py:865-873 (RMSNorm
 *                          jit_shared_adaln.py:20-30, modulate local_thc.py:37-38), without its Linear
 *   oracle_final_bwd       autograd of the line above
 *   oracle_branch_fwd      WorkspaceSharedAdaLNBranch.forward's output sum   local_thc.py:318-323,
 *                          then lazy_workspace_update                        :1325-1328
 *   oracle_branch_bwd      autograd of the two lines above
 *
 * Arithmetic: inputs are widened to fp32 exactly; per-element sums over the 16
 * cell positions or the L layers accumulate in fp32 with fused multiply-add in
 * the reference Triton order (base first, then l = 0, 1, ...; positions
 * r = 0..15); reductions over cells accumulate in fp64.  Results are rounded
 * once (round-to-nearest-even) to the output dtype.
 *
 * Geometry: residual NHWC [B, 4G, 4G, C]; workspace [B, G*G, C]; cell weights
 * [C, 16] with position r = 4*row + col inside the 4x4 cell.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define DT_F32 0
#define DT_BF16 1
#define DT_F16 2

/* ---- exact dtype conversions (IEEE 754 bit manipulation) ------------------ */
static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = ((uint32_t)h) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u >> 16) | 0x40u); /* NaN */
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb; /* round to nearest, ties to even */
  return (uint16_t)(u >> 16);
}
static inline float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t u;
  if (exp == 0) {
    if (man == 0) {
      u = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do {
        man <<= 1;
        e++;
      } while (!(man & 0x400u));
      man &= 0x3ffu;
      u = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    u = sign | 0x7f800000u | (man << 13);
  } else {
    u = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static inline uint16_t f32_to_f16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  uint32_t sign = (u >> 16) & 0x8000u;
  int32_t exp = (int32_t)((u >> 23) & 0xffu);
  uint32_t man = u & 0x7fffffu;
  if (exp == 255) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0));
  int32_t e = exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  if (e <= 0) { /* subnormal or zero */
    if (e < -10) return (uint16_t)sign;
    man |= 0x800000u;
    uint32_t shift = (uint32_t)(14 - e);
    uint32_t half = man >> shift;
    uint32_t rem = man & ((1u << shift) - 1u);
    uint32_t mid = 1u << (shift - 1);
    if (rem > mid || (rem == mid && (half & 1u))) half++;
    return (uint16_t)(sign | half);
  }
  uint32_t half = sign | ((uint32_t)e << 10) | (man >> 13);
  uint32_t rem = man & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (half & 1u))) half++;
  return (uint16_t)half;
}

static inline float ld(const void* p, int dt, int64_t i) {
  if (dt == DT_BF16) return bf16_to_f32(((const uint16_t*)p)[i]);
  if (dt == DT_F16) return f16_to_f32(((const uint16_t*)p)[i]);
  return ((const float*)p)[i];
}
static inline void st(void* p, int dt, int64_t i, float v) {
  if (dt == DT_BF16)
    ((uint16_t*)p)[i] = f32_to_bf16(v);
  else if (dt == DT_F16)
    ((uint16_t*)p)[i] = f32_to_f16(v);
  else
    ((float*)p)[i] = v;
}

/* Element offset of channel 0 at position r of cell m in the NHWC residual. */
static inline int64_t tok_off(int64_t m, int64_t G, int64_t C, int r) {
  int64_t GG = G * G, H = 4 * G;
  int64_t b = m / GG, rem = m % GG, wy = rem / G, wx = rem % G;
  return ((b * H + 4 * wy + (r >> 2)) * H + 4 * wx + (r & 3)) * C;
}

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void oracle_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* z[m, c] = sum_r w[c, r] * x[m, r, c] */
void oracle_read(const void* x, const void* w, int wdt, void* z, int64_t B, int64_t G, int64_t C, int dt) {
  int64_t cells = B * G * G;
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < cells; ++m) {
    int64_t off[16];
    for (int r = 0; r < 16; ++r) off[r] = tok_off(m, G, C, r);
    for (int64_t c = 0; c < C; ++c) {
      float acc = 0.f;
      for (int r = 0; r < 16; ++r) acc = fmaf(ld(w, wdt, c * 16 + r), ld(x, dt, off[r] + c), acc);
      st(z, dt, m * C + c, acc);
    }
  }
}

/* out = base + sum_{l<L} w_l[c, r] * dz_l[m, c]; base may be NULL (zero). */
void oracle_materialise(const void* base, const void* const* dz, const void* const* w, int wdt, int L, void* out,
                        int64_t B, int64_t G, int64_t C, int dt) {
  int64_t cells = B * G * G;
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < cells; ++m) {
    for (int r = 0; r < 16; ++r) {
      int64_t off = tok_off(m, G, C, r);
      for (int64_t c = 0; c < C; ++c) {
        float acc = base ? ld(base, dt, off + c) : 0.f;
        for (int l = 0; l < L; ++l) acc = fmaf(ld(w[l], wdt, c * 16 + r), ld(dz[l], dt, m * C + c), acc);
        st(out, dt, off + c, acc);
      }
    }
  }
}

void oracle_write(const void* dz, const void* w, int wdt, void* out, int64_t B, int64_t G, int64_t C, int dt) {
  const void* dzs[1] = {dz};
  const void* ws[1] = {w};
  oracle_materialise(NULL, dzs, ws, wdt, 1, out, B, G, C, dt);
}

void oracle_write_add(const void* x, const void* dz, const void* w, int wdt, void* out, int64_t B, int64_t G,
                      int64_t C, int dt) {
  const void* dzs[1] = {dz};
  const void* ws[1] = {w};
  oracle_materialise(x, dzs, ws, wdt, 1, out, B, G, C, dt);
}

/* gw[l, c, r] = sum_m high[m, r, c] * low_l[m, c]   (fp64 accumulation) */
void oracle_weight_grad(const void* high, const void* const* low, int L, float* gw, int64_t B, int64_t G,
                        int64_t C, int dt) {
  int64_t cells = B * G * G;
#pragma omp parallel for schedule(static)
  for (int64_t c = 0; c < C; ++c) {
    double acc[12][16];
    memset(acc, 0, sizeof(acc));
    for (int64_t m = 0; m < cells; ++m) {
      double h[16];
      for (int r = 0; r < 16; ++r) h[r] = ld(high, dt, tok_off(m, G, C, r) + c);
      for (int l = 0; l < L; ++l) {
        double v = ld(low[l], dt, m * C + c);
        for (int r = 0; r < 16; ++r) acc[l][r] += h[r] * v;
      }
    }
    for (int l = 0; l < L; ++l)
      for (int r = 0; r < 16; ++r) gw[((int64_t)l * C + c) * 16 + r] = (float)acc[l][r];
  }
}

/* grad_dz_l[m, c] = sum_r w_l[c, r] * gout[m, r, c]  and  grad_w (weight_grad). */
void oracle_materialise_bwd(const void* gout, const void* const* dz, const void* const* w, int wdt, int L,
                            void* const* gdz, float* gw, int64_t B, int64_t G, int64_t C, int dt) {
  int64_t cells = B * G * G;
  if (gdz) {
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < cells; ++m) {
      int64_t off[16];
      for (int r = 0; r < 16; ++r) off[r] = tok_off(m, G, C, r);
      for (int64_t c = 0; c < C; ++c) {
        float g[16];
        for (int r = 0; r < 16; ++r) g[r] = ld(gout, dt, off[r] + c);
        for (int l = 0; l < L; ++l) {
          float acc = 0.f;
          for (int r = 0; r < 16; ++r) acc = fmaf(ld(w[l], wdt, c * 16 + r), g[r], acc);
          st(gdz[l], dt, m * C + c, acc);
        }
      }
    }
  }
  if (gw) oracle_weight_grad(gout, dz, L, gw, B, G, C, dt);
}

static inline float gamma_of(const void* a, int adt, const void* b, int bdt, int64_t c) {
  float g = 0.f;
  for (int r = 0; r < 16; ++r) g = fmaf(ld(a, adt, c * 16 + r), ld(b, bdt, c * 16 + r), g);
  return g;
}

/* out[n, c] = z[n, c] + gamma[c] * dz[n, c],  gamma[c] = sum_r a[c, r] * b[c, r] */
void oracle_lazy_fwd(const void* z, const void* dz, const void* a, int adt, const void* b, int bdt, void* out,
                     int64_t N, int64_t C, int dt) {
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    for (int64_t c = 0; c < C; ++c) {
      float g = gamma_of(a, adt, b, bdt, c);
      st(out, dt, n * C + c, fmaf(g, ld(dz, dt, n * C + c), ld(z, dt, n * C + c)));
    }
  }
}

/* grad_dz = gamma * gzo; ggamma[c] = sum_n gzo*dz (fp64); ga = ggamma*b; gb = ggamma*a */
void oracle_lazy_bwd(const void* gzo, const void* dz, const void* a, int adt, const void* b, int bdt, void* gdz,
                     float* ga, float* gb, int64_t N, int64_t C, int dt) {
#pragma omp parallel for schedule(static)
  for (int64_t c = 0; c < C; ++c) {
    float g = gamma_of(a, adt, b, bdt, c);
    double acc = 0.0;
    for (int64_t n = 0; n < N; ++n) {
      float gv = ld(gzo, dt, n * C + c);
      st(gdz, dt, n * C + c, g * gv);
      acc += (double)gv * (double)ld(dz, dt, n * C + c);
    }
    float s = (float)acc;
    for (int r = 0; r < 16; ++r) {
      if (ga) ga[c * 16 + r] = s * ld(b, bdt, c * 16 + r);
      if (gb) gb[c * 16 + r] = s * ld(a, adt, c * 16 + r);
    }
  }
}

/* ---- final-layer prologue ---------------------------------------------------
 * FinalLayerSharedAdaLN.forward (local_thc.py:865-873) without its Linear:
 *   RMSNorm (jit_shared_adaln.py:20-30): xf = x.float();
 *     r = rsqrt(mean(xf^2) + eps); n = (xf * r * w).to(dtype)
 *   modulate (local_thc.py:37-38): m = n * (1 + scale[b]) + shift[b], each op
 *     rounded to the activation dtype (torch's 16-bit elementwise rule).
 * The mean of squares is summed in fp64 and rounded once; rsqrt is evaluated in
 * fp64 and rounded.  x/out: [B, T, C]; w: [C] (wdt); shift/scale: rows of
 * stride ms (elements) in the activation dtype. */
static inline float rnd(float v, int dt) {
  if (dt == DT_BF16) return bf16_to_f32(f32_to_bf16(v));
  if (dt == DT_F16) return f16_to_f32(f32_to_f16(v));
  return v;
}

static inline float token_rstd(const void* x, int dt, int64_t row, int64_t C, float eps) {
  double ss = 0.0;
  for (int64_t c = 0; c < C; ++c) {
    float v = ld(x, dt, row + c);
    ss += (double)(v * v);
  }
  float ms = (float)ss * (1.0f / (float)C);
  return (float)(1.0 / sqrt((double)(ms + eps)));
}

void oracle_final_fwd(const void* x, const void* w, int wdt, const void* shift, const void* scale, int64_t ms,
                      void* out, int64_t B, int64_t T, int64_t C, float eps, int dt) {
#pragma omp parallel for schedule(static)
  for (int64_t bt = 0; bt < B * T; ++bt) {
    int64_t b = bt / T, row = bt * C;
    float r = token_rstd(x, dt, row, C, eps);
    for (int64_t c = 0; c < C; ++c) {
      float n = rnd((ld(x, dt, row + c) * r) * ld(w, wdt, c), dt);
      float s1 = rnd(1.0f + ld(scale, dt, b * ms + c), dt);
      float p = rnd(n * s1, dt);
      st(out, dt, row + c, p + ld(shift, dt, b * ms + c));
    }
  }
}

/* Autograd of the expression above, op by op (torch derivative formulas):
 *   g_n = (g_m * s1) rounded;  g_scale[b] = sum_t (g_m * n) rounded;  g_shift[b] = sum_t g_m
 *   g_t = g_n * w;  g_w = sum_{b,t} g_n * t   (t = x * r)
 *   g_r = sum_c g_t * x;  g_v = -0.5 * g_r * r^3;  g_sq = g_v / C
 *   g_x = (g_t * r + g_sq * (2 x)) rounded to the activation dtype
 * Sums over tokens and channels accumulate in fp64. */
void oracle_final_bwd(const void* x, const void* w, int wdt, const void* scale, int64_t ms, const void* gm,
                      void* gx, float* gw, float* gsh, float* gsc, int64_t B, int64_t T, int64_t C, float eps,
                      int dt) {
  float* rs = (float*)malloc(sizeof(float) * (size_t)(B * T > 0 ? B * T : 1));
  if (!rs) return;
#pragma omp parallel for schedule(static)
  for (int64_t bt = 0; bt < B * T; ++bt) rs[bt] = token_rstd(x, dt, bt * C, C, eps);
#pragma omp parallel for schedule(static)
  for (int64_t bt = 0; bt < B * T; ++bt) {
    int64_t b = bt / T, row = bt * C;
    float r = rs[bt];
    double dot = 0.0;
    for (int64_t c = 0; c < C; ++c) {
      float xv = ld(x, dt, row + c);
      float s1 = rnd(1.0f + ld(scale, dt, b * ms + c), dt);
      float gn = rnd(ld(gm, dt, row + c) * s1, dt);
      dot += (double)((gn * ld(w, wdt, c)) * xv);
    }
    float gv = (-0.5f * (float)dot) * ((r * r) * r);
    float gsq = gv / (float)C;
    for (int64_t c = 0; c < C; ++c) {
      float xv = ld(x, dt, row + c);
      float s1 = rnd(1.0f + ld(scale, dt, b * ms + c), dt);
      float gn = rnd(ld(gm, dt, row + c) * s1, dt);
      float gt = gn * ld(w, wdt, c);
      st(gx, dt, row + c, gt * r + gsq * (2.0f * xv));
    }
  }
#pragma omp parallel for schedule(static)
  for (int64_t c = 0; c < C; ++c) {
    double aw = 0.0;
    float wc = ld(w, wdt, c);
    for (int64_t b = 0; b < B; ++b) {
      double ash = 0.0, asc = 0.0;
      float s1 = rnd(1.0f + ld(scale, dt, b * ms + c), dt);
      for (int64_t t = 0; t < T; ++t) {
        int64_t row = (b * T + t) * C;
        float tt = ld(x, dt, row + c) * rs[b * T + t];
        float n = rnd(tt * wc, dt);
        float g = ld(gm, dt, row + c);
        float gn = rnd(g * s1, dt);
        ash += (double)g;
        asc += (double)rnd(g * n, dt);
        aw += (double)(gn * tt);
      }
      if (gsh) gsh[b * C + c] = (float)ash;
      if (gsc) gsc[b * C + c] = (float)asc;
    }
    if (gw) gw[c] = (float)aw;
  }
  free(rs);
}

/* ---- branch epilogue + lazy update --------------------------------------------
 * WorkspaceSharedAdaLNBranch.forward's last lines (local_thc.py:318-323):
 *   dz = dz_attn + gate * mlp_out     (the product and the sum each rounded)
 * then lazy_workspace_update (:1325-1328): z' = z + gamma * dz (fmaf, one rounding).
 * Rows n of B images of T rows; gate rows of stride gs. */
void oracle_branch_fwd(const void* z, const void* attn, const void* mlp, const void* gate, int64_t gs, const void* a,
                       int adt, const void* b, int bdt, void* dz_out, void* z_out, int64_t B, int64_t T, int64_t C,
                       int dt) {
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < B * T; ++n) {
    int64_t img = n / T;
    for (int64_t c = 0; c < C; ++c) {
      float g = gamma_of(a, adt, b, bdt, c);
      float gm = rnd(ld(gate, dt, img * gs + c) * ld(mlp, dt, n * C + c), dt);
      float dz = rnd(ld(attn, dt, n * C + c) + gm, dt);
      st(dz_out, dt, n * C + c, dz);
      st(z_out, dt, n * C + c, fmaf(g, dz, ld(z, dt, n * C + c)));
    }
  }
}

/* Its autograd: g_tot = g_dz + round(gamma * g_zo); grad_attn = g_tot;
 * grad_mlp = round(gate * g_tot); grad_gate[b] = sum_rows round(g_tot * mlp);
 * ggamma = sum_rows g_zo * dz; grad_a = ggamma * b, grad_b = ggamma * a (fp64 sums). */
void oracle_branch_bwd(const void* g_dz, const void* g_zo, const void* dz, const void* mlp, const void* gate,
                       int64_t gs, const void* a, int adt, const void* b, int bdt, void* g_attn, void* g_mlp,
                       float* g_gate, float* ga, float* gb, int64_t B, int64_t T, int64_t C, int dt) {
#pragma omp parallel for schedule(static)
  for (int64_t c = 0; c < C; ++c) {
    float g = gamma_of(a, adt, b, bdt, c);
    double gam = 0.0;
    for (int64_t img = 0; img < B; ++img) {
      double gg = 0.0;
      float gt = ld(gate, dt, img * gs + c);
      for (int64_t t = 0; t < T; ++t) {
        int64_t i = (img * T + t) * C + c;
        float zo = ld(g_zo, dt, i);
        float from_lazy = rnd(g * zo, dt);
        float tot = g_dz ? rnd(ld(g_dz, dt, i) + from_lazy, dt) : from_lazy;
        st(g_attn, dt, i, tot);
        st(g_mlp, dt, i, gt * tot);
        gg += (double)rnd(tot * ld(mlp, dt, i), dt);
        gam += (double)zo * (double)ld(dz, dt, i);
      }
      if (g_gate) g_gate[img * C + c] = (float)gg;
    }
    float s = (float)gam;
    for (int r = 0; r < 16; ++r) {
      if (ga) ga[c * 16 + r] = s * ld(b, bdt, c * 16 + r);
      if (gb) gb[c * 16 + r] = s * ld(a, adt, c * 16 + r);
    }
  }
}
