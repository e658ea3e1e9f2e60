// C ABI of the LTHC kernels: argument validation, grid sizing and dtype/depth
// dispatch.  The library never allocates device memory; scratch for the
// two-stage weight-gradient reductions is passed in by the caller.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <type_traits>

#include <cudaTypedefs.h>

#include "lthc_b200.h"
#include "lthc_common.cuh"
#include "lthc_kernels.cuh"
#include "lthc_tma.cuh"
#include "lthc_broadcast_tma.cuh"
#include "lthc_pool_tma.cuh"
#include "lthc_final.cuh"
#include "lthc_umma.cuh"
#include "lthc_embed.cuh"
#include "lthc_branch.cuh"
#include "lthc_matbwd_tc.cuh"

namespace lthc {

namespace {

thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

struct DeviceInfo {
  int sms = 0;
  int major = 0;
  bool ok = false;
};

constexpr int kMaxDevices = 64;
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

// Returns LTHC_OK and fills *sms for the current device, or LTHC_ERR_DEVICE.
int current_device(int* sms) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return fail(LTHC_ERR_DEVICE, "no current CUDA device");
  }
  {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    DeviceInfo& d = g_dev[dev];
    if (!d.ok) {
      int sm = 0, major = 0;
      if (cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
          cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) {
        cudaGetLastError();
        return fail(LTHC_ERR_DEVICE, "cannot query CUDA device %d", dev);
      }
      d.sms = sm;
      d.major = major;
      d.ok = true;
    }
    if (d.major != 10) return fail(LTHC_ERR_DEVICE, "device %d is sm_%d0, this library is built for sm_100a", dev, d.major);
    *sms = d.sms;
  }
  return LTHC_OK;
}

// SM count used for grid sizing in workspace queries; falls back to the B200
// count when no device is current (the query then only over-estimates).
int sms_for_sizing() {
  int sms = 0;
  if (current_device(&sms) != LTHC_OK) {
    g_last_error[0] = '\0';
    return 148;
  }
  return sms;
}

bool valid_act(int dt) { return dt == LTHC_DTYPE_F32 || dt == LTHC_DTYPE_BF16 || dt == LTHC_DTYPE_F16; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_geometry(int64_t B, int64_t G, int64_t C, int act_dtype) {
  if (B < 0) return fail(LTHC_ERR_SHAPE, "batch must be >= 0, got %lld", (long long)B);
  if (G < 1 || G > 4096) return fail(LTHC_ERR_SHAPE, "workspace grid must be in [1, 4096], got %lld", (long long)G);
  if (C < 8 || C > 16384 || C % 8 != 0)
    return fail(LTHC_ERR_SHAPE, "channels must be a multiple of 8 in [8, 16384], got %lld", (long long)C);
  if (!valid_act(act_dtype)) return fail(LTHC_ERR_DTYPE, "unknown activation dtype code %d", act_dtype);
  return LTHC_OK;
}

int check_ptr(const void* p, const char* name) {
  if (!p) return fail(LTHC_ERR_NULL_POINTER, "%s is NULL", name);
  if (!aligned16(p)) return fail(LTHC_ERR_ALIGNMENT, "%s is not 16-byte aligned", name);
  return LTHC_OK;
}

// Activation tensors may be NULL when they are empty (torch gives empty tensors a
// null data pointer); everything else is checked like check_ptr.
int check_act(const void* p, const char* name, bool nonempty) {
  if (!p) return nonempty ? fail(LTHC_ERR_NULL_POINTER, "%s is NULL", name) : LTHC_OK;
  if (!aligned16(p)) return fail(LTHC_ERR_ALIGNMENT, "%s is not 16-byte aligned", name);
  return LTHC_OK;
}

int check_layers(int L) {
  if (L < 1 || L > kMaxLayers) return fail(LTHC_ERR_SHAPE, "n_layers must be in [1, %d], got %d", kMaxLayers, L);
  return LTHC_OK;
}

int launched(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(LTHC_ERR_LAUNCH, "%s launch failed: %s", what, cudaGetErrorString(e));
  return LTHC_OK;
}

#define LTHC_TRY(expr)           \
  do {                           \
    int _st = (expr);            \
    if (_st != LTHC_OK) return _st; \
  } while (0)

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
int64_t slices_of(int64_t C) { return ceil_div(C, kSliceCh); }

// ---- grid plans (pure functions of the problem size and the SM count) ------

// Weight-gradient partials: one [L][C][16] fp32 block per CTA column of the read
// kernel, whose grid is fixed at two CTAs per SM so that the workspace size is a
// pure function of the shape and the SM count.
#ifndef LTHC_WGRAD_CTAS_PER_SM
#define LTHC_WGRAD_CTAS_PER_SM 2
#endif
constexpr int kWgradCtasPerSm = LTHC_WGRAD_CTAS_PER_SM;

int64_t strips_of(int64_t B, int64_t G) { return B * G * ceil_div(G, kStripCells); }

// CTA columns for `per_sm` resident CTAs per SM: rounded down so that the whole
// grid (columns x channel slices) fits in one wave.
int64_t one_wave_columns(int64_t strips, int64_t C, int sms, int per_sm) {
  const int64_t nx = std::max<int64_t>(1, std::min<int64_t>(static_cast<int64_t>(sms) * per_sm / slices_of(C), strips));
  return ceil_div(strips, ceil_div(strips, nx));
}

int64_t wgrad_blocks(int64_t strips, int64_t C, int sms) { return one_wave_columns(strips, C, sms, kWgradCtasPerSm); }

// CTA columns of the one-pass read backward (one partial block per column): one
// wave of its resident CTAs (BcastShape<1, base, true>).
int64_t read_bwd_blocks(int64_t strips, int64_t C, int sms, bool base) {
  return one_wave_columns(strips, C, sms, base ? LTHC_READBWD_BASE_CTAS_PER_SM : LTHC_READBWD_CTAS_PER_SM);
}

size_t wgrad_ws_bytes(int64_t B, int64_t G, int64_t C, int L, int sms) {
  if (B <= 0) return 0;
  return static_cast<size_t>(wgrad_blocks(strips_of(B, G), C, sms)) * L * C * kPos * sizeof(float);
}

// Workspace of the read backward: the partials of the one-pass kernel or of the
// weight-gradient kernel, whichever the call uses.
size_t read_bwd_ws_bytes(int64_t B, int64_t G, int64_t C, int sms) {
  if (B <= 0) return 0;
  const int64_t nx = std::max(read_bwd_blocks(strips_of(B, G), C, sms, true),
                              read_bwd_blocks(strips_of(B, G), C, sms, false));
  return std::max(static_cast<size_t>(nx) * C * kPos * sizeof(float), wgrad_ws_bytes(B, G, C, 1, sms));
}

// Lazy-update grid: CTAs of 8 warps over (row blocks) x (channel slices of 32
// 16-byte vectors).  The fp32 slice (128 channels) is the narrowest, so the row
// block count below is an upper bound for every dtype; the partial buffer is
// sized with it.
int64_t lazy_slices(int64_t C, int esize) { return ceil_div(C, 32 * (16 / esize)); }

int64_t lazy_row_blocks(int64_t N, int64_t C, int sms) {
  const int64_t slices = lazy_slices(C, 4);
  const int64_t bx = std::max<int64_t>(1, static_cast<int64_t>(sms) * 4 / slices);
  return std::max<int64_t>(1, std::min<int64_t>(bx, ceil_div(N, kLazyWarps)));
}

size_t lazy_ws_bytes(int64_t N, int64_t C, int sms) {
  if (N <= 0) return 0;
  return static_cast<size_t>(lazy_row_blocks(N, C, sms)) * C * sizeof(float);
}

// ---- TMA tensor maps ---------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q{};
    void* f = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    cudaGetLastError();
  });
  return fn;
}

#ifndef LTHC_L2_PROMOTION
#define LTHC_L2_PROMOTION 0  // 0 none, 1 128 B, 2 256 B
#endif
constexpr CUtensorMapL2promotion kL2Promotion =
    LTHC_L2_PROMOTION == 0 ? CU_TENSOR_MAP_L2_PROMOTION_NONE
                           : (LTHC_L2_PROMOTION == 1 ? CU_TENSOR_MAP_L2_PROMOTION_L2_128B : CU_TENSOR_MAP_L2_PROMOTION_L2_256B);

template <typename T>
CUtensorMapDataType tmap_dtype() {
  if constexpr (sizeof(T) == 4) return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  else if constexpr (std::is_same_v<T, __nv_bfloat16>) return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  else return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

// NHWC residual [B, 4G, 4G, C] as a 4-D map (C, W, H, B); box = 64 channels x
// 4*kStripCells columns x 4 rows x 1 image (one strip of cells).
template <typename T>
int encode_residual_map(CUtensorMap* m, const void* ptr, int64_t B, int64_t G, int64_t C) {
  auto enc = tmap_encoder();
  if (!enc) return fail(LTHC_ERR_DEVICE, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t es = sizeof(T);
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(4 * G),
                              static_cast<cuuint64_t>(4 * G), static_cast<cuuint64_t>(B)};
  const cuuint64_t strides[3] = {C * es, 4 * G * C * es, 16 * G * G * C * es};
  const cuuint32_t box[4] = {kSliceCh, kBoxCols, 4, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, tmap_dtype<T>(), 4, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, kL2Promotion,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LTHC_ERR_LAUNCH, "cuTensorMapEncodeTiled (residual) failed with %d", (int)r);
  return LTHC_OK;
}

// Workspace [rows, C] as a 2-D map; box = 64 channels x kStripCells rows (one strip).
template <typename T>
int encode_workspace_map(CUtensorMap* m, const void* ptr, int64_t rows, int64_t C) {
  auto enc = tmap_encoder();
  if (!enc) return fail(LTHC_ERR_DEVICE, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t es = sizeof(T);
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {C * es};
  const cuuint32_t box[2] = {kSliceCh, kStripCells};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, tmap_dtype<T>(), 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, kL2Promotion,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LTHC_ERR_LAUNCH, "cuTensorMapEncodeTiled (workspace) failed with %d", (int)r);
  return LTHC_OK;
}

// Per-device, per-kernel, per-launch-shape set-up (cached): opt in to the dynamic
// shared memory the launch needs (the attribute only ever grows, so launches of
// the same kernel with other shapes stay valid) and record how many CTAs of that
// shape fit on one SM.
template <typename Kernel>
int resident_ctas(Kernel kern, int threads, int smem_bytes, int* out) {
  static std::mutex mu;
  static std::map<std::tuple<int, const void*, int, int>, int> cache;
  static std::map<std::pair<int, const void*>, int> smem_set;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return launched("cudaGetDevice");
  const void* fn = reinterpret_cast<const void*>(kern);
  const auto key = std::make_tuple(dev, fn, threads, smem_bytes);
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(key);
  if (it == cache.end()) {
    int& cur = smem_set[std::make_pair(dev, fn)];
    if (smem_bytes > cur) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) != cudaSuccess)
        return launched("cudaFuncSetAttribute");
      cur = smem_bytes;
    }
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, threads, smem_bytes) != cudaSuccess)
      return launched("cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    it = cache.emplace(key, std::max(n, 1)).first;
  }
  *out = it->second;
  return LTHC_OK;
}

// ---- dispatch helpers -----------------------------------------------------
template <typename T, int LT, bool HB, bool WG = false>
int launch_broadcast_tma(BcastTmaParams& p, int sms, cudaStream_t s, int64_t* nx_out = nullptr) {
  using Lay = BcastLayout<T, LT, HB, WG>;
  constexpr int kThreads = Lay::Shape::kThreads;
  auto kern = broadcast_tma_kernel<T, LT, HB, WG>;
  int per_sm = 1;
  LTHC_TRY(resident_ctas(kern, kThreads, Lay::kSmemBytes, &per_sm));
  const int64_t slices = slices_of(p.C);
  // the fused read backward writes one partial block per CTA column: the
  // weight-gradient grid, which the workspace query sizes
  int64_t nx = WG ? read_bwd_blocks(p.strips, p.C, sms, HB) : one_wave_columns(p.strips, p.C, sms, per_sm);
  p.strips_per_cta = ceil_div(p.strips, nx);
  nx = ceil_div(p.strips, p.strips_per_cta);
  if (nx_out) *nx_out = nx;
  kern<<<dim3(static_cast<unsigned>(nx), static_cast<unsigned>(slices)), kThreads, Lay::kSmemBytes, s>>>(p);
  return launched(WG ? "read backward (TMA, one pass)" : "broadcast (TMA)");
}

// grad_x = (grad_x_in +) alpha (.) grad_z and grad_alpha in one pass over x.
template <typename T>
int read_bwd_fused_t(const void* x, const void* grad_z, const void* alpha, int alpha_dtype, const void* grad_x_in,
                     void* grad_x, float* grad_alpha, void* ws, int64_t B, int64_t G, int64_t C, int sms,
                     cudaStream_t s) {
  BcastTmaParams p;
  memset(&p, 0, sizeof(p));
  if (grad_x_in) LTHC_TRY(encode_residual_map<T>(&p.tm_base, grad_x_in, B, G, C));
  LTHC_TRY(encode_residual_map<T>(&p.tm_out, grad_x, B, G, C));
  LTHC_TRY(encode_residual_map<T>(&p.tm_x, x, B, G, C));
  LTHC_TRY(encode_workspace_map<T>(&p.tm_dz[0], grad_z, B * G * G, C));
  p.w[0] = alpha;
  p.partial = static_cast<float*>(ws);
  p.out = grad_x;
  p.w_dtype = alpha_dtype;
  p.L = 1;
  p.G = static_cast<int>(G);
  p.strips_per_row = static_cast<int>(ceil_div(G, kStripCells));
  p.C = C;
  p.strips = B * G * p.strips_per_row;
  int64_t nx = 0;
  if (grad_x_in)
    LTHC_TRY((launch_broadcast_tma<T, 1, true, true>(p, sms, s, &nx)));
  else
    LTHC_TRY((launch_broadcast_tma<T, 1, false, true>(p, sms, s, &nx)));
  const int64_t n = C * kPos;
  const int64_t rb = std::min<int64_t>(ceil_div(n, 256), static_cast<int64_t>(sms) * 8);
  reduce_partials_kernel<<<static_cast<unsigned>(rb), 256, 0, s>>>(p.partial, grad_alpha, n, static_cast<int>(nx));
  return launched("weight-grad reduce");
}

template <typename T>
int broadcast_t(const void* base, const void* const* dz, const void* const* w, int w_dtype, int L, void* out,
                int64_t B, int64_t G, int64_t C, int sms, cudaStream_t s) {
  BcastTmaParams p;
  memset(&p, 0, sizeof(p));
  if (base) LTHC_TRY(encode_residual_map<T>(&p.tm_base, base, B, G, C));
  LTHC_TRY(encode_residual_map<T>(&p.tm_out, out, B, G, C));
  for (int l = 0; l < L; ++l) {
    LTHC_TRY(encode_workspace_map<T>(&p.tm_dz[l], dz[l], B * G * G, C));
    p.w[l] = w[l];
  }
  p.out = out;
  p.w_dtype = w_dtype;
  p.L = L;
  p.G = static_cast<int>(G);
  p.strips_per_row = static_cast<int>(ceil_div(G, kStripCells));
  p.C = C;
  p.strips = B * G * p.strips_per_row;
  const bool hb = base != nullptr;
  if (L == 12) return hb ? launch_broadcast_tma<T, 12, true>(p, sms, s) : launch_broadcast_tma<T, 12, false>(p, sms, s);
  if (L == 1) return hb ? launch_broadcast_tma<T, 1, true>(p, sms, s) : launch_broadcast_tma<T, 1, false>(p, sms, s);
  return hb ? launch_broadcast_tma<T, 0, true>(p, sms, s) : launch_broadcast_tma<T, 0, false>(p, sms, s);
}

// out = base + sum_{l<L} w_l (.) dz_l  (base may be NULL)
int broadcast(const void* base, const void* const* dz, const void* const* w, int w_dtype, int L, void* out, int64_t B,
              int64_t G, int64_t C, int act, cudaStream_t s) {
  int sms = 0;
  LTHC_TRY(current_device(&sms));
  switch (act) {
    case LTHC_DTYPE_F32: return broadcast_t<float>(base, dz, w, w_dtype, L, out, B, G, C, sms, s);
    case LTHC_DTYPE_BF16: return broadcast_t<__nv_bfloat16>(base, dz, w, w_dtype, L, out, B, G, C, sms, s);
    default: return broadcast_t<__half>(base, dz, w, w_dtype, L, out, B, G, C, sms, s);
  }
}

// ---- materialisation backward on the tensor cores ---------------------------------

#ifndef LTHC_MATBWD_TC
#define LTHC_MATBWD_TC 1  // 0: every materialisation backward runs the CUDA-core read-family kernel
#endif
#ifndef LTHC_MATBWD_DZ_STAGES
#define LTHC_MATBWD_DZ_STAGES 2  // dz ring of the plan (the smallest shared memory a call may need)
#endif
#ifndef LTHC_MATBWD_DZ_STAGES_WGRAD
#define LTHC_MATBWD_DZ_STAGES_WGRAD 3  // dz ring of a call that forms the weight gradient
#endif

// Launch plan of matbwd_tc_kernel; ok = false when the shape or dtype is not one
// it takes (fp32, a single layer, C not a multiple of 16, a grid side that does
// not tile into 32-cell stages, or a cell count that is not a whole number of
// 128-cell tiles): those run the CUDA-core kernel.
struct MbPlan {
  bool ok = false;
  int Gq = 0, Rq = 0, Lp = 0, gstages = 0, dstages = 0, visits = 0;
  int64_t S = 0, Tc = 0, parts = 0, grid = 0;
  size_t smem = 0, ws = 0;
};

MbPlan mb_plan(int64_t B, int64_t G, int64_t C, int L, int act, int sms) {
  MbPlan m;
  if (!LTHC_MATBWD_TC || act == LTHC_DTYPE_F32 || L < 2 || L > kMaxLayers || C % kMbSliceCh || B < 1) return m;
  if (G < 8 || (G <= 32 ? 32 % G : G % 32)) return m;
  const int64_t cells = B * G * G;
  if (cells % kMbTileCells || cells > INT32_MAX) return m;
  m.Gq = static_cast<int>(std::min<int64_t>(G, 32));
  m.Rq = 32 / m.Gq;
  m.Lp = L + (L & 1);
  // two T buffers, the weight operands, a dz ring of LTHC_MATBWD_DZ_STAGES and as
  // deep a grad X_L ring as the rest of the shared memory holds (B = 64, L = 12:
  // 3 grad X_L + 2 dz slots)
  const size_t dz = static_cast<size_t>(L) * kMbDzLayerBytes;
  const size_t fixed = 2 * kMbTRegion + kMbBetaBytes + kMbBarriers * 8 + 16 + kMbSmemAlign;  // + alignment slack
  const size_t budget = 227 * 1024;
  m.dstages = LTHC_MATBWD_DZ_STAGES;
  if (fixed + m.dstages * dz > budget) return m;
  m.gstages = static_cast<int>(std::min<size_t>(kMbMaxStages, (budget - fixed - m.dstages * dz) / kMbGxBytes));
  if (m.gstages < 2) return m;
  m.smem = fixed + m.dstages * dz + m.gstages * kMbGxBytes;
  m.Tc = cells / kMbTileCells;
  m.S = C / kMbSliceCh;
  // parts CTAs per slice (each a contiguous cell range), or one CTA per SM over
  // several slices when there are more slices than SMs
  m.parts = std::max<int64_t>(1, std::min<int64_t>(sms / m.S, m.Tc));
  m.grid = std::min<int64_t>(m.parts * m.S, sms);
  m.visits = static_cast<int>(ceil_div(m.S, m.grid));
  m.ws = static_cast<size_t>(m.grid) * m.visits * L * kMbSliceCh * kPos * sizeof(float);
  m.ok = true;
  return m;
}

template <typename T>
int matbwd_tc_t(const MbPlan& m, const void* grad_out, const void* const* dz, const void* const* beta, int beta_dtype,
                int L, void* const* grad_dz, float* grad_beta, void* ws, int64_t B, int64_t G, int64_t C,
                cudaStream_t s) {
  auto enc = tmap_encoder();
  if (!enc) return fail(LTHC_ERR_DEVICE, "cuTensorMapEncodeTiled is not available from the driver");
  MatBwdTcParams p;
  memset(&p, 0, sizeof(p));
  const cuuint64_t es = sizeof(T);
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  {
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(4 * G),
                                static_cast<cuuint64_t>(4 * G), static_cast<cuuint64_t>(B)};
    const cuuint64_t strides[3] = {C * es, 4 * G * C * es, 16 * G * G * C * es};
    const cuuint32_t box[4] = {kMbSliceCh, static_cast<cuuint32_t>(4 * m.Gq), static_cast<cuuint32_t>(4 * m.Rq), 1};
    CUresult r = enc(&p.tm_gx, tmap_dtype<T>(), 4, const_cast<void*>(grad_out), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, kL2Promotion,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(LTHC_ERR_LAUNCH, "cuTensorMapEncodeTiled (grad X_L tiles) failed with %d", (int)r);
  }
  const bool wgrad = grad_beta != nullptr;
  for (int l = 0; l < L; ++l) {
    if (wgrad) p.dz[l] = dz[l];
    if (grad_dz) {
      const cuuint64_t dims[2] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(B * G * G)};
      const cuuint64_t strides[1] = {C * es};
      const cuuint32_t box[2] = {kMbSliceCh, kMbTileCells};
      CUresult r = enc(&p.tm_gdz[l], tmap_dtype<T>(), 2, grad_dz[l], dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, kL2Promotion,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r != CUDA_SUCCESS) return fail(LTHC_ERR_LAUNCH, "cuTensorMapEncodeTiled (grad_dz) failed with %d", (int)r);
    }
  }
  for (int l = 0; l < L; ++l)
    if (grad_dz) p.beta[l] = beta[l];
  p.partial = wgrad ? static_cast<float*>(ws) : nullptr;
  p.beta_dtype = beta_dtype;
  p.L = L;
  p.Lp = m.Lp;
  p.G = static_cast<int>(G);
  p.Gq = m.Gq;
  p.Rq = m.Rq;
  // ring depths of this call: with the weight gradient a deeper dz ring (the dz
  // copies are the slower stream), without it no dz ring and a deeper grad X_L ring
  {
    const size_t dzb = static_cast<size_t>(L) * kMbDzLayerBytes;
    const size_t fixed = m.smem - m.dstages * dzb - m.gstages * kMbGxBytes;
    const size_t budget = 227 * 1024;
    const int dst = wgrad ? LTHC_MATBWD_DZ_STAGES_WGRAD : 1;
    const int gst = static_cast<int>(std::min<size_t>(kMbMaxStages, (budget - fixed - dst * dzb) / kMbGxBytes));
    if (gst >= 2 && fixed + dst * dzb <= budget) {
      p.gstages = gst;
      p.dstages = dst;
    } else {
      p.gstages = m.gstages;
      p.dstages = m.dstages;
    }
  }
  const size_t smem = (m.smem - m.dstages * static_cast<size_t>(L) * kMbDzLayerBytes - m.gstages * kMbGxBytes) +
                      p.dstages * static_cast<size_t>(L) * kMbDzLayerBytes + p.gstages * kMbGxBytes;
  p.need_pool = grad_dz != nullptr;
  p.need_wgrad = wgrad;
  p.visits = m.visits;
  p.C = C;
  p.S = m.S;
  p.Tc = m.Tc;
  p.parts = m.parts;
  int per_sm = 0;
  LTHC_TRY(resident_ctas(matbwd_tc_kernel<T>, kMbThreads, static_cast<int>(smem), &per_sm));
  if (per_sm < 1) return fail(LTHC_ERR_LAUNCH, "the tensor-core backward does not fit on an SM");
  matbwd_tc_kernel<T><<<static_cast<unsigned>(m.grid), kMbThreads, smem, s>>>(p);
  LTHC_TRY(launched("materialisation backward (tensor cores)"));
  if (wgrad) {
    const int64_t n = static_cast<int64_t>(L) * C * kPos;
    const int64_t blocks = std::min<int64_t>(ceil_div(n, 256), m.grid * 4);
    matbwd_tc_finalize_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(static_cast<const float*>(ws), grad_beta,
                                                                            L, C, m.S, m.parts, m.grid, m.visits);
    LTHC_TRY(launched("materialisation backward weight-gradient finalize"));
  }
  return LTHC_OK;
}

// ---- materialisation fused with the final norm + modulate (clusters) ----------
// ---- read family -------------------------------------------------------------
struct ReadJob {
  const void* h;               // residual-sized input
  const void* const* w;        // POOL weights
  int w_dtype;
  void* const* out;            // POOL outputs (nullptr: no pooling)
  const void* const* low;      // WGRAD workspace-sized inputs
  float* grad_w;               // WGRAD result [L][C][16] (nullptr: no weight gradient)
  void* ws;                    // WGRAD partials
  int L;
  int64_t B, G, C;
};

template <typename T, int LT, bool POOL, bool WGRAD, int CPP>
int launch_read_t(PoolTmaParams& p, float* grad_w, int sms, cudaStream_t s) {
  using Lay = PoolLayout<T, (LT > 0 ? LT : kMaxLayers), POOL, WGRAD, CPP>;
  auto kern = pool_tma_kernel<T, LT, POOL, WGRAD, CPP>;
  int per_sm = 1;
  LTHC_TRY(resident_ctas(kern, Lay::kThreads, Lay::kSmemBytes, &per_sm));
  const int64_t slices = slices_of(p.C);
  int64_t nx = WGRAD ? wgrad_blocks(p.strips, p.C, sms) : one_wave_columns(p.strips, p.C, sms, per_sm);
  p.strips_per_cta = ceil_div(p.strips, nx);
  nx = ceil_div(p.strips, p.strips_per_cta);
  kern<<<dim3(static_cast<unsigned>(nx), static_cast<unsigned>(slices)), Lay::kThreads, Lay::kSmemBytes, s>>>(p);
  LTHC_TRY(launched("read family (TMA)"));
  if (WGRAD) {
    const int64_t n = static_cast<int64_t>(p.L) * p.C * kPos;
    const int64_t rb = std::min<int64_t>(ceil_div(n, 256), static_cast<int64_t>(sms) * 8);
    reduce_partials_kernel<<<static_cast<unsigned>(rb), 256, 0, s>>>(p.partial, grad_w, n, static_cast<int>(nx));
    LTHC_TRY(launched("weight-grad reduce"));
  }
  return LTHC_OK;
}

template <typename T, bool POOL, bool WGRAD>
int launch_read_l(PoolTmaParams& p, float* grad_w, int sms, cudaStream_t s) {
  if (p.L == 1) return launch_read_t<T, 1, POOL, WGRAD, 1>(p, grad_w, sms, s);
  if (p.L == 12) return launch_read_t<T, 12, POOL, WGRAD, LTHC_POOL_CELLS_DEEP>(p, grad_w, sms, s);
  return launch_read_t<T, 0, POOL, WGRAD, LTHC_POOL_CELLS_DEEP>(p, grad_w, sms, s);
}

template <typename T>
int read_family_t(const ReadJob& j, int sms, cudaStream_t s) {
  PoolTmaParams p;
  memset(&p, 0, sizeof(p));
  const bool pool = j.out != nullptr;
  const bool wgrad = j.grad_w != nullptr;
  LTHC_TRY(encode_residual_map<T>(&p.tm_h, j.h, j.B, j.G, j.C));
  for (int l = 0; l < j.L; ++l) {
    if (pool) {
      p.w[l] = j.w[l];
      p.out[l] = j.out[l];
    }
    if (wgrad) LTHC_TRY(encode_workspace_map<T>(&p.tm_low[l], j.low[l], j.B * j.G * j.G, j.C));
  }
  p.partial = wgrad ? static_cast<float*>(j.ws) : nullptr;
  p.w_dtype = j.w_dtype;
  p.L = j.L;
  p.G = static_cast<int>(j.G);
  p.strips_per_row = static_cast<int>(ceil_div(j.G, kStripCells));
  p.C = j.C;
  p.strips = strips_of(j.B, j.G);
  if (pool && wgrad) return launch_read_l<T, true, true>(p, j.grad_w, sms, s);
  if (pool) return launch_read_l<T, true, false>(p, nullptr, sms, s);
  return launch_read_l<T, false, true>(p, j.grad_w, sms, s);
}

// Runs the read-family kernel (pooling and/or weight gradient).  The caller has
// validated pointers; this checks the workspace and handles the empty batch.
int read_family(const ReadJob& j, size_t ws_bytes, int act, cudaStream_t s) {
  if (!j.out && !j.grad_w) return LTHC_OK;
  int sms = 0;
  LTHC_TRY(current_device(&sms));
  if (j.B == 0) {
    // Empty batch: pooled outputs are empty, the weight gradient is exactly zero.
    if (j.grad_w && cudaMemsetAsync(j.grad_w, 0, sizeof(float) * j.L * j.C * kPos, s) != cudaSuccess)
      return launched("memset");
    return LTHC_OK;
  }
  if (j.grad_w) {
    const size_t need = wgrad_ws_bytes(j.B, j.G, j.C, j.L, sms);
    if (!j.ws || ws_bytes < need)
      return fail(LTHC_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu bytes required", ws_bytes, need);
    if (!aligned16(j.ws)) return fail(LTHC_ERR_ALIGNMENT, "workspace is not 16-byte aligned");
  }
  switch (act) {
    case LTHC_DTYPE_F32: return read_family_t<float>(j, sms, s);
    case LTHC_DTYPE_BF16: return read_family_t<__nv_bfloat16>(j, sms, s);
    default: return read_family_t<__half>(j, sms, s);
  }
}

int check_weight_dtype(int dt, const char* name) {
  if (!valid_act(dt)) return fail(LTHC_ERR_DTYPE, "unknown %s dtype code %d", name, dt);
  return LTHC_OK;
}

// ---- branch epilogue fused with the lazy update -------------------------------

// Backward CTAs per image (each owns a contiguous row range of one image); a
// pure function of the shape and the SM count, so that the workspace query and
// the launch agree.
// CTAs per image of the branch backward (each owns a contiguous row range of one
// image): close to two full waves of its two resident CTAs per SM, counted with
// the 16-bit slice width (the same count for every dtype, so the workspace
// query needs no dtype).
int64_t branch_ctas_per_image(int64_t B, int64_t T, int64_t C, int sms) {
  if (B <= 0 || T <= 0) return 1;
  const int64_t slots = 2 * static_cast<int64_t>(sms);
  const int64_t k = std::max<int64_t>(1, std::min<int64_t>(2 * slots / (B * lazy_slices(C, 2)),
                                                           ceil_div(T, kLazyWarps)));
  return ceil_div(T, ceil_div(T, k));
}

size_t branch_ws_bytes(int64_t B, int64_t T, int64_t C, int sms) {
  if (B <= 0 || T <= 0) return 0;
  return static_cast<size_t>(B * branch_ctas_per_image(B, T, C, sms)) * 2 * C * sizeof(float);
}

int check_branch(int64_t B, int64_t T, int64_t C, int64_t gstride, int act, int adt, int bdt) {
  if (B < 0 || T < 0) return fail(LTHC_ERR_SHAPE, "batch and rows per image must be >= 0");
  if (C < 8 || C > 16384 || C % 8) return fail(LTHC_ERR_SHAPE, "channels must be a multiple of 8 in [8, 16384]");
  if (gstride < C || gstride % 8) return fail(LTHC_ERR_SHAPE, "gate row stride %lld must be >= C and a multiple of 8",
                                              (long long)gstride);
  if (!valid_act(act)) return fail(LTHC_ERR_DTYPE, "unknown activation dtype code %d", act);
  LTHC_TRY(check_weight_dtype(adt, "alpha"));
  return check_weight_dtype(bdt, "beta");
}

// ---- patch embedding fused with the shared read (tensor cores) -----------------

// X0 NHWC [B, H, H, C] bf16 as a 4-D map (C, W, H, B) for the staged tile stores:
// box = 64 channels x 32 columns x 4 rows, 128-byte swizzle (the UMMA operand
// layout of the staging buffer).
int encode_embed_store_map(CUtensorMap* m, void* ptr, int64_t B, int64_t H, int64_t C) {
  auto enc = tmap_encoder();
  if (!enc) return fail(LTHC_ERR_DEVICE, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t es = 2;
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(H),
                              static_cast<cuuint64_t>(B)};
  const cuuint64_t strides[3] = {C * es, H * C * es, H * H * C * es};
  const cuuint32_t box[4] = {64, static_cast<cuuint32_t>(kEmbedTileCols), 4, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LTHC_ERR_LAUNCH, "cuTensorMapEncodeTiled (embed store) failed with %d", (int)r);
  return LTHC_OK;
}

// ---- final-layer prologue (RMSNorm + modulate) --------------------------------

// Launch shape: one thread per channel pair (at least 4 warps); tiles of two
// tokens per warp (forward) or one (backward, two tensors per token), 3 stages;
// the tile shrinks for wide rows so that a CTA's ring stays within
// kFinalSmemBudget (two CTAs per SM).  Measured on B200 at B = 64, T = 4096,
// C = 768 bf16: 3 stages beat 4 or 6 (bigger tiles amortise the per-tile
// barrier), and a 72 KB budget (3 CTAs per SM, smaller tiles) is slower.
struct FinalShape {
  int threads, tile, stages;
  size_t smem;
};
#ifndef LTHC_FINAL_SMEM_BUDGET_KB
#define LTHC_FINAL_SMEM_BUDGET_KB 110
#endif
#ifndef LTHC_FINAL_FWD_TOKENS_PER_WARP
#define LTHC_FINAL_FWD_TOKENS_PER_WARP 2
#endif
#ifndef LTHC_FINAL_FWD_STAGES
#define LTHC_FINAL_FWD_STAGES 3
#endif
#ifndef LTHC_FINAL_BWD_STAGES
#define LTHC_FINAL_BWD_STAGES 3
#endif
constexpr size_t kFinalSmemBudget = LTHC_FINAL_SMEM_BUDGET_KB * 1024;
// The ring refills the stage of tile i - 1 at the end of tile i (after that
// tile's bulk store has read it) with tile i - 1 + stages, while tile i + 1 must
// already be loading: fewer than 3 stages would wait on a tile never requested.
static_assert(LTHC_FINAL_FWD_STAGES >= 3 && LTHC_FINAL_BWD_STAGES >= 3, "the final-layer ring needs 3 or more stages");

FinalShape final_shape(int64_t C, int es, bool bwd) {
  FinalShape f;
  const int warps = static_cast<int>(std::min<int64_t>(kFinalMaxThreads / 32, std::max<int64_t>(4, ceil_div(C, 64))));
  f.threads = 32 * warps;
  f.stages = bwd ? LTHC_FINAL_BWD_STAGES : LTHC_FINAL_FWD_STAGES;
  f.tile = bwd ? warps : LTHC_FINAL_FWD_TOKENS_PER_WARP * warps;
  while (f.tile > 1 && FinalSmem(C, es, f.tile, f.stages, bwd).total > kFinalSmemBudget) --f.tile;
  f.smem = FinalSmem(C, es, f.tile, f.stages, bwd).total;
  return f;
}

// CTAs per image: about two per SM over the whole batch, each with whole tiles.
// The backward's workspace is sized with tile = 1 (an upper bound on the count).
constexpr int kFinalCtasPerSm = 2;

int64_t final_tokens_per_cta(int64_t B, int64_t T, int tile, int sms) {
  const int64_t want = std::max<int64_t>(1, static_cast<int64_t>(sms) * kFinalCtasPerSm / std::max<int64_t>(B, 1));
  const int64_t k = std::max<int64_t>(1, std::min<int64_t>(want, ceil_div(T, tile)));
  return ceil_div(ceil_div(T, k), tile) * tile;
}

int64_t final_ctas_per_image(int64_t B, int64_t T, int tile, int sms) {
  if (T <= 0) return 1;
  return ceil_div(T, final_tokens_per_cta(B, T, tile, sms));
}

size_t final_ws_bytes(int64_t B, int64_t T, int64_t C, int sms) {
  if (B <= 0 || T <= 0) return 0;
  return static_cast<size_t>(B * final_ctas_per_image(B, T, 1, sms)) * 3 * C * sizeof(float);
}

int check_final(int64_t B, int64_t T, int64_t C, int64_t mod_stride, int act_dtype, int w_dtype, float eps) {
  if (B < 0 || T < 0) return fail(LTHC_ERR_SHAPE, "batch and tokens must be >= 0, got %lld, %lld", (long long)B,
                                  (long long)T);
  if (B > 65535) return fail(LTHC_ERR_SHAPE, "batch must be <= 65535, got %lld", (long long)B);
  if (C < 8 || C > kFinalChunk * kFinalMaxChunks || C % 8 != 0)
    return fail(LTHC_ERR_SHAPE, "channels must be a multiple of 8 in [8, %d], got %lld", kFinalChunk * kFinalMaxChunks,
                (long long)C);
  if (mod_stride < C) return fail(LTHC_ERR_SHAPE, "shift/scale row stride %lld is below C = %lld",
                                  (long long)mod_stride, (long long)C);
  if (!valid_act(act_dtype)) return fail(LTHC_ERR_DTYPE, "unknown activation dtype code %d", act_dtype);
  if (!valid_act(w_dtype)) return fail(LTHC_ERR_DTYPE, "unknown norm weight dtype code %d", w_dtype);
  if (!(eps >= 0.f)) return fail(LTHC_ERR_SHAPE, "eps must be >= 0");
  return LTHC_OK;
}

template <typename T, bool BWD>
int final_launch(FinalParams& p, int64_t B, int sms, int64_t* ctas_per_image, cudaStream_t s) {
  const FinalShape f = final_shape(p.C, sizeof(T), BWD);
  p.tile = f.tile;
  p.stages = f.stages;
  auto go = [&](auto kern) -> int {
    int per_sm = 0;
    LTHC_TRY(resident_ctas(kern, f.threads, static_cast<int>(f.smem), &per_sm));
    // forward: one wave of resident CTAs; backward: the workspace plan's count
    const int ctas_per_sm = BWD ? kFinalCtasPerSm : per_sm;
    p.tokens_per_cta = final_tokens_per_cta(B, p.T, f.tile, sms * ctas_per_sm / kFinalCtasPerSm);
    const int64_t K = ceil_div(p.T, p.tokens_per_cta);
    *ctas_per_image = K;
    const dim3 grid(static_cast<unsigned>(K), static_cast<unsigned>(B));
    kern<<<grid, f.threads, f.smem, s>>>(p);
    return launched(BWD ? "final norm/modulate backward" : "final norm/modulate forward");
  };
  switch (ceil_div(p.C, kFinalChunk)) {
    case 1: return go(final_norm_modulate_kernel<T, BWD, 1>);
    case 2: return go(final_norm_modulate_kernel<T, BWD, 2>);
    case 3: return go(final_norm_modulate_kernel<T, BWD, 3>);
    default: return go(final_norm_modulate_kernel<T, BWD, 4>);
  }
}

template <bool BWD>
int final_dispatch(FinalParams& p, int64_t B, int sms, int64_t* K, int act, cudaStream_t s) {
  switch (act) {
    case LTHC_DTYPE_F32: return final_launch<float, BWD>(p, B, sms, K, s);
    case LTHC_DTYPE_BF16: return final_launch<__nv_bfloat16, BWD>(p, B, sms, K, s);
    default: return final_launch<__half, BWD>(p, B, sms, K, s);
  }
}

FinalParams final_params(const void* x, const void* w, int w_dtype, const void* shift, const void* scale,
                         int64_t mod_stride, int64_t T, int64_t C, float eps) {
  FinalParams p;
  memset(&p, 0, sizeof(p));
  p.x = x;
  p.w = w;
  p.w_dtype = w_dtype;
  p.shift = shift;
  p.scale = scale;
  p.mod_stride = mod_stride;
  p.T = T;
  p.C = C;
  p.eps = eps;
  p.inv_c = 1.0f / static_cast<float>(C);
  p.c_f = static_cast<float>(C);
  return p;
}

}  // namespace
}  // namespace lthc

using namespace lthc;

extern "C" {

int lthc_version(void) { return 100; }

const char* lthc_status_string(int status) {
  switch (status) {
    case LTHC_OK: return "ok";
    case LTHC_ERR_NULL_POINTER: return "null pointer";
    case LTHC_ERR_SHAPE: return "unsupported shape";
    case LTHC_ERR_DTYPE: return "unsupported dtype";
    case LTHC_ERR_ALIGNMENT: return "misaligned pointer";
    case LTHC_ERR_WORKSPACE: return "workspace too small";
    case LTHC_ERR_LAUNCH: return "kernel launch failed";
    case LTHC_ERR_DEVICE: return "no usable sm_100 device";
    case LTHC_ERR_TIMEOUT: return "device-side wait timed out";
    default: return "unknown status";
  }
}

const char* lthc_last_error_message(void) { return g_last_error; }

int lthc_device_status(int* status_out, void* stream) {
  if (!status_out) return fail(LTHC_ERR_NULL_POINTER, "status_out is NULL");
  int sms = 0;
  LTHC_TRY(current_device(&sms));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int host = 0;
  const int zero = 0;
  if (cudaMemcpyFromSymbolAsync(&host, g_device_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaMemcpyToSymbolAsync(g_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return launched("device status read");
  *status_out = host ? LTHC_ERR_TIMEOUT : LTHC_OK;
  return LTHC_OK;
}

int lthc_selftest_wait_timeout(int limit_ms, int* result_dev, void* stream) {
  if (limit_ms < 1 || limit_ms > 5000) return fail(LTHC_ERR_SHAPE, "limit_ms must be in [1, 5000], got %d", limit_ms);
  LTHC_TRY(check_ptr(result_dev, "result_dev"));
  int sms = 0;
  LTHC_TRY(current_device(&sms));
  wait_timeout_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<unsigned long long>(limit_ms) * 1000000ull, result_dev);
  return launched("wait-timeout self-test");
}

int lthc_selftest_umma(const void* A, const void* B, float* D, int N, int K, int* status_dev, void* stream) {
  if (!A || !B || !D || !status_dev) return fail(LTHC_ERR_NULL_POINTER, "A, B, D and status must be set");
  if (!(N == 64 || N == 128 || N == 256)) return fail(LTHC_ERR_SHAPE, "N must be 64, 128 or 256, got %d", N);
  if (K < 64 || K > 256 || K % 64) return fail(LTHC_ERR_SHAPE, "K must be 64, 128, 192 or 256, got %d", K);
  int sms = 0;
  LTHC_TRY(current_device(&sms));
  const int smem = 1024 + (K / 64) * (128 + N) * 128 + 16;
  int per_sm = 0;
  LTHC_TRY(resident_ctas(umma_selftest_kernel, 128, smem, &per_sm));
  umma_selftest_kernel<<<1, 128, smem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(A), static_cast<const __nv_bfloat16*>(B), D, N, K, status_dev);
  return launched("tcgen05 self-test");
}

int lthc_selftest_umma_desc(const void* a_img, int a_bytes, const void* b_img, int b_bytes, const uint64_t* a_desc,
                            const uint64_t* b_desc, int steps, uint32_t idesc, int N, float* D, int* status_dev,
                            void* stream) {
  if (!a_img || !b_img || !a_desc || !b_desc || !D || !status_dev)
    return fail(LTHC_ERR_NULL_POINTER, "images, descriptors, D and status must be set");
  if (!aligned16(a_img) || !aligned16(b_img)) return fail(LTHC_ERR_ALIGNMENT, "operand images must be 16-byte aligned");
  if (a_bytes < 16 || a_bytes > kUmmaProbeRegion || a_bytes % 16 || b_bytes < 16 || b_bytes > kUmmaProbeRegion ||
      b_bytes % 16)
    return fail(LTHC_ERR_SHAPE, "operand images must be 16..%d bytes, multiples of 16", kUmmaProbeRegion);
  if (steps < 1 || steps > kUmmaProbeMaxSteps) return fail(LTHC_ERR_SHAPE, "steps must be in [1, %d]", kUmmaProbeMaxSteps);
  if (N < 16 || N > 256 || N % 16) return fail(LTHC_ERR_SHAPE, "N must be a multiple of 16 in [16, 256], got %d", N);
  if (((idesc >> 24) & 31u) != 8u || ((idesc >> 17) & 63u) != static_cast<uint32_t>(N >> 3))
    return fail(LTHC_ERR_SHAPE, "the instruction descriptor must encode M = 128 and N = %d", N);
  UmmaProbeParams p;
  memset(&p, 0, sizeof(p));
  for (int s = 0; s < steps; ++s) {
    // start addresses are region-relative and must stay inside the region (the
    // kernel adds the region's shared address to the 14-bit field)
    if ((a_desc[s] & 0x3FFFu) * 16 >= static_cast<uint64_t>(kUmmaProbeRegion) ||
        (b_desc[s] & 0x3FFFu) * 16 >= static_cast<uint64_t>(kUmmaProbeRegion))
      return fail(LTHC_ERR_SHAPE, "step %d starts outside its operand region", s);
    p.a_desc[s] = a_desc[s];
    p.b_desc[s] = b_desc[s];
  }
  p.steps = steps;
  p.idesc = idesc;
  p.N = N;
  p.a_bytes = a_bytes;
  p.b_bytes = b_bytes;
  int sms = 0;
  LTHC_TRY(current_device(&sms));
  int per_sm = 0;
  LTHC_TRY(resident_ctas(umma_probe_kernel, 128, kUmmaProbeSmem, &per_sm));
  umma_probe_kernel<<<1, 128, kUmmaProbeSmem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(a_img), static_cast<const uint4*>(b_img), p, D, status_dev);
  return launched("tcgen05 descriptor self-test");
}

// ------------------------------ write family ---------------------------------

int lthc_write_fwd(const void* dz, const void* beta, int beta_dtype, void* out, int64_t B, int64_t G, int64_t C,
                   int act_dtype, void* stream) {
  LTHC_TRY(check_geometry(B, G, C, act_dtype));
  LTHC_TRY(check_weight_dtype(beta_dtype, "beta"));
  LTHC_TRY(check_act(dz, "dz", B > 0));
  LTHC_TRY(check_ptr(beta, "beta"));
  LTHC_TRY(check_act(out, "out", B > 0));
  if (B == 0) return LTHC_OK;
  const void* dzs[1] = {dz};
  const void* ws[1] = {beta};
  return broadcast(nullptr, dzs, ws, beta_dtype, 1, out, B, G, C, act_dtype, static_cast<cudaStream_t>(stream));
}

int lthc_write_add_fwd(const void* x, const void* dz, const void* beta, int beta_dtype, void* out, int64_t B,
                       int64_t G, int64_t C, int act_dtype, void* stream) {
  LTHC_TRY(check_geometry(B, G, C, act_dtype));
  LTHC_TRY(check_weight_dtype(beta_dtype, "beta"));
  LTHC_TRY(check_act(x, "x", B > 0));
  LTHC_TRY(check_act(dz, "dz", B > 0));
  LTHC_TRY(check_ptr(beta, "beta"));
  LTHC_TRY(check_act(out, "out", B > 0));
  if (B == 0) return LTHC_OK;
  const void* dzs[1] = {dz};
  const void* ws[1] = {beta};
  return broadcast(x, dzs, ws, beta_dtype, 1, out, B, G, C, act_dtype, static_cast<cudaStream_t>(stream));
}

int lthc_materialise_fwd(const void* x0, const void* const* dz, const void* const* beta, int beta_dtype,
                         int n_layers, void* out, int64_t B, int64_t G, int64_t C, int act_dtype, void* stream) {
  LTHC_TRY(check_geometry(B, G, C, act_dtype));
  LTHC_TRY(check_weight_dtype(beta_dtype, "beta"));
  LTHC_TRY(check_layers(n_layers));
  if (!dz || !beta) return fail(LTHC_ERR_NULL_POINTER, "dz / beta pointer arrays are NULL");
  if (x0) LTHC_TRY(check_act(x0, "x0", B > 0));
  LTHC_TRY(check_act(out, "out", B > 0));
  for (int l = 0; l < n_layers; ++l) {
    LTHC_TRY(check_act(dz[l], "dz[l]", B > 0));
    LTHC_TRY(check_ptr(beta[l], "beta[l]"));
  }
  if (B == 0) return LTHC_OK;
  return broadcast(x0, dz, beta, beta_dtype, n_layers, out, B, G, C, act_dtype, static_cast<cudaStream_t>(stream));
}

int lthc_materialise12_fwd(const void* x0, const void* const* dz, const void* const* beta, int beta_dtype,
                           void* out, int64_t B, int64_t G, int64_t C, int act_dtype, void* stream) {
  return lthc_materialise_fwd(x0, dz, beta, beta_dtype, 12, out, B, G, C, act_dtype, stream);
}

size_t lthc_materialise_bwd_workspace_bytes(int64_t B, int64_t G, int64_t C, int n_layers) {
  if (B <= 0 || G <= 0 || C <= 0 || n_layers < 1 || n_layers > kMaxLayers) return 0;
  const int sms = sms_for_sizing();
  // the larger of the two kernels' needs (the query does not know the dtype)
  const MbPlan m = mb_plan(B, G, C, n_layers, LTHC_DTYPE_BF16, sms);
  return std::max(wgrad_ws_bytes(B, G, C, n_layers, sms), m.ok ? m.ws : size_t{0});
}

int lthc_materialise_bwd_uses_tensor_cores(int64_t B, int64_t G, int64_t C, int n_layers, int act_dtype) {
  if (B < 1 || G < 1 || C < 8 || !valid_act(act_dtype)) return 0;
  return mb_plan(B, G, C, n_layers, act_dtype, sms_for_sizing()).ok ? 1 : 0;
}

int lthc_materialise_bwd(const void* grad_out, const void* const* dz, const void* const* beta, int beta_dtype,
                         int n_layers, void* const* grad_dz, float* grad_beta, void* workspace,
                         size_t workspace_bytes, int64_t B, int64_t G, int64_t C, int act_dtype, void* stream) {
  LTHC_TRY(check_geometry(B, G, C, act_dtype));
  LTHC_TRY(check_weight_dtype(beta_dtype, "beta"));
  LTHC_TRY(check_layers(n_layers));
  LTHC_TRY(check_act(grad_out, "grad_out", B > 0));
  if (!grad_dz && !grad_beta) return LTHC_OK;
  if (grad_dz) {
    if (!beta) return fail(LTHC_ERR_NULL_POINTER, "beta pointer array is NULL");
    for (int l = 0; l < n_layers; ++l) {
      LTHC_TRY(check_ptr(beta[l], "beta[l]"));
      LTHC_TRY(check_act(grad_dz[l], "grad_dz[l]", B > 0));
    }
  }
  if (grad_beta) {
    if (!dz) return fail(LTHC_ERR_NULL_POINTER, "dz pointer array is NULL");
    LTHC_TRY(check_ptr(grad_beta, "grad_beta"));
    for (int l = 0; l < n_layers; ++l) LTHC_TRY(check_act(dz[l], "dz[l]", B > 0));
  }
  if (B == 0) {
    ReadJob j{grad_out, beta, beta_dtype, grad_dz, dz, grad_beta, workspace, n_layers, B, G, C};
    return read_family(j, workspace_bytes, act_dtype, static_cast<cudaStream_t>(stream));
  }
  int sms = 0;
  LTHC_TRY(current_device(&sms));
  const MbPlan m = mb_plan(B, G, C, n_layers, act_dtype, sms);
  if (m.ok) {
    // One pass over grad_out on the tensor cores produces both gradients.
    if (grad_beta) {
      if (!workspace || workspace_bytes < m.ws)
        return fail(LTHC_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu bytes required",
                    workspace_bytes, m.ws);
      if (!aligned16(workspace)) return fail(LTHC_ERR_ALIGNMENT, "workspace is not 16-byte aligned");
    }
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (act_dtype == LTHC_DTYPE_BF16)
      return matbwd_tc_t<__nv_bfloat16>(m, grad_out, dz, beta, beta_dtype, n_layers, grad_dz, grad_beta, workspace,
                                        B, G, C, s);
    return matbwd_tc_t<__half>(m, grad_out, dz, beta, beta_dtype, n_layers, grad_dz, grad_beta, workspace, B, G, C,
                               s);
  }
  // One pass over grad_out produces both gradients.
  ReadJob j{grad_out, beta, beta_dtype, grad_dz, dz, grad_beta, workspace, n_layers, B, G, C};
  return read_family(j, workspace_bytes, act_dtype, static_cast<cudaStream_t>(stream));
}

size_t lthc_write_bwd_workspace_bytes(int64_t B, int64_t G, int64_t C) {
  return lthc_materialise_bwd_workspace_bytes(B, G, C, 1);
}

int lthc_write_bwd(const void* grad_out, const void* dz, const void* beta, int beta_dtype, void* grad_dz,
                   float* grad_beta, void* workspace, size_t workspace_bytes, int64_t B, int64_t G, int64_t C,
                   int act_dtype, void* stream) {
  const void* dzs[1] = {dz};
  const void* betas[1] = {beta};
  void* gdzs[1] = {grad_dz};
  return lthc_materialise_bwd(grad_out, dzs, betas, beta_dtype, 1, grad_dz ? gdzs : nullptr, grad_beta, workspace,
                              workspace_bytes, B, G, C, act_dtype, stream);
}

// ------------------------------ read family ----------------------------------

int lthc_read_fwd(const void* x, const void* alpha, int alpha_dtype, void* z, int64_t B, int64_t G, int64_t C,
                  int act_dtype, void* stream) {
  LTHC_TRY(check_geometry(B, G, C, act_dtype));
  LTHC_TRY(check_weight_dtype(alpha_dtype, "alpha"));
  LTHC_TRY(check_act(x, "x", B > 0));
  LTHC_TRY(check_ptr(alpha, "alpha"));
  LTHC_TRY(check_act(z, "z", B > 0));
  if (B == 0) return LTHC_OK;
  const void* w[1] = {alpha};
  void* out[1] = {z};
  ReadJob j{x, w, alpha_dtype, out, nullptr, nullptr, nullptr, 1, B, G, C};
  return read_family(j, 0, act_dtype, static_cast<cudaStream_t>(stream));
}

size_t lthc_weight_grad_workspace_bytes(int64_t B, int64_t G, int64_t C, int n_layers) {
  return lthc_materialise_bwd_workspace_bytes(B, G, C, n_layers);
}

int lthc_weight_grad(const void* high, const void* const* low, int n_layers, float* grad_w, void* workspace,
                     size_t workspace_bytes, int64_t B, int64_t G, int64_t C, int act_dtype, void* stream) {
  LTHC_TRY(check_geometry(B, G, C, act_dtype));
  LTHC_TRY(check_layers(n_layers));
  LTHC_TRY(check_act(high, "high", B > 0));
  LTHC_TRY(check_ptr(grad_w, "grad_w"));
  if (!low) return fail(LTHC_ERR_NULL_POINTER, "low pointer array is NULL");
  for (int l = 0; l < n_layers; ++l) LTHC_TRY(check_act(low[l], "low[l]", B > 0));
  ReadJob j{high, nullptr, LTHC_DTYPE_F32, nullptr, low, grad_w, workspace, n_layers, B, G, C};
  return read_family(j, workspace_bytes, act_dtype, static_cast<cudaStream_t>(stream));
}

// ---- weight gradient without caller scratch -------------------------------------
// The per-CTA partials of lthc_weight_grad_noalloc live in this fixed buffer, so
// the call needs no workspace and allocates nothing.  Host code cannot use the
// symbol itself as a device pointer: its device address is looked up once per
// device with cudaGetSymbolAddress (with that device current) and cached.
static __device__ __align__(256) float g_noalloc_scratch[LTHC_NOALLOC_SCRATCH_BYTES / sizeof(float)];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[lthc::kMaxDevices] = {};

static int noalloc_scratch(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= lthc::kMaxDevices) {
    cudaGetLastError();
    return fail(LTHC_ERR_DEVICE, "no current CUDA device");
  }
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      return fail(LTHC_ERR_DEVICE, "cudaGetSymbolAddress of the internal scratch buffer failed on device %d: %s", dev,
                  cudaGetErrorString(e));
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return LTHC_OK;
}

int lthc_weight_grad_noalloc(const void* high, const void* const* low, int n_layers, float* grad_w, int64_t B,
                             int64_t G, int64_t C, int act_dtype, void* stream) {
  LTHC_TRY(check_geometry(B, G, C, act_dtype));
  LTHC_TRY(check_layers(n_layers));
  LTHC_TRY(check_act(high, "high", B > 0));
  LTHC_TRY(check_ptr(grad_w, "grad_w"));
  if (!low) return fail(LTHC_ERR_NULL_POINTER, "low pointer array is NULL");
  for (int l = 0; l < n_layers; ++l) LTHC_TRY(check_act(low[l], "low[l]", B > 0));
  int sms = 0;
  LTHC_TRY(current_device(&sms));
  const size_t need = wgrad_ws_bytes(B, G, C, n_layers, sms);
  if (need > LTHC_NOALLOC_SCRATCH_BYTES)
    return fail(LTHC_ERR_WORKSPACE,
                "lthc_weight_grad_noalloc: this shape needs %zu bytes of partial sums, more than the fixed %u-byte "
                "device buffer; call lthc_weight_grad with a caller-provided workspace instead",
                need, LTHC_NOALLOC_SCRATCH_BYTES);
  void* ws = nullptr;
  if (B > 0) LTHC_TRY(noalloc_scratch(&ws));
  ReadJob j{high, nullptr, LTHC_DTYPE_F32, nullptr, low, grad_w, ws, n_layers, B, G, C};
  return read_family(j, LTHC_NOALLOC_SCRATCH_BYTES, act_dtype, static_cast<cudaStream_t>(stream));
}

size_t lthc_read_bwd_workspace_bytes(int64_t B, int64_t G, int64_t C) {
  if (B <= 0 || G <= 0 || C <= 0) return 0;
  return read_bwd_ws_bytes(B, G, C, sms_for_sizing());
}

int lthc_read_bwd(const void* x, const void* grad_z, const void* alpha, int alpha_dtype, const void* grad_x_in,
                  void* grad_x, float* grad_alpha, void* workspace, size_t workspace_bytes, int64_t B, int64_t G,
                  int64_t C, int act_dtype, void* stream) {
  LTHC_TRY(check_geometry(B, G, C, act_dtype));
  LTHC_TRY(check_weight_dtype(alpha_dtype, "alpha"));
  LTHC_TRY(check_act(grad_z, "grad_z", B > 0));
  LTHC_TRY(check_ptr(alpha, "alpha"));
  if (grad_x_in) LTHC_TRY(check_act(grad_x_in, "grad_x_in", B > 0));
  if (grad_alpha) LTHC_TRY(check_act(x, "x", B > 0));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (grad_alpha) {
    // validate the workspace before anything is enqueued
    int sms = 0;
    LTHC_TRY(current_device(&sms));
    const size_t need = grad_x ? read_bwd_ws_bytes(B, G, C, sms) : wgrad_ws_bytes(B, G, C, 1, sms);
    if (B > 0 && (!workspace || workspace_bytes < need))
      return fail(LTHC_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu bytes required", workspace_bytes,
                  need);
  }
  if (grad_x) LTHC_TRY(check_act(grad_x, "grad_x", B > 0));
  if (grad_x && grad_alpha && B > 0) {
    // both gradients: one pass reads x and grad_z once and writes grad_x
    if (!aligned16(workspace)) return fail(LTHC_ERR_ALIGNMENT, "workspace is not 16-byte aligned");
    int sms = 0;
    LTHC_TRY(current_device(&sms));
    switch (act_dtype) {
      case LTHC_DTYPE_F32:
        return read_bwd_fused_t<float>(x, grad_z, alpha, alpha_dtype, grad_x_in, grad_x, grad_alpha, workspace, B, G,
                                       C, sms, s);
      case LTHC_DTYPE_BF16:
        return read_bwd_fused_t<__nv_bfloat16>(x, grad_z, alpha, alpha_dtype, grad_x_in, grad_x, grad_alpha,
                                               workspace, B, G, C, sms, s);
      default:
        return read_bwd_fused_t<__half>(x, grad_z, alpha, alpha_dtype, grad_x_in, grad_x, grad_alpha, workspace, B,
                                        G, C, sms, s);
    }
  }
  if (grad_x) {
    if (B > 0) {
      const void* dzs[1] = {grad_z};
      const void* ws[1] = {alpha};
      LTHC_TRY(broadcast(grad_x_in, dzs, ws, alpha_dtype, 1, grad_x, B, G, C, act_dtype, s));
    }
  }
  if (grad_alpha) {
    const void* low[1] = {grad_z};
    ReadJob j{x, nullptr, LTHC_DTYPE_F32, nullptr, low, grad_alpha, workspace, 1, B, G, C};
    LTHC_TRY(read_family(j, workspace_bytes, act_dtype, s));
  }
  return LTHC_OK;
}

// ------------------------------ lazy recurrence ------------------------------

static int check_lazy(int64_t N, int64_t C, int act_dtype, int a_dtype, int b_dtype) {
  if (N < 0) return fail(LTHC_ERR_SHAPE, "rows must be >= 0, got %lld", (long long)N);
  if (C < 8 || C > 16384 || C % 8 != 0)
    return fail(LTHC_ERR_SHAPE, "channels must be a multiple of 8 in [8, 16384], got %lld", (long long)C);
  if (!valid_act(act_dtype)) return fail(LTHC_ERR_DTYPE, "unknown activation dtype code %d", act_dtype);
  LTHC_TRY(check_weight_dtype(a_dtype, "alpha"));
  LTHC_TRY(check_weight_dtype(b_dtype, "beta"));
  return LTHC_OK;
}

int lthc_lazy_update_fwd(const void* z, const void* dz, const void* alpha, int alpha_dtype, const void* beta,
                         int beta_dtype, void* z_out, int64_t N, int64_t C, int act_dtype, void* stream) {
  LTHC_TRY(check_lazy(N, C, act_dtype, alpha_dtype, beta_dtype));
  LTHC_TRY(check_act(z, "z", N > 0));
  LTHC_TRY(check_act(dz, "dz", N > 0));
  LTHC_TRY(check_ptr(alpha, "alpha"));
  LTHC_TRY(check_ptr(beta, "beta"));
  LTHC_TRY(check_act(z_out, "z_out", N > 0));
  if (N == 0) return LTHC_OK;
  int sms = 0;
  LTHC_TRY(current_device(&sms));
  LazyParams p{z, dz, alpha, beta, z_out, nullptr, alpha_dtype, beta_dtype, N, C};
  const int es = act_dtype == LTHC_DTYPE_F32 ? 4 : 2;
  dim3 grid(static_cast<unsigned>(lazy_row_blocks(N, C, sms)), static_cast<unsigned>(lazy_slices(C, es)));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (act_dtype) {
    case LTHC_DTYPE_F32: lazy_fwd_kernel<float><<<grid, 32 * kLazyWarps, 0, s>>>(p); break;
    case LTHC_DTYPE_BF16: lazy_fwd_kernel<__nv_bfloat16><<<grid, 32 * kLazyWarps, 0, s>>>(p); break;
    default: lazy_fwd_kernel<__half><<<grid, 32 * kLazyWarps, 0, s>>>(p); break;
  }
  return launched("lazy update");
}

size_t lthc_lazy_update_bwd_workspace_bytes(int64_t N, int64_t C) {
  if (N <= 0 || C <= 0) return 0;
  return lazy_ws_bytes(N, C, sms_for_sizing());
}

int lthc_lazy_update_bwd(const void* grad_z_out, const void* dz, const void* alpha, int alpha_dtype,
                         const void* beta, int beta_dtype, void* grad_dz, float* grad_alpha, float* grad_beta,
                         void* workspace, size_t workspace_bytes, int64_t N, int64_t C, int act_dtype,
                         void* stream) {
  LTHC_TRY(check_lazy(N, C, act_dtype, alpha_dtype, beta_dtype));
  LTHC_TRY(check_act(grad_z_out, "grad_z_out", N > 0));
  LTHC_TRY(check_act(dz, "dz", N > 0));
  LTHC_TRY(check_ptr(alpha, "alpha"));
  LTHC_TRY(check_ptr(beta, "beta"));
  LTHC_TRY(check_act(grad_dz, "grad_dz", N > 0));
  if (grad_alpha) LTHC_TRY(check_ptr(grad_alpha, "grad_alpha"));
  if (grad_beta) LTHC_TRY(check_ptr(grad_beta, "grad_beta"));
  int sms = 0;
  LTHC_TRY(current_device(&sms));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (N == 0) {
    if (grad_alpha && cudaMemsetAsync(grad_alpha, 0, sizeof(float) * C * kPos, s) != cudaSuccess)
      return launched("memset");
    if (grad_beta && cudaMemsetAsync(grad_beta, 0, sizeof(float) * C * kPos, s) != cudaSuccess)
      return launched("memset");
    return LTHC_OK;
  }
  const size_t need = lazy_ws_bytes(N, C, sms);
  if (!workspace || workspace_bytes < need)
    return fail(LTHC_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu bytes required", workspace_bytes,
                need);
  if (!aligned16(workspace)) return fail(LTHC_ERR_ALIGNMENT, "workspace is not 16-byte aligned");
  const int64_t nblk = lazy_row_blocks(N, C, sms);
  LazyParams p{grad_z_out, dz, alpha, beta, grad_dz, static_cast<float*>(workspace), alpha_dtype, beta_dtype, N, C};
  const int es = act_dtype == LTHC_DTYPE_F32 ? 4 : 2;
  dim3 grid(static_cast<unsigned>(nblk), static_cast<unsigned>(lazy_slices(C, es)));
  switch (act_dtype) {
    case LTHC_DTYPE_F32: lazy_bwd_kernel<float><<<grid, 32 * kLazyWarps, 0, s>>>(p); break;
    case LTHC_DTYPE_BF16: lazy_bwd_kernel<__nv_bfloat16><<<grid, 32 * kLazyWarps, 0, s>>>(p); break;
    default: lazy_bwd_kernel<__half><<<grid, 32 * kLazyWarps, 0, s>>>(p); break;
  }
  LTHC_TRY(launched("lazy update backward"));
  if (grad_alpha || grad_beta) {
    lazy_bwd_finalize_kernel<<<static_cast<unsigned>(ceil_div(C, 32)), 32 * kGammaFinalizeWarps, 0, s>>>(
        p, static_cast<int>(nblk), grad_alpha, grad_beta);
    LTHC_TRY(launched("lazy update backward finalize"));
  }
  return LTHC_OK;
}

// ------------------- branch epilogue fused with the lazy update ----------------

int lthc_branch_lazy_fwd(const void* z, const void* dz_attn, const void* mlp_out, const void* gate,
                         int64_t gate_stride, const void* alpha, int alpha_dtype, const void* beta, int beta_dtype,
                         void* dz_out, void* z_out, int64_t B, int64_t T, int64_t C, int act_dtype, void* stream) {
  LTHC_TRY(check_branch(B, T, C, gate_stride, act_dtype, alpha_dtype, beta_dtype));
  const bool ne = B > 0 && T > 0;
  LTHC_TRY(check_act(z, "z", ne));
  LTHC_TRY(check_act(dz_attn, "dz_attn", ne));
  LTHC_TRY(check_act(mlp_out, "mlp_out", ne));
  LTHC_TRY(check_act(gate, "gate", ne));
  LTHC_TRY(check_act(dz_out, "dz_out", ne));
  LTHC_TRY(check_act(z_out, "z_out", ne));
  LTHC_TRY(check_ptr(alpha, "alpha"));
  LTHC_TRY(check_ptr(beta, "beta"));
  if (!ne) return LTHC_OK;
  int sms = 0;
  LTHC_TRY(current_device(&sms));
  BranchLazyParams p;
  memset(&p, 0, sizeof(p));
  p.z = z;
  p.attn = dz_attn;
  p.mlp = mlp_out;
  p.gate = gate;
  p.a = alpha;
  p.b = beta;
  p.a_dtype = alpha_dtype;
  p.b_dtype = beta_dtype;
  p.out0 = dz_out;
  p.out1 = z_out;
  p.N = B * T;
  p.C = C;
  p.T = T;
  p.gstride = gate_stride;
  const int es = act_dtype == LTHC_DTYPE_F32 ? 4 : 2;
  const dim3 grid(static_cast<unsigned>(lazy_row_blocks(p.N, C, sms)), static_cast<unsigned>(lazy_slices(C, es)));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (act_dtype) {
    case LTHC_DTYPE_F32: branch_lazy_fwd_kernel<float><<<grid, 32 * kLazyWarps, 0, s>>>(p); break;
    case LTHC_DTYPE_BF16: branch_lazy_fwd_kernel<__nv_bfloat16><<<grid, 32 * kLazyWarps, 0, s>>>(p); break;
    default: branch_lazy_fwd_kernel<__half><<<grid, 32 * kLazyWarps, 0, s>>>(p); break;
  }
  return launched("branch epilogue + lazy update");
}

size_t lthc_branch_lazy_bwd_workspace_bytes(int64_t B, int64_t T, int64_t C) {
  if (C <= 0) return 0;
  return branch_ws_bytes(B, T, C, sms_for_sizing());
}

int lthc_branch_lazy_bwd(const void* grad_dz, const void* grad_z_out, const void* dz, const void* mlp_out,
                         const void* gate, int64_t gate_stride, const void* alpha, int alpha_dtype, const void* beta,
                         int beta_dtype, void* grad_attn, void* grad_mlp, float* grad_gate, float* grad_alpha,
                         float* grad_beta, void* workspace, size_t workspace_bytes, int64_t B, int64_t T, int64_t C,
                         int act_dtype, void* stream) {
  LTHC_TRY(check_branch(B, T, C, gate_stride, act_dtype, alpha_dtype, beta_dtype));
  const bool ne = B > 0 && T > 0;
  if (grad_dz) LTHC_TRY(check_act(grad_dz, "grad_dz", ne));
  LTHC_TRY(check_act(grad_z_out, "grad_z_out", ne));
  LTHC_TRY(check_act(dz, "dz", ne));
  LTHC_TRY(check_act(mlp_out, "mlp_out", ne));
  LTHC_TRY(check_act(gate, "gate", ne));
  LTHC_TRY(check_act(grad_attn, "grad_attn", ne));
  LTHC_TRY(check_act(grad_mlp, "grad_mlp", ne));
  LTHC_TRY(check_ptr(alpha, "alpha"));
  LTHC_TRY(check_ptr(beta, "beta"));
  if (!ne && !grad_alpha && !grad_beta && (B == 0 || !grad_gate)) return LTHC_OK;
  int sms = 0;
  LTHC_TRY(current_device(&sms));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!ne) {
    if (grad_alpha && cudaMemsetAsync(grad_alpha, 0, sizeof(float) * C * kPos, s) != cudaSuccess)
      return launched("memset");
    if (grad_beta && cudaMemsetAsync(grad_beta, 0, sizeof(float) * C * kPos, s) != cudaSuccess)
      return launched("memset");
    if (B > 0 && grad_gate && cudaMemsetAsync(grad_gate, 0, sizeof(float) * B * C, s) != cudaSuccess)
      return launched("memset");
    return LTHC_OK;
  }
  const size_t need = branch_ws_bytes(B, T, C, sms);
  if (!workspace || workspace_bytes < need)
    return fail(LTHC_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu bytes required", workspace_bytes,
                need);
  if (!aligned16(workspace)) return fail(LTHC_ERR_ALIGNMENT, "workspace is not 16-byte aligned");
  const int64_t per_image = branch_ctas_per_image(B, T, C, sms);
  BranchLazyParams p;
  memset(&p, 0, sizeof(p));
  p.mlp = mlp_out;
  p.gate = gate;
  p.a = alpha;
  p.b = beta;
  p.a_dtype = alpha_dtype;
  p.b_dtype = beta_dtype;
  p.dz = dz;
  p.g_dz = grad_dz;
  p.g_zo = grad_z_out;
  p.out0 = grad_attn;
  p.out1 = grad_mlp;
  p.partial = static_cast<float*>(workspace);
  p.N = B * T;
  p.C = C;
  p.T = T;
  p.gstride = gate_stride;
  p.rows_per_cta = ceil_div(T, per_image);
  const int es = act_dtype == LTHC_DTYPE_F32 ? 4 : 2;
  const dim3 grid(static_cast<unsigned>(B * per_image), static_cast<unsigned>(lazy_slices(C, es)));
  switch (act_dtype) {
    case LTHC_DTYPE_F32: branch_lazy_bwd_kernel<float><<<grid, 32 * kLazyWarps, 0, s>>>(p); break;
    case LTHC_DTYPE_BF16: branch_lazy_bwd_kernel<__nv_bfloat16><<<grid, 32 * kLazyWarps, 0, s>>>(p); break;
    default: branch_lazy_bwd_kernel<__half><<<grid, 32 * kLazyWarps, 0, s>>>(p); break;
  }
  LTHC_TRY(launched("branch epilogue + lazy update backward"));
  const int64_t gate_blocks = grad_gate ? std::min<int64_t>(ceil_div(B * C, 32 * kGammaFinalizeWarps),
                                                             static_cast<int64_t>(sms) * 4) : 0;
  const int64_t blocks = ceil_div(C, 32) + gate_blocks;
  branch_lazy_bwd_finalize_kernel<<<static_cast<unsigned>(blocks), 32 * kGammaFinalizeWarps, 0, s>>>(
      p, B, per_image, grad_gate, grad_alpha, grad_beta);
  return launched("branch epilogue + lazy update backward finalize");
}

// ------------------- patch embedding fused with the shared read ----------------

int lthc_patch_embed_read_fwd(const void* img, int img_dtype, const void* w1, const void* w2, const void* b2,
                              const void* alpha, void* x0, void* z, int64_t B, int in_ch, int64_t H, int64_t C,
                              void* stream) {
  if (B < 0 || B > 65535) return fail(LTHC_ERR_SHAPE, "batch must be in [0, 65535], got %lld", (long long)B);
  if (in_ch < 1 || in_ch > 4) return fail(LTHC_ERR_SHAPE, "input channels must be in [1, 4], got %d", in_ch);
  if (H < kEmbedTileCols || H % kEmbedTileCols || H > 1024)
    return fail(LTHC_ERR_SHAPE, "token grid side must be a multiple of %d in [%d, 1024], got %lld", kEmbedTileCols,
                kEmbedTileCols, (long long)H);
  if (C < kEmbedChunk || C % kEmbedChunk || C > 4096)
    return fail(LTHC_ERR_SHAPE, "embed channels must be a multiple of %d in [%d, 4096], got %lld", kEmbedChunk,
                kEmbedChunk, (long long)C);
  if (img_dtype != LTHC_DTYPE_F32 && img_dtype != LTHC_DTYPE_BF16)
    return fail(LTHC_ERR_DTYPE, "image dtype must be fp32 or bf16, got code %d", img_dtype);
  const bool nonempty = B > 0;
  LTHC_TRY(check_act(img, "img", nonempty));
  LTHC_TRY(check_act(x0, "x0", nonempty));
  LTHC_TRY(check_act(z, "z", nonempty));
  LTHC_TRY(check_ptr(w1, "w1"));
  LTHC_TRY(check_ptr(w2, "w2"));
  LTHC_TRY(check_ptr(b2, "b2"));
  LTHC_TRY(check_ptr(alpha, "alpha"));
  if (!nonempty) return LTHC_OK;
  int sms = 0;
  LTHC_TRY(current_device(&sms));
  EmbedParams p;
  memset(&p, 0, sizeof(p));
  LTHC_TRY(encode_embed_store_map(&p.tm_x0, x0, B, H, C));
  p.img = img;
  p.w1 = static_cast<const __nv_bfloat16*>(w1);
  p.w2 = static_cast<const __nv_bfloat16*>(w2);
  p.b2 = static_cast<const __nv_bfloat16*>(b2);
  p.alpha = static_cast<const __nv_bfloat16*>(alpha);
  p.z = static_cast<__nv_bfloat16*>(z);
  p.img_f32 = img_dtype == LTHC_DTYPE_F32;
  p.in_ch = in_ch;
  p.H = static_cast<int>(H);
  p.C = static_cast<int>(C);
  p.B = B;
  p.tiles = B * (H / 4) * (H / kEmbedTileCols);
  const int nchunks = static_cast<int>(C / kEmbedChunk);
  int per_sm = 0;
  LTHC_TRY(resident_ctas(patch_embed_read_kernel, kEmbedThreads, static_cast<int>(EmbedSmem::kTotal), &per_sm));
  const int64_t per_chunk = std::max<int64_t>(1, std::min<int64_t>(sms / nchunks, p.tiles));
  const unsigned grid = static_cast<unsigned>(per_chunk * nchunks);
  patch_embed_read_kernel<<<grid, kEmbedThreads, EmbedSmem::kTotal, static_cast<cudaStream_t>(stream)>>>(p);
  return launched("patch embedding + read (tensor cores)");
}

// ------------------------- final-layer prologue --------------------------------

int lthc_final_norm_modulate_fwd(const void* x, const void* norm_weight, int w_dtype, const void* shift,
                                 const void* scale, int64_t mod_stride, void* out, int64_t B, int64_t T, int64_t C,
                                 float eps, int act_dtype, void* stream) {
  LTHC_TRY(check_final(B, T, C, mod_stride, act_dtype, w_dtype, eps));
  const bool nonempty = B > 0 && T > 0;
  LTHC_TRY(check_act(x, "x", nonempty));
  LTHC_TRY(check_act(out, "out", nonempty));
  // shift / scale are [B, C]: NULL is valid for an empty batch only
  if (!norm_weight || (B > 0 && (!shift || !scale)))
    return fail(LTHC_ERR_NULL_POINTER, "norm_weight, shift and scale must be set");
  if (!nonempty) return LTHC_OK;
  int sms = 0;
  LTHC_TRY(current_device(&sms));
  FinalParams p = final_params(x, norm_weight, w_dtype, shift, scale, mod_stride, T, C, eps);
  p.out = out;
  int64_t K = 0;
  return final_dispatch<false>(p, B, sms, &K, act_dtype, static_cast<cudaStream_t>(stream));
}

size_t lthc_final_norm_modulate_bwd_workspace_bytes(int64_t B, int64_t T, int64_t C) {
  if (C <= 0) return 0;
  return final_ws_bytes(B, T, C, sms_for_sizing());
}

int lthc_final_norm_modulate_bwd(const void* x, const void* norm_weight, int w_dtype, const void* scale,
                                 int64_t mod_stride, const void* grad_out, void* grad_x, float* grad_weight,
                                 float* grad_shift, float* grad_scale, void* workspace, size_t workspace_bytes,
                                 int64_t B, int64_t T, int64_t C, float eps, int act_dtype, void* stream) {
  LTHC_TRY(check_final(B, T, C, mod_stride, act_dtype, w_dtype, eps));
  const bool nonempty = B > 0 && T > 0;
  LTHC_TRY(check_act(x, "x", nonempty));
  LTHC_TRY(check_act(grad_out, "grad_out", nonempty));
  LTHC_TRY(check_act(grad_x, "grad_x", nonempty));
  if (!norm_weight || (B > 0 && !scale)) return fail(LTHC_ERR_NULL_POINTER, "norm_weight and scale must be set");
  if (!nonempty && !grad_weight && (B == 0 || (!grad_shift && !grad_scale))) return LTHC_OK;
  int sms = 0;
  LTHC_TRY(current_device(&sms));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!nonempty) {
    if (grad_weight && cudaMemsetAsync(grad_weight, 0, sizeof(float) * C, s) != cudaSuccess) return launched("memset");
    if (B > 0 && grad_shift && cudaMemsetAsync(grad_shift, 0, sizeof(float) * B * C, s) != cudaSuccess)
      return launched("memset");
    if (B > 0 && grad_scale && cudaMemsetAsync(grad_scale, 0, sizeof(float) * B * C, s) != cudaSuccess)
      return launched("memset");
    return LTHC_OK;
  }
  const size_t need = final_ws_bytes(B, T, C, sms);
  if (!workspace || workspace_bytes < need)
    return fail(LTHC_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu bytes required", workspace_bytes,
                need);
  if (!aligned16(workspace)) return fail(LTHC_ERR_ALIGNMENT, "workspace is not 16-byte aligned");
  FinalParams p = final_params(x, norm_weight, w_dtype, nullptr, scale, mod_stride, T, C, eps);
  p.grad_out = grad_out;
  p.out = grad_x;
  p.partial = static_cast<float*>(workspace);
  int64_t K = 0;
  LTHC_TRY(final_dispatch<true>(p, B, sms, &K, act_dtype, s));
  if (grad_weight || grad_shift || grad_scale) {
    const int64_t img_blocks = (grad_shift || grad_scale)
                                   ? std::min<int64_t>(ceil_div(2 * B * C, 32 * kGammaFinalizeWarps),
                                                       static_cast<int64_t>(sms) * 4)
                                   : 0;
    const int64_t blocks = ceil_div(C, 32) + img_blocks;
    final_bwd_finalize_kernel<<<static_cast<unsigned>(blocks), 32 * kGammaFinalizeWarps, 0, s>>>(
        p.partial, grad_weight, grad_shift, grad_scale, B, K, C);
    LTHC_TRY(launched("final norm/modulate backward finalize"));
  }
  return LTHC_OK;
}

}  // extern "C"
