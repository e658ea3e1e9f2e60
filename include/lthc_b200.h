/*
 * lthc_b200.h — C ABI of the B200 (sm_100a) Local Token Hyper-Connection kernels.
 *
 * Every entry point takes plain device pointers, sizes, dtype codes and a CUDA
 * stream handle passed as `void*` (a cudaStream_t; NULL means the legacy default
 * stream).  Nothing here allocates device memory: outputs and scratch
 * ("workspace") are owned by the caller, who sizes the workspace with the
 * matching *_workspace_bytes() query.  Kernels are enqueued on `stream` and the
 * call returns without synchronising.  Inputs are never written.
 *
 * Geometry (the B/4 shape of the reference is B x 64 x 64 x C, G = 16):
 *   residual   X  : NHWC [B, 4G, 4G, C]   (a "cell" is a 4x4 block of tokens)
 *   workspace  Z  : [B, G*G, C]           (one row per cell, row-major cells)
 *   cell weights  : [C, 16]               (position r = 4*row + col inside a cell)
 *   weight grads  : float32 [L, C, 16]
 * Constraints: C % 8 == 0, 8 <= C <= 16384, G >= 1, 1 <= L <= 12, every pointer
 * 16-byte aligned, every tensor contiguous.  B == 0 is a valid empty call.
 *
 * All entry points return an lthc_status code (0 = success).  A failed call
 * enqueues nothing.  lthc_last_error_message() gives a one-line reason for the
 * most recent failure on the calling host thread.
 *
 * Reference interfaces replaced (paths are inside tongtongliang/flowmatching_lthc):
 *   flowmatching_lthc/models/local_thc.py                  (eager modules)
 *   flowmatching_lthc/models/local_thc_triton_kernels.py   (jit_thc:: Triton ops)
 * Each declaration below cites the function it stands in for.
 */
#ifndef LTHC_B200_H
#define LTHC_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LTHC_API __attribute__((visibility("default")))
#else
#define LTHC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- dtype codes (activation and weight element types) ------------------ */
#define LTHC_DTYPE_F32 0
#define LTHC_DTYPE_BF16 1
#define LTHC_DTYPE_F16 2

/* ---- status codes -------------------------------------------------------- */
#define LTHC_OK 0
#define LTHC_ERR_NULL_POINTER 1   /* a required pointer was NULL               */
#define LTHC_ERR_SHAPE 2          /* B/G/C/L outside the supported range       */
#define LTHC_ERR_DTYPE 3          /* unknown or unsupported dtype code         */
#define LTHC_ERR_ALIGNMENT 4      /* a pointer is not 16-byte aligned          */
#define LTHC_ERR_WORKSPACE 5      /* workspace missing or smaller than needed  */
#define LTHC_ERR_LAUNCH 6         /* the CUDA launch itself failed             */
#define LTHC_ERR_DEVICE 7         /* no usable sm_100 device is current        */
#define LTHC_ERR_TIMEOUT 8        /* a bounded device-side wait gave up        */

#define LTHC_MAX_LAYERS 12

/* Library version (major*10000 + minor*100 + patch). */
LTHC_API int lthc_version(void);

/* Human-readable name of a status code (static storage). */
LTHC_API const char* lthc_status_string(int status);

/* One-line description of the last failure on this host thread ("" if none). */
LTHC_API const char* lthc_last_error_message(void);

/* Reads and clears the device-side error word that kernels set when a bounded
 * wait gives up or a kernel meets an index it refuses to touch.  Synchronises
 * `stream`.  *status_out receives LTHC_OK or LTHC_ERR_TIMEOUT. */
LTHC_API int lthc_device_status(int* status_out, void* stream);

/* Diagnostic: enqueues a one-block kernel that waits on a barrier nothing will
 * complete, giving up after limit_ms milliseconds (1..5000) the same way every
 * kernel's bounded waits do: it sets the device error word (seen afterwards by
 * lthc_device_status as LTHC_ERR_TIMEOUT), writes 1 to *result_dev (a device int)
 * and returns, leaving the CUDA context usable.  No counterpart in the reference
 * (whose failure handling is host-side only, scripts/evaluate_fid.py:333-351). */
LTHC_API int lthc_selftest_wait_timeout(int limit_ms, int* result_dev, void* stream);

/* ======================= write family: workspace -> residual ============== */

/* out[b,cell,r,c] = beta[c,r] * dz[b,cell,c]
 * Replaces LayerLocalWrite.write (local_thc.py:1261-1273) and
 * jit_thc::local_read_traceable (local_thc_triton_kernels.py:2686-2696, kernel
 * _read_fwd_kernel :63-95; "read" is that file's legacy name for the write). */
LTHC_API int lthc_write_fwd(const void* dz, const void* beta, int beta_dtype, void* out,
                   int64_t B, int64_t G, int64_t C, int act_dtype, void* stream);

/* out = x + beta (.) dz broadcast over each cell; out may equal x (in place).
 * Replaces LayerLocalWrite.write_add (local_thc.py:1275-1276) and
 * jit_thc::local_read_add_traceable (local_thc_triton_kernels.py:2713-2723,
 * kernel _read_add_cell_fwd_kernel :134-164). */
LTHC_API int lthc_write_add_fwd(const void* x, const void* dz, const void* beta, int beta_dtype,
                       void* out, int64_t B, int64_t G, int64_t C, int act_dtype,
                       void* stream);

/* Fused materialisation X_L = X_0 + sum_{l<L} beta_l (.) dz_l, fp32 accumulation,
 * one rounding to the activation dtype.  dz[l] / beta[l] are arrays of L device
 * pointers (host arrays).  x0 may be NULL (then X_0 = 0).
 * Replaces SharedReadFusedFinal12LocalTHCSharedAdaLNJiT.final_accumulate_reference
 * (local_thc.py:1416-1420) -> jit_thc::final_accumulate_b4_12_traceable
 * (local_thc_triton_kernels.py:1669-1736, kernel :317-405) for L = 12, and
 * jit_thc::final_accumulate_b4_traceable (:1578-1598, kernel :202-238) for any L. */
LTHC_API int lthc_materialise_fwd(const void* x0, const void* const* dz, const void* const* beta,
                         int beta_dtype, int n_layers, void* out, int64_t B, int64_t G,
                         int64_t C, int act_dtype, void* stream);

/* Fixed-depth alias of lthc_materialise_fwd with n_layers = 12 (the released
 * jit_thc::final_accumulate_b4_12_traceable signature). */
LTHC_API int lthc_materialise12_fwd(const void* x0, const void* const* dz, const void* const* beta,
                           int beta_dtype, void* out, int64_t B, int64_t G, int64_t C,
                           int act_dtype, void* stream);

/* Backward of the materialisation (and, with L = 1, of write / write_add):
 *   grad_dz[l][b,cell,c] = sum_r beta_l[c,r] * grad_out[b,cell,r,c]
 *   grad_beta[l,c,r]     = sum_{b,cell} grad_out[b,cell,r,c] * dz_l[b,cell,c]  (fp32)
 * grad_X_0 is grad_out itself (the reference aliases it) and is not written.
 * grad_dz may be NULL (weight gradient only); grad_beta may be NULL (grad_dz only).
 * The weight gradient is reduced in a fixed order: repeated calls give identical
 * bits on the same device.
 * 16-bit activations with 2 <= n_layers, C % 16 == 0, G in {8, 16, 32} or a
 * multiple of 32, and B*G*G a multiple of 128 run on the tensor cores
 * (lthc_materialise_bwd_uses_tensor_cores): each fp32 beta enters as two 16-bit
 * parts (hi + lo, 16 / 22 significant bits for bf16 / fp16) and the position sum
 * of grad_dz is accumulated by the tensor core, so grad_dz may differ from a
 * sequential fp32 sum by one unit in the last place of the 16-bit output on a
 * small fraction of elements; every other case sums in fp32 in position order.
 * Replaces _backward_final_accumulate_12 (local_thc_triton_kernels.py:1897-1912):
 * jit_thc::final_accumulate_b4_12_grad_dz_ptr (:1800-1845, kernel :512-595) and
 * jit_thc::final_accumulate_b4_12_grad_beta_ptr (:1848-1894, kernel :598-680). */
LTHC_API size_t lthc_materialise_bwd_workspace_bytes(int64_t B, int64_t G, int64_t C, int n_layers);
LTHC_API int lthc_materialise_bwd(const void* grad_out, const void* const* dz,
                         const void* const* beta, int beta_dtype, int n_layers,
                         void* const* grad_dz, float* grad_beta, void* workspace,
                         size_t workspace_bytes, int64_t B, int64_t G, int64_t C,
                         int act_dtype, void* stream);
/* 1 if lthc_materialise_bwd runs this shape and dtype on the tensor cores, else 0. */
LTHC_API int lthc_materialise_bwd_uses_tensor_cores(int64_t B, int64_t G, int64_t C, int n_layers, int act_dtype);

/* Backward of write / write_add for one layer (grad of x_hi is grad_out itself).
 * Replaces the eager autograd of local_thc.py:1261-1276 and
 * _backward_read_add (local_thc_triton_kernels.py:2738-2744). */
LTHC_API size_t lthc_write_bwd_workspace_bytes(int64_t B, int64_t G, int64_t C);
LTHC_API int lthc_write_bwd(const void* grad_out, const void* dz, const void* beta, int beta_dtype,
                   void* grad_dz, float* grad_beta, void* workspace, size_t workspace_bytes,
                   int64_t B, int64_t G, int64_t C, int act_dtype, void* stream);

/* ======================= read family: residual -> workspace =============== */

/* z[b,cell,c] = sum_r alpha[c,r] * x[b,cell,r,c]  (fp32 accumulation)
 * Replaces SharedLocalRead.read (local_thc.py:1211-1223) and
 * jit_thc::local_write_traceable (local_thc_triton_kernels.py:2673-2683, kernel
 * _write_fwd_kernel :27-60; "write" is that file's legacy name for the read). */
LTHC_API int lthc_read_fwd(const void* x, const void* alpha, int alpha_dtype, void* z,
                  int64_t B, int64_t G, int64_t C, int act_dtype, void* stream);

/* grad_w[l,c,r] = sum_{b,cell} high[b,cell,r,c] * low[l][b,cell,c]  (fp32, fixed order)
 * Replaces jit_thc::local_weight_grad_traceable (local_thc_triton_kernels.py:
 * 2699-2710, kernel _cell_weight_grad_kernel :167-199, which uses atomics). */
LTHC_API size_t lthc_weight_grad_workspace_bytes(int64_t B, int64_t G, int64_t C, int n_layers);
LTHC_API int lthc_weight_grad(const void* high, const void* const* low, int n_layers, float* grad_w,
                     void* workspace, size_t workspace_bytes, int64_t B, int64_t G,
                     int64_t C, int act_dtype, void* stream);

/* Size of the fixed device buffer behind lthc_weight_grad_noalloc (per GPU). */
#define LTHC_NOALLOC_SCRATCH_BYTES (4u * 1024u * 1024u)

/* Same result as lthc_weight_grad, but the caller passes no workspace and the
 * library allocates nothing: the per-CTA partial sums live in a fixed
 * LTHC_NOALLOC_SCRATCH_BYTES buffer compiled into the library (every GPU that
 * loads the library holds it until the process exits).  No counterpart in the
 * reference; it exists for callers that cannot allocate device memory at the
 * call site: hosts that give an operator only its input and output buffers and
 * own all other device memory, and callers that must not call cudaMalloc on
 * that path because it can synchronise the device and stall other streams.
 * Limits and behaviour:
 *  - shapes whose partials do not fit the buffer (it grows with L, C and the
 *    SM count; at C = 768 on 148 SMs it fits L <= 3) are rejected with
 *    LTHC_ERR_WORKSPACE before anything is enqueued;
 *  - the first call on each device looks up the buffer's device address
 *    (a one-time set-up); make that first call before any stream capture;
 *  - all calls on a device share the buffer: calls that may overlap on the GPU
 *    (different streams, or threads without ordering) race and must be
 *    serialised.  Each call writes every partial it later reads, so nothing is
 *    carried over from the previous call. */
LTHC_API int lthc_weight_grad_noalloc(const void* high, const void* const* low, int n_layers, float* grad_w,
                                      int64_t B, int64_t G, int64_t C, int act_dtype, void* stream);

/* Backward of the read:
 *   grad_x = (grad_x_in +) alpha (.) grad_z broadcast over each cell
 *   grad_alpha[c,r] = sum_{b,cell} x[b,cell,r,c] * grad_z[b,cell,c]   (fp32)
 * grad_x_in may be NULL; grad_x may equal grad_x_in (accumulate in place).
 * grad_alpha may be NULL.  Replaces the eager autograd of local_thc.py:1219-1222
 * and _backward_write (local_thc_triton_kernels.py:2726-2730). */
LTHC_API size_t lthc_read_bwd_workspace_bytes(int64_t B, int64_t G, int64_t C);
LTHC_API int lthc_read_bwd(const void* x, const void* grad_z, const void* alpha, int alpha_dtype,
                  const void* grad_x_in, void* grad_x, float* grad_alpha, void* workspace,
                  size_t workspace_bytes, int64_t B, int64_t G, int64_t C, int act_dtype,
                  void* stream);

/* ======================= lazy shared-read workspace recurrence ============ */

/* z_out[n,c] = z[n,c] + gamma[c] * dz[n,c],  gamma[c] = sum_r alpha[c,r]*beta[c,r]
 * over N = B*G*G workspace rows.  z_out may equal z (in place).
 * Replaces SharedReadLocalTHCSharedAdaLNJiTBlock.lazy_workspace_update
 * (local_thc.py:1325-1328) with LayerLocalWrite.gamma_from_alpha (:1278-1283). */
LTHC_API int lthc_lazy_update_fwd(const void* z, const void* dz, const void* alpha, int alpha_dtype,
                         const void* beta, int beta_dtype, void* z_out, int64_t N, int64_t C,
                         int act_dtype, void* stream);

/* Backward of the lazy update (grad of z is grad_z_out itself):
 *   grad_dz = gamma (.) grad_z_out
 *   ggamma[c] = sum_n grad_z_out[n,c] * dz[n,c]     (fp32, fixed order)
 *   grad_alpha[c,r] = ggamma[c] * beta[c,r];  grad_beta[c,r] = ggamma[c] * alpha[c,r]
 * grad_alpha / grad_beta are fp32 [C,16].  Replaces the eager autograd of
 * local_thc.py:1278-1283, 1325-1328. */
LTHC_API size_t lthc_lazy_update_bwd_workspace_bytes(int64_t N, int64_t C);
LTHC_API int lthc_lazy_update_bwd(const void* grad_z_out, const void* dz, const void* alpha,
                         int alpha_dtype, const void* beta, int beta_dtype, void* grad_dz,
                         float* grad_alpha, float* grad_beta, void* workspace,
                         size_t workspace_bytes, int64_t N, int64_t C, int act_dtype,
                         void* stream);

/* Tensor-core self-test: D[128 x N] = A[128 x K] * B[N x K]^T with A, B row-major
 * bf16 and D fp32 on the 5th-generation tensor cores (tcgen05, TMEM), one CTA.
 * N in {64, 128, 256}; K in {64, 128, 192, 256}.  *status_dev receives 0, or 1
 * if the bounded wait for the MMA gave up.  Validates the operand descriptors
 * used by the tensor-core kernels of this library. */
LTHC_API int lthc_selftest_umma(const void* A, const void* B, float* D, int N, int K, int* status_dev,
                         void* stream);

/* Raw-descriptor tensor-core self-test: a_img / b_img (device, 16-byte aligned,
 * a_bytes / b_bytes <= 65536, multiples of 16) are copied verbatim into two
 * shared-memory regions; then `steps` (1..8) MMAs run with the given
 * shared-memory descriptors (host arrays; start addresses relative to their
 * region) and instruction descriptor (M = 128, N a multiple of 16 up to 256),
 * accumulating after the first, and D[128 x N] fp32 receives the result.
 * *status_dev receives 0, or 1 if the bounded wait gave up.  Pins the
 * no-swizzle operand layouts of the tensor-core materialisation backward. */
LTHC_API int lthc_selftest_umma_desc(const void* a_img, int a_bytes, const void* b_img, int b_bytes,
                                     const uint64_t* a_desc, const uint64_t* b_desc, int steps, uint32_t idesc,
                                     int N, float* D, int* status_dev, void* stream);

/* ======================= branch epilogue fused with the lazy update ========== */

/* dz = dz_attn + gate (.) mlp_out   (each op rounded to the activation dtype)
 * z_out = z + gamma (.) dz,  gamma[c] = sum_r alpha[c,r] * beta[c,r]
 * over B images of T workspace rows [B*T, C]; gate holds one row per image
 * (row stride gate_stride elements, e.g. a chunk of t6).  dz and z_out are
 * written; z_out may equal z.  Replaces the end of
 * WorkspaceSharedAdaLNBranch.forward (local_thc.py:318-323) followed by
 * SharedReadLocalTHCSharedAdaLNJiTBlock.lazy_workspace_update (:1325-1328). */
LTHC_API int lthc_branch_lazy_fwd(const void* z, const void* dz_attn, const void* mlp_out, const void* gate,
                         int64_t gate_stride, const void* alpha, int alpha_dtype, const void* beta,
                         int beta_dtype, void* dz_out, void* z_out, int64_t B, int64_t T, int64_t C,
                         int act_dtype, void* stream);

/* Backward: grad_dz (from the materialisation; may be NULL) and grad_z_out give
 *   g_tot = grad_dz + gamma (.) grad_z_out;  grad_attn = g_tot;
 *   grad_mlp = gate (.) g_tot;  grad_gate [B,C] = sum_rows g_tot (.) mlp_out (fp32);
 *   grad_alpha / grad_beta [C,16] from sum_rows grad_z_out (.) dz (fp32, fixed order).
 * grad_gate, grad_alpha and grad_beta may be NULL.  The grad of z is grad_z_out. */
LTHC_API size_t lthc_branch_lazy_bwd_workspace_bytes(int64_t B, int64_t T, int64_t C);
LTHC_API int lthc_branch_lazy_bwd(const void* grad_dz, const void* grad_z_out, const void* dz,
                         const void* mlp_out, const void* gate, int64_t gate_stride,
                         const void* alpha, int alpha_dtype, const void* beta, int beta_dtype,
                         void* grad_attn, void* grad_mlp, float* grad_gate, float* grad_alpha,
                         float* grad_beta, void* workspace, size_t workspace_bytes, int64_t B,
                         int64_t T, int64_t C, int act_dtype, void* stream);

/* ======================= patch embedding fused with the shared read ========= */

/* X0 = NHWC(conv1x1(conv4x4/4(img; w1); w2) + b2) and Z = read(X0; alpha) in one
 * pass on the tensor cores (tcgen05, bf16 operands, fp32 accumulation; the
 * bottleneck h1 and X0 rounded to bf16 as under bf16 autocast).
 *   img   [B, in_ch, 4H, 4H] fp32 or bf16 (img_dtype), in_ch in 1..4
 *   w1    [128, in_ch*16] bf16 (proj1 weight, flattened), w2 [C, 128] bf16,
 *   b2    [C] bf16, alpha [C, 16] bf16 (the shared read's weights)
 *   x0    [B, H, H, C] bf16 out;  z [B, (H/4)^2, C] bf16 out
 * H a multiple of 32 (64 at B/4), C a multiple of 256.  Z is computed from the
 * bf16 X0 with the arithmetic of lthc_read_fwd (equal bits).
 * Replaces BottleneckPatchEmbedNHWC.forward (local_thc.py:64-89) followed by
 * SharedLocalRead.read (:1211-1223), as called by forward_lazy (:1378-1379). */
LTHC_API int lthc_patch_embed_read_fwd(const void* img, int img_dtype, const void* w1, const void* w2,
                         const void* b2, const void* alpha, void* x0, void* z, int64_t B,
                         int in_ch, int64_t H, int64_t C, void* stream);

/* ======================= final-layer prologue on the residual =============== */

/* m[b,t,:] = modulate(RMSNorm(x[b,t,:]), shift[b,:], scale[b,:]) over the
 * materialised residual x [B, T, C] (T = tokens per image), i.e.
 *   n = (x * rsqrt(mean_c(x^2) + eps) * norm_weight)   in fp32, rounded to the activation dtype
 *   m = n * (1 + scale[b]) + shift[b]                   each op rounded to the activation dtype
 * shift / scale are rows of row stride mod_stride (elements) in the activation
 * dtype (the two halves of t2 = shared_final_modulation(c)); norm_weight is [C]
 * of w_dtype.  C is a multiple of 8, at most 1024.  Replaces the eager
 * norm_final + modulate of FinalLayerSharedAdaLN.forward (local_thc.py:865-873;
 * RMSNorm jit_shared_adaln.py:20-30; modulate local_thc.py:37-38); the final
 * Linear stays a library GEMM. */
LTHC_API int lthc_final_norm_modulate_fwd(const void* x, const void* norm_weight, int w_dtype,
                         const void* shift, const void* scale, int64_t mod_stride, void* out,
                         int64_t B, int64_t T, int64_t C, float eps, int act_dtype, void* stream);

/* Backward of lthc_final_norm_modulate_fwd given grad_out = dL/dm:
 *   grad_x [B,T,C] (activation dtype), and, each optional (NULL: not computed),
 *   grad_weight [C], grad_shift [B,C], grad_scale [B,C] as fp32 sums over tokens
 *   (fixed order, run-to-run reproducible).
 * Follows the reference autograd of the same expression op by op. */
LTHC_API size_t lthc_final_norm_modulate_bwd_workspace_bytes(int64_t B, int64_t T, int64_t C);
LTHC_API int lthc_final_norm_modulate_bwd(const void* x, const void* norm_weight, int w_dtype,
                         const void* scale, int64_t mod_stride, const void* grad_out, void* grad_x,
                         float* grad_weight, float* grad_shift, float* grad_scale, void* workspace,
                         size_t workspace_bytes, int64_t B, int64_t T, int64_t C, float eps,
                         int act_dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LTHC_B200_H */
