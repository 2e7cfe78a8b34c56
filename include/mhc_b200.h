/*
 * mhc_b200.h -- C ABI of the B200 (sm_100a) mHC hot path.
 *
 * The reference (svdrecbd/mhc-mlx) launches its kernels through
 * mx.fast.metal_kernel(...) from mhc_mlx/metal.py; every launcher there takes
 * row-contiguous device arrays and lets MLX allocate the outputs.  This header
 * is the boundary that replaces those launchers: plain pointers and sizes, no
 * framework types.  Each entry point names the reference launcher it stands in
 * for (file:line in the reference project).
 *
 * Conventions
 *   - Every function returns 0 on success, a nonzero MHC_ERR_* code otherwise;
 *     mhc_last_error() returns a thread-local message for the last failure.
 *   - The caller owns every buffer, including workspaces; the library keeps no
 *     device allocation between calls, except the fixed scratch array that
 *     mhc_bwd_noalloc uses.  All work is enqueued on `stream`
 *     (a cudaStream_t passed as void*; NULL = legacy default stream) and no
 *     call synchronises the host.
 *   - Tensors are row-contiguous.  x / out / dx are [T, n, C] (T = tokens,
 *     n = streams, C = channels per stream) in the dtype given by the
 *     matching *_dtype argument (MHC_F32, MHC_F16, MHC_BF16).  All math is
 *     fp32.  Parameter vectors (H_*, M, rms_weight, gradients) are fp32.
 *   - 1 <= n <= 64 (reference metal.py:71 _MAX_N_ALLOWED), C >= 1, T >= 0.
 *   - Results are deterministic: cross-block reductions are two-stage with a
 *     fixed summation order, no floating-point atomics.
 */
#ifndef MHC_B200_H
#define MHC_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(MHC_BUILDING_LIB)
#define MHC_API __attribute__((visibility("default")))
#else
#define MHC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum mhc_dtype { MHC_F32 = 0, MHC_F16 = 1, MHC_BF16 = 2 };

enum mhc_status {
  MHC_OK = 0,
  MHC_ERR_INVALID = 1,     /* bad shape / dtype / pointer / size argument */
  MHC_ERR_CUDA = 2,        /* a CUDA runtime call or kernel launch failed */
  MHC_ERR_UNSUPPORTED = 3, /* valid arguments outside what this build covers */
  MHC_ERR_WORKSPACE = 4    /* workspace smaller than *_workspace_bytes() */
};

/* ---- library info ------------------------------------------------------ */
MHC_API const char* mhc_last_error(void);
MHC_API int mhc_version(void);
/* Hash of the sources and compiler flags this library was built from (no
 * counterpart in the reference): lets a loader check that the binary it
 * maps matches the source tree next to it. */
MHC_API const char* mhc_build_id(void);
/* Number of SMs of the current device (used to size workspaces). */
MHC_API int mhc_device_sm_count(int* sm_count);
/* Self-test of the reciprocal the Sinkhorn kernels use for their row and
 * column scales (a hardware approximation refined by one Newton-Raphson
 * step, instead of an IEEE division): y[i] = 1 / x[i] for count floats.  No
 * counterpart in the reference; it exists so that tests can bound the
 * reciprocal against CUDA's division (within 1 ulp). */
MHC_API int mhc_selftest_reciprocal(const float* x, float* y, int64_t count, void* stream);

/* ---- parameters: activations + Sinkhorn-Knopp (single n x n matrix) ----
 * Replaces reference.py:51-55 activate_pre_post and reference.py:58-69
 * mixing_matrix_from_logits (Metal: metal.py:1525 sinkhorn_knopp_metal).
 *   H_pre_act = sigmoid(H_pre_raw), H_post_act = 2 sigmoid(H_post_raw),
 *   M = SK(exp(H_res_raw - rowmax)), `iters` row/col normalisations; a row
 *   whose sum is <= eps keeps scale 1, a column whose sum is <= eps gets 0.
 * Any of H_pre_raw/H_post_raw (with their outputs) may be NULL to skip them.
 * tape (nullable, mhc_sinkhorn_tape_floats(n, iters) floats) records the
 * forward for mhc_params_bwd. */
MHC_API size_t mhc_sinkhorn_tape_floats(int n, int iters);
MHC_API int mhc_params_fwd(const float* H_pre_raw, const float* H_post_raw,
                   const float* H_res_raw, int n, int iters, float eps,
                   float* H_pre_act, float* H_post_act, float* M,
                   float* tape, void* stream);

/* Backward of mhc_params_fwd: dH_res_raw from dM through the Sinkhorn
 * iterations (reference metal.py:1978 sinkhorn_knopp_backward_metal), and the
 * sigmoid chains for H_pre/H_post (reference.py:51-55 under autodiff).
 * tape must hold the record written by mhc_params_fwd for the same H_res_raw,
 * n, iters, eps.  Pass NULL for a pre/post pair to skip it. */
MHC_API int mhc_params_bwd(const float* H_pre_raw, const float* H_post_raw,
                   const float* H_res_raw, const float* tape, int n, int iters,
                   float eps, const float* dH_pre_act, const float* dH_post_act,
                   const float* dM, float* dH_pre_raw, float* dH_post_raw,
                   float* dH_res_raw, void* stream);

/* ---- batched Sinkhorn-Knopp: [batch, n, n] independent matrices --------
 * New surface (the reference accepts one 2-D matrix, reference.py:64-65);
 * per matrix identical to mhc_params_fwd's M.  The backward replays the
 * forward itself (like reference sinkhorn_knopp_backward.metal) and needs a
 * workspace of mhc_sinkhorn_batched_workspace_bytes() bytes (0 for the
 * register/shared-memory path used when n divides 32). */
MHC_API size_t mhc_sinkhorn_batched_workspace_bytes(int64_t batch, int n, int iters);
MHC_API int mhc_sinkhorn_batched_fwd(const float* H_res_raw, int64_t batch, int n,
                             int iters, float eps, float* M, void* stream);
MHC_API int mhc_sinkhorn_batched_bwd(const float* H_res_raw, const float* dM,
                             int64_t batch, int n, int iters, float eps,
                             float* dH_res_raw, void* workspace,
                             size_t workspace_bytes, void* stream);

/* ---- fused layer forward: aggregate + RMSNorm + mix + residual add ------
 * Replaces metal.py:1823 mhc_forward_fused_metal (its 1-kernel and 3-kernel
 * strategies, kernels mhc_fused / mhc_forward_agg / mhc_forward_rms_reduce /
 * stream_mix_add_rms_col[_bf16]); math of reference.py:148-161:
 *   y[t,c]   = sum_i H_pre_act[i] x[t,i,c]
 *   inv[t]   = 1 / sqrt(mean_c y^2 + eps)
 *   out[t,i,c] = sum_j M[i,j] x[t,j,c] + H_post_act[i] * (y*inv[t]) * w[c]
 * One read of x and one write of out per call.  out_dtype is MHC_F32, or
 * equal to x_dtype for half outputs (metal.py:1610-1616). */
MHC_API int mhc_fwd(const void* x, int x_dtype, const float* M, const float* H_pre_act,
            const float* H_post_act, const float* rms_weight, void* out,
            int out_dtype, int64_t T, int n, int C, float eps, void* stream);

/* ---- fused layer backward --------------------------------------------------
 * Replaces the VJP at metal.py:2787-2857 (prep_tile, rms_reduce, dx_col, dM,
 * dH_pre, dH_post, d_rms_weight kernels).  One pass over x and d_out writes
 * dx (in dx_dtype, normally x's dtype) and per-block partial sums of
 * dM, dH_pre_act, dH_post_act and d_rms_weight into `workspace`;
 * mhc_bwd_finalize reduces them in a fixed order.  The workspace must stay
 * untouched between the two calls. */
MHC_API size_t mhc_bwd_workspace_bytes(int64_t T, int n, int C);
MHC_API int mhc_bwd(const void* x, int x_dtype, const void* d_out, int dout_dtype,
            const float* M, const float* H_pre_act, const float* H_post_act,
            const float* rms_weight, void* dx, int dx_dtype, int64_t T, int n,
            int C, float eps, void* workspace, size_t workspace_bytes,
            void* stream);

/* Reduce the partials of mhc_bwd into dM[n*n], dH_pre_act[n], dH_post_act[n],
 * d_rms_weight[C].  If H_res_raw and tape are non-NULL it also runs the
 * parameter chain of mhc_params_bwd in the same launch and writes
 * dH_pre_raw/dH_post_raw/dH_res_raw (any of the *_act/dM outputs may then be
 * NULL). */
MHC_API int mhc_bwd_finalize(const void* workspace, int n, int C, float* dM,
                     float* dH_pre_act, float* dH_post_act, float* d_rms_weight,
                     const float* H_pre_raw, const float* H_post_raw,
                     const float* H_res_raw, const float* tape, int iters,
                     float eps, float* dH_pre_raw, float* dH_post_raw,
                     float* dH_res_raw, void* stream);

/* ---- fused layer backward without caller-provided memory ------------------
 * No counterpart in the reference.  Same result as mhc_bwd followed by
 * mhc_bwd_finalize (activated-parameter gradients), for callers that cannot
 * allocate device memory: a plugin boundary that hands a kernel only its
 * inputs and outputs (as the reference's mx.fast.metal_kernel boundary
 * does), or a runtime whose allocator may not be called on this path.
 * The per-block partial sums live in one file-scope device array of
 * MHC_NOALLOC_SCRATCH_BYTES that every GPU loading the library keeps until
 * process exit; the call allocates nothing.  It fails with MHC_ERR_WORKSPACE
 * when mhc_bwd_workspace_bytes(T, n, C) exceeds that size.  That size is a
 * 256-byte header, then G * (n*n + 2n) * 4 bytes rounded up to a multiple of
 * 256, then G * C * 4 bytes, with G = min(4 * SMs, 8 * T) partial rows: on a
 * 148-SM B200, n = 4 fits any T up to C = 7,060.  The first call on a device
 * looks up the array's device address (once per device): make it before any
 * stream capture.  A first call whose lookup failed returns MHC_ERR_CUDA and
 * may be retried.  All calls share the array, so calls that overlap on the
 * GPU (different streams, or several host threads) race: serialise them. */
#define MHC_NOALLOC_SCRATCH_BYTES ((size_t)16 << 20)
MHC_API int mhc_bwd_noalloc(const void* x, int x_dtype, const void* d_out, int dout_dtype,
                            const float* M, const float* H_pre_act, const float* H_post_act,
                            const float* rms_weight, void* dx, int dx_dtype, float* dM,
                            float* dH_pre_act, float* dH_post_act, float* d_rms_weight,
                            int64_t T, int n, int C, float eps, void* stream);

/* ---- stream mix + add (MHCRewire post-combine) ---------------------------
 * Replaces metal.py:954 stream_mix_add_metal (kernel stream_mix_add.metal):
 *   out[t,i,c] = sum_j M[i,j] x[t,j,c] + y_dist[t,i,c]
 * and its VJP metal.py:2661-2690 (stream_mix_backward_dx + mhc_backward_dM):
 *   dx = M^T d_out, dM = sum d_out x^T (d_y_dist = d_out, not computed). */
MHC_API int mhc_mix_add_fwd(const void* x, int x_dtype, const float* M,
                    const void* y_dist, int y_dtype, void* out, int out_dtype,
                    int64_t T, int n, int C, void* stream);
MHC_API size_t mhc_mix_bwd_workspace_bytes(int64_t T, int n, int C);
MHC_API int mhc_mix_add_bwd(const void* x, int x_dtype, const float* M,
                    const void* d_out, int dout_dtype, void* dx, int dx_dtype,
                    float* dM, int64_t T, int n, int C, void* workspace,
                    size_t workspace_bytes, void* stream);

/* ---- fused MHCRewire post-combine -----------------------------------------
 * layer.py:302-337 post_combine with the H_pre/H_post folding done in-kernel:
 *   out[t,i,c] = H_post_act[i] * (y_inner[t,i,c] + sum_j M[i,j] H_pre_act[j] x[t,j,c])
 * Backward writes dx (mix branch only), dy_inner, and reduces
 * dM, dH_pre_act, dH_post_act (fp32) with a fixed order. */
MHC_API int mhc_rewire_combine_fwd(const void* x, int x_dtype, const void* y_inner,
                           int y_dtype, const float* M, const float* H_pre_act,
                           const float* H_post_act, void* out, int out_dtype,
                           int64_t T, int n, int C, void* stream);
MHC_API size_t mhc_rewire_bwd_workspace_bytes(int64_t T, int n, int C);
MHC_API int mhc_rewire_combine_bwd(const void* x, int x_dtype, const void* y_inner,
                           int y_dtype, const void* d_out, int dout_dtype,
                           const float* M, const float* H_pre_act,
                           const float* H_post_act, void* dx, int dx_dtype,
                           void* dy_inner, int dy_dtype, float* dM,
                           float* dH_pre_act, float* dH_post_act, int64_t T,
                           int n, int C, void* workspace,
                           size_t workspace_bytes, void* stream);

/* ---- MHCRewire backward end to end -----------------------------------------
 * The reference differentiates MHCRewire.__call__ (layer.py:469-492) as two
 * separate pieces: the pre-scale x * H_pre (layer.py:478-480) and the
 * post-combine (layer.py:312-337, VJP metal.py:2661-2709), each producing a
 * dx and a dH_pre contribution that MLX then adds.  These two calls bracket
 * the inner module's backward instead, so dx is written once and dH_pre is
 * one reduction:
 *   mhc_rewire_bwd_dy (before the inner backward):
 *     dy_inner[t,i,c] = H_post_act[i] * d_out[t,i,c], and partial sums of
 *     R_i = sum d_out_i * y_inner_i into `workspace`;
 *   mhc_rewire_bwd_dx (after it, with d_xpre = the inner module's input
 *   gradient, NULL for zero):
 *     dx[t,j,c] = H_pre_act[j] * (sum_i M[i,j] H_post_act[i] d_out[t,i,c] + d_xpre[t,j,c])
 *     dM[i,j]   = H_post_act[i] H_pre_act[j] Q[i,j],   Q = sum d_out x^T
 *     dH_pre_act[j]  = sum_i H_post_act[i] M[i,j] Q[i,j] + sum d_xpre_j x_j
 *     dH_post_act[i] = R_i + sum_j M[i,j] H_pre_act[j] Q[i,j]
 *   (fixed summation order; dx may be NULL when only the parameter gradients
 *   are wanted).  Both calls take the same workspace of
 *   mhc_rewire_fused_bwd_workspace_bytes(), untouched in between.  d_out and
 *   d_xpre are fp32 or x's dtype; dy_inner has y_inner's dtype. */
MHC_API size_t mhc_rewire_fused_bwd_workspace_bytes(int64_t T, int n, int C);
MHC_API int mhc_rewire_bwd_dy(const void* y_inner, int y_dtype, const void* d_out,
                              int dout_dtype, const float* H_post_act, void* dy_inner,
                              int dy_dtype, int64_t T, int n, int C, void* workspace,
                              size_t workspace_bytes, void* stream);
MHC_API int mhc_rewire_bwd_dx(const void* x, int x_dtype, const void* d_out, int dout_dtype,
                              const void* d_xpre, int dxpre_dtype, const float* M,
                              const float* H_pre_act, const float* H_post_act, void* dx,
                              int dx_dtype, float* dM, float* dH_pre_act, float* dH_post_act,
                              const float* H_pre_raw, const float* H_post_raw,
                              const float* H_res_raw, const float* tape,
                              const float* jacobian, int iters, float eps, float* dH_pre_raw,
                              float* dH_post_raw, float* dH_res_raw, int64_t T, int n, int C,
                              void* workspace, size_t workspace_bytes, void* stream);
/* The raw-parameter arguments of mhc_rewire_bwd_dx carry the chain rule on
 * to H_pre_raw / H_post_raw / H_res_raw (what mhc_params_bwd does with the
 * activation gradients) in the same finalize launch: pass the raw parameters,
 * the tape of mhc_rewire_in_fwd or mhc_params_fwd, the forward's iters and
 * eps, and three outputs; all NULL to stop at the activation gradients.
 * jacobian (nullable, n <= 4): the one mhc_rewire_in_fwd wrote, turning the
 * Sinkhorn backward into n^2 dot products. */

/* ---- MHCRewire input side ----------------------------------------------------
 * layer.py:474-480 (MHCRewire.__call__: the wrapped MHCLayer's activations,
 * then x * H_pre_act) in one call:
 *   H_pre_act, H_post_act, M and the tape exactly as mhc_params_fwd;
 *   x_pre[t,i,c] = x[t,i,c] * H_pre_act[i]  (as mhc_prescale_fwd).
 * For n in {1, 2, 4, 8} this is one launch: one block runs the parameter chain
 * while the others pre-scale.  Otherwise the parameter kernel, then the
 * pre-scale.  jacobian (nullable; n in {1, 2, 4} only,
 * mhc_rewire_jacobian_floats(n) floats) receives the transposed Jacobian
 * dM/dH_res_raw for mhc_rewire_bwd_dx; tape is required when iters > 0. */
MHC_API size_t mhc_rewire_jacobian_floats(int n);
MHC_API int mhc_rewire_in_fwd(const void* x, int x_dtype, const float* H_pre_raw,
                              const float* H_post_raw, const float* H_res_raw, int iters,
                              float eps, float* H_pre_act, float* H_post_act, float* M,
                              float* tape, float* jacobian, void* x_pre, int out_dtype,
                              int64_t T, int n, int C, void* stream);

/* ---- stream pre-scale (MHCRewire input side) ------------------------------
 * layer.py:478-480: x_pre[t,i,c] = x[t,i,c] * H_pre_act[i].  Backward:
 * dx = H_pre_act[i] * d_xpre, dH_pre_act[i] = sum d_xpre * x (fixed order). */
MHC_API int mhc_prescale_fwd(const void* x, int x_dtype, const float* H_pre_act,
                     void* x_pre, int out_dtype, int64_t T, int n, int C,
                     void* stream);
MHC_API int mhc_prescale_bwd(const void* x, int x_dtype, const void* d_xpre,
                     int d_dtype, const float* H_pre_act, void* dx,
                     int dx_dtype, float* dH_pre_act, int64_t T, int n, int C,
                     void* workspace, size_t workspace_bytes, void* stream);

/* ---- residual add + aggregate ----------------------------------------------
 * Replaces metal.py:1673 residual_add_agg_metal (kernel residual_add_agg.metal,
 * utils.py:4-24):  out = x + res;  y_agg[t,c] = sum_i H_pre[i] out[t,i,c]. */
MHC_API int mhc_residual_add_agg(const void* x, int x_dtype, const void* res,
                         int res_dtype, const float* H_pre, void* out,
                         int out_dtype, float* y_agg, int64_t T, int n, int C,
                         void* stream);

/* Backward of mhc_residual_add_agg (the reference registers no VJP for it):
 *   dx = dres = d_out + H_pre[i] * d_y,   dH_pre[i] = sum d_y * out_i
 * out is the forward's output (dtype out_dtype); d_out (same dtype as out)
 * and d_y ([T, C] fp32) may each be NULL (treated as zero).  dx is written in
 * dx_dtype; dH_pre is reduced in a fixed order.  Workspace:
 * mhc_mix_bwd_workspace_bytes(T, n, C). */
MHC_API int mhc_residual_add_agg_bwd(const void* out, int out_dtype, const void* d_out,
                                     int dout_dtype, const float* d_y, const float* H_pre,
                                     void* dx, int dx_dtype, float* dH_pre, int64_t T, int n,
                                     int C, void* workspace, size_t workspace_bytes,
                                     void* stream);

/* ---- quantized linear layer (the module MHCRewire wraps) -------------------
 * The 4-bit affine group-wise QuantizedLinear that the reference wraps
 * (tests/test_quantized.py:15 QuantizedLinear.from_linear(..., group_size=64,
 * bits=4), examples/patch_llama_mock.py:90, patching.py:74-80), with the
 * weight dequantised tile by tile inside a tensor-core GEMM (the [out, in]
 * weight is never written to memory):
 *   W[n, k] = scales[n, k/64] * q[n, k] + biases[n, k/64],  q in [0, 15]
 * w_packed is [N][K/8] 32-bit words, code k%8 of row n in bits [4(k%8), 4(k%8)+4)
 * of word k/8; scales / biases are [N][K/64] in scales_dtype (MHC_BF16 or
 * MHC_F16).  Each weight is q * scale + bias, one fused multiply-add in the
 * activations' dtype (the tensor-core operand type; scale and bias are
 * rounded to it first when stored in the other 16-bit type).
 *   mhc_qlinear_fwd:    y[M, N]  = x[M, K] W^T (+ bias[N], x's dtype, may be NULL)
 *   mhc_qlinear_bwd_dx: dx[M, K] = dy[M, N] W
 * x / dy / y / dx are row-contiguous bf16 or fp16 (one dtype per call);
 * fp32 accumulation.  Covered: bits = 4, group_size = 64, N and K multiples
 * of 128, 16-byte aligned x / dy, w_packed and outputs (MHC_ERR_UNSUPPORTED
 * or MHC_ERR_INVALID otherwise). */
MHC_API int mhc_qlinear_fwd(const void* x, int x_dtype, const uint32_t* w_packed,
                            const void* scales, const void* biases, int scales_dtype,
                            const void* bias, void* y, int64_t M, int N, int K,
                            int group_size, int bits, void* stream);
MHC_API int mhc_qlinear_bwd_dx(const void* dy, int dy_dtype, const uint32_t* w_packed,
                               const void* scales, const void* biases, int scales_dtype,
                               void* dx, int64_t M, int N, int K, int group_size, int bits,
                               void* stream);

/* The same input gradient from the transposed layouts of the frozen weight
 * (no counterpart in the reference: a derived, cacheable copy for the
 * backward), which let the dequantised rows of W^T live in tensor memory:
 *   wt_packed  [K][N/8] 32-bit words, code n%8 of row k in bits
 *              [4(n%8), 4(n%8)+4) of word n/8 (the codes of W^T);
 *   scales_t, biases_t  [K/64][N] in dy's dtype (scales[n][g] at [g][n]).
 * Same coverage as mhc_qlinear_bwd_dx; scales_t / biases_t 16-byte aligned. */
/* Builds wt_packed ([K][N/8]) from w_packed ([N][K/8]) on the device: the
 * one-time layout step of mhc_qlinear_bwd_dx_t (no counterpart in the
 * reference).  N and K multiples of 8. */
MHC_API int mhc_qlinear_transpose_pack(const uint32_t* w_packed, uint32_t* wt_packed, int N,
                                       int K, void* stream);
MHC_API int mhc_qlinear_bwd_dx_t(const void* dy, int dy_dtype, const uint32_t* wt_packed,
                                 const void* scales_t, const void* biases_t, void* dx,
                                 int64_t M, int N, int K, int group_size, int bits,
                                 void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MHC_B200_H */
