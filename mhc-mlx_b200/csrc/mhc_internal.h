// Host-side internals shared by the .cu files: error reporting, device
// queries and the launcher declarations that mhc_capi.cu validates and calls.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

#include "mhc_b200.h"

namespace mhc {

// Thread-local last-error text (returned by mhc_last_error()).
int set_error(int code, const char* fmt, ...);
// Checks cudaGetLastError() after a launch; returns MHC_OK or MHC_ERR_CUDA.
int check_launch(const char* what);

// Current device's SM count (cached per device).
int sm_count();
// Max dynamic shared memory per block (opt-in) of the current device.
int max_smem_optin();

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Launch-attribute caches (mhc_capi.cu): the attribute call and the
// occupancy query cost microseconds of host time, so each is made once per
// kernel, device and shape and remembered.  Thread-safe.
bool dyn_smem_cached(const void* kernel, size_t dyn);
void dyn_smem_remember(const void* kernel, size_t dyn);
int occupancy_cached(const void* kernel, int threads, size_t smem);  // -1: unknown
void occupancy_remember(const void* kernel, int threads, size_t smem, int per_sm);

// Allow `dyn` bytes of dynamic shared memory for `kernel`.  Needed whenever
// static + dynamic shared memory exceeds the 48 KB default; the attribute is
// per kernel and device, so it is set again only when a launch needs more.
template <typename K>
inline cudaError_t allow_dyn_smem(K kernel, size_t dyn) {
  if (dyn == 0) return cudaSuccess;
  const void* k = reinterpret_cast<const void*>(kernel);
  if (dyn_smem_cached(k, dyn)) return cudaSuccess;
  const cudaError_t e =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn);
  if (e == cudaSuccess) dyn_smem_remember(k, dyn);
  return e;
}

// Resident blocks per SM of `kernel` at this block size and shared memory.
template <typename K>
inline int blocks_per_sm(K kernel, int threads, size_t smem) {
  const void* k = reinterpret_cast<const void*>(kernel);
  int per_sm = occupancy_cached(k, threads, smem);
  if (per_sm >= 0) return per_sm;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess)
    return 1;  // not remembered: the query is retried on the next launch
  occupancy_remember(k, threads, smem, per_sm);
  return per_sm;
}

// Launch with programmatic stream serialisation: the kernel may start while
// the previous kernel of the stream finishes (it calls pdl_wait() before
// touching memory).  MHC_B200_PDL=0 launches without the attribute.
bool pdl_enabled();
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

inline int dtype_size(int dt) { return dt == MHC_F32 ? 4 : 2; }
inline bool dtype_ok(int dt) { return dt == MHC_F32 || dt == MHC_F16 || dt == MHC_BF16; }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Upper bound of partial rows a backward launch may use; sizes workspaces.
int max_partial_rows(int64_t T);

// ---- Sinkhorn / parameters (mhc_sinkhorn.cu) ----------------------------
// The parameter forward folded into another launch: raw parameters in, the
// activations, M, the Sinkhorn tape and (nullable, n <= 4) the transposed
// Jacobian of M out.
struct ParamsFwd {
  const float* hpre_raw;
  const float* hpost_raw;
  const float* hres_raw;
  int iters;
  float eps;
  float* hpre;
  float* hpost;
  float* M;
  float* tape;
  float* jac;
  int stage;  // set by the launcher: the block keeps the tape in dynamic shared memory
};
// The parameter backward folded into a finalize: raw parameters, the
// forward's tape / Jacobian, and the raw gradients (all null: not folded).
struct ParamsBwd {
  const float* hpre_raw;
  const float* hpost_raw;
  const float* hres_raw;
  const float* tape;
  const float* jac;
  int iters;
  float eps;
  float* dhpre_raw;
  float* dhpost_raw;
  float* dhres_raw;
  __host__ __device__ bool any() const { return dhpre_raw || dhpost_raw || dhres_raw; }
};
size_t sk_tape_floats(int n, int iters);
int launch_selftest_reciprocal(const float* x, float* y, int64_t count, cudaStream_t st);
int launch_params_fwd(const float* hpre_raw, const float* hpost_raw, const float* hres_raw,
                      int n, int iters, float eps, float* hpre, float* hpost, float* M,
                      float* tape, cudaStream_t st);
int launch_params_bwd(const float* hpre_raw, const float* hpost_raw, const float* hres_raw,
                      const float* tape, int n, int iters, float eps, const float* dhpre,
                      const float* dhpost, const float* dM, float* dhpre_raw,
                      float* dhpost_raw, float* dhres_raw, cudaStream_t st);
size_t sk_batched_ws_bytes(int64_t batch, int n, int iters);
int launch_sk_batched_fwd(const float* H, int64_t batch, int n, int iters, float eps, float* M,
                          void* ws, size_t ws_bytes, cudaStream_t st);
int launch_sk_batched_bwd(const float* H, const float* dM, int64_t batch, int n, int iters,
                          float eps, float* dH, void* ws, size_t ws_bytes, cudaStream_t st);

// ---- layer forward / backward (mhc_layer.cu) ------------------------------
int launch_fwd(const void* x, int xdt, const float* M, const float* hpre, const float* hpost,
               const float* w, void* out, int odt, int64_t T, int n, int C, float eps,
               cudaStream_t st);
size_t bwd_ws_bytes(int64_t T, int n, int C);
int launch_bwd(const void* x, int xdt, const void* dout, int ddt, const float* M,
               const float* hpre, const float* hpost, const float* w, void* dx, int dxdt,
               int64_t T, int n, int C, float eps, void* ws, size_t ws_bytes, cudaStream_t st);
int launch_finalize(const void* ws, int n, int C, float* dM, float* dhpre, float* dhpost,
                    float* dw, const float* hpre_raw, const float* hpost_raw,
                    const float* hres_raw, const float* tape, int iters, float eps,
                    float* dhpre_raw, float* dhpost_raw, float* dhres_raw, cudaStream_t st);

// ---- mix / rewire / prescale / residual (mhc_mix.cu) ------------------------
int launch_mix_add_fwd(const void* x, int xdt, const float* M, const void* y, int ydt, void* out,
                       int odt, int64_t T, int n, int C, cudaStream_t st);
size_t mix_ws_bytes(int64_t T, int n, int C);
int launch_mix_add_bwd(const void* x, int xdt, const float* M, const void* dout, int ddt,
                       void* dx, int dxdt, float* dM, int64_t T, int n, int C, void* ws,
                       size_t ws_bytes, cudaStream_t st);
int launch_rewire_fwd(const void* x, int xdt, const void* y, int ydt, const float* M,
                      const float* hpre, const float* hpost, void* out, int odt, int64_t T,
                      int n, int C, cudaStream_t st);
int launch_rewire_bwd(const void* x, int xdt, const void* y, int ydt, const void* dout, int ddt,
                      const float* M, const float* hpre, const float* hpost, void* dx, int dxdt,
                      void* dy, int dydt, float* dM, float* dhpre, float* dhpost, int64_t T,
                      int n, int C, void* ws, size_t ws_bytes, cudaStream_t st);
size_t rewire_fused_ws_bytes(int64_t T, int n, int C);
int launch_rewire_bwd_dy(const void* y, int ydt, const void* d, int ddt, const float* hpost,
                         void* dy, int dydt, int64_t T, int n, int C, void* ws, size_t ws_bytes,
                         cudaStream_t st);
int launch_rewire_bwd_dx(const void* x, int xdt, const void* d, int ddt, const void* p, int pdt,
                         const float* M, const float* hpre, const float* hpost, void* dx, int dxdt,
                         float* dM, float* dhpre, float* dhpost, const ParamsBwd& pb, int64_t T,
                         int n, int C, void* ws, size_t ws_bytes, cudaStream_t st);
int launch_prescale_fwd(const void* x, int xdt, const float* hpre, void* xo, int odt, int64_t T,
                        int n, int C, cudaStream_t st);
int launch_rewire_in_fwd(const void* x, int xdt, const ParamsFwd& pf, void* xo, int odt, int64_t T,
                         int n, int C, cudaStream_t st);
int launch_prescale_bwd(const void* x, int xdt, const void* d, int ddt, const float* hpre,
                        void* dx, int dxdt, float* dhpre, int64_t T, int n, int C, void* ws,
                        size_t ws_bytes, cudaStream_t st);
int launch_residual_add_agg(const void* x, int xdt, const void* res, int rdt, const float* hpre,
                            void* out, int odt, float* yagg, int64_t T, int n, int C,
                            cudaStream_t st);
int launch_residual_add_agg_bwd(const void* out, int odt, const void* dout, int ddt,
                                const float* dy, const float* hpre, void* dx, int dxdt,
                                float* dhpre, int64_t T, int n, int C, void* ws, size_t ws_bytes,
                                cudaStream_t st);

// ---- quantized linear (mhc_qmm.cu) ------------------------------------------
int launch_qlinear_fwd(const void* x, int xdt, const uint32_t* wq, const void* scales,
                       const void* biases, int sdt, const void* bias, void* y, int64_t M, int N,
                       int K, int group_size, int bits, cudaStream_t st);
int launch_qlinear_transpose_pack(const uint32_t* w, uint32_t* wt, int N, int K, cudaStream_t st);
int launch_qlinear_bwd_dx_t(const void* dy, int dydt, const uint32_t* wt, const void* scales_t,
                            const void* biases_t, void* dx, int64_t M, int N, int K,
                            int group_size, int bits, cudaStream_t st);
int launch_qlinear_bwd_dx(const void* dy, int dydt, const uint32_t* wq, const void* scales,
                          const void* biases, int sdt, void* dx, int64_t M, int N, int K,
                          int group_size, int bits, cudaStream_t st);

}  // namespace mhc
