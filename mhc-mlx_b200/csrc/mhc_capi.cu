// extern "C" boundary of libmhc_b200.so: argument validation, error codes
// and the thread-local error text, then a call into the launchers.  The
// checks mirror the ValueError conditions of the reference launchers in
// mhc_mlx/metal.py (n in [1, 64] via _validate_n metal.py:826-833, shape and
// dtype agreement, output dtype fp32 or matching a half input
// metal.py:1610-1616).
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

#include "mhc_internal.h"
#include "mhc_sinkhorn.cuh"

namespace mhc {

static thread_local char g_err[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(MHC_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return MHC_OK;
}

static constexpr int kMaxDevices = 64;
static int g_sm[kMaxDevices];
static int g_smem[kMaxDevices];
static std::once_flag g_once[kMaxDevices];

static int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kMaxDevices) d = 0;
  return d;
}

static void query(int d) {
  int v = 0;
  g_sm[d] = (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d) == cudaSuccess && v > 0) ? v : 148;
  v = 0;
  g_smem[d] = (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, d) == cudaSuccess && v > 0) ? v : 48 * 1024;
}

int sm_count() {
  const int d = current_device();
  std::call_once(g_once[d], query, d);
  return g_sm[d];
}

int max_smem_optin() {
  const int d = current_device();
  std::call_once(g_once[d], query, d);
  return g_smem[d];
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("MHC_B200_PDL");
    return !(v && *v == '0');
  }();
  return on;
}

// Launch-attribute caches keyed on (kernel, device[, block, shared bytes]).
namespace {
std::mutex g_attr_mu;
std::map<std::pair<const void*, int>, size_t> g_dyn;  // largest dynamic smem allowed so far
std::map<std::tuple<const void*, int, int, size_t>, int> g_occ;  // resident blocks per SM
}  // namespace

bool dyn_smem_cached(const void* kernel, size_t dyn) {
  std::lock_guard<std::mutex> lk(g_attr_mu);
  auto it = g_dyn.find({kernel, current_device()});
  return it != g_dyn.end() && it->second >= dyn;
}

void dyn_smem_remember(const void* kernel, size_t dyn) {
  std::lock_guard<std::mutex> lk(g_attr_mu);
  size_t& v = g_dyn[{kernel, current_device()}];
  if (dyn > v) v = dyn;
}

int occupancy_cached(const void* kernel, int threads, size_t smem) {
  std::lock_guard<std::mutex> lk(g_attr_mu);
  auto it = g_occ.find({kernel, current_device(), threads, smem});
  return it == g_occ.end() ? -1 : it->second;
}

void occupancy_remember(const void* kernel, int threads, size_t smem, int per_sm) {
  std::lock_guard<std::mutex> lk(g_attr_mu);
  g_occ[{kernel, current_device(), threads, smem}] = per_sm;
}

}  // namespace mhc

using namespace mhc;

#define MHC_TRY_BEGIN try {
#define MHC_TRY_END                                                        \
  }                                                                        \
  catch (...) {                                                            \
    return set_error(MHC_ERR_CUDA, "%s: unexpected C++ exception", __func__); \
  }

static int check_common(const char* fn, int64_t T, int n, int C) {
  if (n < 1 || n > 64) return set_error(MHC_ERR_INVALID, "%s: n=%d must be in [1, 64]", fn, n);
  if (C < 1) return set_error(MHC_ERR_INVALID, "%s: C=%d must be positive", fn, C);
  if (T < 0) return set_error(MHC_ERR_INVALID, "%s: T=%lld must be >= 0", fn, (long long)T);
  return MHC_OK;
}

static int check_dtype(const char* fn, const char* what, int dt) {
  if (!dtype_ok(dt)) return set_error(MHC_ERR_INVALID, "%s: %s dtype %d is not one of MHC_F32/F16/BF16", fn, what, dt);
  return MHC_OK;
}

#define MHC_REQ(cond, ...) \
  do { if (!(cond)) return set_error(MHC_ERR_INVALID, __VA_ARGS__); } while (0)
#define MHC_CHK(expr) \
  do { const int _r = (expr); if (_r != MHC_OK) return _r; } while (0)

extern "C" {

const char* mhc_last_error(void) { return g_err; }

int mhc_version(void) { return 10000; }  // 1.0.0

#ifndef MHC_BUILD_ID
#define MHC_BUILD_ID "unknown"
#endif
const char* mhc_build_id(void) { return MHC_BUILD_ID; }

int mhc_device_sm_count(int* out) {
  MHC_REQ(out, "mhc_device_sm_count: NULL output");
  *out = sm_count();
  return MHC_OK;
}

int mhc_selftest_reciprocal(const float* x, float* y, int64_t count, void* stream) {
  MHC_TRY_BEGIN
  MHC_REQ(count >= 0, "mhc_selftest_reciprocal: count must be >= 0");
  MHC_REQ(count == 0 || (x && y), "mhc_selftest_reciprocal: NULL pointer");
  if (count == 0) return MHC_OK;
  return launch_selftest_reciprocal(x, y, count, as_stream(stream));
  MHC_TRY_END
}

size_t mhc_sinkhorn_tape_floats(int n, int iters) {
  if (n < 1 || n > 64 || iters < 0) return 0;
  return sk_tape_floats(n, iters);
}

int mhc_params_fwd(const float* H_pre_raw, const float* H_post_raw, const float* H_res_raw, int n,
                   int iters, float eps, float* H_pre_act, float* H_post_act, float* M,
                   float* tape, void* stream) {
  MHC_TRY_BEGIN
  MHC_CHK(check_common(__func__, 1, n, 1));
  MHC_REQ(iters >= 0, "%s: iters=%d must be >= 0", __func__, iters);
  MHC_REQ(!H_pre_raw == !H_pre_act, "%s: H_pre_raw and H_pre_act must both be given or both NULL", __func__);
  MHC_REQ(!H_post_raw == !H_post_act, "%s: H_post_raw and H_post_act must both be given or both NULL", __func__);
  MHC_REQ(!H_res_raw || M, "%s: M is NULL", __func__);
  return launch_params_fwd(H_pre_raw, H_post_raw, H_res_raw, n, iters, eps, H_pre_act, H_post_act,
                           M, H_res_raw ? tape : nullptr, as_stream(stream));
  MHC_TRY_END
}

int mhc_params_bwd(const float* H_pre_raw, const float* H_post_raw, const float* H_res_raw,
                   const float* tape, int n, int iters, float eps, const float* dH_pre_act,
                   const float* dH_post_act, const float* dM, float* dH_pre_raw,
                   float* dH_post_raw, float* dH_res_raw, void* stream) {
  MHC_TRY_BEGIN
  MHC_CHK(check_common(__func__, 1, n, 1));
  MHC_REQ(iters >= 0, "%s: iters=%d must be >= 0", __func__, iters);
  MHC_REQ(!(H_pre_raw && dH_pre_act) || dH_pre_raw, "%s: dH_pre_raw is NULL", __func__);
  MHC_REQ(!(H_post_raw && dH_post_act) || dH_post_raw, "%s: dH_post_raw is NULL", __func__);
  if (H_res_raw && dM) {
    MHC_REQ(dH_res_raw, "%s: dH_res_raw is NULL", __func__);
    MHC_REQ(tape || iters == 0, "%s: tape is NULL (record it with mhc_params_fwd)", __func__);
  }
  return launch_params_bwd(H_pre_raw, H_post_raw, H_res_raw, tape, n, iters, eps, dH_pre_act,
                           dH_post_act, dM, dH_pre_raw, dH_post_raw, dH_res_raw,
                           as_stream(stream));
  MHC_TRY_END
}

size_t mhc_sinkhorn_batched_workspace_bytes(int64_t batch, int n, int iters) {
  if (n < 1 || n > 64 || iters < 0 || batch < 0) return 0;
  return sk_batched_ws_bytes(batch, n, iters);
}

int mhc_sinkhorn_batched_fwd(const float* H_res_raw, int64_t batch, int n, int iters, float eps,
                             float* M, void* stream) {
  MHC_TRY_BEGIN
  MHC_CHK(check_common(__func__, batch, n, 1));
  MHC_REQ(iters >= 0, "%s: iters=%d must be >= 0", __func__, iters);
  MHC_REQ(batch == 0 || (H_res_raw && M), "%s: NULL pointer", __func__);
  MHC_REQ(batch * n <= (int64_t)INT32_MAX * 64, "%s: batch too large", __func__);
  return launch_sk_batched_fwd(H_res_raw, batch, n, iters, eps, M, nullptr, 0, as_stream(stream));
  MHC_TRY_END
}

int mhc_sinkhorn_batched_bwd(const float* H_res_raw, const float* dM, int64_t batch, int n,
                             int iters, float eps, float* dH_res_raw, void* workspace,
                             size_t workspace_bytes, void* stream) {
  MHC_TRY_BEGIN
  MHC_CHK(check_common(__func__, batch, n, 1));
  MHC_REQ(iters >= 0, "%s: iters=%d must be >= 0", __func__, iters);
  MHC_REQ(batch == 0 || (H_res_raw && dM && dH_res_raw), "%s: NULL pointer", __func__);
  return launch_sk_batched_bwd(H_res_raw, dM, batch, n, iters, eps, dH_res_raw, workspace,
                               workspace_bytes, as_stream(stream));
  MHC_TRY_END
}

int mhc_fwd(const void* x, int x_dtype, const float* M, const float* H_pre_act,
            const float* H_post_act, const float* rms_weight, void* out, int out_dtype, int64_t T,
            int n, int C, float eps, void* stream) {
  MHC_TRY_BEGIN
  MHC_CHK(check_common(__func__, T, n, C));
  MHC_CHK(check_dtype(__func__, "x", x_dtype));
  MHC_CHK(check_dtype(__func__, "out", out_dtype));
  MHC_REQ(out_dtype == MHC_F32 || out_dtype == x_dtype,
          "%s: out dtype must be fp32 or equal to x's dtype", __func__);
  MHC_REQ(M && H_pre_act && H_post_act && rms_weight, "%s: NULL parameter pointer", __func__);
  MHC_REQ(T == 0 || (x && out), "%s: NULL x/out", __func__);
  return launch_fwd(x, x_dtype, M, H_pre_act, H_post_act, rms_weight, out, out_dtype, T, n, C, eps,
                    as_stream(stream));
  MHC_TRY_END
}

size_t mhc_bwd_workspace_bytes(int64_t T, int n, int C) {
  if (n < 1 || n > 64 || C < 1 || T < 0) return 0;
  return bwd_ws_bytes(T, n, C);
}

int mhc_bwd(const void* x, int x_dtype, const void* d_out, int dout_dtype, const float* M,
            const float* H_pre_act, const float* H_post_act, const float* rms_weight, void* dx,
            int dx_dtype, int64_t T, int n, int C, float eps, void* workspace,
            size_t workspace_bytes, void* stream) {
  MHC_TRY_BEGIN
  MHC_CHK(check_common(__func__, T, n, C));
  MHC_CHK(check_dtype(__func__, "x", x_dtype));
  MHC_CHK(check_dtype(__func__, "d_out", dout_dtype));
  MHC_CHK(check_dtype(__func__, "dx", dx_dtype));
  MHC_REQ(M && H_pre_act && H_post_act && rms_weight, "%s: NULL parameter pointer", __func__);
  MHC_REQ(T == 0 || (x && d_out && dx), "%s: NULL x/d_out/dx", __func__);
  return launch_bwd(x, x_dtype, d_out, dout_dtype, M, H_pre_act, H_post_act, rms_weight, dx,
                    dx_dtype, T, n, C, eps, workspace, workspace_bytes, as_stream(stream));
  MHC_TRY_END
}

int mhc_bwd_finalize(const void* workspace, int n, int C, float* dM, float* dH_pre_act,
                     float* dH_post_act, float* d_rms_weight, const float* H_pre_raw,
                     const float* H_post_raw, const float* H_res_raw, const float* tape,
                     int iters, float eps, float* dH_pre_raw, float* dH_post_raw,
                     float* dH_res_raw, void* stream) {
  MHC_TRY_BEGIN
  MHC_CHK(check_common(__func__, 0, n, C));
  MHC_REQ(workspace, "%s: NULL workspace", __func__);
  MHC_REQ(iters >= 0, "%s: iters=%d must be >= 0", __func__, iters);
  if (H_res_raw && dH_res_raw)
    MHC_REQ(tape || iters == 0, "%s: tape is NULL (record it with mhc_params_fwd)", __func__);
  return launch_finalize(workspace, n, C, dM, dH_pre_act, dH_post_act, d_rms_weight, H_pre_raw,
                         H_post_raw, H_res_raw, tape, iters, eps, dH_pre_raw, dH_post_raw,
                         dH_res_raw, as_stream(stream));
  MHC_TRY_END
}

int mhc_mix_add_fwd(const void* x, int x_dtype, const float* M, const void* y_dist, int y_dtype,
                    void* out, int out_dtype, int64_t T, int n, int C, void* stream) {
  MHC_TRY_BEGIN
  MHC_CHK(check_common(__func__, T, n, C));
  MHC_CHK(check_dtype(__func__, "x", x_dtype));
  MHC_CHK(check_dtype(__func__, "y_dist", y_dtype));
  MHC_CHK(check_dtype(__func__, "out", out_dtype));
  MHC_REQ(M, "%s: NULL M", __func__);
  MHC_REQ(T == 0 || (x && y_dist && out), "%s: NULL tensor pointer", __func__);
  return launch_mix_add_fwd(x, x_dtype, M, y_dist, y_dtype, out, out_dtype, T, n, C,
                            as_stream(stream));
  MHC_TRY_END
}

size_t mhc_mix_bwd_workspace_bytes(int64_t T, int n, int C) {
  if (n < 1 || n > 64 || C < 1 || T < 0) return 0;
  return mix_ws_bytes(T, n, C);
}

int mhc_mix_add_bwd(const void* x, int x_dtype, const float* M, const void* d_out, int dout_dtype,
                    void* dx, int dx_dtype, float* dM, int64_t T, int n, int C, void* workspace,
                    size_t workspace_bytes, void* stream) {
  MHC_TRY_BEGIN
  MHC_CHK(check_common(__func__, T, n, C));
  MHC_CHK(check_dtype(__func__, "x", x_dtype));
  MHC_CHK(check_dtype(__func__, "d_out", dout_dtype));
  MHC_CHK(check_dtype(__func__, "dx", dx_dtype));
  MHC_REQ(M && dM, "%s: NULL M/dM", __func__);
  MHC_REQ(T == 0 || (x && d_out && dx), "%s: NULL tensor pointer", __func__);
  return launch_mix_add_bwd(x, x_dtype, M, d_out, dout_dtype, dx, dx_dtype, dM, T, n, C, workspace,
                            workspace_bytes, as_stream(stream));
  MHC_TRY_END
}

int mhc_rewire_combine_fwd(const void* x, int x_dtype, const void* y_inner, int y_dtype,
                           const float* M, const float* H_pre_act, const float* H_post_act,
                           void* out, int out_dtype, int64_t T, int n, int C, void* stream) {
  MHC_TRY_BEGIN
  MHC_CHK(check_common(__func__, T, n, C));
  MHC_CHK(check_dtype(__func__, "x", x_dtype));
  MHC_CHK(check_dtype(__func__, "y_inner", y_dtype));
  MHC_CHK(check_dtype(__func__, "out", out_dtype));
  MHC_REQ(M && H_pre_act && H_post_act, "%s: NULL parameter pointer", __func__);
  MHC_REQ(T == 0 || (x && y_inner && out), "%s: NULL tensor pointer", __func__);
  return launch_rewire_fwd(x, x_dtype, y_inner, y_dtype, M, H_pre_act, H_post_act, out, out_dtype,
                           T, n, C, as_stream(stream));
  MHC_TRY_END
}

size_t mhc_rewire_bwd_workspace_bytes(int64_t T, int n, int C) {
  return mhc_mix_bwd_workspace_bytes(T, n, C);
}

int mhc_rewire_combine_bwd(const void* x, int x_dtype, const void* y_inner, int y_dtype,
                           const void* d_out, int dout_dtype, const float* M,
                           const float* H_pre_act, const float* H_post_act, void* dx, int dx_dtype,
                           void* dy_inner, int dy_dtype, float* dM, float* dH_pre_act,
                           float* dH_post_act, int64_t T, int n, int C, void* workspace,
                           size_t workspace_bytes, void* stream) {
  MHC_TRY_BEGIN
  MHC_CHK(check_common(__func__, T, n, C));
  MHC_CHK(check_dtype(__func__, "x", x_dtype));
  MHC_CHK(check_dtype(__func__, "y_inner", y_dtype));
  MHC_CHK(check_dtype(__func__, "d_out", dout_dtype));
  MHC_CHK(check_dtype(__func__, "dx", dx_dtype));
  MHC_CHK(check_dtype(__func__, "dy_inner", dy_dtype));
  MHC_REQ(M && H_pre_act && H_post_act, "%s: NULL parameter pointer", __func__);
  MHC_REQ(dM && dH_pre_act && dH_post_act, "%s: NULL gradient pointer", __func__);
  MHC_REQ(T == 0 || (x && y_inner && d_out && dx && dy_inner), "%s: NULL tensor pointer", __func__);
  return launch_rewire_bwd(x, x_dtype, y_inner, y_dtype, d_out, dout_dtype, M, H_pre_act,
                           H_post_act, dx, dx_dtype, dy_inner, dy_dtype, dM, dH_pre_act,
                           dH_post_act, T, n, C, workspace, workspace_bytes, as_stream(stream));
  MHC_TRY_END
}

size_t mhc_rewire_fused_bwd_workspace_bytes(int64_t T, int n, int C) {
  if (n < 1 || n > 64 || C < 1 || T < 0) return 0;
  return rewire_fused_ws_bytes(T, n, C);
}

int mhc_rewire_bwd_dy(const void* y_inner, int y_dtype, const void* d_out, int dout_dtype,
                      const float* H_post_act, void* dy_inner, int dy_dtype, int64_t T, int n,
                      int C, void* workspace, size_t workspace_bytes, void* stream) {
  MHC_TRY_BEGIN
  MHC_CHK(check_common(__func__, T, n, C));
  MHC_CHK(check_dtype(__func__, "y_inner", y_dtype));
  MHC_CHK(check_dtype(__func__, "d_out", dout_dtype));
  MHC_CHK(check_dtype(__func__, "dy_inner", dy_dtype));
  MHC_REQ(H_post_act, "%s: NULL parameter pointer", __func__);
  MHC_REQ(T == 0 || (y_inner && d_out && dy_inner), "%s: NULL tensor pointer", __func__);
  return launch_rewire_bwd_dy(y_inner, y_dtype, d_out, dout_dtype, H_post_act, dy_inner, dy_dtype,
                              T, n, C, workspace, workspace_bytes, as_stream(stream));
  MHC_TRY_END
}

int mhc_rewire_bwd_dx(const void* x, int x_dtype, const void* d_out, int dout_dtype,
                      const void* d_xpre, int dxpre_dtype, const float* M, const float* H_pre_act,
                      const float* H_post_act, void* dx, int dx_dtype, float* dM,
                      float* dH_pre_act, float* dH_post_act, const float* H_pre_raw,
                      const float* H_post_raw, const float* H_res_raw, const float* tape,
                      const float* jacobian, int iters, float eps, float* dH_pre_raw,
                      float* dH_post_raw, float* dH_res_raw, int64_t T, int n, int C,
                      void* workspace, size_t workspace_bytes, void* stream) {
  MHC_TRY_BEGIN
  MHC_CHK(check_common(__func__, T, n, C));
  MHC_CHK(check_dtype(__func__, "x", x_dtype));
  MHC_CHK(check_dtype(__func__, "d_out", dout_dtype));
  MHC_CHK(check_dtype(__func__, "d_xpre", dxpre_dtype));
  MHC_CHK(check_dtype(__func__, "dx", dx_dtype));
  MHC_REQ(M && H_pre_act && H_post_act, "%s: NULL parameter pointer", __func__);
  MHC_REQ(dM && dH_pre_act && dH_post_act, "%s: NULL gradient pointer", __func__);
  MHC_REQ(T == 0 || (x && d_out), "%s: NULL tensor pointer", __func__);
  MHC_REQ(!H_pre_raw == !dH_pre_raw, "%s: H_pre_raw and dH_pre_raw must both be given or both NULL", __func__);
  MHC_REQ(!H_post_raw == !dH_post_raw, "%s: H_post_raw and dH_post_raw must both be given or both NULL", __func__);
  MHC_REQ(!H_res_raw == !dH_res_raw, "%s: H_res_raw and dH_res_raw must both be given or both NULL", __func__);
  if (H_res_raw) {
    MHC_REQ(iters >= 0, "%s: iters=%d must be >= 0", __func__, iters);
    MHC_REQ(tape || jacobian || iters == 0, "%s: tape is NULL (record it with mhc_rewire_in_fwd)", __func__);
  }
  MHC_REQ(!jacobian || sk_lane_ok(n), "%s: a Jacobian exists for n in {1, 2, 4} only (n=%d)", __func__, n);
  const ParamsBwd pb{H_pre_raw, H_post_raw, H_res_raw, tape, jacobian, iters, eps,
                     dH_pre_raw, dH_post_raw, dH_res_raw};
  return launch_rewire_bwd_dx(x, x_dtype, d_out, dout_dtype, d_xpre, dxpre_dtype, M, H_pre_act,
                              H_post_act, dx, dx_dtype, dM, dH_pre_act, dH_post_act, pb, T, n, C,
                              workspace, workspace_bytes, as_stream(stream));
  MHC_TRY_END
}

size_t mhc_rewire_jacobian_floats(int n) {
  if (n < 1 || n > 64) return 0;
  return sk_jacobian_floats(n);
}

int mhc_rewire_in_fwd(const void* x, int x_dtype, const float* H_pre_raw, const float* H_post_raw,
                      const float* H_res_raw, int iters, float eps, float* H_pre_act,
                      float* H_post_act, float* M, float* tape, float* jacobian, void* x_pre,
                      int out_dtype, int64_t T, int n, int C, void* stream) {
  MHC_TRY_BEGIN
  MHC_CHK(check_common(__func__, T, n, C));
  MHC_CHK(check_dtype(__func__, "x", x_dtype));
  MHC_CHK(check_dtype(__func__, "x_pre", out_dtype));
  MHC_REQ(iters >= 0, "%s: iters=%d must be >= 0", __func__, iters);
  MHC_REQ(H_pre_raw && H_post_raw && H_res_raw, "%s: NULL raw parameter pointer", __func__);
  MHC_REQ(H_pre_act && H_post_act && M, "%s: NULL activation pointer", __func__);
  MHC_REQ(tape || iters == 0, "%s: tape is NULL", __func__);
  MHC_REQ(!jacobian || sk_lane_ok(n), "%s: a Jacobian exists for n in {1, 2, 4} only (n=%d)", __func__, n);
  MHC_REQ(T == 0 || (x && x_pre), "%s: NULL tensor pointer", __func__);
  const ParamsFwd pf{H_pre_raw, H_post_raw, H_res_raw, iters, eps, H_pre_act, H_post_act, M,
                     tape, jacobian, 0};
  return launch_rewire_in_fwd(x, x_dtype, pf, x_pre, out_dtype, T, n, C, as_stream(stream));
  MHC_TRY_END
}

int mhc_prescale_fwd(const void* x, int x_dtype, const float* H_pre_act, void* x_pre,
                     int out_dtype, int64_t T, int n, int C, void* stream) {
  MHC_TRY_BEGIN
  MHC_CHK(check_common(__func__, T, n, C));
  MHC_CHK(check_dtype(__func__, "x", x_dtype));
  MHC_CHK(check_dtype(__func__, "x_pre", out_dtype));
  MHC_REQ(H_pre_act, "%s: NULL H_pre_act", __func__);
  MHC_REQ(T == 0 || (x && x_pre), "%s: NULL tensor pointer", __func__);
  return launch_prescale_fwd(x, x_dtype, H_pre_act, x_pre, out_dtype, T, n, C, as_stream(stream));
  MHC_TRY_END
}

int mhc_prescale_bwd(const void* x, int x_dtype, const void* d_xpre, int d_dtype,
                     const float* H_pre_act, void* dx, int dx_dtype, float* dH_pre_act, int64_t T,
                     int n, int C, void* workspace, size_t workspace_bytes, void* stream) {
  MHC_TRY_BEGIN
  MHC_CHK(check_common(__func__, T, n, C));
  MHC_CHK(check_dtype(__func__, "x", x_dtype));
  MHC_CHK(check_dtype(__func__, "d_xpre", d_dtype));
  MHC_CHK(check_dtype(__func__, "dx", dx_dtype));
  MHC_REQ(H_pre_act && dH_pre_act, "%s: NULL parameter pointer", __func__);
  MHC_REQ(T == 0 || (x && d_xpre && dx), "%s: NULL tensor pointer", __func__);
  return launch_prescale_bwd(x, x_dtype, d_xpre, d_dtype, H_pre_act, dx, dx_dtype, dH_pre_act, T, n,
                             C, workspace, workspace_bytes, as_stream(stream));
  MHC_TRY_END
}

int mhc_qlinear_fwd(const void* x, int x_dtype, const uint32_t* w_packed, const void* scales,
                    const void* biases, int scales_dtype, const void* bias, void* y, int64_t M,
                    int N, int K, int group_size, int bits, void* stream) {
  MHC_TRY_BEGIN
  return launch_qlinear_fwd(x, x_dtype, w_packed, scales, biases, scales_dtype, bias, y, M, N, K,
                            group_size, bits, as_stream(stream));
  MHC_TRY_END
}

int mhc_qlinear_bwd_dx(const void* dy, int dy_dtype, const uint32_t* w_packed,
                       const void* scales, const void* biases, int scales_dtype, void* dx,
                       int64_t M, int N, int K, int group_size, int bits, void* stream) {
  MHC_TRY_BEGIN
  return launch_qlinear_bwd_dx(dy, dy_dtype, w_packed, scales, biases, scales_dtype, dx, M, N, K,
                               group_size, bits, as_stream(stream));
  MHC_TRY_END
}

int mhc_qlinear_transpose_pack(const uint32_t* w_packed, uint32_t* wt_packed, int N, int K,
                               void* stream) {
  MHC_TRY_BEGIN
  return launch_qlinear_transpose_pack(w_packed, wt_packed, N, K, as_stream(stream));
  MHC_TRY_END
}

int mhc_qlinear_bwd_dx_t(const void* dy, int dy_dtype, const uint32_t* wt_packed,
                         const void* scales_t, const void* biases_t, void* dx, int64_t M, int N,
                         int K, int group_size, int bits, void* stream) {
  MHC_TRY_BEGIN
  return launch_qlinear_bwd_dx_t(dy, dy_dtype, wt_packed, scales_t, biases_t, dx, M, N, K,
                                 group_size, bits, as_stream(stream));
  MHC_TRY_END
}

int mhc_residual_add_agg(const void* x, int x_dtype, const void* res, int res_dtype,
                         const float* H_pre, void* out, int out_dtype, float* y_agg, int64_t T,
                         int n, int C, void* stream) {
  MHC_TRY_BEGIN
  MHC_CHK(check_common(__func__, T, n, C));
  MHC_CHK(check_dtype(__func__, "x", x_dtype));
  MHC_CHK(check_dtype(__func__, "res", res_dtype));
  MHC_CHK(check_dtype(__func__, "out", out_dtype));
  MHC_REQ(H_pre, "%s: NULL H_pre", __func__);
  MHC_REQ(T == 0 || (x && res && out && y_agg), "%s: NULL tensor pointer", __func__);
  return launch_residual_add_agg(x, x_dtype, res, res_dtype, H_pre, out, out_dtype, y_agg, T, n, C,
                                 as_stream(stream));
  MHC_TRY_END
}

int mhc_residual_add_agg_bwd(const void* out, int out_dtype, const void* d_out, int dout_dtype,
                             const float* d_y, const float* H_pre, void* dx, int dx_dtype,
                             float* dH_pre, int64_t T, int n, int C, void* workspace,
                             size_t workspace_bytes, void* stream) {
  MHC_TRY_BEGIN
  MHC_CHK(check_common(__func__, T, n, C));
  MHC_CHK(check_dtype(__func__, "out", out_dtype));
  MHC_CHK(check_dtype(__func__, "dx", dx_dtype));
  if (d_out) MHC_CHK(check_dtype(__func__, "d_out", dout_dtype));
  MHC_REQ(H_pre && dH_pre, "%s: NULL H_pre/dH_pre", __func__);
  MHC_REQ(T == 0 || (out && dx), "%s: NULL out/dx", __func__);
  return launch_residual_add_agg_bwd(out, out_dtype, d_out, d_out ? dout_dtype : out_dtype, d_y,
                                     H_pre, dx, dx_dtype, dH_pre, T, n, C, workspace,
                                     workspace_bytes, as_stream(stream));
  MHC_TRY_END
}

}  // extern "C"
