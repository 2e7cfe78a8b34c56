// MHCRewire-side kernels for sm_100a: stream mix + add (reference
// stream_mix_add.metal, metal.py:954-1014), its backward (reference
// stream_mix_backward_dx.metal + mhc_backward_dM.metal, metal.py:2661-2690),
// the fused post-combine of layer.py:302-337 (H_pre/H_post folded in-kernel),
// the input pre-scale of layer.py:478-480, and residual_add_agg
// (reference residual_add_agg.metal, metal.py:1673-1731, utils.py:4-24).
//
// All of these are elementwise over columns with an n x n mix across the
// streams of one token: thread = (token, VEC consecutive columns), the n
// stream values of those columns in registers, one read of every input and
// one write of every output.  Parameter gradients are reduced per CTA into a
// partial row and summed in a fixed order by a one-CTA finalize.
//
// Combined forward (rewire form; the plain mix is hpre = hpost = 1):
//   out_i = hpost_i * (y_i + sum_j M_ij (hpre_j x_j))
// Combined backward:
//   dz_i = hpost_i d_i,  dy_i = dz_i,  dx_j = hpre_j sum_i M_ij dz_i
//   Q_ij = sum d_i x_j,  R_i = sum d_i y_i          (partials)
//   dM_ij = hpost_i hpre_j Q_ij
//   dhpre_j = sum_i hpost_i M_ij Q_ij
//   dhpost_i = R_i + sum_j M_ij hpre_j Q_ij
//
// MHCRewire end to end (pre-scale, inner module, post-combine) runs its
// backward as two passes around the inner module's backward, so that dx is
// written once and dH_pre comes out of one reduction:
//   dy side (before the inner backward): dy_i = hpost_i d_i, R_i = sum d_i y_i
//   x side  (after it, p = d_xpre):      dx_j = hpre_j (sum_i M_ij hpost_i d_i + p_j)
//                                        Q_ij = sum d_i x_j, S_j = sum p_j x_j
//   finalize: dM, dhpost as above; dhpre_j = sum_i hpost_i M_ij Q_ij + S_j
// The two passes write their partial rows into one workspace: the dy side
// rows [0, G1) (header word 0 = G1), the x side rows [G1, G1 + G2) (word 2 =
// G2); a row is [Q (n*n) | R (n) | S (n)] with the other side's slots zero.
#include <algorithm>
#include <cstdlib>

#include "mhc_common.cuh"
#include "mhc_internal.h"
#include "mhc_sinkhorn.cuh"

namespace mhc {

constexpr int kMixBD = 256;

// Loop helper: with EXACT the stream count is the compile-time MAXN, else a
// runtime n <= MAXN handled with predicated, fully unrolled loops (the
// register arrays stay in registers).
#define MHC_FOR_N(j) _Pragma("unroll") for (int j = 0; j < MAXN; ++j) if (EXACT || j < n)

template <typename T, int V>
__device__ __forceinline__ void load_or_zero(const T* p, bool ok, float (&o)[V]) {
  if (ok) load_vec<T, V>(p, o);
  else
#pragma unroll
    for (int v = 0; v < V; ++v) o[v] = 0.f;
}

// ------------------------------------------------------------ combine fwd --
template <int MAXN, bool EXACT, typename XT, typename YT, typename OT, int VEC>
__global__ void __launch_bounds__(kMixBD)
k_combine_fwd(const XT* __restrict__ x, const YT* __restrict__ y, const float* __restrict__ Mg,
              const float* __restrict__ hpre_g, const float* __restrict__ hpost_g,
              OT* __restrict__ out, int64_t T, int n, int C) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sM[MAXN * MAXN];
  __shared__ float shpre[MAXN], shpost[MAXN];
  const int nr = EXACT ? MAXN : n;
  for (int e = threadIdx.x; e < nr * nr; e += blockDim.x) sM[e] = Mg[e];
  for (int e = threadIdx.x; e < nr; e += blockDim.x) {
    shpre[e] = hpre_g ? hpre_g[e] : 1.0f;
    shpost[e] = hpost_g ? hpost_g[e] : 1.0f;
  }
  __syncthreads();
  const int groups = (C + VEC - 1) / VEC;
  const int64_t items = T * groups;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < items;
       q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = q / groups;
    const int col = (int)(q - t * groups) * VEC;
    const int64_t base = t * (int64_t)nr * C + col;
    float xs[MAXN][VEC];
    MHC_FOR_N(j) {
      load_vec<XT, VEC>(x + base + (int64_t)j * C, xs[j]);
#pragma unroll
      for (int v = 0; v < VEC; ++v) xs[j][v] *= shpre[j];
    }
    MHC_FOR_N(i) {
      float yv[VEC], o[VEC];
      load_vec<YT, VEC>(y + base + (int64_t)i * C, yv);
#pragma unroll
      for (int v = 0; v < VEC; ++v) o[v] = 0.f;
      MHC_FOR_N(j) {
        const float mij = sM[i * nr + j];
#pragma unroll
        for (int v = 0; v < VEC; ++v) o[v] = fmaf(mij, xs[j][v], o[v]);
      }
#pragma unroll
      for (int v = 0; v < VEC; ++v) o[v] = shpost[i] * (yv[v] + o[v]);
      store_vec<OT, VEC>(out + base + (int64_t)i * C, o);
    }
  }
}

// ----------------------------------------------------------- prescale fwd --
// PARAMS (MHCRewire's input side, n in {1, 2, 4, 8}): the parameter kernel
// rides along as block 0 -- sigmoids, the Sinkhorn forward with its tape and,
// for n <= 4, the transposed Jacobian of M (sk_jacobian_lane) -- while blocks
// 1.. pre-scale with H_pre_act = sigmoid(H_pre_raw) evaluated in-block by the
// same function (the same bits block 0 stores).  The one-warp latency chain
// of the Sinkhorn iterations then overlaps the streaming instead of
// preceding it.
template <int MAXN, bool EXACT, typename XT, typename OT, int VEC, bool PARAMS = false>
__global__ void __launch_bounds__(kMixBD, PARAMS ? 8 : 1)  // PARAMS: keep 8 blocks per SM
k_prescale_fwd(const XT* __restrict__ x, const float* __restrict__ hpre_g, OT* __restrict__ xo,
               int64_t T, int n, int C, ParamsFwd pf) {
  pdl_wait();
  pdl_trigger();
  __shared__ float shpre[MAXN];
  const int nr = EXACT ? MAXN : n;
  int b0 = 0;
  if constexpr (PARAMS) {
    static_assert(EXACT && MAXN <= 8, "the parameter block runs the one-warp Sinkhorn paths");
    if (blockIdx.x == 0) {
      const int tid = threadIdx.x;
      if (tid < MAXN) {
        pf.hpre[tid] = sigmoidf_(pf.hpre_raw[tid]);
        pf.hpost[tid] = 2.0f * sigmoidf_(pf.hpost_raw[tid]);
      }
      if constexpr (MAXN <= 4) {
        // pf.stage: the tape goes to shared memory first (the Jacobian's
        // sweep reads it there) and then to the global record
        extern __shared__ float s_tape[];
        float* tp = pf.stage ? s_tape : pf.tape;
        if (tid < 32) sk_forward_lane<MAXN>(pf.hres_raw, pf.iters, pf.eps, tp, pf.M);
        if (pf.jac || pf.stage) {  // kernel arguments: uniform over the block
          __syncthreads();  // tape stored
          if (pf.stage) {
            const int tf = pf.iters * (MAXN * MAXN + 2 * MAXN);
            for (int e = tid; e < tf; e += blockDim.x) pf.tape[e] = s_tape[e];
          }
          if (pf.jac) sk_jacobian_lane<MAXN>(pf.hres_raw, tp, pf.iters, pf.eps, pf.jac, !pf.stage);
        }
      } else {
        if (tid < 32) sk_forward_warp<MAXN>(pf.hres_raw, pf.iters, pf.eps, pf.tape, pf.M);
      }
      return;
    }
    b0 = 1;
    for (int e = threadIdx.x; e < nr; e += blockDim.x) shpre[e] = sigmoidf_(pf.hpre_raw[e]);
  } else {
    for (int e = threadIdx.x; e < nr; e += blockDim.x) shpre[e] = hpre_g[e];
  }
  __syncthreads();
  const int groups = (C + VEC - 1) / VEC;
  const int64_t items = T * groups;
  for (int64_t q = (int64_t)(blockIdx.x - b0) * blockDim.x + threadIdx.x; q < items;
       q += (int64_t)(gridDim.x - b0) * blockDim.x) {
    const int64_t t = q / groups;
    const int col = (int)(q - t * groups) * VEC;
    const int64_t base = t * (int64_t)nr * C + col;
    MHC_FOR_N(i) {
      float v_[VEC];
      load_vec<XT, VEC>(x + base + (int64_t)i * C, v_);
#pragma unroll
      for (int v = 0; v < VEC; ++v) v_[v] *= shpre[i];
      store_vec<OT, VEC>(xo + base + (int64_t)i * C, v_);
    }
  }
}

// ------------------------------------------------------- residual add agg --
// out = x + res (fp32 add, stored as OT); y_agg = sum_i hpre_i (x + res)_i in
// fp32 from the unrounded sums, as residual_add_agg.metal does.
template <int MAXN, bool EXACT, typename XT, typename RT, typename OT, int VEC>
__global__ void __launch_bounds__(kMixBD)
k_residual_add_agg(const XT* __restrict__ x, const RT* __restrict__ res,
                   const float* __restrict__ hpre_g, OT* __restrict__ out,
                   float* __restrict__ yagg, int64_t T, int n, int C) {
  __shared__ float shpre[MAXN];
  const int nr = EXACT ? MAXN : n;
  for (int e = threadIdx.x; e < nr; e += blockDim.x) shpre[e] = hpre_g[e];
  __syncthreads();
  const int groups = (C + VEC - 1) / VEC;
  const int64_t items = T * groups;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < items;
       q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = q / groups;
    const int col = (int)(q - t * groups) * VEC;
    const int64_t base = t * (int64_t)nr * C + col;
    float agg[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) agg[v] = 0.f;
    MHC_FOR_N(i) {
      float a[VEC], b[VEC];
      load_vec<XT, VEC>(x + base + (int64_t)i * C, a);
      load_vec<RT, VEC>(res + base + (int64_t)i * C, b);
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        a[v] += b[v];
        agg[v] = fmaf(a[v], shpre[i], agg[v]);
      }
      store_vec<OT, VEC>(out + base + (int64_t)i * C, a);
    }
    // y_agg rows are C fp32 values; VEC is 1, 4 or 8 and C % VEC == 0
    store_vec<float, VEC>(yagg + t * C + col, agg);
  }
}

// ------------------------------------------------------- combine bwd (fast) --
// Thread-per-(token, VEC columns) with the Q / R partials in registers
// (n <= 8).  HAS_Y: accumulate R_i = sum d_i y_i (rewire mode).
template <int N, typename XT, typename YT, typename DT, typename DXT, typename DYT, int VEC,
          bool HAS_Y>
__global__ void __launch_bounds__(kMixBD)
k_combine_bwd_fast(const XT* __restrict__ x, const YT* __restrict__ y,
                   const DT* __restrict__ dout, const float* __restrict__ Mg,
                   const float* __restrict__ hpre_g, const float* __restrict__ hpost_g,
                   DXT* __restrict__ dx, DYT* __restrict__ dy, int64_t T, int C,
                   float* __restrict__ ws_p, int* __restrict__ ws_hdr) {
  constexpr int P = N * N + 2 * N;
  __shared__ float sM[N * N];
  __shared__ float sacc[(kMixBD / 32) * P];
  for (int e = threadIdx.x; e < N * N; e += blockDim.x) sM[e] = Mg[e];
  float hpre[N], hpost[N];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    hpre[i] = hpre_g ? __ldg(hpre_g + i) : 1.0f;
    hpost[i] = hpost_g ? __ldg(hpost_g + i) : 1.0f;
  }
  __syncthreads();
  float aQ[N][N], aR[N];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    aR[i] = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) aQ[i][j] = 0.f;
  }
  const int groups = (C + VEC - 1) / VEC;
  const int64_t items = T * groups;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < items;
       q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = q / groups;
    const int col = (int)(q - t * groups) * VEC;
    const int64_t base = t * (int64_t)N * C + col;
    float xr[N][VEC], dr[N][VEC];
#pragma unroll
    for (int i = 0; i < N; ++i) {
      load_vec<XT, VEC>(x + base + (int64_t)i * C, xr[i]);
      load_vec<DT, VEC>(dout + base + (int64_t)i * C, dr[i]);
    }
#pragma unroll
    for (int i = 0; i < N; ++i) {
      if constexpr (HAS_Y) {
        float yv[VEC];
        load_vec<YT, VEC>(y + base + (int64_t)i * C, yv);
#pragma unroll
        for (int v = 0; v < VEC; ++v) aR[i] = fmaf(dr[i][v], yv[v], aR[i]);
      }
#pragma unroll
      for (int j = 0; j < N; ++j)
#pragma unroll
        for (int v = 0; v < VEC; ++v) aQ[i][j] = fmaf(dr[i][v], xr[j][v], aQ[i][j]);
    }
    // dz overwrites d; dy = dz
#pragma unroll
    for (int i = 0; i < N; ++i) {
#pragma unroll
      for (int v = 0; v < VEC; ++v) dr[i][v] *= hpost[i];
      if (dy) store_vec<DYT, VEC>(dy + base + (int64_t)i * C, dr[i]);
    }
#pragma unroll
    for (int j = 0; j < N; ++j) {
      float o[VEC];
#pragma unroll
      for (int v = 0; v < VEC; ++v) o[v] = 0.f;
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const float mij = sM[i * N + j];
#pragma unroll
        for (int v = 0; v < VEC; ++v) o[v] = fmaf(mij, dr[i][v], o[v]);
      }
#pragma unroll
      for (int v = 0; v < VEC; ++v) o[v] *= hpre[j];
      store_vec<DXT, VEC>(dx + base + (int64_t)j * C, o);
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int i = 0; i < N; ++i) {
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const float v = warp_sum(aQ[i][j]);
      if (lane == 0) sacc[warp * P + i * N + j] = v;
    }
    const float r = warp_sum(aR[i]);
    if (lane == 0) { sacc[warp * P + N * N + i] = r; sacc[warp * P + N * N + N + i] = 0.f; }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < P; e += blockDim.x) {
    float s = 0.f;
    for (int w = 0; w < nw; ++w) s += sacc[w * P + e];
    ws_p[(size_t)blockIdx.x * P + e] = s;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) ws_hdr[0] = gridDim.x;
}

// ---------------------------------------------------- combine bwd (generic) --
// Any n <= 64: a tile of kMixGenBD columns of d and x is staged in shared
// memory (plus the products d_i y_i when y is given); each thread writes
// dx / dy for its column, then the CTA accumulates Q = D X^T with 4x4
// register blocks and thread i (< n) sums the product row i into R_i.
constexpr int kMixGenBD = 128;
constexpr int kMixGenLD = kMixGenBD + 1;
constexpr int kMixRB = 4;
constexpr int kMixMaxBlk = 2;  // ceil(16 * 16 / 128)

__host__ __device__ inline size_t mix_gen_smem(int n) {
  return ((size_t)n * n + 2 * (size_t)n + 3 * (size_t)n * kMixGenLD) * sizeof(float);
}

// TAIL = the x side of the end-to-end MHCRewire backward: `y` is then d_xpre
// (p, may be NULL), sp holds p_j (not a product), dx_j gains hpre_j p_j, no dy
// is written, the per-stream sums are S_j = sum p_j x_j (slot n*n + n), and
// the rows start after the dy side's (header word 0).
template <typename XT, typename YT, typename DT, typename DXT, typename DYT, bool TAIL = false>
__global__ void __launch_bounds__(kMixGenBD)
k_combine_bwd_generic(const XT* __restrict__ x, const YT* __restrict__ y,
                      const DT* __restrict__ dout, const float* __restrict__ Mg,
                      const float* __restrict__ hpre_g, const float* __restrict__ hpost_g,
                      DXT* __restrict__ dx, DYT* __restrict__ dy, int64_t T, int n, int C,
                      float* __restrict__ ws_p, int* __restrict__ ws_hdr) {
  extern __shared__ float smem[];
  float* sM = smem;
  float* shpre = sM + n * n;
  float* shpost = shpre + n;
  float* sx = shpost + n;            // n x LD
  float* sd = sx + n * kMixGenLD;    // n x LD
  float* sp = sd + n * kMixGenLD;    // n x LD  (d_i * y_i, or p_j with TAIL)
  const int tid = threadIdx.x;
  const int row0 = TAIL ? ws_hdr[0] : 0;
  for (int e = tid; e < n * n; e += kMixGenBD) sM[e] = Mg[e];
  for (int e = tid; e < n; e += kMixGenBD) {
    shpre[e] = hpre_g ? hpre_g[e] : 1.0f;
    shpost[e] = hpost_g ? hpost_g[e] : 1.0f;
  }
  const int nb = (n + kMixRB - 1) / kMixRB;
  const int nblk = nb * nb;
  float acc[kMixMaxBlk][kMixRB][kMixRB];
#pragma unroll
  for (int q = 0; q < kMixMaxBlk; ++q)
#pragma unroll
    for (int a = 0; a < kMixRB; ++a)
#pragma unroll
      for (int b = 0; b < kMixRB; ++b) acc[q][a][b] = 0.f;
  float accR = 0.f;
  __syncthreads();
  const int tiles = (C + kMixGenBD - 1) / kMixGenBD;
  const int64_t ntile = T * tiles;
  for (int64_t tt = blockIdx.x; tt < ntile; tt += gridDim.x) {
    const int64_t t = tt / tiles;
    const int c0 = (int)(tt - t * tiles) * kMixGenBD;
    const int c = c0 + tid;
    const bool ok = c < C;
    const int64_t base = t * (int64_t)n * C + c;
    for (int i = 0; i < n; ++i) {
      const float dv = ok ? to_f(dout[base + (int64_t)i * C]) : 0.f;
      sx[i * kMixGenLD + tid] = ok ? to_f(x[base + (int64_t)i * C]) : 0.f;
      sd[i * kMixGenLD + tid] = dv;
      if (TAIL) sp[i * kMixGenLD + tid] = (ok && y) ? to_f(y[base + (int64_t)i * C]) : 0.f;
      else if (y) sp[i * kMixGenLD + tid] = ok ? dv * to_f(y[base + (int64_t)i * C]) : 0.f;
    }
    if (ok) {
      if (dx)
        for (int j = 0; j < n; ++j) {
          float o = 0.f;
          for (int i = 0; i < n; ++i)
            o = fmaf(sM[i * n + j], shpost[i] * sd[i * kMixGenLD + tid], o);
          if (TAIL) o += sp[j * kMixGenLD + tid];
          dx[base + (int64_t)j * C] = from_f<DXT>(o * shpre[j]);
        }
      if (!TAIL && dy)
        for (int i = 0; i < n; ++i)
          dy[base + (int64_t)i * C] = from_f<DYT>(shpost[i] * sd[i * kMixGenLD + tid]);
    }
    __syncthreads();
    const int width = min(kMixGenBD, C - c0);
#pragma unroll
    for (int q = 0; q < kMixMaxBlk; ++q) {
      const int blk = tid + q * kMixGenBD;
      if (blk >= nblk) break;
      const int i0 = (blk / nb) * kMixRB, j0 = (blk % nb) * kMixRB;
      for (int cc = 0; cc < width; ++cc) {
        float dv[kMixRB], xv[kMixRB];
#pragma unroll
        for (int a = 0; a < kMixRB; ++a) {
          dv[a] = (i0 + a < n) ? sd[(i0 + a) * kMixGenLD + cc] : 0.f;
          xv[a] = (j0 + a < n) ? sx[(j0 + a) * kMixGenLD + cc] : 0.f;
        }
#pragma unroll
        for (int a = 0; a < kMixRB; ++a)
#pragma unroll
          for (int b = 0; b < kMixRB; ++b) acc[q][a][b] = fmaf(dv[a], xv[b], acc[q][a][b]);
      }
    }
    if (TAIL && y && tid < n)
      for (int cc = 0; cc < width; ++cc)
        accR = fmaf(sp[tid * kMixGenLD + cc], sx[tid * kMixGenLD + cc], accR);
    else if (!TAIL && y && tid < n)
      for (int cc = 0; cc < width; ++cc) accR += sp[tid * kMixGenLD + cc];
    __syncthreads();
  }
  const int P = n * n + 2 * n;
  float* pr = ws_p + (size_t)(row0 + blockIdx.x) * P;
  if (tid < n) {
    pr[n * n + tid] = TAIL ? 0.f : accR;
    pr[n * n + n + tid] = TAIL ? accR : 0.f;
  }
#pragma unroll
  for (int q = 0; q < kMixMaxBlk; ++q) {
    const int blk = tid + q * kMixGenBD;
    if (blk >= nblk) break;
    const int i0 = (blk / nb) * kMixRB, j0 = (blk % nb) * kMixRB;
#pragma unroll
    for (int a = 0; a < kMixRB; ++a)
#pragma unroll
      for (int b = 0; b < kMixRB; ++b) {
        const int i = i0 + a, j = j0 + b;
        if (i < n && j < n) pr[i * n + j] = acc[q][a][b];
      }
  }
  if (blockIdx.x == 0 && tid == 0) ws_hdr[TAIL ? 2 : 0] = gridDim.x;
}

// ------------------------------------------- rewire backward, x side (fast) --
// The finalize of MHCRewire's end-to-end backward when the x side's last CTA
// runs it (on = 1): the activation gradients (each nullable) and the
// raw-parameter chain rule of pb.
struct RewireFin {
  float* dM;
  float* dhpre;
  float* dhpost;
  ParamsBwd pb;
  int on;
};

// Run by the last CTA of the x side (n in {1, 2, 4}) once every CTA's row
// is visible: sums the G rows of P floats -- each already holding its share
// of the dy side's rows -- in a fixed order (16-byte columns of a row over S
// interleaved row slices, then the slices of an entry by a warp butterfly),
// so the result does not depend on which CTA came last.  Then the mode-3
// finalize of k_combine_finalize and the raw-parameter tail: sigmoid chain
// rule, and dH_res from the Jacobian's dot products or the lane-path
// reverse sweep.  The rows were written in this launch: L2 loads.
template <int N>
__device__ __forceinline__ void rewire_fin_last(const float* rows, int G, const float* sM,
                                                const float* __restrict__ hpre_g,
                                                const float* __restrict__ hpost_g,
                                                const RewireFin& fin) {
  constexpr int NN = N * N, P = NN + 2 * N;
  constexpr int W = (P % 4 == 0) ? 4 : 1;  // floats per load
  constexpr int CW = P / W;                // loads per row
  constexpr int S = kMixBD / CW;           // row slices
  __shared__ float red[S * P];
  __shared__ float fq[P], fa[P];
  const int tid = threadIdx.x, c = tid % CW, r = tid / CW;
  if (r < S) {
    float a[W];
#pragma unroll
    for (int k = 0; k < W; ++k) a[k] = 0.f;
#pragma unroll 8
    for (int g = r; g < G; g += S) {
      const float* src = rows + (size_t)g * P + c * W;
      if constexpr (W == 4) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(src));
        a[0] += v.x; a[1] += v.y; a[2] += v.z; a[3] += v.w;
      } else {
        a[0] += __ldcg(src);
      }
    }
#pragma unroll
    for (int k = 0; k < W; ++k) red[r * P + c * W + k] = a[k];
  }
  __syncthreads();
  const int lane = tid & 31, warp = tid >> 5;
  for (int e = warp; e < P; e += (int)(blockDim.x >> 5)) {
    float s = 0.f;
    for (int q = lane; q < S; q += 32) s += red[q * P + e];
    s = warp_sum(s);
    if (lane == 0) fq[e] = s;
  }
  __syncthreads();
  // Q = fq[0, NN), R = fq[NN, NN + N), S = fq[NN + N, P)
  if (tid < NN) {
    const int i = tid / N, j = tid % N;
    const float v = (hpost_g[i] * hpre_g[j]) * fq[tid];
    fa[tid] = v;
    if (fin.dM) fin.dM[tid] = v;
  } else if (tid < NN + N) {
    const int j = tid - NN;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i) s = fmaf(hpost_g[i] * sM[i * N + j], fq[i * N + j], s);
    s += fq[NN + N + j];
    fa[tid] = s;
    if (fin.dhpre) fin.dhpre[j] = s;
  } else if (tid < P) {
    const int i = tid - NN - N;
    float s = fq[NN + i];
#pragma unroll
    for (int j = 0; j < N; ++j) s = fmaf(sM[i * N + j] * hpre_g[j], fq[i * N + j], s);
    fa[tid] = s;
    if (fin.dhpost) fin.dhpost[i] = s;
  }
  const ParamsBwd& pb = fin.pb;
  if (!pb.any()) return;
  __syncthreads();  // fa complete
  if (tid < N) {
    if (pb.dhpre_raw) {
      const float sg = sigmoidf_(pb.hpre_raw[tid]);
      pb.dhpre_raw[tid] = fa[NN + tid] * (1.0f - sg) * sg;
    }
    if (pb.dhpost_raw) {
      const float sg = sigmoidf_(pb.hpost_raw[tid]);
      pb.dhpost_raw[tid] = (2.0f * fa[NN + N + tid]) * (1.0f - sg) * sg;
    }
  }
  if (!pb.dhres_raw) return;
  if (pb.jac) {
    if (tid < NN) {
      float s = 0.f;
#pragma unroll
      for (int u = 0; u < NN; ++u) s = fmaf(fa[u], pb.jac[u * NN + tid], s);
      pb.dhres_raw[tid] = s;
    }
  } else if (tid < 32 && (pb.tape || pb.iters == 0)) {
    const bool act = tid < NN;
    const float d = sk_backward_lane<N>(pb.hres_raw, pb.tape, pb.iters, pb.eps, act ? fa[tid] : 0.f);
    if (act) pb.dhres_raw[tid] = d;
  }
}

// End of an x-side CTA: Q and S reduced over its threads (fixed-order warp
// butterflies, then the warps in order) into its partial row [Q | 0 | S] --
// with fin.on plus its share of the dy side's rows b, b + G2, ... (written by
// the previous launch) -- and, with fin.on, the last CTA to finish (a ticket
// in header word 3, zeroed by the dy side) runs the finalize.
template <int N>
__device__ __forceinline__ void rewire_x_rows(float (&aQ)[N][N], float (&aS)[N], const float* sM,
                                              const float* __restrict__ hpre_g,
                                              const float* __restrict__ hpost_g,
                                              float* __restrict__ ws_p, int* __restrict__ ws_hdr,
                                              int row0, const RewireFin& fin) {
  constexpr int P = N * N + 2 * N;
  __shared__ float sacc[32 * P];  // up to 1,024 threads
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int i = 0; i < N; ++i) {
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const float v = warp_sum(aQ[i][j]);
      if (lane == 0) sacc[warp * P + i * N + j] = v;
    }
    const float r = warp_sum(aS[i]);
    if (lane == 0) { sacc[warp * P + N * N + i] = 0.f; sacc[warp * P + N * N + N + i] = r; }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < P; e += blockDim.x) {
    float s = 0.f;
    for (int w = 0; w < nw; ++w) s += sacc[w * P + e];
    if (fin.on)  // this CTA's share of the dy side's rows (written by the previous launch)
      for (int r = blockIdx.x; r < row0; r += gridDim.x) s += ws_p[(size_t)r * P + e];
    ws_p[(size_t)(row0 + blockIdx.x) * P + e] = s;
  }
  if (!fin.on) {
    if (blockIdx.x == 0 && threadIdx.x == 0) ws_hdr[2] = gridDim.x;
    return;
  }
  __shared__ int s_last;
  __threadfence();  // this CTA's row is visible device-wide before its ticket
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(ws_hdr + 3, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  rewire_fin_last<N>(ws_p + (size_t)row0 * P, (int)gridDim.x, sM, hpre_g, hpost_g, fin);
  if (threadIdx.x == 0) ws_hdr[3] = 0;  // the workspace may be finalized again
}

// n in {1, 2, 4}, 16-byte vectors: thread = (token, VEC columns) with the
// x rows and the dx accumulators of all n streams in registers, Q and S in
// registers across the thread's items.  p (d_xpre) may be NULL (zero), dx
// may be NULL (only the parameter partials are wanted).  Ends in
// rewire_x_rows (partial rows, and with fin.on the last-CTA finalize).
template <int N, typename XT, typename DT, typename PT, int VEC>
__global__ void __launch_bounds__(kMixBD, 2)
k_rewire_bwd_x_fast(const XT* __restrict__ x, const DT* __restrict__ dout,
                    const PT* __restrict__ dp, const float* __restrict__ Mg,
                    const float* __restrict__ hpre_g, const float* __restrict__ hpost_g,
                    XT* __restrict__ dx, int64_t T, int C, float* __restrict__ ws_p,
                    int* __restrict__ ws_hdr, RewireFin fin) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sM[N * N];
  const int row0 = ws_hdr[0];
  for (int e = threadIdx.x; e < N * N; e += blockDim.x) sM[e] = Mg[e];
  float hpre[N], hpost[N];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    hpre[i] = __ldg(hpre_g + i);
    hpost[i] = __ldg(hpost_g + i);
  }
  __syncthreads();
  float aQ[N][N], aS[N];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    aS[i] = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) aQ[i][j] = 0.f;
  }
  // (token, column group) of linear item q = thread + k * stride, stepped
  // incrementally: no per-item 64-bit division
  const int groups = C / VEC;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t q0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t t = q0 / groups;
  int g = (int)(q0 - t * groups);
  const int64_t dt = stride / groups;
  const int dg = (int)(stride - dt * groups);
  for (; t < T;) {
    const int64_t base = t * (int64_t)N * C + (int64_t)g * VEC;
    // every load of the item first, then the arithmetic
    float xr[N][VEC], dr[N][VEC], pv[N][VEC];
#pragma unroll
    for (int j = 0; j < N; ++j) load_vec<XT, VEC>(x + base + (int64_t)j * C, xr[j]);
#pragma unroll
    for (int i = 0; i < N; ++i) load_vec<DT, VEC>(dout + base + (int64_t)i * C, dr[i]);
    if (dp) {
#pragma unroll
      for (int j = 0; j < N; ++j) load_vec<PT, VEC>(dp + base + (int64_t)j * C, pv[j]);
    } else {
#pragma unroll
      for (int j = 0; j < N; ++j)
#pragma unroll
        for (int v = 0; v < VEC; ++v) pv[j][v] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
      for (int j = 0; j < N; ++j)
#pragma unroll
        for (int v = 0; v < VEC; ++v) aQ[i][j] = fmaf(dr[i][v], xr[j][v], aQ[i][j]);
#pragma unroll
    for (int j = 0; j < N; ++j) {
      float o[VEC];
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        aS[j] = fmaf(pv[j][v], xr[j][v], aS[j]);
        float a = pv[j][v];
#pragma unroll
        for (int i = 0; i < N; ++i) a = fmaf(sM[i * N + j] * hpost[i], dr[i][v], a);
        o[v] = a * hpre[j];
      }
      if (dx) store_vec<XT, VEC>(dx + base + (int64_t)j * C, o);
    }
    g += dg;
    t += dt;
    if (g >= groups) { g -= groups; ++t; }
  }
  rewire_x_rows<N>(aQ, aS, sM, hpre_g, hpost_g, ws_p, ws_hdr, row0, fin);
}

// Shared-memory 4-column loads of the staged rows (plain ld.shared: the
// load_vec helpers use global-memory cache hints).
template <typename T>
__device__ __forceinline__ void lds4(const T* p, float (&o)[4]) {
  if constexpr (sizeof(T) == 4) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = to_f(h[k]);
  }
}

// x side with bulk-copy staging (n in {1, 2, 4}): one CTA of 512 threads per
// SM takes the tokens b, b + G, ... of the sequence; a token's x, d_out and
// d_xpre rows are each one contiguous run, so thread 0 stages a whole token
// with three 1-D bulk copies (plain loads of this GPU's memory) into a ring
// of NS buffers completing on mbarriers, NS tokens ahead.  The CTA's TPI
// parts take TPI consecutive tokens of the sequence per step (16 warps per
// SM to hide the shared-memory and FMA latencies of ~220 instructions per
// 4-column group; more tokens per step, fewer block barriers per token);
// thread t of a part owns its column groups t, t + 512 / TPI, ...  A step's
// buffers are refilled after the block barrier that follows their last
// reads.  The loads no longer occupy registers, so the bytes in flight
// per SM are the ring's.  Waits are bounded: a copy that never lands makes the
// CTA wait (bounded) for its other copies in flight, write NaN into its dx
// tokens from there on and into its partial row, so the parameter gradients
// come out NaN.
constexpr int kXBulkMaxStages = 8;
constexpr int kXBulkBD = 512;

template <int N, typename XT, typename DT, typename PT, int TPI>
__global__ void __launch_bounds__(kXBulkBD, 1)
k_rewire_bwd_x_bulk(const XT* __restrict__ x, const DT* __restrict__ dout,
                    const PT* __restrict__ dp, const float* __restrict__ Mg,
                    const float* __restrict__ hpre_g, const float* __restrict__ hpost_g,
                    XT* __restrict__ dx, int64_t T, int C, int NS, float* __restrict__ ws_p,
                    int* __restrict__ ws_hdr, RewireFin fin) {
  pdl_wait();
  pdl_trigger();
  constexpr int HB = kXBulkBD / TPI;  // threads per token of a step
  extern __shared__ __align__(16) unsigned char s_ring[];
  __shared__ float sM[N * N];
  __shared__ __align__(16) float sWT[N][4];  // sWT[j][i] = M_ij H_post_i
  __shared__ __align__(8) uint64_t s_full[kXBulkMaxStages];
  __shared__ int s_abort;
  const int tid = threadIdx.x, hf = tid / HB, lt = tid % HB;
  const int row0 = ws_hdr[0];
  const int64_t G = gridDim.x, RS = (int64_t)N * C;
  const unsigned bx = (unsigned)(RS * sizeof(XT)), bdo = (unsigned)(RS * sizeof(DT));
  const unsigned bp = dp ? (unsigned)(RS * sizeof(PT)) : 0u;
  const unsigned sb = bx + bdo + bp;  // bytes per stage (multiples of 16: launcher)
  if (tid == 0) {
    for (int b = 0; b < NS; ++b) mbar_init(&s_full[b], 1);
    s_abort = 0;
    mbar_init_fence();
  }
  for (int e = tid; e < N * N; e += blockDim.x) {
    sM[e] = Mg[e];
    sWT[e % N][e / N] = Mg[e] * __ldg(hpost_g + e / N);
  }
  float hpre[N];
#pragma unroll
  for (int i = 0; i < N; ++i) hpre[i] = __ldg(hpre_g + i);
  __syncthreads();
  const int64_t ntok = (int64_t)blockIdx.x < T ? (T - 1 - blockIdx.x) / G + 1 : 0;
  auto issue = [&](int64_t k) {  // thread 0: token k of this CTA's sequence
    const int64_t tok = blockIdx.x + k * G;
    const int slot = (int)(k % NS);
    unsigned char* dst = s_ring + (size_t)slot * sb;
    mbar_arrive_expect_tx(&s_full[slot], sb);
    bulk_g2s(dst, x + tok * RS, bx, &s_full[slot]);
    bulk_g2s(dst + bx, dout + tok * RS, bdo, &s_full[slot]);
    if (dp) bulk_g2s(dst + bx + bdo, dp + tok * RS, bp, &s_full[slot]);
  };
  int64_t issued = 0;  // meaningful in thread 0
  if (tid == 0)
    for (; issued < NS && issued < ntok; ++issued) issue(issued);

  float aQ[N][N], aS[N];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    aS[i] = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) aQ[i][j] = 0.f;
  }
  const int groups = C / 4;
  int64_t k0 = 0;
  bool aborted = false;
  for (; k0 < ntok; k0 += TPI) {
    const int64_t k = k0 + hf;  // this part's token of the step
    if (k < ntok) {
      const int slot = (int)(k % NS);
      if (!mbar_wait(&s_full[slot], (unsigned)((k / NS) & 1))) s_abort = 1;
      const unsigned char* src = s_ring + (size_t)slot * sb;
      const XT* sx = reinterpret_cast<const XT*>(src);
      const DT* sd = reinterpret_cast<const DT*>(src + bx);
      const PT* sp = reinterpret_cast<const PT*>(src + bx + bdo);
      XT* dxt = dx ? dx + (blockIdx.x + k * G) * RS : nullptr;
      for (int g = lt; g < groups; g += HB) {
        float xr[N][4], dr[N][4], pv[N][4];
#pragma unroll
        for (int j = 0; j < N; ++j) lds4<XT>(sx + (int64_t)j * C + 4 * g, xr[j]);
#pragma unroll
        for (int i = 0; i < N; ++i) lds4<DT>(sd + (int64_t)i * C + 4 * g, dr[i]);
        if (dp) {
#pragma unroll
          for (int j = 0; j < N; ++j) lds4<PT>(sp + (int64_t)j * C + 4 * g, pv[j]);
        } else {
#pragma unroll
          for (int j = 0; j < N; ++j)
#pragma unroll
            for (int v = 0; v < 4; ++v) pv[j][v] = 0.f;
        }
#pragma unroll
        for (int i = 0; i < N; ++i)
#pragma unroll
          for (int j = 0; j < N; ++j)
#pragma unroll
            for (int v = 0; v < 4; ++v) aQ[i][j] = fmaf(dr[i][v], xr[j][v], aQ[i][j]);
#pragma unroll
        for (int j = 0; j < N; ++j) {
          const float4 w4 = *reinterpret_cast<const float4*>(sWT[j]);
          const float wj[4] = {w4.x, w4.y, w4.z, w4.w};
          float o[4];
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            aS[j] = fmaf(pv[j][v], xr[j][v], aS[j]);
            float a = pv[j][v];
#pragma unroll
            for (int i = 0; i < N; ++i) a = fmaf(wj[i], dr[i][v], a);
            o[v] = a * hpre[j];
          }
          if (dxt) store_vec<XT, 4>(dxt + (int64_t)j * C + 4 * g, o);
        }
      }
    }
    __syncthreads();  // every read of the pair's buffers done; s_abort agreed
    if (s_abort) { aborted = true; break; }
    if (tid == 0) {
      fence_proxy_async_smem();
      for (; issued < ntok && issued < k0 + TPI + NS; ++issued) issue(issued);
    }
  }
  if (aborted) {
    if (tid == 0)
      for (int64_t q = k0; q < issued; ++q)
        (void)mbar_wait(&s_full[q % NS], (unsigned)((q / NS) & 1));
    const float nan = __int_as_float(0x7fc00000);
    if (dx) {
      float o[4] = {nan, nan, nan, nan};
      for (int64_t k = k0 + hf; k < ntok; k += TPI)
        for (int g = lt; g < groups; g += HB)
#pragma unroll
          for (int j = 0; j < N; ++j)
            store_vec<XT, 4>(dx + (blockIdx.x + k * G) * RS + (int64_t)j * C + 4 * g, o);
    }
#pragma unroll
    for (int i = 0; i < N; ++i) {
      aS[i] = nan;
#pragma unroll
      for (int j = 0; j < N; ++j) aQ[i][j] = nan;
    }
  }
  rewire_x_rows<N>(aQ, aS, sM, hpre_g, hpost_g, ws_p, ws_hdr, row0, fin);
}

// ----------------------------------------------------------- prescale bwd --
// dx_i = hpre_i d_i;  R_i = sum d_i x_i  (-> dH_pre_act)
template <int MAXN, bool EXACT, typename XT, typename DT, typename DXT, int VEC>
__global__ void __launch_bounds__(kMixBD)
k_prescale_bwd(const XT* __restrict__ x, const DT* __restrict__ dout,
               const float* __restrict__ hpre_g, DXT* __restrict__ dx, int64_t T, int n, int C,
               float* __restrict__ ws_p, int* __restrict__ ws_hdr) {
  pdl_wait();
  pdl_trigger();
  __shared__ float shpre[MAXN];
  __shared__ float sacc[(kMixBD / 32) * MAXN];
  const int nr = EXACT ? MAXN : n;
  for (int e = threadIdx.x; e < nr; e += blockDim.x) shpre[e] = hpre_g[e];
  __syncthreads();
  float aR[MAXN];
#pragma unroll
  for (int i = 0; i < MAXN; ++i) aR[i] = 0.f;
  const int groups = (C + VEC - 1) / VEC;
  const int64_t items = T * groups;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < items;
       q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = q / groups;
    const int col = (int)(q - t * groups) * VEC;
    const int64_t base = t * (int64_t)nr * C + col;
    MHC_FOR_N(i) {
      float a[VEC], d[VEC];
      load_vec<XT, VEC>(x + base + (int64_t)i * C, a);
      load_vec<DT, VEC>(dout + base + (int64_t)i * C, d);
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        aR[i] = fmaf(d[v], a[v], aR[i]);
        d[v] *= shpre[i];
      }
      store_vec<DXT, VEC>(dx + base + (int64_t)i * C, d);
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  MHC_FOR_N(i) {
    const float v = warp_sum(aR[i]);
    if (lane == 0) sacc[warp * MAXN + i] = v;
  }
  __syncthreads();
  const int P = nr * nr + 2 * nr;
  float* pr = ws_p + (size_t)blockIdx.x * P;
  for (int e = threadIdx.x; e < P; e += blockDim.x) {
    float s = 0.f;
    if (e >= nr * nr && e < nr * nr + nr)
      for (int w = 0; w < nw; ++w) s += sacc[w * MAXN + (e - nr * nr)];
    pr[e] = s;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    ws_hdr[0] = gridDim.x;
    ws_hdr[3] = 0;  // ticket of the rewire x side's last-CTA finalize
  }
}

// ------------------------------------------------- residual add agg bwd --
// Backward of out = x + res, y_agg = sum_i hpre_i out_i (the reference
// registers no VJP for residual_add_agg; this adds it):
//   dx = dres = d_out + hpre_i * d_y;  dH_pre_i = sum d_y * out_i.
// out is read from the forward's saved output; d_out or d_y may be absent.
template <int MAXN, bool EXACT, typename OT, typename DT, typename DXT, int VEC>
__global__ void __launch_bounds__(kMixBD)
k_residual_bwd(const OT* __restrict__ out, const DT* __restrict__ dout,
               const float* __restrict__ dy, const float* __restrict__ hpre_g,
               DXT* __restrict__ dx, int64_t T, int n, int C, float* __restrict__ ws_p,
               int* __restrict__ ws_hdr) {
  __shared__ float shpre[MAXN];
  __shared__ float sacc[(kMixBD / 32) * MAXN];
  const int nr = EXACT ? MAXN : n;
  for (int e = threadIdx.x; e < nr; e += blockDim.x) shpre[e] = hpre_g[e];
  __syncthreads();
  float aR[MAXN];
#pragma unroll
  for (int i = 0; i < MAXN; ++i) aR[i] = 0.f;
  const int groups = (C + VEC - 1) / VEC;
  const int64_t items = T * groups;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < items;
       q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = q / groups;
    const int col = (int)(q - t * groups) * VEC;
    const int64_t base = t * (int64_t)nr * C + col;
    float g[VEC];
    if (dy) load_vec<float, VEC>(dy + t * C + col, g);
    else
#pragma unroll
      for (int v = 0; v < VEC; ++v) g[v] = 0.f;
    MHC_FOR_N(i) {
      float o[VEC], d[VEC];
      if (dout) load_vec<DT, VEC>(dout + base + (int64_t)i * C, d);
      else
#pragma unroll
        for (int v = 0; v < VEC; ++v) d[v] = 0.f;
      if (dy) {
        load_vec<OT, VEC>(out + base + (int64_t)i * C, o);
#pragma unroll
        for (int v = 0; v < VEC; ++v) aR[i] = fmaf(g[v], o[v], aR[i]);
      }
#pragma unroll
      for (int v = 0; v < VEC; ++v) d[v] = fmaf(shpre[i], g[v], d[v]);
      store_vec<DXT, VEC>(dx + base + (int64_t)i * C, d);
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  MHC_FOR_N(i) {
    const float v = warp_sum(aR[i]);
    if (lane == 0) sacc[warp * MAXN + i] = v;
  }
  __syncthreads();
  const int P = nr * nr + 2 * nr;
  float* pr = ws_p + (size_t)blockIdx.x * P;
  for (int e = threadIdx.x; e < P; e += blockDim.x) {
    float s = 0.f;
    if (e >= nr * nr && e < nr * nr + nr)
      for (int w = 0; w < nw; ++w) s += sacc[w * MAXN + (e - nr * nr)];
    pr[e] = s;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) ws_hdr[0] = gridDim.x;
}

// --------------------------------------------------------------- finalize --
// One CTA: sums the partial rows (fixed order) into Q (n*n) and R (n), then
//   mode 0 (mix):      dM = Q
//   mode 1 (rewire):   dM_ij = hpost_i hpre_j Q_ij, dhpre_j = sum_i hpost_i M_ij Q_ij,
//                      dhpost_i = R_i + sum_j M_ij hpre_j Q_ij
//   mode 2 (prescale): dhpre = R
//   mode 3 (rewire end to end): as mode 1 with dhpre_j += S_j; the rows of
//                      both passes are summed (header words 0 and 2)
// and, in modes 1 and 3 with pb.any(), carries on to the raw-parameter
// gradients (sigmoid chain rule, Sinkhorn backward: sk_params_bwd_tail) in
// the same launch.  Dynamic shared memory: [D (n * sk_ld(n)) | staged tape],
// D only for n > 8 without a Jacobian, the staged tape only when stage_sk.
// Thread t sums entry e = t % EW of a block of EW consecutive entries over the
// interleaved row slice t / EW (slice r takes rows r, r + S, ...; S = 1024 /
// EW slices), then the slices are added in order: a fixed order for a given
// row count.  EW is the entry count rounded up to a warp, at most 1024, so a
// few entries (n = 4: 24) get 32 slices of the rows (a one-CTA kernel is a
// latency chain: fewer dependent loads per thread) and many entries (n = 32:
// 1088) take two passes instead of one pass per 32 entries.
constexpr int kCFinBD = 1024;

__global__ void __launch_bounds__(kCFinBD)
k_combine_finalize(const char* __restrict__ ws, int n, const float* __restrict__ M,
                   const float* __restrict__ hpre, const float* __restrict__ hpost, int mode,
                   float* __restrict__ dM, float* __restrict__ dhpre, float* __restrict__ dhpost,
                   ParamsBwd pb, int stage_sk) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sQ[kMaxN * kMaxN + 2 * kMaxN];
  __shared__ float sA[kMaxN * kMaxN + 2 * kMaxN];  // [dM | dhpre | dhpost] for the tail
  __shared__ float part[kCFinBD];
  extern __shared__ float s_dyn[];
  const int* hdr = reinterpret_cast<const int*>(ws);
  const int G = mode == 3 ? hdr[0] + hdr[2] : hdr[0];
  const int P = n * n + 2 * n;
  const int E = mode == 3 ? P : n * n + n;  // entries summed
  const float* wp = reinterpret_cast<const float*>(ws + WsLayout::params_off());
  const int EW = min((E + 31) / 32 * 32, kCFinBD);
  const int S = kCFinBD / EW;
  const int el = threadIdx.x % EW, r0 = threadIdx.x / EW;
  for (int e0 = 0; e0 < E; e0 += EW) {
    const int e = e0 + el;
    float s = 0.f;
    if (e < E && r0 < S) {
#pragma unroll 8
      for (int g = r0; g < G; g += S) s += wp[(size_t)g * P + e];
    }
    part[threadIdx.x] = s;
    __syncthreads();
    if (r0 == 0 && e < E) {
      float t = 0.f;
      for (int q = 0; q < S; ++q) t += part[q * EW + el];
      sQ[e] = t;
    }
    __syncthreads();
  }
  const float* sR = sQ + n * n;
  if (mode == 0) {
    for (int e = threadIdx.x; e < n * n; e += blockDim.x) dM[e] = sQ[e];
    return;
  }
  if (mode == 2) {
    for (int e = threadIdx.x; e < n; e += blockDim.x) dhpre[e] = sR[e];
    return;
  }
  for (int e = threadIdx.x; e < n * n; e += blockDim.x) {
    const int i = e / n, j = e % n;
    const float v = (hpost[i] * hpre[j]) * sQ[e];
    sA[e] = v;
    if (dM) dM[e] = v;
  }
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    float s = 0.f;
    for (int i = 0; i < n; ++i) s = fmaf(hpost[i] * M[i * n + j], sQ[i * n + j], s);
    if (mode == 3) s += sR[n + j];
    sA[n * n + j] = s;
    if (dhpre) dhpre[j] = s;
  }
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float s = sR[i];
    for (int j = 0; j < n; ++j) s = fmaf(M[i * n + j] * hpre[j], sQ[i * n + j], s);
    sA[n * n + n + i] = s;
    if (dhpost) dhpost[i] = s;
  }
  if (!pb.any()) return;  // kernel argument: uniform over the block
  __syncthreads();        // sA complete
  const bool dreg = !sk_warp_ok(n) && !pb.jac;
  sk_params_bwd_tail<kCFinBD>(sA, n, pb.hpre_raw, pb.hpost_raw, pb.hres_raw, pb.tape, pb.jac,
                              pb.iters, pb.eps, stage_sk, s_dyn + (dreg ? n * sk_ld(n) : 0), s_dyn,
                              pb.dhpre_raw, pb.dhpost_raw, pb.dhres_raw);
}

// ================================================================= launch ==
static int mix_rows_cap() { return sm_count() * 4; }

static int elem_grid(int64_t items, int cap) {
  int64_t b = (items + kMixBD - 1) / kMixBD;
  if (b > cap) b = cap;
  return (int)(b < 1 ? 1 : b);
}

static bool all_aligned(std::initializer_list<const void*> ps) {
  for (const void* p : ps)
    if (p && !aligned16(p)) return false;
  return true;
}

// ---- combine forward (plain mix: hpre = hpost = NULL) ----------------------
template <typename XT, typename YT, typename OT>
static int combine_fwd_t(const void* xv, const void* yv, const float* M, const float* hpre,
                         const float* hpost, void* ov, int64_t T, int n, int C,
                         cudaStream_t st) {
  constexpr int VX = VecOf<XT>::value;
  const XT* x = static_cast<const XT*>(xv);
  const YT* y = static_cast<const YT*>(yv);
  OT* o = static_cast<OT*>(ov);
  const bool vec = (C % VX == 0) && all_aligned({xv, yv, ov});
  const int cap = sm_count() * 8;
  const int gv = elem_grid(T * (C / VX), cap), g1 = elem_grid(T * C, cap);
#define MHC_CF(NN, EX, V, G) \
  launch_pdl(k_combine_fwd<NN, EX, XT, YT, OT, V>, G, kMixBD, 0, st, x, y, M, hpre, hpost, o, T, n, C)
  switch (n) {
    case 1: if (vec) MHC_CF(1, true, VX, gv); else MHC_CF(1, true, 1, g1); break;
    case 2: if (vec) MHC_CF(2, true, VX, gv); else MHC_CF(2, true, 1, g1); break;
    case 4: if (vec) MHC_CF(4, true, VX, gv); else MHC_CF(4, true, 1, g1); break;
    case 8: if (vec) MHC_CF(8, true, VX, gv); else MHC_CF(8, true, 1, g1); break;
    case 16: MHC_CF(16, true, 1, g1); break;
    case 32: MHC_CF(32, true, 1, g1); break;
    default: MHC_CF(64, false, 1, g1); break;
  }
#undef MHC_CF
  return check_launch("combine_fwd");
}

// dtype triples: y in {x, f32}; out in {f32, x}
template <typename XT>
static int combine_fwd_x(const void* x, const void* y, int ydt, const float* M, const float* hpre,
                         const float* hpost, void* o, int odt, int64_t T, int n, int C,
                         cudaStream_t st, int xdt) {
  const bool y32 = ydt == MHC_F32, o32 = odt == MHC_F32;
  if (!y32 && ydt != xdt) return set_error(MHC_ERR_UNSUPPORTED, "mix: y dtype must be fp32 or x's dtype");
  if (!o32 && odt != xdt) return set_error(MHC_ERR_UNSUPPORTED, "mix: out dtype must be fp32 or x's dtype");
  if (y32 && o32) return combine_fwd_t<XT, float, float>(x, y, M, hpre, hpost, o, T, n, C, st);
  if (y32) return combine_fwd_t<XT, float, XT>(x, y, M, hpre, hpost, o, T, n, C, st);
  if (o32) return combine_fwd_t<XT, XT, float>(x, y, M, hpre, hpost, o, T, n, C, st);
  return combine_fwd_t<XT, XT, XT>(x, y, M, hpre, hpost, o, T, n, C, st);
}

static int combine_fwd(const void* x, int xdt, const void* y, int ydt, const float* M,
                       const float* hpre, const float* hpost, void* o, int odt, int64_t T, int n,
                       int C, cudaStream_t st) {
  if (T == 0) return MHC_OK;
  switch (xdt) {
    case MHC_F32: return combine_fwd_x<float>(x, y, ydt, M, hpre, hpost, o, odt, T, n, C, st, xdt);
    case MHC_BF16: return combine_fwd_x<bf16>(x, y, ydt, M, hpre, hpost, o, odt, T, n, C, st, xdt);
    default: return combine_fwd_x<f16>(x, y, ydt, M, hpre, hpost, o, odt, T, n, C, st, xdt);
  }
}

int launch_mix_add_fwd(const void* x, int xdt, const float* M, const void* y, int ydt, void* out,
                       int odt, int64_t T, int n, int C, cudaStream_t st) {
  return combine_fwd(x, xdt, y, ydt, M, nullptr, nullptr, out, odt, T, n, C, st);
}

int launch_rewire_fwd(const void* x, int xdt, const void* y, int ydt, const float* M,
                      const float* hpre, const float* hpost, void* out, int odt, int64_t T,
                      int n, int C, cudaStream_t st) {
  return combine_fwd(x, xdt, y, ydt, M, hpre, hpost, out, odt, T, n, C, st);
}

// ---- combine backward --------------------------------------------------------
size_t mix_ws_bytes(int64_t T, int n, int C) {
  (void)T; (void)C;
  return WsLayout::bytes(mix_rows_cap(), n, 0);
}

template <typename XT, typename YT, typename DT>
static int combine_bwd_t(const void* xv, const void* yv, const void* dv, const float* M,
                         const float* hpre, const float* hpost, void* dxv, void* dyv, int64_t T,
                         int n, int C, void* ws, cudaStream_t st) {
  using DXT = XT;
  using DYT = YT;
  constexpr int VX = VecOf<XT>::value;
  const XT* x = static_cast<const XT*>(xv);
  const YT* y = static_cast<const YT*>(yv);
  const DT* d = static_cast<const DT*>(dv);
  DXT* dx = static_cast<DXT*>(dxv);
  DYT* dy = static_cast<DYT*>(dyv);
  char* b = static_cast<char*>(ws);
  float* wp = reinterpret_cast<float*>(b + WsLayout::params_off());
  int* hdr = reinterpret_cast<int*>(b);
  const int cap = mix_rows_cap();
  const bool vec = (C % VX == 0) && all_aligned({xv, yv, dv, dxv, dyv});
  const int gv = elem_grid(T * (C / VX), cap), g1 = elem_grid(T * C, cap);
  const bool has_y = y != nullptr;
#define MHC_CB(NN, V, HY, G)                                                                    \
  k_combine_bwd_fast<NN, XT, YT, DT, DXT, DYT, V, HY><<<G, kMixBD, 0, st>>>(x, y, d, M, hpre,  \
                                                                            hpost, dx, dy, T, \
                                                                            C, wp, hdr)
#define MHC_CB2(NN, V, G) \
  do { if (has_y) MHC_CB(NN, V, true, G); else MHC_CB(NN, V, false, G); } while (0)
  switch (n) {
    case 1: if (vec) MHC_CB2(1, VX, gv); else MHC_CB2(1, 1, g1); return check_launch("combine_bwd");
    case 2: if (vec) MHC_CB2(2, VX, gv); else MHC_CB2(2, 1, g1); return check_launch("combine_bwd");
    case 4: if (vec) MHC_CB2(4, VX, gv); else MHC_CB2(4, 1, g1); return check_launch("combine_bwd");
    case 8: MHC_CB2(8, 1, g1); return check_launch("combine_bwd");
    default: break;
  }
#undef MHC_CB2
#undef MHC_CB
  const size_t smem = mix_gen_smem(n);
  auto kern = k_combine_bwd_generic<XT, YT, DT, DXT, DYT>;
  {
    cudaError_t e = allow_dyn_smem(kern, smem);
    if (e != cudaSuccess) return set_error(MHC_ERR_CUDA, "combine_bwd: %s", cudaGetErrorString(e));
  }
  const int64_t ntile = T * ((C + kMixGenBD - 1) / kMixGenBD);
  const int G = (int)(ntile < cap ? (ntile < 1 ? 1 : ntile) : cap);
  kern<<<G, kMixGenBD, smem, st>>>(x, y, d, M, hpre, hpost, dx, dy, T, n, C, wp, hdr);
  return check_launch("combine_bwd(generic)");
}

template <typename XT>
static int combine_bwd_x(const void* x, int xdt, const void* y, int ydt, const void* d, int ddt,
                         const float* M, const float* hpre, const float* hpost, void* dx,
                         void* dy, int64_t T, int n, int C, void* ws, cudaStream_t st) {
  const bool y32 = (y == nullptr) || ydt == MHC_F32;
  const bool d32 = ddt == MHC_F32;
  if (y && !y32 && ydt != xdt) return set_error(MHC_ERR_UNSUPPORTED, "mix bwd: y dtype must be fp32 or x's dtype");
  if (!d32 && ddt != xdt) return set_error(MHC_ERR_UNSUPPORTED, "mix bwd: d_out dtype must be fp32 or x's dtype");
  if (y32 && d32) return combine_bwd_t<XT, float, float>(x, y, d, M, hpre, hpost, dx, dy, T, n, C, ws, st);
  if (y32) return combine_bwd_t<XT, float, XT>(x, y, d, M, hpre, hpost, dx, dy, T, n, C, ws, st);
  if (d32) return combine_bwd_t<XT, XT, float>(x, y, d, M, hpre, hpost, dx, dy, T, n, C, ws, st);
  return combine_bwd_t<XT, XT, XT>(x, y, d, M, hpre, hpost, dx, dy, T, n, C, ws, st);
}

static int combine_bwd(const void* x, int xdt, const void* y, int ydt, const void* d, int ddt,
                       const float* M, const float* hpre, const float* hpost, void* dx, int dxdt,
                       void* dy, int dydt, int mode, float* dM, float* dhpre, float* dhpost,
                       int64_t T, int n, int C, void* ws, size_t ws_bytes, cudaStream_t st) {
  const size_t need = mix_ws_bytes(T, n, C);
  if (!ws || ws_bytes < need)
    return set_error(MHC_ERR_WORKSPACE, "mix bwd: workspace %zu < %zu bytes", ws_bytes, need);
  if (dxdt != xdt) return set_error(MHC_ERR_UNSUPPORTED, "mix bwd: dx dtype must equal x dtype");
  if (dy && dydt != (y ? ydt : dydt))
    return set_error(MHC_ERR_UNSUPPORTED, "mix bwd: dy dtype must equal y dtype");
  int r;
  switch (xdt) {
    case MHC_F32: r = combine_bwd_x<float>(x, xdt, y, ydt, d, ddt, M, hpre, hpost, dx, dy, T, n, C, ws, st); break;
    case MHC_BF16: r = combine_bwd_x<bf16>(x, xdt, y, ydt, d, ddt, M, hpre, hpost, dx, dy, T, n, C, ws, st); break;
    default: r = combine_bwd_x<f16>(x, xdt, y, ydt, d, ddt, M, hpre, hpost, dx, dy, T, n, C, ws, st); break;
  }
  if (r != MHC_OK) return r;
  k_combine_finalize<<<1, kCFinBD, 0, st>>>(static_cast<const char*>(ws), n, M, hpre, hpost, mode,
                                            dM, dhpre, dhpost, ParamsBwd{}, 0);
  return check_launch("combine_finalize");
}

int launch_mix_add_bwd(const void* x, int xdt, const float* M, const void* dout, int ddt,
                       void* dx, int dxdt, float* dM, int64_t T, int n, int C, void* ws,
                       size_t ws_bytes, cudaStream_t st) {
  return combine_bwd(x, xdt, nullptr, MHC_F32, dout, ddt, M, nullptr, nullptr, dx, dxdt, nullptr,
                     MHC_F32, 0, dM, nullptr, nullptr, T, n, C, ws, ws_bytes, st);
}

int launch_rewire_bwd(const void* x, int xdt, const void* y, int ydt, const void* dout, int ddt,
                      const float* M, const float* hpre, const float* hpost, void* dx, int dxdt,
                      void* dy, int dydt, float* dM, float* dhpre, float* dhpost, int64_t T,
                      int n, int C, void* ws, size_t ws_bytes, cudaStream_t st) {
  return combine_bwd(x, xdt, y, ydt, dout, ddt, M, hpre, hpost, dx, dxdt, dy, dydt, 1, dM,
                     dhpre, dhpost, T, n, C, ws, ws_bytes, st);
}

// ---- pre-scale -----------------------------------------------------------------
template <typename XT, typename OT>
static int prescale_fwd_t(const void* xv, const float* hpre, void* ov, int64_t T, int n, int C,
                          const ParamsFwd* pf, cudaStream_t st) {
  constexpr int VX = VecOf<XT>::value;
  const XT* x = static_cast<const XT*>(xv);
  OT* o = static_cast<OT*>(ov);
  const bool vec = (C % VX == 0) && all_aligned({xv, ov});
  const int cap = sm_count() * 8;
  const int gv = elem_grid(T * (C / VX), cap), g1 = elem_grid(T * C, cap);
  if (pf) {  // n in {1, 2, 4, 8}: one more block for the parameters
    // with a Jacobian to compute, the tape is staged in shared memory when it
    // is small (every block gets the allocation: at most 8 KB)
    ParamsFwd q = *pf;
    const size_t tb = sk_tape_floats(n, q.iters) * sizeof(float);
    q.stage = (q.jac && sk_lane_ok(n) && q.iters > 0 && tb <= 8 * 1024) ? 1 : 0;
    const size_t smem = q.stage ? tb : 0;
    // the streaming blocks plus the parameter block fill one wave of 8 per SM
    // (a streaming block beyond it would start only when the parameter block
    // ends and finish that much later)
    const int pv = std::max(1, std::min(gv, cap - 1)), p1 = std::max(1, std::min(g1, cap - 1));
#define MHC_PP(NN, V, G) \
  launch_pdl(k_prescale_fwd<NN, true, XT, OT, V, true>, G + 1, kMixBD, smem, st, x, nullptr, o, T, n, C, q)
    switch (n) {
      case 1: if (vec) MHC_PP(1, VX, pv); else MHC_PP(1, 1, p1); break;
      case 2: if (vec) MHC_PP(2, VX, pv); else MHC_PP(2, 1, p1); break;
      case 4: if (vec) MHC_PP(4, VX, pv); else MHC_PP(4, 1, p1); break;
      default: if (vec) MHC_PP(8, VX, pv); else MHC_PP(8, 1, p1); break;
    }
#undef MHC_PP
    return check_launch("rewire_in_fwd");
  }
#define MHC_PF(NN, EX, V, G) \
  launch_pdl(k_prescale_fwd<NN, EX, XT, OT, V>, G, kMixBD, 0, st, x, hpre, o, T, n, C, ParamsFwd{})
  switch (n) {
    case 1: if (vec) MHC_PF(1, true, VX, gv); else MHC_PF(1, true, 1, g1); break;
    case 2: if (vec) MHC_PF(2, true, VX, gv); else MHC_PF(2, true, 1, g1); break;
    case 4: if (vec) MHC_PF(4, true, VX, gv); else MHC_PF(4, true, 1, g1); break;
    case 8: if (vec) MHC_PF(8, true, VX, gv); else MHC_PF(8, true, 1, g1); break;
    case 16: if (vec) MHC_PF(16, true, VX, gv); else MHC_PF(16, true, 1, g1); break;
    case 32: if (vec) MHC_PF(32, true, VX, gv); else MHC_PF(32, true, 1, g1); break;
    default: if (vec) MHC_PF(64, false, VX, gv); else MHC_PF(64, false, 1, g1); break;
  }
#undef MHC_PF
  return check_launch("prescale_fwd");
}

static int prescale_fwd_any(const void* x, int xdt, const float* hpre, void* xo, int odt,
                            int64_t T, int n, int C, const ParamsFwd* pf, cudaStream_t st) {
  if (odt != xdt && odt != MHC_F32)
    return set_error(MHC_ERR_UNSUPPORTED, "prescale: out dtype must be fp32 or x's dtype");
  switch (xdt) {
    case MHC_F32: return prescale_fwd_t<float, float>(x, hpre, xo, T, n, C, pf, st);
    case MHC_BF16:
      return odt == MHC_F32 ? prescale_fwd_t<bf16, float>(x, hpre, xo, T, n, C, pf, st)
                            : prescale_fwd_t<bf16, bf16>(x, hpre, xo, T, n, C, pf, st);
    default:
      return odt == MHC_F32 ? prescale_fwd_t<f16, float>(x, hpre, xo, T, n, C, pf, st)
                            : prescale_fwd_t<f16, f16>(x, hpre, xo, T, n, C, pf, st);
  }
}

int launch_prescale_fwd(const void* x, int xdt, const float* hpre, void* xo, int odt, int64_t T,
                        int n, int C, cudaStream_t st) {
  if (T == 0) return MHC_OK;
  return prescale_fwd_any(x, xdt, hpre, xo, odt, T, n, C, nullptr, st);
}

// MHCRewire's input side: parameters + pre-scale in one launch for n <= 8
// (the one-warp Sinkhorn paths), else the parameter kernel and then the
// pre-scale.  The Jacobian is written for n <= 4 when pf.jac is given.
int launch_rewire_in_fwd(const void* x, int xdt, const ParamsFwd& pf, void* xo, int odt, int64_t T,
                         int n, int C, cudaStream_t st) {
  if (sk_warp_ok(n))  // T = 0 too: the parameter block still runs
    return prescale_fwd_any(x, xdt, nullptr, xo, odt, T, n, C, &pf, st);
  int r = launch_params_fwd(pf.hpre_raw, pf.hpost_raw, pf.hres_raw, n, pf.iters, pf.eps, pf.hpre,
                            pf.hpost, pf.M, pf.tape, st);
  if (r != MHC_OK || T == 0) return r;
  return prescale_fwd_any(x, xdt, pf.hpre, xo, odt, T, n, C, nullptr, st);
}

template <typename XT, typename DT>
static int prescale_bwd_t(const void* xv, const void* dv, const float* hpre, void* dxv, int64_t T,
                          int n, int C, void* ws, cudaStream_t st) {
  constexpr int VX = VecOf<XT>::value;
  const XT* x = static_cast<const XT*>(xv);
  const DT* d = static_cast<const DT*>(dv);
  XT* dx = static_cast<XT*>(dxv);
  char* b = static_cast<char*>(ws);
  float* wp = reinterpret_cast<float*>(b + WsLayout::params_off());
  int* hdr = reinterpret_cast<int*>(b);
  const bool vec = (C % VX == 0) && all_aligned({xv, dv, dxv});
  const int cap = mix_rows_cap();
  const int gv = elem_grid(T * (C / VX), cap), g1 = elem_grid(T * C, cap);
#define MHC_PB(NN, EX, V, G) \
  launch_pdl(k_prescale_bwd<NN, EX, XT, DT, XT, V>, G, kMixBD, 0, st, x, d, hpre, dx, T, n, C, wp, hdr)
  switch (n) {
    case 1: if (vec) MHC_PB(1, true, VX, gv); else MHC_PB(1, true, 1, g1); break;
    case 2: if (vec) MHC_PB(2, true, VX, gv); else MHC_PB(2, true, 1, g1); break;
    case 4: if (vec) MHC_PB(4, true, VX, gv); else MHC_PB(4, true, 1, g1); break;
    case 8: if (vec) MHC_PB(8, true, VX, gv); else MHC_PB(8, true, 1, g1); break;
    case 16: MHC_PB(16, true, 1, g1); break;
    case 32: MHC_PB(32, true, 1, g1); break;
    default: MHC_PB(64, false, 1, g1); break;
  }
#undef MHC_PB
  return check_launch("prescale_bwd");
}

int launch_prescale_bwd(const void* x, int xdt, const void* d, int ddt, const float* hpre,
                        void* dx, int dxdt, float* dhpre, int64_t T, int n, int C, void* ws,
                        size_t ws_bytes, cudaStream_t st) {
  const size_t need = mix_ws_bytes(T, n, C);
  if (!ws || ws_bytes < need)
    return set_error(MHC_ERR_WORKSPACE, "prescale bwd: workspace %zu < %zu bytes", ws_bytes, need);
  if (dxdt != xdt) return set_error(MHC_ERR_UNSUPPORTED, "prescale bwd: dx dtype must equal x dtype");
  if (ddt != xdt && ddt != MHC_F32)
    return set_error(MHC_ERR_UNSUPPORTED, "prescale bwd: d dtype must be fp32 or x's dtype");
  int r;
  switch (xdt) {
    case MHC_F32: r = prescale_bwd_t<float, float>(x, d, hpre, dx, T, n, C, ws, st); break;
    case MHC_BF16:
      r = ddt == MHC_F32 ? prescale_bwd_t<bf16, float>(x, d, hpre, dx, T, n, C, ws, st)
                         : prescale_bwd_t<bf16, bf16>(x, d, hpre, dx, T, n, C, ws, st);
      break;
    default:
      r = ddt == MHC_F32 ? prescale_bwd_t<f16, float>(x, d, hpre, dx, T, n, C, ws, st)
                         : prescale_bwd_t<f16, f16>(x, d, hpre, dx, T, n, C, ws, st);
      break;
  }
  if (r != MHC_OK) return r;
  k_combine_finalize<<<1, kCFinBD, 0, st>>>(static_cast<const char*>(ws), n, nullptr, nullptr,
                                            nullptr, 2, nullptr, dhpre, nullptr, ParamsBwd{}, 0);
  return check_launch("prescale_finalize");
}

// ---- MHCRewire end to end: dy side and x side ------------------------------------
size_t rewire_fused_ws_bytes(int64_t T, int n, int C) {
  (void)T; (void)C;
  return WsLayout::bytes(2 * mix_rows_cap(), n, 0);
}

// dy_i = hpost_i d_i and R_i = sum d_i y_i: the pre-scale backward's
// arithmetic with (y, hpost, dy) in place of (x, hpre, dx); its rows carry R
// in slot n*n and zeros elsewhere, and it records G1 in header word 0.
int launch_rewire_bwd_dy(const void* y, int ydt, const void* d, int ddt, const float* hpost,
                         void* dy, int dydt, int64_t T, int n, int C, void* ws, size_t ws_bytes,
                         cudaStream_t st) {
  const size_t need = rewire_fused_ws_bytes(T, n, C);
  if (!ws || ws_bytes < need)
    return set_error(MHC_ERR_WORKSPACE, "rewire bwd: workspace %zu < %zu bytes", ws_bytes, need);
  if (dydt != ydt) return set_error(MHC_ERR_UNSUPPORTED, "rewire bwd: dy dtype must equal y dtype");
  if (ddt != ydt && ddt != MHC_F32)
    return set_error(MHC_ERR_UNSUPPORTED, "rewire bwd: d_out dtype must be fp32 or y's dtype");
  switch (ydt) {
    case MHC_F32: return prescale_bwd_t<float, float>(y, d, hpost, dy, T, n, C, ws, st);
    case MHC_BF16:
      return ddt == MHC_F32 ? prescale_bwd_t<bf16, float>(y, d, hpost, dy, T, n, C, ws, st)
                            : prescale_bwd_t<bf16, bf16>(y, d, hpost, dy, T, n, C, ws, st);
    default:
      return ddt == MHC_F32 ? prescale_bwd_t<f16, float>(y, d, hpost, dy, T, n, C, ws, st)
                            : prescale_bwd_t<f16, f16>(y, d, hpost, dy, T, n, C, ws, st);
  }
}

// *finished: the x side's last CTA ran the finalize (fast path, fin.on).
template <typename XT, typename DT, typename PT>
static int rewire_x_t(const void* xv, const void* dv, const void* pv, const float* M,
                      const float* hpre, const float* hpost, void* dxv, int64_t T, int n, int C,
                      void* ws, RewireFin fin, bool* finished, cudaStream_t st) {
  constexpr int VX = VecOf<XT>::value;
  // 4 columns per item: all of an item's loads fit in registers at once
  constexpr int V4 = 4;
  const XT* x = static_cast<const XT*>(xv);
  const DT* d = static_cast<const DT*>(dv);
  const PT* p = static_cast<const PT*>(pv);
  XT* dx = static_cast<XT*>(dxv);
  char* b = static_cast<char*>(ws);
  float* wp = reinterpret_cast<float*>(b + WsLayout::params_off());
  int* hdr = reinterpret_cast<int*>(b);
  const int cap = mix_rows_cap();
  const bool vec = (C % VX == 0) && all_aligned({xv, dv, pv, dxv});
  if (vec && (n == 1 || n == 2 || n == 4)) {
    fin.on = aligned16(ws) ? 1 : 0;  // the last CTA's 16-byte row loads
    *finished = fin.on != 0;
    // Bulk-copy staging when a token's rows are whole 16-byte runs and at
    // least three tokens fit in the ring (MHC_B200_XBULK=0: the register
    // kernel below, for comparison).
    const int64_t RS = (int64_t)n * C;
    const bool runs16 = C % 4 == 0 && (RS * (int64_t)sizeof(XT)) % 16 == 0 &&
                        (RS * (int64_t)sizeof(DT)) % 16 == 0 &&
                        (!pv || (RS * (int64_t)sizeof(PT)) % 16 == 0);
    const int64_t sb = RS * (int64_t)(sizeof(XT) + sizeof(DT) + (pv ? sizeof(PT) : 0));
    const int64_t budget = (int64_t)max_smem_optin() - 12 * 1024;  // static shared memory aside
    const int NS = sb > 0 ? (int)std::min<int64_t>(kXBulkMaxStages, budget / sb) : 0;
    static const bool bulk_on = [] {
      const char* v = getenv("MHC_B200_XBULK");
      return !(v && *v == '0');
    }();
    // tokens per step (MHC_B200_XBULK_TPI: 2 or 4); the ring must hold a step
    // and at least one token ahead
    static const int tpi = [] {
      const char* v = getenv("MHC_B200_XBULK_TPI");
      return (v && *v == '2') ? 2 : 4;
    }();
    if (bulk_on && runs16 && NS >= tpi + 1) {
      const int G = (int)std::max<int64_t>(1, std::min<int64_t>(sm_count(), T));
      const size_t smem = (size_t)NS * (size_t)sb;
#define MHC_RB(NN)                                                                            \
  do {                                                                                        \
    auto kern = tpi == 2 ? k_rewire_bwd_x_bulk<NN, XT, DT, PT, 2>                             \
                         : k_rewire_bwd_x_bulk<NN, XT, DT, PT, 4>;                            \
    const cudaError_t e = allow_dyn_smem(kern, smem);                                         \
    if (e != cudaSuccess)                                                                     \
      return set_error(MHC_ERR_CUDA, "rewire_bwd_x_bulk: %s", cudaGetErrorString(e));        \
    launch_pdl(kern, G, kXBulkBD, smem, st, x, d, p, M, hpre, hpost, dx, T, C, NS, wp, hdr, fin); \
  } while (0)
      if (n == 1) MHC_RB(1);
      else if (n == 2) MHC_RB(2);
      else MHC_RB(4);
#undef MHC_RB
      return check_launch("rewire_bwd_x_bulk");
    }
    const int G = elem_grid(T * (C / V4), cap);
#define MHC_RX(NN) \
  launch_pdl(k_rewire_bwd_x_fast<NN, XT, DT, PT, V4>, G, kMixBD, 0, st, x, d, p, M, hpre, hpost, dx, T, C, wp, hdr, fin)
    if (n == 1) MHC_RX(1);
    else if (n == 2) MHC_RX(2);
    else MHC_RX(4);
#undef MHC_RX
    return check_launch("rewire_bwd_x");
  }
  const size_t smem = mix_gen_smem(n);
  auto kern = k_combine_bwd_generic<XT, PT, DT, XT, XT, true>;
  {
    cudaError_t e = allow_dyn_smem(kern, smem);
    if (e != cudaSuccess) return set_error(MHC_ERR_CUDA, "rewire_bwd_x: %s", cudaGetErrorString(e));
  }
  const int64_t ntile = T * ((C + kMixGenBD - 1) / kMixGenBD);
  const int G = (int)(ntile < cap ? (ntile < 1 ? 1 : ntile) : cap);
  kern<<<G, kMixGenBD, smem, st>>>(x, p, d, M, hpre, hpost, dx, nullptr, T, n, C, wp, hdr);
  return check_launch("rewire_bwd_x(generic)");
}

template <typename XT>
static int rewire_x_x(const void* x, int xdt, const void* d, int ddt, const void* p, int pdt,
                      const float* M, const float* hpre, const float* hpost, void* dx, int64_t T,
                      int n, int C, void* ws, const RewireFin& fin, bool* fd, cudaStream_t st) {
  const bool d32 = ddt == MHC_F32, p32 = (p == nullptr) || pdt == MHC_F32;
  if (!d32 && ddt != xdt) return set_error(MHC_ERR_UNSUPPORTED, "rewire bwd: d_out dtype must be fp32 or x's dtype");
  if (!p32 && pdt != xdt) return set_error(MHC_ERR_UNSUPPORTED, "rewire bwd: d_xpre dtype must be fp32 or x's dtype");
  if (d32 && p32) return rewire_x_t<XT, float, float>(x, d, p, M, hpre, hpost, dx, T, n, C, ws, fin, fd, st);
  if (d32) return rewire_x_t<XT, float, XT>(x, d, p, M, hpre, hpost, dx, T, n, C, ws, fin, fd, st);
  if (p32) return rewire_x_t<XT, XT, float>(x, d, p, M, hpre, hpost, dx, T, n, C, ws, fin, fd, st);
  return rewire_x_t<XT, XT, XT>(x, d, p, M, hpre, hpost, dx, T, n, C, ws, fin, fd, st);
}

int launch_rewire_bwd_dx(const void* x, int xdt, const void* d, int ddt, const void* p, int pdt,
                         const float* M, const float* hpre, const float* hpost, void* dx, int dxdt,
                         float* dM, float* dhpre, float* dhpost, const ParamsBwd& pb, int64_t T,
                         int n, int C, void* ws, size_t ws_bytes, cudaStream_t st) {
  const size_t need = rewire_fused_ws_bytes(T, n, C);
  if (!ws || ws_bytes < need)
    return set_error(MHC_ERR_WORKSPACE, "rewire bwd: workspace %zu < %zu bytes", ws_bytes, need);
  if (dx && dxdt != xdt) return set_error(MHC_ERR_UNSUPPORTED, "rewire bwd: dx dtype must equal x dtype");
  // The fast x side (n <= 4) finalizes in its last CTA, the Jacobian or the
  // lane-path sweep included; otherwise the one-CTA finalize kernel follows.
  const RewireFin fin{dM, dhpre, dhpost, pb, 0};
  bool finished = false;
  int r;
  switch (xdt) {
    case MHC_F32: r = rewire_x_x<float>(x, xdt, d, ddt, p, pdt, M, hpre, hpost, dx, T, n, C, ws, fin, &finished, st); break;
    case MHC_BF16: r = rewire_x_x<bf16>(x, xdt, d, ddt, p, pdt, M, hpre, hpost, dx, T, n, C, ws, fin, &finished, st); break;
    default: r = rewire_x_x<f16>(x, xdt, d, ddt, p, pdt, M, hpre, hpost, dx, T, n, C, ws, fin, &finished, st); break;
  }
  if (r != MHC_OK || finished) return r;
  // The raw-parameter chain rule runs in the finalize when its thread count
  // suits the Sinkhorn path of n, else as the separate parameter kernel on
  // the activation gradients the finalize wrote.
  const bool fold = pb.any() && sk_tail_ok(n, kCFinBD);
  size_t dyn = 0;
  int stage = 0;
  if (fold && !pb.jac && pb.hres_raw && pb.dhres_raw && pb.tape) {
    if (!sk_warp_ok(n)) dyn += (size_t)n * sk_ld(n) * sizeof(float);
    const size_t sb = sk_stage_floats(n, pb.iters) * sizeof(float);
    if (dyn + sb <= 150 * 1024) {
      dyn += sb;
      stage = 1;
    }
  } else if (fold && !pb.jac && !sk_warp_ok(n)) {
    dyn = (size_t)n * sk_ld(n) * sizeof(float);
  }
  {
    const cudaError_t e = allow_dyn_smem(k_combine_finalize, dyn);
    if (e != cudaSuccess)
      return set_error(MHC_ERR_CUDA, "rewire_bwd_finalize: %s", cudaGetErrorString(e));
  }
  launch_pdl(k_combine_finalize, 1, kCFinBD, dyn, st, static_cast<const char*>(ws), n, M, hpre,
             hpost, 3, dM, dhpre, dhpost, fold ? pb : ParamsBwd{}, stage);
  r = check_launch("rewire_bwd_finalize");
  if (r != MHC_OK || !pb.any() || fold) return r;
  return launch_params_bwd(pb.hpre_raw, pb.hpost_raw, pb.hres_raw, pb.tape, n, pb.iters, pb.eps,
                           dhpre, dhpost, dM, pb.dhpre_raw, pb.dhpost_raw, pb.dhres_raw, st);
}

// ---- residual add + aggregate ----------------------------------------------------
template <typename XT, typename RT, typename OT>
static int residual_t(const void* xv, const void* rv, const float* hpre, void* ov, float* yagg,
                      int64_t T, int n, int C, cudaStream_t st) {
  constexpr int VX = VecOf<XT>::value;
  const XT* x = static_cast<const XT*>(xv);
  const RT* r = static_cast<const RT*>(rv);
  OT* o = static_cast<OT*>(ov);
  const bool vec = (C % VX == 0) && all_aligned({xv, rv, ov, yagg});
  const int cap = sm_count() * 8;
  const int gv = elem_grid(T * (C / VX), cap), g1 = elem_grid(T * C, cap);
#define MHC_RA(NN, EX, V, G) \
  k_residual_add_agg<NN, EX, XT, RT, OT, V><<<G, kMixBD, 0, st>>>(x, r, hpre, o, yagg, T, n, C)
  switch (n) {
    case 1: if (vec) MHC_RA(1, true, VX, gv); else MHC_RA(1, true, 1, g1); break;
    case 2: if (vec) MHC_RA(2, true, VX, gv); else MHC_RA(2, true, 1, g1); break;
    case 4: if (vec) MHC_RA(4, true, VX, gv); else MHC_RA(4, true, 1, g1); break;
    case 8: if (vec) MHC_RA(8, true, VX, gv); else MHC_RA(8, true, 1, g1); break;
    case 16: if (vec) MHC_RA(16, true, VX, gv); else MHC_RA(16, true, 1, g1); break;
    case 32: if (vec) MHC_RA(32, true, VX, gv); else MHC_RA(32, true, 1, g1); break;
    default: MHC_RA(64, false, 1, g1); break;
  }
#undef MHC_RA
  return check_launch("residual_add_agg");
}

template <typename XT>
static int residual_x(const void* x, int xdt, const void* r, int rdt, const float* hpre, void* o,
                      int odt, float* yagg, int64_t T, int n, int C, cudaStream_t st) {
  if (rdt != xdt) return set_error(MHC_ERR_UNSUPPORTED, "residual_add_agg: res dtype must equal x dtype");
  if (odt == MHC_F32) return residual_t<XT, XT, float>(x, r, hpre, o, yagg, T, n, C, st);
  if (odt == MHC_BF16) return residual_t<XT, XT, bf16>(x, r, hpre, o, yagg, T, n, C, st);
  return residual_t<XT, XT, f16>(x, r, hpre, o, yagg, T, n, C, st);
}

int launch_residual_add_agg(const void* x, int xdt, const void* res, int rdt, const float* hpre,
                            void* out, int odt, float* yagg, int64_t T, int n, int C,
                            cudaStream_t st) {
  if (T == 0) return MHC_OK;
  switch (xdt) {
    case MHC_F32: return residual_x<float>(x, xdt, res, rdt, hpre, out, odt, yagg, T, n, C, st);
    case MHC_BF16: return residual_x<bf16>(x, xdt, res, rdt, hpre, out, odt, yagg, T, n, C, st);
    default: return residual_x<f16>(x, xdt, res, rdt, hpre, out, odt, yagg, T, n, C, st);
  }
}

// ---- residual add + aggregate: backward -----------------------------------------
template <typename OT, typename DT, typename DXT>
static int residual_bwd_t(const void* ov, const void* dv, const float* dy, const float* hpre,
                          void* dxv, int64_t T, int n, int C, void* ws, cudaStream_t st) {
  constexpr int VO = VecOf<OT>::value, VD = VecOf<DT>::value, VX = VecOf<DXT>::value;
  constexpr int V = VO < VD ? (VO < VX ? VO : VX) : (VD < VX ? VD : VX);  // fp32 anywhere -> 4
  const OT* o = static_cast<const OT*>(ov);
  const DT* d = static_cast<const DT*>(dv);
  DXT* dx = static_cast<DXT*>(dxv);
  char* b = static_cast<char*>(ws);
  float* wp = reinterpret_cast<float*>(b + WsLayout::params_off());
  int* hdr = reinterpret_cast<int*>(b);
  const bool vec = (C % 4 == 0) && (C % V == 0) && all_aligned({ov, dv, dy, dxv});
  const int cap = mix_rows_cap();
  const int gv = elem_grid(T * (C / V), cap), g1 = elem_grid(T * C, cap);
#define MHC_RB(NN, EX, VV, G) \
  k_residual_bwd<NN, EX, OT, DT, DXT, VV><<<G, kMixBD, 0, st>>>(o, d, dy, hpre, dx, T, n, C, wp, hdr)
  switch (n) {
    case 1: if (vec) MHC_RB(1, true, V, gv); else MHC_RB(1, true, 1, g1); break;
    case 2: if (vec) MHC_RB(2, true, V, gv); else MHC_RB(2, true, 1, g1); break;
    case 4: if (vec) MHC_RB(4, true, V, gv); else MHC_RB(4, true, 1, g1); break;
    case 8: if (vec) MHC_RB(8, true, V, gv); else MHC_RB(8, true, 1, g1); break;
    case 16: MHC_RB(16, true, 1, g1); break;
    case 32: MHC_RB(32, true, 1, g1); break;
    default: MHC_RB(64, false, 1, g1); break;
  }
#undef MHC_RB
  return check_launch("residual_add_agg_bwd");
}

template <typename OT>
static int residual_bwd_o(const void* o, const void* d, int ddt, const float* dy,
                          const float* hpre, void* dx, int dxdt, int64_t T, int n, int C,
                          void* ws, cudaStream_t st, int odt) {
  // d_out has out's dtype (or is absent); dx has the dtype chosen by the caller
  if (d && ddt != odt) return set_error(MHC_ERR_UNSUPPORTED, "residual_add_agg_bwd: d_out dtype must equal out dtype");
  switch (dxdt) {
    case MHC_F32: return residual_bwd_t<OT, OT, float>(o, d, dy, hpre, dx, T, n, C, ws, st);
    case MHC_BF16: return residual_bwd_t<OT, OT, bf16>(o, d, dy, hpre, dx, T, n, C, ws, st);
    default: return residual_bwd_t<OT, OT, f16>(o, d, dy, hpre, dx, T, n, C, ws, st);
  }
}

int launch_residual_add_agg_bwd(const void* out, int odt, const void* dout, int ddt,
                                const float* dy, const float* hpre, void* dx, int dxdt,
                                float* dhpre, int64_t T, int n, int C, void* ws, size_t ws_bytes,
                                cudaStream_t st) {
  const size_t need = mix_ws_bytes(T, n, C);
  if (!ws || ws_bytes < need)
    return set_error(MHC_ERR_WORKSPACE, "residual_add_agg_bwd: workspace %zu < %zu bytes", ws_bytes, need);
  int r;
  switch (odt) {
    case MHC_F32: r = residual_bwd_o<float>(out, dout, ddt, dy, hpre, dx, dxdt, T, n, C, ws, st, odt); break;
    case MHC_BF16: r = residual_bwd_o<bf16>(out, dout, ddt, dy, hpre, dx, dxdt, T, n, C, ws, st, odt); break;
    default: r = residual_bwd_o<f16>(out, dout, ddt, dy, hpre, dx, dxdt, T, n, C, ws, st, odt); break;
  }
  if (r != MHC_OK) return r;
  k_combine_finalize<<<1, kCFinBD, 0, st>>>(static_cast<const char*>(ws), n, nullptr, nullptr,
                                            nullptr, 2, nullptr, dhpre, nullptr, ParamsBwd{}, 0);
  return check_launch("residual_add_agg_bwd_finalize");
}

}  // namespace mhc
