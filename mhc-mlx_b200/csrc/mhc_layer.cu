// Fused mHC layer kernels for sm_100a: forward (aggregate + RMSNorm + mix +
// residual add), backward (dx plus per-CTA partials of every parameter
// gradient) and the finalize reduction (+ Sinkhorn / sigmoid chain).
//
// Reference math: reference.py:72-161.  Reference launch structure being
// replaced: metal.py:1823-1975 (forward strategy selector: 1 or 3 kernels)
// and metal.py:2787-2857 (backward: 7 kernels, dM/dH reductions on n^2 / n
// threadgroups).  Here the forward is one pass (x read once, out written
// once) and the backward is one pass (x, d_out read once, dx written once)
// followed by a small deterministic reduction.
//
// Mapping ("fast" kernels, n in {1,2,4,8[,16,32]}): persistent CTAs, one token
// row [n, C] at a time per CTA.  Thread t owns the column groups
// g = t + k*blockDim (k < ITEMS), VEC columns each, for all n streams, so the
// whole row sits in registers between the load and the store; the RMS sum
// (and in the backward the RMS-gradient dot product) is one block reduction.
// The "generic" kernels cover any n <= 64 and any C with two passes per row.
#include <cstdlib>

#include <cooperative_groups.h>

#include "mhc_common.cuh"
#include "mhc_sinkhorn.cuh"
#include "mhc_internal.h"

namespace mhc {

// ===================================================================== fwd ==
// PIPE: the next token's x is prefetched with cp.async into thread-private
// shared-memory slots once the current token's values are in registers.
template <int N, typename InT, typename OutT, int VEC, int ITEMS, int MAXT, bool PIPE>
__global__ void __launch_bounds__(MAXT)
k_fwd_fast(const InT* __restrict__ x, const float* __restrict__ Mg,
           const float* __restrict__ hpre_g, const float* __restrict__ hpost_g,
           const float* __restrict__ w, OutT* __restrict__ out, int64_t T, int C, float eps) {
  static_assert(!PIPE || VEC * sizeof(InT) == 16, "16-byte chunks");
  extern __shared__ uint4 s_stage[];
  constexpr bool kMReg = N <= 8;
  __shared__ float sM[N * N];
  __shared__ float red[2][32];
  for (int e = threadIdx.x; e < N * N; e += blockDim.x) sM[e] = Mg[e];
  float hpre[N], hpost[N];
#pragma unroll
  for (int i = 0; i < N; ++i) { hpre[i] = __ldg(hpre_g + i); hpost[i] = __ldg(hpost_g + i); }
  __syncthreads();
  float Mr[kMReg ? N : 1][kMReg ? N : 1];
  if constexpr (kMReg) {
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
      for (int j = 0; j < N; ++j) Mr[i][j] = sM[i * N + j];
  }

  int col[ITEMS];
  bool ok[ITEMS];
  float wv[ITEMS][VEC];
#pragma unroll
  for (int it = 0; it < ITEMS; ++it) {
    col[it] = (threadIdx.x + it * blockDim.x) * VEC;
    ok[it] = col[it] < C;
    if (ok[it]) load_f32<VEC>(w + col[it], wv[it]);
    else
#pragma unroll
      for (int v = 0; v < VEC; ++v) wv[it][v] = 0.f;
  }

  const int64_t rs = (int64_t)N * C;
  auto slot = [&](int it, int i) -> uint4* {
    return s_stage + (it * N + i) * blockDim.x + threadIdx.x;
  };
  auto prefetch = [&](int64_t tp) {
#pragma unroll
    for (int it = 0; it < ITEMS; ++it) {
      if (!ok[it]) continue;
#pragma unroll
      for (int i = 0; i < N; ++i) cp_async16(slot(it, i), x + tp * rs + (int64_t)i * C + col[it]);
    }
    cp_async_commit();
  };
  if constexpr (PIPE) {
    if ((int64_t)blockIdx.x < T) prefetch(blockIdx.x);
  }
  int par = 0;
  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    const InT* xt = x + t * rs;
    float xr[ITEMS][N][VEC];
    if constexpr (PIPE) cp_async_wait_all();
#pragma unroll
    for (int it = 0; it < ITEMS; ++it)
#pragma unroll
      for (int i = 0; i < N; ++i) {
        if (ok[it]) {
          if constexpr (PIPE) unpack16<InT, VEC>(*slot(it, i), xr[it][i]);
          else load_vec<InT, VEC>(xt + (int64_t)i * C + col[it], xr[it][i]);
        } else {
#pragma unroll
          for (int v = 0; v < VEC; ++v) xr[it][i][v] = 0.f;
        }
      }
    float y[ITEMS][VEC];
    float ss = 0.f;
#pragma unroll
    for (int it = 0; it < ITEMS; ++it)
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < N; ++i) a = fmaf(hpre[i], xr[it][i][v], a);
        y[it][v] = a;
        ss = fmaf(a, a, ss);
      }
    // the staged chunks are all in registers now: refill with the next token
    if constexpr (PIPE) {
      if (t + gridDim.x < T) prefetch(t + gridDim.x);
    }
    ss = block_sum(ss, red[par]);
    par ^= 1;
    const float inv = inv_rms(ss, C, eps);
    OutT* ot = out + t * rs;
#pragma unroll
    for (int it = 0; it < ITEMS; ++it) {
      if (!ok[it]) continue;
      float yn[VEC];
#pragma unroll
      for (int v = 0; v < VEC; ++v) yn[v] = (y[it][v] * inv) * wv[it][v];
#pragma unroll
      for (int i = 0; i < N; ++i) {
        float o[VEC];
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          float m = 0.f;
#pragma unroll
          for (int j = 0; j < N; ++j) {
            const float mij = kMReg ? Mr[kMReg ? i : 0][kMReg ? j : 0] : sM[i * N + j];
            m = fmaf(mij, xr[it][j][v], m);
          }
          o[v] = m + hpost[i] * yn[v];
        }
        store_vec<OutT, VEC>(ot + (int64_t)i * C + col[it], o);
      }
    }
  }
}

// Generic forward: any n <= MAXN, any C, any alignment.  Pass 1 computes the
// row's sum of squares, pass 2 re-reads the row (L2-resident) and writes out.
template <int MAXN, typename InT, typename OutT>
__global__ void __launch_bounds__(256)
k_fwd_generic(const InT* __restrict__ x, const float* __restrict__ Mg,
              const float* __restrict__ hpre_g, const float* __restrict__ hpost_g,
              const float* __restrict__ w, OutT* __restrict__ out, int64_t T, int n, int C,
              float eps) {
  __shared__ float sM[MAXN * MAXN];
  __shared__ float shpre[MAXN], shpost[MAXN];
  __shared__ float red[2][32];
  for (int e = threadIdx.x; e < n * n; e += blockDim.x) sM[e] = Mg[e];
  for (int e = threadIdx.x; e < n; e += blockDim.x) { shpre[e] = hpre_g[e]; shpost[e] = hpost_g[e]; }
  __syncthreads();
  const int64_t rs = (int64_t)n * C;
  int par = 0;
  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    const InT* xt = x + t * rs;
    float ss = 0.f;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
      float a = 0.f;
      for (int i = 0; i < n; ++i) a = fmaf(shpre[i], to_f(xt[(int64_t)i * C + c]), a);
      ss = fmaf(a, a, ss);
    }
    ss = block_sum(ss, red[par]);
    par ^= 1;
    const float inv = inv_rms(ss, C, eps);
    OutT* ot = out + t * rs;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
      float xc[MAXN];
      float a = 0.f;
#pragma unroll
      for (int j = 0; j < MAXN; ++j) {
        xc[j] = j < n ? to_f(xt[(int64_t)j * C + c]) : 0.f;
        if (j < n) a = fmaf(shpre[j], xc[j], a);
      }
      const float yn = (a * inv) * __ldg(w + c);
      for (int i = 0; i < n; ++i) {
        float m = 0.f;
#pragma unroll
        for (int j = 0; j < MAXN; ++j)
          if (j < n) m = fmaf(sM[i * n + j], xc[j], m);
        ot[(int64_t)i * C + c] = from_f<OutT>(m + shpost[i] * yn);
      }
    }
  }
}

// Cluster-split forward for n in {16, 32, 64}: the columns of one token are
// split over the CTAs of a thread-block cluster (cluster size cs = 1..8,
// chosen at launch so that a few CTAs per SM are in flight even when there
// are few tokens).  Each CTA reduces sum(y^2) over its columns; the cs
// partials are summed through distributed shared memory between two cluster
// barriers (the second keeps every CTA's partial alive until all have read
// it), then each CTA writes its columns: out_i = sum_j M_ij x_j + hpost_i yn,
// with the slice of x re-read from L2.  No workspace and no atomics; the
// partials are summed in rank order, so results are deterministic.
template <int N, typename InT, typename OutT>
__global__ void __launch_bounds__(256)
k_fwd_split(const InT* __restrict__ x, const float* __restrict__ Mg,
            const float* __restrict__ hpre_g, const float* __restrict__ hpost_g,
            const float* __restrict__ w, OutT* __restrict__ out, int64_t T, int C, float eps) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  const int cs = (int)cl.num_blocks(), rank = (int)cl.block_rank();
  __shared__ __align__(16) float sMT[N * N];  // sMT[j * N + i] = M[i][j]
  __shared__ float shpre[N], shpost[N];
  __shared__ float red[2][32];
  __shared__ float s_part;
  for (int e = threadIdx.x; e < N * N; e += blockDim.x) sMT[(e % N) * N + e / N] = Mg[e];
  for (int e = threadIdx.x; e < N; e += blockDim.x) { shpre[e] = hpre_g[e]; shpost[e] = hpost_g[e]; }
  __syncthreads();
  const int64_t t = blockIdx.x / cs;
  const int chunk = (C + cs - 1) / cs, c0 = rank * chunk, c1 = min(C, c0 + chunk);
  const InT* xt = x + t * (int64_t)N * C;
  float ss = 0.f;
  for (int c = c0 + threadIdx.x; c < c1; c += blockDim.x) {
    float a = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i) a = fmaf(shpre[i], to_f(xt[(int64_t)i * C + c]), a);
    ss = fmaf(a, a, ss);
  }
  ss = block_sum(ss, red[0]);
  if (threadIdx.x == 0) s_part = ss;
  cl.sync();  // every CTA's partial is written
  float tot = 0.f;
  for (int r = 0; r < cs; ++r) tot += *cl.map_shared_rank(&s_part, r);
  const float inv = inv_rms(tot, C, eps);
  OutT* ot = out + t * (int64_t)N * C;
  // M^T staged once more so that one float4 holds M[i..i+3][j]: four output
  // streams advance with two packed FMAs per column j (same per-stream order
  // over j as a scalar chain, bit-identical)
  const float4* sMT4 = reinterpret_cast<const float4*>(sMT);
  for (int c = c0 + threadIdx.x; c < c1; c += blockDim.x) {
    float xc[N], a = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) {
      xc[j] = to_f(xt[(int64_t)j * C + c]);
      a = fmaf(shpre[j], xc[j], a);
    }
    const float yn = (a * inv) * __ldg(w + c);
#pragma unroll 2
    for (int i = 0; i < N; i += 4) {
      float m0 = 0.f, m1 = 0.f, m2 = 0.f, m3 = 0.f;
#pragma unroll
      for (int j = 0; j < N; ++j) {
        const float4 r4 = sMT4[(j * N + i) / 4];
        fma2(m0, m1, r4.x, r4.y, xc[j], xc[j]);
        fma2(m2, m3, r4.z, r4.w, xc[j], xc[j]);
      }
      ot[(int64_t)i * C + c] = from_f<OutT>(m0 + shpost[i] * yn);
      ot[(int64_t)(i + 1) * C + c] = from_f<OutT>(m1 + shpost[i + 1] * yn);
      ot[(int64_t)(i + 2) * C + c] = from_f<OutT>(m2 + shpost[i + 2] * yn);
      ot[(int64_t)(i + 3) * C + c] = from_f<OutT>(m3 + shpost[i + 3] * yn);
    }
  }
  cl.sync();  // no CTA leaves while another may still read its partial
}

// ===================================================================== bwd ==
// Per token (y = sum_i hpre_i x_i, dyn = sum_i hpost_i d_i, both per column):
//   ss = sum_c y^2, pd = sum_c dyn w y, inv = 1/sqrt(ss/C + eps)
//   dya = dyn w inv - (pd inv^3 / C) y
//   dx_j = sum_i M_ij d_i + hpre_j dya
// Accumulated over tokens and columns (per CTA, then finalize):
//   dM_ij += d_i x_j, dHpre_j += dya x_j, dHpost_i += d_i (y inv w),
//   dw_c += dyn (y inv)
//
// PIPE: the next token's x and d_out chunks are prefetched with cp.async into
// thread-private shared-memory slots (one 16-byte chunk per (item, stream))
// as soon as the current token's values have been consumed by the first
// pass, so HBM keeps streaming while the CTA reduces, computes and stores.
template <int N, typename XT, typename DT, typename DXT, int VEC, int ITEMS, int MAXT, bool PIPE>
__global__ void __launch_bounds__(MAXT)
k_bwd_fast(const XT* __restrict__ x, const DT* __restrict__ dout, const float* __restrict__ Mg,
           const float* __restrict__ hpre_g, const float* __restrict__ hpost_g,
           const float* __restrict__ w, DXT* __restrict__ dx, int64_t T, int C, float eps,
           float* __restrict__ ws_p, float* __restrict__ ws_c, int* __restrict__ ws_hdr) {
  static_assert(!PIPE || (VEC * sizeof(XT) == 16 && VEC * sizeof(DT) == 16), "16-byte chunks");
  extern __shared__ uint4 s_stage[];
  constexpr int P = N * N + 2 * N;
  __shared__ float sM[N * N];
  __shared__ float red[2][64];
  __shared__ float sacc[32 * P];
  for (int e = threadIdx.x; e < N * N; e += blockDim.x) sM[e] = Mg[e];
  float hpre[N], hpost[N];
#pragma unroll
  for (int i = 0; i < N; ++i) { hpre[i] = __ldg(hpre_g + i); hpost[i] = __ldg(hpost_g + i); }
  __syncthreads();

  int col[ITEMS];
  bool ok[ITEMS];
#pragma unroll
  for (int it = 0; it < ITEMS; ++it) {
    col[it] = (threadIdx.x + it * blockDim.x) * VEC;
    ok[it] = col[it] < C;
  }
  float aM[N][N], aPre[N], aPost[N], aW[ITEMS][VEC];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    aPre[i] = 0.f; aPost[i] = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) aM[i][j] = 0.f;
  }
#pragma unroll
  for (int it = 0; it < ITEMS; ++it)
#pragma unroll
    for (int v = 0; v < VEC; ++v) aW[it][v] = 0.f;

  const int64_t rs = (int64_t)N * C;
  const float invC = 1.0f / (float)C;
  // slot(kind, it, i): kind 0 = x, 1 = d_out; thread index fastest
  auto slot = [&](int kind, int it, int i) -> uint4* {
    return s_stage + ((kind * ITEMS + it) * N + i) * blockDim.x + threadIdx.x;
  };
  auto prefetch = [&](int64_t tp) {
#pragma unroll
    for (int it = 0; it < ITEMS; ++it) {
      if (!ok[it]) continue;
#pragma unroll
      for (int i = 0; i < N; ++i) {
        cp_async16(slot(0, it, i), x + tp * rs + (int64_t)i * C + col[it]);
        cp_async16(slot(1, it, i), dout + tp * rs + (int64_t)i * C + col[it]);
      }
    }
    cp_async_commit();
  };
  if constexpr (PIPE) {
    if ((int64_t)blockIdx.x < T) prefetch(blockIdx.x);
  }
  int par = 0;
  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    const XT* xt = x + t * rs;
    const DT* dt = dout + t * rs;
    float xr[ITEMS][N][VEC], dr[ITEMS][N][VEC];
    if constexpr (PIPE) cp_async_wait_all();
#pragma unroll
    for (int it = 0; it < ITEMS; ++it)
#pragma unroll
      for (int i = 0; i < N; ++i) {
        if (ok[it]) {
          if constexpr (PIPE) {
            unpack16<XT, VEC>(*slot(0, it, i), xr[it][i]);
            unpack16<DT, VEC>(*slot(1, it, i), dr[it][i]);
          } else {
            load_vec<XT, VEC>(xt + (int64_t)i * C + col[it], xr[it][i]);
            load_vec<DT, VEC>(dt + (int64_t)i * C + col[it], dr[it][i]);
          }
        } else {
#pragma unroll
          for (int v = 0; v < VEC; ++v) { xr[it][i][v] = 0.f; dr[it][i][v] = 0.f; }
        }
      }
    float ss = 0.f, pd = 0.f;
#pragma unroll
    for (int it = 0; it < ITEMS; ++it) {
      float wv[VEC];
      if (ok[it]) load_f32<VEC>(w + col[it], wv);
      else
#pragma unroll
        for (int v = 0; v < VEC; ++v) wv[v] = 0.f;
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        float y = 0.f, dyn = 0.f;
#pragma unroll
        for (int i = 0; i < N; ++i) {
          y = fmaf(hpre[i], xr[it][i][v], y);
          dyn = fmaf(hpost[i], dr[it][i][v], dyn);
        }
        ss = fmaf(y, y, ss);
        pd = fmaf(dyn * wv[v], y, pd);
      }
    }
    // every staged value has been consumed above: refill the slots with the
    // next token while this one is reduced, computed and stored
    if constexpr (PIPE) {
      if (t + gridDim.x < T) prefetch(t + gridDim.x);
    }
    const float2 red2 = block_sum2(ss, pd, red[par]);
    par ^= 1;
    const float inv = inv_rms(red2.x, C, eps);
    const float k2 = (red2.y * (inv * inv * inv)) * invC;

    float dya[ITEMS][VEC];
#pragma unroll
    for (int it = 0; it < ITEMS; ++it) {
      float wv[VEC];
      if (ok[it]) load_f32<VEC>(w + col[it], wv);
      else
#pragma unroll
        for (int v = 0; v < VEC; ++v) wv[v] = 0.f;
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        float y = 0.f, dyn = 0.f;
#pragma unroll
        for (int i = 0; i < N; ++i) {
          y = fmaf(hpre[i], xr[it][i][v], y);
          dyn = fmaf(hpost[i], dr[it][i][v], dyn);
        }
        const float yi = y * inv;
        const float yn = yi * wv[v];
        aW[it][v] = fmaf(dyn, yi, aW[it][v]);
        const float g = (dyn * wv[v]) * inv - k2 * y;
        dya[it][v] = g;
#pragma unroll
        for (int i = 0; i < N; ++i) {
          aPost[i] = fmaf(dr[it][i][v], yn, aPost[i]);
          aPre[i] = fmaf(g, xr[it][i][v], aPre[i]);
#pragma unroll
          for (int j = 0; j < N; ++j) aM[i][j] = fmaf(dr[it][i][v], xr[it][j][v], aM[i][j]);
        }
      }
    }
    DXT* dxt = dx + t * rs;
#pragma unroll
    for (int it = 0; it < ITEMS; ++it) {
      if (!ok[it]) continue;
#pragma unroll
      for (int j = 0; j < N; ++j) {
        float o[VEC];
#pragma unroll
        for (int v = 0; v < VEC; ++v) o[v] = hpre[j] * dya[it][v];
#pragma unroll
        for (int i = 0; i < N; ++i) {
          const float mij = sM[i * N + j];
#pragma unroll
          for (int v = 0; v < VEC; ++v) o[v] = fmaf(mij, dr[it][i][v], o[v]);
        }
        store_vec<DXT, VEC>(dxt + (int64_t)j * C + col[it], o);
      }
    }
  }

  // ---- per-CTA partials: fixed-order warp butterfly + ordered warp sum ----
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int i = 0; i < N; ++i) {
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const float v = warp_sum(aM[i][j]);
      if (lane == 0) sacc[warp * P + i * N + j] = v;
    }
    const float a = warp_sum(aPre[i]);
    const float b = warp_sum(aPost[i]);
    if (lane == 0) { sacc[warp * P + N * N + i] = a; sacc[warp * P + N * N + N + i] = b; }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < P; e += blockDim.x) {
    float s = 0.f;
    for (int q = 0; q < nw; ++q) s += sacc[q * P + e];
    ws_p[(size_t)blockIdx.x * P + e] = s;
  }
#pragma unroll
  for (int it = 0; it < ITEMS; ++it)
    if (ok[it]) store_vec<float, VEC, false>(ws_c + (size_t)blockIdx.x * C + col[it], aW[it]);
  if (blockIdx.x == 0 && threadIdx.x == 0) { ws_hdr[0] = gridDim.x; ws_hdr[1] = 1; }
}

// Full-row backward for 16-bit rows: x, d_out and dx share one 16-bit type T
// and C = 8 * BD, so thread t owns columns 8t..8t+7 of every stream with no
// tail.  Same math and partial-row output as k_bwd_fast; the differences:
//   - staging: BULK = false copies the next token's x and d_out rows with
//     per-thread 16-byte cp.async (NBUF = 2 double-buffers the slots: token
//     t + G is requested before token t is processed; NBUF = 1 refills the
//     single buffer once the first pass has read it, as k_bwd_fast does).
//     BULK = true has one thread issue a 1-D bulk copy (cp.async.bulk, the TMA
//     unit) per stream row into NBUF >= 2 buffers, each completing on its own
//     mbarrier; a buffer is refilled with token t + NBUF * G right after the
//     block reduction of token t, when every thread has read it.  The waits
//     are bounded: a copy that never lands makes the CTA write NaN into its
//     dx rows and partial rows (so the gradients come out NaN, visibly) and
//     return;
//   - y and dyn of the first pass stay in registers for the second; w is
//     staged once in shared memory and M is kept transposed there, so the
//     per-token parameter reads are shared-memory vector loads;
//   - the two per-token block sums take one barrier and a warp butterfly;
//   - MMA (n = 4): dM = sum d x^T runs on the tensor cores from the staged
//     rows.  Per warp and 64-column group, ldmatrix gives A = d_out rows
//     (stream i, 16-column block b) and B = x columns (stream j, block b'),
//     and two m16n8k16 products accumulate D[(i,b)][(j,b')]; only the
//     b == b' entries are dM partials (the others are never read).  Rows of A
//     and columns of B are ordered, and stream rows padded by one 16-byte
//     chunk, so that each 8x8 matrix load touches 8 distinct bank groups.
//     bf16 x bf16 (or f16 x f16) products are exact in fp32.
// Dynamic shared layout: w as [2][BD] float4 (thread t's columns 8t..8t+3
// and 8t+4..8t+7, conflict-free), then [NBUF][x rows N | d_out rows N][SB
// chunks of 16 bytes].
template <int N, typename T, int BD, bool MMA, int NBUF, bool BULK = false>
__global__ void __launch_bounds__(BD, 512 / BD)
k_bwd_rows(const T* __restrict__ x, const T* __restrict__ dout, const float* __restrict__ Mg,
           const float* __restrict__ hpre_g, const float* __restrict__ hpost_g,
           const float* __restrict__ w, T* __restrict__ dx, int64_t T_, float eps,
           float* __restrict__ ws_p, float* __restrict__ ws_c, int* __restrict__ ws_hdr) {
  static_assert(sizeof(T) == 2, "16-bit rows");
  static_assert(!MMA || N == 4, "the tensor-core dM layout is for n = 4");
  static_assert(BULK ? (NBUF == 2 || NBUF == 3) : (NBUF == 1 || NBUF == 2), "staging buffers");
  constexpr int C = 8 * BD, P = N * N + 2 * N, NW = BD / 32;
  constexpr int SB = BD + (MMA ? 1 : 0);  // chunks per staged stream row
  constexpr int BUF = 2 * N * SB;         // chunks per buffer
  constexpr int64_t RS = (int64_t)N * C;  // elements per token
  constexpr unsigned kRowBytes = BD * 16, kTokBytes = 2 * N * kRowBytes;
  extern __shared__ uint4 s_dyn[];
  float4* s_w = reinterpret_cast<float4*>(s_dyn);
  uint4* s_stage = s_dyn + 2 * BD;
  __shared__ __align__(16) float sMT[N * N];  // sMT[j * N + i] = M[i][j]
  __shared__ float red[2][64];
  __shared__ float sacc[NW * P];
  __shared__ __align__(8) uint64_t s_full[BULK ? NBUF : 1];
  __shared__ int s_abort;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t G = gridDim.x;
  if constexpr (BULK) {
    if (tid == 0) {
#pragma unroll
      for (int b = 0; b < NBUF; ++b) mbar_init(&s_full[b], 1);
      s_abort = 0;
      mbar_init_fence();
    }
  }
  for (int e = tid; e < N * N; e += BD) sMT[(e % N) * N + e / N] = Mg[e];
  s_w[tid] = __ldg(reinterpret_cast<const float4*>(w) + 2 * tid);
  s_w[BD + tid] = __ldg(reinterpret_cast<const float4*>(w) + 2 * tid + 1);
  float hpre[N], hpost[N];
#pragma unroll
  for (int i = 0; i < N; ++i) { hpre[i] = __ldg(hpre_g + i); hpost[i] = __ldg(hpost_g + i); }
  __syncthreads();
  auto load_w = [&](float (&wv)[8]) {
    const float4 a = s_w[tid], b = s_w[BD + tid];
    wv[0] = a.x; wv[1] = a.y; wv[2] = a.z; wv[3] = a.w;
    wv[4] = b.x; wv[5] = b.y; wv[6] = b.z; wv[7] = b.w;
  };

  const int col = tid * 8;
  float aM[MMA ? 1 : N][MMA ? 1 : N], aPre[N], aPost[N], aW[8];
  float accA[4] = {0.f, 0.f, 0.f, 0.f}, accB[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < N; ++i) { aPre[i] = 0.f; aPost[i] = 0.f; }
#pragma unroll
  for (int i = 0; i < (MMA ? 1 : N); ++i)
#pragma unroll
    for (int j = 0; j < (MMA ? 1 : N); ++j) aM[i][j] = 0.f;
#pragma unroll
  for (int v = 0; v < 8; ++v) aW[v] = 0.f;

  // per-thread cp.async staging of token tp into buffer buf
  auto prefetch = [&](int64_t tp, int buf) {
    uint4* s = s_stage + buf * BUF + tid;
    const T* xs = x + tp * RS + col;
    const T* ds = dout + tp * RS + col;
#pragma unroll
    for (int i = 0; i < N; ++i) {
      cp_async16(s + i * SB, xs + (int64_t)i * C);
      cp_async16(s + (N + i) * SB, ds + (int64_t)i * C);
    }
  };
  // one thread: bulk copies of token tp's 2N rows into buffer buf
  auto issue = [&](int64_t tp, int buf) {
    uint4* s = s_stage + buf * BUF;
    mbar_arrive_expect_tx(&s_full[buf], kTokBytes);
#pragma unroll
    for (int i = 0; i < N; ++i) {
      bulk_g2s(s + i * SB, x + tp * RS + (int64_t)i * C, kRowBytes, &s_full[buf]);
      bulk_g2s(s + (N + i) * SB, dout + tp * RS + (int64_t)i * C, kRowBytes, &s_full[buf]);
    }
  };
  if constexpr (BULK) {
    if (tid == 0)
#pragma unroll
      for (int k = 0; k < NBUF; ++k)
        if ((int64_t)blockIdx.x + k * G < T_) issue(blockIdx.x + k * G, k);
  } else {
    if ((int64_t)blockIdx.x < T_) prefetch(blockIdx.x, 0);
    cp_async_commit();
  }
  int par = 0, buf = 0;
  unsigned use = 0;  // BULK: tokens consumed so far (buffer use = use / NBUF)
  bool aborted = false;
  int64_t t = blockIdx.x;
  for (; t < T_; t += G) {
    if constexpr (BULK) {
      buf = (int)(use % NBUF);
      if (!mbar_wait(&s_full[buf], (use / NBUF) & 1u)) s_abort = 1;
    } else if constexpr (NBUF == 2) {
      // the other buffer was last read before the previous token's barrier
      if (t + G < T_) prefetch(t + G, buf ^ 1);
      cp_async_commit();
      cp_async_wait_group<1>();
    } else {
      cp_async_wait_all();
    }
    const uint4* sb = s_stage + buf * BUF;
    if constexpr (MMA) {
      __syncwarp();  // every lane's chunks of this buffer are visible to the warp
      const int q = lane >> 3, rr = lane & 7, wbase = tid & ~31;
      // A: row (stream rr&3, block 2*(rr>>2) + (q&1)), k-half q>>1
      // B: col (stream rr&3, block 2*(rr>>2) + (q>>1)), k-half q&1
      const uint4* pa = sb + (N + (rr & 3)) * SB + wbase + 2 * (2 * (rr >> 2) + (q & 1)) + (q >> 1);
      const uint4* pb = sb + (rr & 3) * SB + wbase + 2 * (2 * (rr >> 2) + (q >> 1)) + (q & 1);
#pragma unroll
      for (int g64 = 0; g64 < 4; ++g64) {
        unsigned a[4], b[4];
        ldmatrix_x4(a, pa + 8 * g64);
        ldmatrix_x4(b, pb + 8 * g64);
        mma_16816<T>(accA, a, b[0], b[1]);
        mma_16816<T>(accB, a, b[2], b[3]);
      }
    }
    float xr[N][8], dr[N][8];
#pragma unroll
    for (int i = 0; i < N; ++i) {
      unpack16<T, 8>(sb[i * SB + tid], xr[i]);
      unpack16<T, 8>(sb[(N + i) * SB + tid], dr[i]);
    }
    if constexpr (!BULK) {
      if constexpr (NBUF == 1) {
        if constexpr (MMA) __syncwarp();  // the warp's ldmatrix reads precede the refill
        if (t + G < T_) prefetch(t + G, 0);
        cp_async_commit();
      } else {
        buf ^= 1;
      }
    }
    float yk[8], dk[8], ss = 0.f, pd = 0.f;
    {
      float wv[8];
      load_w(wv);
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        float y = 0.f, dyn = 0.f;
#pragma unroll
        for (int i = 0; i < N; ++i) {
          y = fmaf(hpre[i], xr[i][v], y);
          dyn = fmaf(hpost[i], dr[i][v], dyn);
        }
        yk[v] = y;
        dk[v] = dyn;
        ss = fmaf(y, y, ss);
        pd = fmaf(dyn * wv[v], y, pd);
      }
    }
    const float2 red2 = block_sum2_bfly<NW>(ss, pd, red[par]);
    par ^= 1;
    if constexpr (BULK) {
      // after the barrier: every thread has read buffer `buf` (the MMA's
      // ldmatrix and the unpack precede it), and s_abort is the same for all
      if (s_abort) { aborted = true; break; }
      if (tid == 0 && t + NBUF * G < T_) {
        fence_proxy_async_smem();
        issue(t + NBUF * G, buf);
      }
      ++use;
    }
    const float inv = inv_rms(red2.x, C, eps);
    const float k2 = (red2.y * (inv * inv * inv)) * (1.0f / (float)C);

    float dya[8];
    {
      float wv[8];
      load_w(wv);
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        const float yi = yk[v] * inv;
        const float yn = yi * wv[v];
        aW[v] = fmaf(dk[v], yi, aW[v]);
        const float g = (dk[v] * wv[v]) * inv - k2 * yk[v];
        dya[v] = g;
#pragma unroll
        for (int i = 0; i < N; ++i) {
          aPost[i] = fmaf(dr[i][v], yn, aPost[i]);
          aPre[i] = fmaf(g, xr[i][v], aPre[i]);
          if constexpr (!MMA) {
#pragma unroll
            for (int j = 0; j < N; ++j) aM[i][j] = fmaf(dr[i][v], xr[j][v], aM[i][j]);
          }
        }
      }
    }
    T* dxt = dx + t * RS + col;
#pragma unroll
    for (int j = 0; j < N; ++j) {
      float mc[N];
#pragma unroll
      for (int i = 0; i < N; ++i) mc[i] = sMT[j * N + i];
      float o[8];
#pragma unroll
      for (int v = 0; v < 8; ++v) o[v] = hpre[j] * dya[v];
#pragma unroll
      for (int i = 0; i < N; ++i)
#pragma unroll
        for (int v = 0; v < 8; ++v) o[v] = fmaf(mc[i], dr[i][v], o[v]);
      store_vec<T, 8>(dxt + (int64_t)j * C, o);
    }
  }
  if constexpr (BULK) {
    if (aborted) {
      // a bulk copy did not land in time: wait (bounded) for the copies this
      // CTA still has in flight, then mark everything it owns as invalid
      if (tid == 0) {
        for (unsigned k = use; k < use + NBUF; ++k)
          if ((int64_t)blockIdx.x + (int64_t)k * G < T_)
            (void)mbar_wait(&s_full[k % NBUF], (k / NBUF) & 1u);
      }
      const float nan = __int_as_float(0x7fc00000);
      float o[8];
#pragma unroll
      for (int v = 0; v < 8; ++v) { o[v] = nan; aW[v] = nan; }
      for (; t < T_; t += G)
#pragma unroll
        for (int j = 0; j < N; ++j) store_vec<T, 8>(dx + t * RS + col + (int64_t)j * C, o);
#pragma unroll
      for (int i = 0; i < N; ++i) { aPre[i] = nan; aPost[i] = nan; }
#pragma unroll
      for (int e = 0; e < 4; ++e) { accA[e] = nan; accB[e] = nan; }
    }
  } else {
    cp_async_wait_all();  // only empty groups can remain; nothing is left in flight at exit
  }

  // ---- per-CTA partials: fixed-order warp reductions + ordered warp sum ----
  if constexpr (MMA) {
    // lane (g, t) holds D[g][2t..2t+1] (accA) and D[g+8][2t..2t+1] (accB):
    // dM partials where (g < 4) == (t < 2), for i = g & 3, j = (2t + e) & 3;
    // lane (g + 4, t + 2) = lane + 18 holds the other half of the same (i, j)
    float v0 = accA[0] + accB[2], v1 = accA[1] + accB[3];
    v0 += __shfl_down_sync(0xffffffffu, v0, 18);
    v1 += __shfl_down_sync(0xffffffffu, v1, 18);
    const int g = lane >> 2, tq = lane & 3;
    if (g < 4 && tq < 2) {
      sacc[warp * P + g * N + 2 * tq] = v0;
      sacc[warp * P + g * N + 2 * tq + 1] = v1;
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
      for (int j = 0; j < N; ++j) {
        const float v = warp_sum(aM[i][j]);
        if (lane == 0) sacc[warp * P + i * N + j] = v;
      }
  }
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const float a = warp_sum(aPre[i]);
    const float b = warp_sum(aPost[i]);
    if (lane == 0) { sacc[warp * P + N * N + i] = a; sacc[warp * P + N * N + N + i] = b; }
  }
  __syncthreads();
  for (int e = tid; e < P; e += BD) {
    float s = 0.f;
#pragma unroll 4
    for (int q = 0; q < NW; ++q) s += sacc[q * P + e];
    ws_p[(size_t)blockIdx.x * P + e] = s;
  }
  store_vec<float, 8, false>(ws_c + (size_t)blockIdx.x * C + col, aW);
  if (blockIdx.x == 0 && tid == 0) { ws_hdr[0] = gridDim.x; ws_hdr[1] = 1; }
}

// Full-row backward for fp32 rows (x, d_out, dx fp32, C = 8 * BD): the
// k_bwd_rows design with the rows staged by bulk copies, in half tokens.  An
// fp32 token is 2N rows of C floats (128 KB at n = 4, C = 4096), too large for
// a ring of whole tokens, so the ring holds NS = 3 half tokens (columns
// [0, C/2) or [C/2, C) of all 2N rows, 64 KB each): thread t owns columns
// 4t .. 4t + 3 of each half, so its shared-memory reads are consecutive
// 16-byte chunks across the warp.  After token t's block reduction both of
// its halves are free and the next two halves of this CTA's sequence are
// requested into them.  dM runs on the fp32 pipe (fp32 products are not exact
// on the tensor cores).  Waits are bounded as in k_bwd_rows: a copy that never
// lands makes the CTA write NaN into its dx rows and partial rows.
template <int N, int BD>
__global__ void __launch_bounds__(BD, 1)
k_bwd_rows32(const float* __restrict__ x, const float* __restrict__ dout,
             const float* __restrict__ Mg, const float* __restrict__ hpre_g,
             const float* __restrict__ hpost_g, const float* __restrict__ w,
             float* __restrict__ dx, int64_t T_, float eps, float* __restrict__ ws_p,
             float* __restrict__ ws_c, int* __restrict__ ws_hdr) {
  constexpr int C = 8 * BD, H = C / 2, P = N * N + 2 * N, NW = BD / 32, NS = 3;
  constexpr int64_t RS = (int64_t)N * C;   // elements per token
  constexpr int SLOT = 2 * N * H;          // floats per half-token slot
  constexpr unsigned kRowBytes = H * 4, kHalfBytes = 2 * N * kRowBytes;
  extern __shared__ float4 s_dyn4[];
  float4* s_w = s_dyn4;                                         // [2][BD]
  float* s_stage = reinterpret_cast<float*>(s_dyn4 + 2 * BD);   // [NS][2N][H]
  __shared__ __align__(16) float sMT[N * N];  // sMT[j * N + i] = M[i][j]
  __shared__ float red[2][64];
  __shared__ float sacc[NW * P];
  __shared__ __align__(8) uint64_t s_full[NS];
  __shared__ int s_abort;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t G = gridDim.x;
  if (tid == 0) {
#pragma unroll
    for (int b = 0; b < NS; ++b) mbar_init(&s_full[b], 1);
    s_abort = 0;
    mbar_init_fence();
  }
  for (int e = tid; e < N * N; e += BD) sMT[(e % N) * N + e / N] = Mg[e];
  s_w[tid] = __ldg(reinterpret_cast<const float4*>(w) + tid);
  s_w[BD + tid] = __ldg(reinterpret_cast<const float4*>(w + H) + tid);
  float hpre[N], hpost[N];
#pragma unroll
  for (int i = 0; i < N; ++i) { hpre[i] = __ldg(hpre_g + i); hpost[i] = __ldg(hpost_g + i); }
  __syncthreads();
  auto load_w = [&](float (&wv)[8]) {
    const float4 a = s_w[tid], b = s_w[BD + tid];
    wv[0] = a.x; wv[1] = a.y; wv[2] = a.z; wv[3] = a.w;
    wv[4] = b.x; wv[5] = b.y; wv[6] = b.z; wv[7] = b.w;
  };

  // this CTA's tokens blockIdx.x, blockIdx.x + G, ...; half k of the
  // sequence is token k / 2, columns [(k % 2) H, (k % 2 + 1) H)
  const int64_t ntok = (int64_t)blockIdx.x < T_ ? (T_ - 1 - blockIdx.x) / G + 1 : 0;
  const unsigned nhalf = (unsigned)(2 * ntok);
  auto issue = [&](unsigned k) {  // one thread
    const int64_t tok = blockIdx.x + (int64_t)(k >> 1) * G;
    const int h = (int)(k & 1u);
    const int slot = (int)(k % NS);
    float* sd = s_stage + slot * SLOT;
    mbar_arrive_expect_tx(&s_full[slot], kHalfBytes);
#pragma unroll
    for (int i = 0; i < N; ++i) {
      bulk_g2s(sd + i * H, x + tok * RS + (int64_t)i * C + h * H, kRowBytes, &s_full[slot]);
      bulk_g2s(sd + (N + i) * H, dout + tok * RS + (int64_t)i * C + h * H, kRowBytes,
               &s_full[slot]);
    }
  };
  unsigned issued = 0;  // meaningful in thread 0
  if (tid == 0)
    for (; issued < NS && issued < nhalf; ++issued) issue(issued);

  float aM[N][N], aPre[N], aPost[N], aW[8];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    aPre[i] = 0.f; aPost[i] = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) aM[i][j] = 0.f;
  }
#pragma unroll
  for (int v = 0; v < 8; ++v) aW[v] = 0.f;

  int par = 0;
  unsigned use = 0;  // halves consumed
  bool aborted = false;
  int64_t t = blockIdx.x;
  for (; t < T_; t += G) {
    // each half's first-pass sums are taken as soon as it lands, so the
    // wait for the second half (requested later) overlaps that arithmetic;
    // y and dyn are recomputed in the second pass (fp32 has issue slots to
    // spare; keeping them would spill at 128 registers)
    float xr[N][8], dr[N][8];
    float ss = 0.f, pd = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int slot = (int)(use % NS);
      if (!mbar_wait(&s_full[slot], (use / NS) & 1u)) s_abort = 1;
      const float* sb = s_stage + slot * SLOT + 4 * tid;
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const float4 a = *reinterpret_cast<const float4*>(sb + i * H);
        const float4 b = *reinterpret_cast<const float4*>(sb + (N + i) * H);
        xr[i][4 * h] = a.x; xr[i][4 * h + 1] = a.y; xr[i][4 * h + 2] = a.z; xr[i][4 * h + 3] = a.w;
        dr[i][4 * h] = b.x; dr[i][4 * h + 1] = b.y; dr[i][4 * h + 2] = b.z; dr[i][4 * h + 3] = b.w;
      }
      ++use;
      const float4 w4 = s_w[h * BD + tid];
      const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
      for (int v = 4 * h; v < 4 * h + 4; ++v) {
        float y = 0.f, dyn = 0.f;
#pragma unroll
        for (int i = 0; i < N; ++i) {
          y = fmaf(hpre[i], xr[i][v], y);
          dyn = fmaf(hpost[i], dr[i][v], dyn);
        }
        ss = fmaf(y, y, ss);
        pd = fmaf(dyn * wv[v - 4 * h], y, pd);
      }
    }
    const float2 red2 = block_sum2_bfly<NW>(ss, pd, red[par]);
    par ^= 1;
    // after the barrier every thread has read both halves, and s_abort is
    // the same for all
    if (s_abort) { aborted = true; break; }
    if (tid == 0) {
      fence_proxy_async_smem();
      for (int k = 0; k < 2 && issued < nhalf; ++k, ++issued) issue(issued);
    }
    const float inv = inv_rms(red2.x, C, eps);
    const float k2 = (red2.y * (inv * inv * inv)) * (1.0f / (float)C);

    float dya[8];
    {
      float wv[8];
      load_w(wv);
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        float yv = 0.f, dv = 0.f;
#pragma unroll
        for (int i = 0; i < N; ++i) {
          yv = fmaf(hpre[i], xr[i][v], yv);
          dv = fmaf(hpost[i], dr[i][v], dv);
        }
        const float yi = yv * inv;
        const float yn = yi * wv[v];
        aW[v] = fmaf(dv, yi, aW[v]);
        const float g = (dv * wv[v]) * inv - k2 * yv;
        dya[v] = g;
#pragma unroll
        for (int i = 0; i < N; ++i) {
          aPost[i] = fmaf(dr[i][v], yn, aPost[i]);
          aPre[i] = fmaf(g, xr[i][v], aPre[i]);
#pragma unroll
          for (int j = 0; j < N; ++j) aM[i][j] = fmaf(dr[i][v], xr[j][v], aM[i][j]);
        }
      }
    }
    float* dxt = dx + t * RS + 4 * tid;
#pragma unroll
    for (int j = 0; j < N; ++j) {
      float mc[N];
#pragma unroll
      for (int i = 0; i < N; ++i) mc[i] = sMT[j * N + i];
      float o[8];
#pragma unroll
      for (int v = 0; v < 8; ++v) o[v] = hpre[j] * dya[v];
#pragma unroll
      for (int i = 0; i < N; ++i)
#pragma unroll
        for (int v = 0; v < 8; ++v) o[v] = fmaf(mc[i], dr[i][v], o[v]);
      __stcs(reinterpret_cast<float4*>(dxt + (int64_t)j * C), make_float4(o[0], o[1], o[2], o[3]));
      __stcs(reinterpret_cast<float4*>(dxt + (int64_t)j * C + H),
             make_float4(o[4], o[5], o[6], o[7]));
    }
  }
  if (aborted) {
    // a bulk copy did not land in time: wait (bounded) for this CTA's other
    // copies in flight, then mark everything it owns as invalid
    if (tid == 0)
      for (unsigned k = use; k < issued; ++k) (void)mbar_wait(&s_full[k % NS], (k / NS) & 1u);
    const float nan = __int_as_float(0x7fc00000);
    const float4 n4 = make_float4(nan, nan, nan, nan);
    for (; t < T_; t += G)
#pragma unroll
      for (int j = 0; j < N; ++j) {
        float* dxt = dx + t * RS + (int64_t)j * C + 4 * tid;
        reinterpret_cast<float4*>(dxt)[0] = n4;
        reinterpret_cast<float4*>(dxt + H)[0] = n4;
      }
#pragma unroll
    for (int i = 0; i < N; ++i) {
      aPre[i] = nan; aPost[i] = nan;
#pragma unroll
      for (int j = 0; j < N; ++j) aM[i][j] = nan;
    }
#pragma unroll
    for (int v = 0; v < 8; ++v) aW[v] = nan;
  }

  // ---- per-CTA partials: fixed-order warp reductions + ordered warp sum ----
#pragma unroll
  for (int i = 0; i < N; ++i) {
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const float v = warp_sum(aM[i][j]);
      if (lane == 0) sacc[warp * P + i * N + j] = v;
    }
    const float a = warp_sum(aPre[i]);
    const float b = warp_sum(aPost[i]);
    if (lane == 0) { sacc[warp * P + N * N + i] = a; sacc[warp * P + N * N + N + i] = b; }
  }
  __syncthreads();
  for (int e = tid; e < P; e += BD) {
    float sum = 0.f;
#pragma unroll 4
    for (int q = 0; q < NW; ++q) sum += sacc[q * P + e];
    ws_p[(size_t)blockIdx.x * P + e] = sum;
  }
  float* wc = ws_c + (size_t)blockIdx.x * C + 4 * tid;
  reinterpret_cast<float4*>(wc)[0] = make_float4(aW[0], aW[1], aW[2], aW[3]);
  reinterpret_cast<float4*>(wc + H)[0] = make_float4(aW[4], aW[5], aW[6], aW[7]);
  if (blockIdx.x == 0 && tid == 0) { ws_hdr[0] = gridDim.x; ws_hdr[1] = 1; }
}

// Generic backward: any n <= 64, any C.  Pass 1 reduces ss and pd for the
// row; pass 2 walks the row in tiles of blockDim columns: each thread stages
// its column of x and d_out in shared memory (plus two extra rows: y inv w
// and dya), writes dx, and the CTA accumulates the (n+1) x (n+1) outer
// product D_aug X_aug^T with 4x4 register blocks:
//   [i<n, j<n] -> dM_ij,  [i<n, j=n] -> dHpost_i,  [i=n, j<n] -> dHpre_j.
// d_rms_weight accumulates in the CTA's own row of the column partials.
//
// Launched as thread-block clusters of cs = 1..8 CTAs: the CTAs of a cluster
// share each of the cluster's tokens, one column slice each (so a few tokens
// still fill the GPU), and the per-token sums (ss, pd) of the cs slices are
// added through distributed shared memory in rank order.  The partial pairs
// are double-buffered by token parity: a CTA cannot write the same buffer
// again before passing the next cluster barrier, which the others reach only
// after reading it.
constexpr int kGenBD = 128;   // threads per CTA (= tile width)
constexpr int kGenLD = kGenBD + 1;
constexpr int kGenRB = 4;     // register block edge
constexpr int kGenMaxBlk = 3; // ceil(ceil(65/4)^2 / 128)

template <typename XT, typename DT, typename DXT>
__global__ void __launch_bounds__(kGenBD)
k_bwd_generic(const XT* __restrict__ x, const DT* __restrict__ dout, const float* __restrict__ Mg,
              const float* __restrict__ hpre_g, const float* __restrict__ hpost_g,
              const float* __restrict__ w, DXT* __restrict__ dx, int64_t T, int n, int C,
              float eps, float* __restrict__ ws_p, float* __restrict__ ws_c,
              int* __restrict__ ws_hdr) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  const int cs = (int)cl.num_blocks(), rank = (int)cl.block_rank();
  const int64_t q0 = blockIdx.x / cs, Q = gridDim.x / cs;  // cluster index / count
  const int chunk = (C + cs - 1) / cs, cl0 = min(C, rank * chunk), cl1 = min(C, cl0 + chunk);
  __shared__ float2 s_part[2];
  extern __shared__ float smem[];
  const int na = n + 1;
  float* sM = smem;                       // n*n
  float* shpre = sM + n * n;              // n
  float* shpost = shpre + n;              // n
  float* sx = shpost + n;                 // na x kGenLD  (row n = y inv w)
  float* sd = sx + na * kGenLD;           // na x kGenLD  (row n = dya)
  __shared__ float red[2][64];
  const int tid = threadIdx.x;
  for (int e = tid; e < n * n; e += kGenBD) sM[e] = Mg[e];
  for (int e = tid; e < n; e += kGenBD) { shpre[e] = hpre_g[e]; shpost[e] = hpost_g[e]; }
  float* wc = ws_c + (size_t)blockIdx.x * C;
  for (int c = tid; c < C; c += kGenBD) wc[c] = 0.f;

  const int nb = (na + kGenRB - 1) / kGenRB;  // blocks per edge
  const int nblk = nb * nb;
  float acc[kGenMaxBlk][kGenRB][kGenRB];
#pragma unroll
  for (int q = 0; q < kGenMaxBlk; ++q)
#pragma unroll
    for (int a = 0; a < kGenRB; ++a)
#pragma unroll
      for (int b = 0; b < kGenRB; ++b) acc[q][a][b] = 0.f;
  __syncthreads();

  const int64_t rs = (int64_t)n * C;
  const float invC = 1.0f / (float)C;
  int par = 0;
  for (int64_t t = q0; t < T; t += Q) {
    const XT* xt = x + t * rs;
    const DT* dt = dout + t * rs;
    float ss = 0.f, pd = 0.f;
    for (int c = cl0 + tid; c < cl1; c += kGenBD) {
      float y = 0.f, dyn = 0.f;
      for (int i = 0; i < n; ++i) {
        y = fmaf(shpre[i], to_f(xt[(int64_t)i * C + c]), y);
        dyn = fmaf(shpost[i], to_f(dt[(int64_t)i * C + c]), dyn);
      }
      ss = fmaf(y, y, ss);
      pd = fmaf(dyn * __ldg(w + c), y, pd);
    }
    const float2 part = block_sum2(ss, pd, red[par]);
    if (tid == 0) s_part[par] = part;
    cl.sync();  // every slice's partial pair of this token is written
    float2 red2 = make_float2(0.f, 0.f);
    for (int r = 0; r < cs; ++r) {
      const float2 v = *cl.map_shared_rank(&s_part[par], r);
      red2.x += v.x;
      red2.y += v.y;
    }
    par ^= 1;
    const float inv = inv_rms(red2.x, C, eps);
    const float k2 = (red2.y * (inv * inv * inv)) * invC;
    DXT* dxt = dx + t * rs;
    for (int c0 = cl0; c0 < cl1; c0 += kGenBD) {
      const int c = c0 + tid;
      const bool ok = c < cl1;
      float y = 0.f, dyn = 0.f;
      for (int i = 0; i < n; ++i) {
        const float xv = ok ? to_f(xt[(int64_t)i * C + c]) : 0.f;
        const float dv = ok ? to_f(dt[(int64_t)i * C + c]) : 0.f;
        sx[i * kGenLD + tid] = xv;
        sd[i * kGenLD + tid] = dv;
        y = fmaf(shpre[i], xv, y);
        dyn = fmaf(shpost[i], dv, dyn);
      }
      const float wv = ok ? __ldg(w + c) : 0.f;
      const float yi = y * inv;
      const float g = (dyn * wv) * inv - k2 * y;
      sx[n * kGenLD + tid] = yi * wv;
      sd[n * kGenLD + tid] = ok ? g : 0.f;
      if (ok) {
        wc[c] = fmaf(dyn, yi, wc[c]);
        for (int j = 0; j < n; ++j) {
          float o = shpre[j] * g;
          for (int i = 0; i < n; ++i) o = fmaf(sM[i * n + j], sd[i * kGenLD + tid], o);
          dxt[(int64_t)j * C + c] = from_f<DXT>(o);
        }
      }
      __syncthreads();
      const int width = min(kGenBD, cl1 - c0);
#pragma unroll
      for (int q = 0; q < kGenMaxBlk; ++q) {
        const int blk = tid + q * kGenBD;
        if (blk >= nblk) break;
        const int i0 = (blk / nb) * kGenRB, j0 = (blk % nb) * kGenRB;
        for (int cc = 0; cc < width; ++cc) {
          float dv[kGenRB], xv[kGenRB];
#pragma unroll
          for (int a = 0; a < kGenRB; ++a) {
            dv[a] = (i0 + a < na) ? sd[(i0 + a) * kGenLD + cc] : 0.f;
            xv[a] = (j0 + a < na) ? sx[(j0 + a) * kGenLD + cc] : 0.f;
          }
#pragma unroll
          for (int a = 0; a < kGenRB; ++a)
#pragma unroll
            for (int b = 0; b < kGenRB; ++b) acc[q][a][b] = fmaf(dv[a], xv[b], acc[q][a][b]);
        }
      }
      __syncthreads();
    }
  }
  // scatter the owned blocks into this CTA's partial row
  const int P = n * n + 2 * n;
  float* pr = ws_p + (size_t)blockIdx.x * P;
#pragma unroll
  for (int q = 0; q < kGenMaxBlk; ++q) {
    const int blk = tid + q * kGenBD;
    if (blk >= nblk) break;
    const int i0 = (blk / nb) * kGenRB, j0 = (blk % nb) * kGenRB;
#pragma unroll
    for (int a = 0; a < kGenRB; ++a)
#pragma unroll
      for (int b = 0; b < kGenRB; ++b) {
        const int i = i0 + a, j = j0 + b;
        if (i < n && j < n) pr[i * n + j] = acc[q][a][b];
        else if (i == n && j < n) pr[n * n + j] = acc[q][a][b];      // dHpre_j
        else if (i < n && j == n) pr[n * n + n + i] = acc[q][a][b];  // dHpost_i
      }
  }
  if (blockIdx.x == 0 && tid == 0) { ws_hdr[0] = gridDim.x; ws_hdr[1] = 1; }
  cl.sync();  // the last token's partial pairs stay readable until every CTA has them
}

// Backward for n in {16, 32}: cluster column slices like k_bwd_generic, in
// two passes over a token's slice with compile-time N, so that the two
// n x n contractions are register-tiled and d_out is the only tensor read
// twice:
//   pass 1, per tile of 128 columns: stage x and d_out; per column y = sum
//     H_pre x, dyn = sum H_post d (kept in shared memory for pass 2) and the
//     token sums ss, pd; dM += d x^T as one 8 x 8 register block per thread
//     over SL = 128 / (N/8)^2 column slices (16 scalar loads for 64 FMAs);
//     and per-token sums that do not need inv yet:
//       U_i = sum d_i y w,  A_j = sum dyn w x_j,  B_j = sum y x_j,
//     since dH_post_i = inv U_i and dH_pre_j = sum dya x_j = inv A_j - k2 B_j
//     (dya = dyn w inv - k2 y), folded in once the token's inv and k2 are
//     known (8 / (N/8) rows and columns per thread);
//   pass 2, per tile: stage d_out and dya, then dx = M^T d + H_pre dya with
//     thread (jg, cg) owning streams 4jg..4jg+3 of DXC groups of 4 columns
//     (one float4 of M and DXC float4s of d per stream feed 16 DXC FMAs).
// PIPE (fp32 x and d_out, 16-byte aligned rows): two staging buffers; the
// next tile (of either pass, or of the next token) is copied with cp.async
// while the current one is computed, so load latency overlaps the
// contractions.  Otherwise each thread loads its column of the tile.
// Both contractions issue packed two-lane FMAs (fma2: bit-identical to fmaf).
// Staged row i starts at wide_row(i) = i * kWideLD + (i / 8) * 8 floats, so
// the 8-row blocks read by one warp fall on distinct banks and every row
// start is 16-byte aligned.  A slice holds at most kWideSlice columns (the
// launcher picks the cluster size).  The slices' dM blocks are added in slice
// order at the end (no atomics: bitwise reproducible).
constexpr int kWideBD = 128;
constexpr int kWideLD = kWideBD + 4;
constexpr int kWideSlice = 4096;
__host__ __device__ constexpr int wide_row(int i) { return i * kWideLD + (i >> 3) * 8; }
// [NBUF buffers: x rows | d rows][3 extra rows: y w, dyn w or dya, y][y, dyn per slice column]
__host__ __device__ constexpr int wide_ex_off(int n, int nbuf) { return nbuf * 2 * wide_row(n); }
__host__ __device__ constexpr size_t wide_smem_bytes(int n, int nbuf) {
  return ((size_t)wide_ex_off(n, nbuf) + 3 * kWideLD + 2 * (size_t)kWideSlice) * sizeof(float);
}

template <int N, typename XT, typename DT, typename DXT, bool PIPE>
__global__ void __launch_bounds__(kWideBD, PIPE ? 2 : 3)
k_bwd_wide(const XT* __restrict__ x, const DT* __restrict__ dout, const float* __restrict__ Mg,
           const float* __restrict__ hpre_g, const float* __restrict__ hpost_g,
           const float* __restrict__ w, DXT* __restrict__ dx, int64_t T, int C, float eps,
           int vec_dx, float* __restrict__ ws_p, float* __restrict__ ws_c,
           int* __restrict__ ws_hdr) {
  static_assert(N == 16 || N == 32, "register tiling for n = 16 and n = 32");
  static_assert(!PIPE || (std::is_same<XT, float>::value && std::is_same<DT, float>::value),
                "cp.async staging copies fp32 rows");
  constexpr int NBUF = PIPE ? 2 : 1;
  constexpr int NB = N / 8;                 // 8 x 8 blocks per edge
  constexpr int SL = kWideBD / (NB * NB);   // column slices of the dM product
  constexpr int HR = 8 / NB;                // dH rows / columns per thread
  constexpr int CG = kWideBD / (N / 4);     // 4-column groups in a dx row pass
  constexpr int DXC = kWideBD / (4 * CG);   // 4-column groups per thread
  constexpr int P = N * N + 2 * N;
  constexpr int BUFSZ = 2 * wide_row(N);
  static_assert(P <= wide_ex_off(N, 1), "partials fit the staging area");
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  const int cs = (int)cl.num_blocks(), rank = (int)cl.block_rank();
  const int64_t q0 = blockIdx.x / cs, Q = gridDim.x / cs;
  const int chunk = (((C + cs - 1) / cs) + 3) & ~3;  // slice starts on 4-column groups
  const int cl0 = min(C, rank * chunk), cl1 = min(C, cl0 + chunk);
  const int K = (cl1 - cl0 + kWideBD - 1) / kWideBD;  // tiles per pass
  __shared__ float2 s_part[2];
  __shared__ float red[2][64];
  __shared__ __align__(16) float sM[N * N];
  __shared__ float shpre[N], shpost[N];
  extern __shared__ __align__(16) float smem[];
  float* ex_yw = smem + wide_ex_off(N, NBUF);  // y w
  float* ex_dw = ex_yw + kWideLD;              // dyn w (pass 1) / dya (pass 2)
  float* ex_y = ex_dw + kWideLD;               // y
  float* sy = ex_y + kWideLD;                  // y of the slice's columns
  float* sdy = sy + kWideSlice;                // dyn of the slice's columns
  const int tid = threadIdx.x;
  for (int e = tid; e < N * N; e += kWideBD) sM[e] = Mg[e];
  if (tid < N) { shpre[tid] = hpre_g[tid]; shpost[tid] = hpost_g[tid]; }
  float* wc = ws_c + (size_t)blockIdx.x * C;
  for (int c = tid; c < C; c += kWideBD) wc[c] = 0.f;

  const int jg = tid / CG, cgi = tid % CG;            // dx roles
  const int sl = tid / (NB * NB), blk = tid % (NB * NB);
  const int bi = blk / NB, bj = blk % NB;              // dM roles
  float acc[8][8], hpo[HR], hpr[HR];
#pragma unroll
  for (int a = 0; a < 8; ++a)
#pragma unroll
    for (int b = 0; b < 8; ++b) acc[a][b] = 0.f;
#pragma unroll
  for (int r = 0; r < HR; ++r) { hpo[r] = 0.f; hpr[r] = 0.f; }
  __syncthreads();

  const int64_t rs = (int64_t)N * C;
  const float invC = 1.0f / (float)C;

  // cp.async of the next tile in the CTA's order (token, pass, tile) into
  // buffer b: pass 0 copies x and d_out rows, pass 1 d_out rows only.  The
  // slice and C are multiples of 4 columns, so a tile is whole 16-byte
  // chunks.  Every call commits one group (empty past the last tile).
  int64_t nt = q0;
  int npass = 0, nk = 0;
  auto issue_next = [&](int b) {
    if constexpr (PIPE) {
      if (K > 0 && nt < T) {
        float* bx = smem + b * BUFSZ;
        float* bd = bx + wide_row(N);
        const int c0 = cl0 + nk * kWideBD, nch = min(kWideBD, cl1 - c0) / 4;
        const float* xs = reinterpret_cast<const float*>(x) + nt * rs + c0;
        const float* ds = reinterpret_cast<const float*>(dout) + nt * rs + c0;
        const int rows = npass == 0 ? 2 * N : N;
        for (int e = tid; e < rows * (kWideBD / 4); e += kWideBD) {
          const int r = e / (kWideBD / 4), ch = e % (kWideBD / 4);
          if (ch < nch) {
            if (npass == 0 && r < N) {
              cp_async16(bx + wide_row(r) + 4 * ch, xs + (int64_t)r * C + 4 * ch);
            } else {
              const int i = npass == 0 ? r - N : r;
              cp_async16(bd + wide_row(i) + 4 * ch, ds + (int64_t)i * C + 4 * ch);
            }
          }
        }
      }
      cp_async_commit();
      if (++nk >= K) { nk = 0; if (++npass == 2) { npass = 0; nt += Q; } }
    }
  };
  int buf = 0;
  issue_next(0);

  int par = 0;
  for (int64_t t = q0; t < T; t += Q) {
    const XT* xt = x + t * rs;
    const DT* dt = dout + t * rs;
    float ss = 0.f, pd = 0.f, U[HR], A[HR], B[HR];
#pragma unroll
    for (int r = 0; r < HR; ++r) { U[r] = 0.f; A[r] = 0.f; B[r] = 0.f; }
    // ---- pass 1 ----
    for (int k = 0; k < K; ++k) {
      const int c0 = cl0 + k * kWideBD, width = min(kWideBD, cl1 - c0);
      float* bx = smem + buf * BUFSZ;
      float* bd = bx + wide_row(N);
      const int c = c0 + tid;
      const bool ok = tid < width;
      float y = 0.f, dyn = 0.f;
      if constexpr (PIPE) {
        issue_next(buf ^ 1);
        cp_async_wait_group<1>();
        __syncthreads();  // this tile's copies from every thread have landed
        if (ok) {
#pragma unroll 8
          for (int i = 0; i < N; ++i) {
            y = fmaf(shpre[i], bx[wide_row(i) + tid], y);
            dyn = fmaf(shpost[i], bd[wide_row(i) + tid], dyn);
          }
        }
      } else {
#pragma unroll 8
        for (int i = 0; i < N; ++i) {
          const float xv = ok ? to_f(xt[(int64_t)i * C + c]) : 0.f;
          const float dv = ok ? to_f(dt[(int64_t)i * C + c]) : 0.f;
          bx[wide_row(i) + tid] = xv;
          bd[wide_row(i) + tid] = dv;
          y = fmaf(shpre[i], xv, y);
          dyn = fmaf(shpost[i], dv, dyn);
        }
      }
      const float wv = ok ? __ldg(w + c) : 0.f;
      ss = fmaf(y, y, ss);
      pd = fmaf(dyn * wv, y, pd);
      ex_yw[tid] = y * wv;
      ex_dw[tid] = dyn * wv;
      ex_y[tid] = y;
      if (ok) { sy[c - cl0] = y; sdy[c - cl0] = dyn; }
      __syncthreads();
      for (int cc = sl; cc < width; cc += SL) {
        float dv[8], xv[8];
#pragma unroll
        for (int a = 0; a < 8; ++a) {
          dv[a] = bd[wide_row(8 * bi + a) + cc];
          xv[a] = bx[wide_row(8 * bj + a) + cc];
        }
#pragma unroll
        for (int a = 0; a < 8; ++a)
#pragma unroll
          for (int b = 0; b < 8; b += 2)
            fma2(acc[a][b], acc[a][b + 1], dv[a], dv[a], xv[b], xv[b + 1]);
        const float yw = ex_yw[cc], dw = ex_dw[cc], yv = ex_y[cc];
#pragma unroll
        for (int r = 0; r < HR; ++r) {
          U[r] = fmaf(bd[wide_row(8 * bi + HR * bj + r) + cc], yw, U[r]);
          const float xj = bx[wide_row(8 * bj + HR * bi + r) + cc];
          A[r] = fmaf(dw, xj, A[r]);
          B[r] = fmaf(yv, xj, B[r]);
        }
      }
      __syncthreads();
      if constexpr (PIPE) buf ^= 1;
    }
    const float2 part = block_sum2(ss, pd, red[par]);
    if (tid == 0) s_part[par] = part;
    cl.sync();  // every slice's partial pair of this token is written
    float2 red2 = make_float2(0.f, 0.f);
    for (int r = 0; r < cs; ++r) {
      const float2 v = *cl.map_shared_rank(&s_part[par], r);
      red2.x += v.x;
      red2.y += v.y;
    }
    par ^= 1;
    const float inv = inv_rms(red2.x, C, eps);
    const float k2 = (red2.y * (inv * inv * inv)) * invC;
#pragma unroll
    for (int r = 0; r < HR; ++r) {
      hpo[r] = fmaf(inv, U[r], hpo[r]);
      hpr[r] += inv * A[r] - k2 * B[r];
    }
    // ---- pass 2: dx ----
    DXT* dxt = dx + t * rs;
    for (int k = 0; k < K; ++k) {
      const int c0 = cl0 + k * kWideBD, width = min(kWideBD, cl1 - c0);
      float* bd = smem + buf * BUFSZ + wide_row(N);
      const int c = c0 + tid;
      const bool ok = tid < width;
      if constexpr (PIPE) {
        issue_next(buf ^ 1);
        cp_async_wait_group<1>();
      } else {
#pragma unroll 16
        for (int i = 0; i < N; ++i) bd[wide_row(i) + tid] = ok ? to_f(dt[(int64_t)i * C + c]) : 0.f;
      }
      if (ok) {
        const float y = sy[c - cl0], dyn = sdy[c - cl0], wv = __ldg(w + c);
        ex_dw[tid] = (dyn * wv) * inv - k2 * y;
        wc[c] = fmaf(dyn, y * inv, wc[c]);
      } else {
        ex_dw[tid] = 0.f;
      }
      __syncthreads();
#pragma unroll
      for (int q = 0; q < DXC; ++q) {
        const int cb = 4 * cgi + 4 * CG * q;
        if (cb < width) {
          float o[4][4];
          const float4 g4 = *reinterpret_cast<const float4*>(ex_dw + cb);
#pragma unroll
          for (int a = 0; a < 4; ++a) {
            const float hp = shpre[4 * jg + a];
            o[a][0] = hp * g4.x; o[a][1] = hp * g4.y; o[a][2] = hp * g4.z; o[a][3] = hp * g4.w;
          }
#pragma unroll 8
          for (int i = 0; i < N; ++i) {
            const float4 m4 = *reinterpret_cast<const float4*>(sM + i * N + 4 * jg);
            const float4 d4 = *reinterpret_cast<const float4*>(bd + wide_row(i) + cb);
            const float mv[4] = {m4.x, m4.y, m4.z, m4.w};
#pragma unroll
            for (int a = 0; a < 4; ++a) {
              fma2(o[a][0], o[a][1], mv[a], mv[a], d4.x, d4.y);
              fma2(o[a][2], o[a][3], mv[a], mv[a], d4.z, d4.w);
            }
          }
#pragma unroll
          for (int a = 0; a < 4; ++a) {
            DXT* dst = dxt + (int64_t)(4 * jg + a) * C + c0 + cb;
            if (vec_dx && cb + 4 <= width) {
              store_vec<DXT, 4, true>(dst, o[a]);
            } else {
#pragma unroll
              for (int v = 0; v < 4; ++v)
                if (cb + v < width) dst[v] = from_f<DXT>(o[a][v]);
            }
          }
        }
      }
      __syncthreads();
      if constexpr (PIPE) buf ^= 1;
    }
  }
  if constexpr (PIPE) cp_async_wait_all();  // only empty groups can remain
  // add the slices' blocks in slice order in the (now free) staging area
  float* sbuf = smem;
  for (int s = 0; s < SL; ++s) {
    if (sl == s) {
#pragma unroll
      for (int a = 0; a < 8; ++a)
#pragma unroll
        for (int b = 0; b < 8; ++b) {
          float& e = sbuf[(8 * bi + a) * N + 8 * bj + b];
          e = (s == 0 ? 0.f : e) + acc[a][b];
        }
#pragma unroll
      for (int r = 0; r < HR; ++r) {
        float& e1 = sbuf[N * N + N + 8 * bi + HR * bj + r];  // dH_post_i
        e1 = (s == 0 ? 0.f : e1) + hpo[r];
        float& e2 = sbuf[N * N + 8 * bj + HR * bi + r];      // dH_pre_j
        e2 = (s == 0 ? 0.f : e2) + hpr[r];
      }
    }
    __syncthreads();
  }
  // The cluster's CTAs add their parameter partials through distributed
  // shared memory in rank order; rank 0 writes the sum, so the finalize reads
  // one parameter row per cluster (header word 1 = cs: rows 0, cs, 2cs, ...).
  // The d_rms_weight rows stay per CTA (each CTA owns its columns).
  cl.sync();  // every CTA's sums are complete; the last token's partial pairs are read
  if (rank == 0) {
    float* pr = ws_p + (size_t)blockIdx.x * P;
    for (int e = tid; e < P; e += kWideBD) {
      float v = 0.f;
      for (int r = 0; r < cs; ++r) v += cl.map_shared_rank(sbuf, r)[e];
      pr[e] = v;
    }
  }
  if (blockIdx.x == 0 && tid == 0) { ws_hdr[0] = gridDim.x; ws_hdr[1] = cs; }
  cl.sync();  // every CTA's shared memory stays alive until rank 0 has read it
}

// ================================================================ finalize ==
// Blocks of BD threads (256, or 1024 for n = 32 so that its Sinkhorn
// backward runs one matrix entry per thread).  Blocks [0, nbc) reduce
// d_rms_weight, 32 columns per block: thread (slice r, column c) sums partial
// rows r, r + S, r + 2S, ... (S = BD / 32 slices) and the slice sums are
// added in slice order -- a fixed order for a given row count, with S times
// fewer dependent loads per thread than a plain column walk.  The last block
// reduces the n*n + 2n parameter partials (sliced the same way when 2P <= BD,
// else whole rows per entry) and optionally runs the parameter chain
// (Sinkhorn backward from a staged tape + sigmoid derivatives).
template <int BD>
__device__ __forceinline__ float sliced_row_sum(const float* __restrict__ base, size_t stride,
                                                int G, int r0) {
  float s = 0.f;
#pragma unroll 4
  for (int g = r0; g < G; g += BD / 32) s += base[(size_t)g * stride];
  return s;
}

template <int BD>
__global__ void __launch_bounds__(BD)
k_finalize(const char* __restrict__ ws, int n, int C, float* __restrict__ dM,
           float* __restrict__ dhpre, float* __restrict__ dhpost, float* __restrict__ dw,
           const float* __restrict__ hpre_raw, const float* __restrict__ hpost_raw,
           const float* __restrict__ hres_raw, const float* __restrict__ tape, int iters,
           float eps, float* __restrict__ dhpre_raw, float* __restrict__ dhpost_raw,
           float* __restrict__ dhres_raw, int stage_sk) {
  const int G = reinterpret_cast<const int*>(ws)[0];
  // parameter partials sit in rows 0, step, 2 step, ... (step > 1 when the
  // CTAs of a cluster combined theirs); d_rms_weight partials in all G rows
  const int step = max(1, reinterpret_cast<const int*>(ws)[1]);
  const int Gp = (G + step - 1) / step;
  const size_t pstride = (size_t)step * (size_t)(n * n + 2 * n);
  const int P = n * n + 2 * n;
  const float* wp = reinterpret_cast<const float*>(ws + WsLayout::params_off());
  const float* wc = reinterpret_cast<const float*>(ws + WsLayout::cols_off(G, n));
  const int nbc = (C + 31) / 32;
  const int tid = threadIdx.x, lane = tid & 31, r0 = tid >> 5;
  __shared__ float part[(BD / 32)][32];
  if ((int)blockIdx.x < nbc) {
    const int c = blockIdx.x * 32 + lane;
    part[r0][lane] = (c < C) ? sliced_row_sum<BD>(wc + c, C, G, r0) : 0.f;
    __syncthreads();
    if (r0 == 0 && c < C && dw) {
      float s = 0.f;
#pragma unroll
      for (int q = 0; q < (BD / 32); ++q) s += part[q][lane];
      dw[c] = s;
    }
    return;
  }
  __shared__ float sP[kMaxN * kMaxN + 2 * kMaxN];
  __shared__ float D[kMaxN * (kMaxN + 1)];
  extern __shared__ float s_fin[];  // optional staged copy of tape + logits
  auto emit = [&](int e, float s) {
    sP[e] = s;
    if (e < n * n) { if (dM) dM[e] = s; }
    else if (e < n * n + n) { if (dhpre) dhpre[e - n * n] = s; }
    else if (dhpost) dhpost[e - n * n - n] = s;
  };
  if (2 * P <= BD) {
    // every thread of the block: S = BD / P slices of the G rows per
    // entry, consecutive threads on consecutive entries of a row
    float* flat = &part[0][0];
    const int S = BD / P, e = tid % P, q = tid / P;
    if (q < S) {
      float s = 0.f;
#pragma unroll 8
      for (int g = q; g < Gp; g += S) s += wp[(size_t)g * pstride + e];
      flat[q * P + e] = s;
    }
    __syncthreads();
    if (tid < P) {
      float s = 0.f;
      for (int k = 0; k < S; ++k) s += flat[k * P + tid];
      emit(tid, s);
    }
    __syncthreads();
  } else {
    // Larger n: thread tid owns entries tid + k * BD and adds their G
    // partial rows in row order, KE entries at a time, so each row step
    // issues KE independent loads (and the unrolled steps several rows'
    // worth) instead of one dependent load per 32-entry group.
    constexpr int KE = BD >= 1024 ? 2 : 5;
    for (int base = 0; base < P; base += KE * BD) {
      float s[KE];
      int ee[KE];
#pragma unroll
      for (int k = 0; k < KE; ++k) { ee[k] = base + tid + k * BD; s[k] = 0.f; }
#pragma unroll 8
      for (int g = 0; g < Gp; ++g) {
        const float* row = wp + (size_t)g * pstride;
#pragma unroll
        for (int k = 0; k < KE; ++k)
          if (ee[k] < P) s[k] += row[ee[k]];
      }
#pragma unroll
      for (int k = 0; k < KE; ++k)
        if (ee[k] < P) emit(ee[k], s[k]);
    }
    __syncthreads();
  }
  sk_params_bwd_tail<BD>(sP, n, hpre_raw, hpost_raw, hres_raw, tape, nullptr, iters, eps,
                         stage_sk, s_fin, D, dhpre_raw, dhpost_raw, dhres_raw);
}

// ================================================================= launch ==
// Environment overrides for tuning sweeps (unset in normal use):
//   MHC_B200_FWD_ITEMS / MHC_B200_BWD_ITEMS  force the ITEMS of the fast path
//   MHC_B200_GENERIC=1                       force the generic kernels
static int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return v && *v ? atoi(v) : dflt;
}

int max_partial_rows(int64_t T) {
  int64_t g = (int64_t)sm_count() * 4;
  if (g > 8 * T) g = 8 * T;  // up to 8 column slices per token (cluster-split backward)
  return (int)(g < 1 ? 1 : g);
}

template <typename K>
static int persistent_grid(K kernel, int threads, size_t smem, int64_t T, int cap) {
  int per_sm = blocks_per_sm(kernel, threads, smem);
  if (per_sm < 1) per_sm = 1;
  int64_t g = (int64_t)per_sm * sm_count();
  if (g > cap) g = cap;
  if (g > T) g = T;
  return (int)(g < 1 ? 1 : g);
}

// Threads per CTA ceiling for a fast instantiation holding `d` fp32 row
// values per thread.
constexpr int fast_maxt(int d) { return d <= 16 ? 1024 : (d <= 64 ? 512 : 256); }

static int round32(int v) { return (v + 31) & ~31; }

// ---- forward dispatch -------------------------------------------------------
template <int N, typename InT, typename OutT, int VEC, int ITEMS>
static int try_fwd_items(const InT* x, const float* M, const float* hpre, const float* hpost,
                         const float* w, OutT* out, int64_t T, int C, float eps, cudaStream_t st) {
  constexpr int d = N * VEC * ITEMS;
  if constexpr (d > 64) {
    return -1;
  } else {
    constexpr int MAXT = fast_maxt(d);
    const int groups = (C + VEC - 1) / VEC;
    const int threads = round32((groups + ITEMS - 1) / ITEMS);
    if (threads > MAXT) return -1;
    const size_t smem = (size_t)ITEMS * N * 16 * threads;
    // Measured on B200 (n=4, C=4096, 64K tokens): staging the next row helps
    // 16-bit inputs (715 -> 685 us) and costs fp32 inputs (1380 -> 1438 us),
    // whose two resident CTAs per SM already overlap load and store phases.
    if constexpr (VEC * sizeof(InT) == 16 && sizeof(InT) == 2) {
      if (env_int("MHC_B200_PIPE", 1) && smem <= (size_t)max_smem_optin()) {
        auto kern = k_fwd_fast<N, InT, OutT, VEC, ITEMS, MAXT, true>;
        cudaError_t e = allow_dyn_smem(kern, smem);
        if (e != cudaSuccess) return set_error(MHC_ERR_CUDA, "mhc_fwd: %s", cudaGetErrorString(e));
        const int grid = persistent_grid(kern, threads, smem, T, 1 << 30);
        kern<<<grid, threads, smem, st>>>(x, M, hpre, hpost, w, out, T, C, eps);
        return check_launch("mhc_fwd");
      }
    }
    auto kern = k_fwd_fast<N, InT, OutT, VEC, ITEMS, MAXT, false>;
    const int grid = persistent_grid(kern, threads, 0, T, 1 << 30);
    kern<<<grid, threads, 0, st>>>(x, M, hpre, hpost, w, out, T, C, eps);
    return check_launch("mhc_fwd");
  }
}

template <int N, typename InT, typename OutT, int VEC>
static int try_fwd_vec(const InT* x, const float* M, const float* hpre, const float* hpost,
                       const float* w, OutT* out, int64_t T, int C, float eps, cudaStream_t st) {
  const int forced = env_int("MHC_B200_FWD_ITEMS", 0);
  const int groups = (C + VEC - 1) / VEC;
  // Default: the fewest ITEMS whose block is at most 512 threads (256 for
  // 16-bit inputs: measured on B200, n=4, C=4096, 64K tokens, bf16 in/out,
  // 687 us with 512 threads x 1 group, 660 us with 256 threads x 2 groups;
  // fp32 is flat between 2 and 4 groups, 1393 / 1389 us).
  const int cap = sizeof(InT) == 2 ? 256 : 512;
  const int order[4] = {1, 2, 4, 8};
  for (int k = 0; k < 4; ++k) {
    const int items = order[k];
    if (forced && items != forced) continue;
    if (!forced && round32((groups + items - 1) / items) > cap && items != 8) continue;
    int r = -1;
    switch (items) {
      case 1: r = try_fwd_items<N, InT, OutT, VEC, 1>(x, M, hpre, hpost, w, out, T, C, eps, st); break;
      case 2: r = try_fwd_items<N, InT, OutT, VEC, 2>(x, M, hpre, hpost, w, out, T, C, eps, st); break;
      case 4: r = try_fwd_items<N, InT, OutT, VEC, 4>(x, M, hpre, hpost, w, out, T, C, eps, st); break;
      case 8: r = try_fwd_items<N, InT, OutT, VEC, 8>(x, M, hpre, hpost, w, out, T, C, eps, st); break;
    }
    if (r >= 0) return r;
  }
  return -1;
}

template <int N, typename InT, typename OutT>
static int fwd_fast(const InT* x, const float* M, const float* hpre, const float* hpost,
                    const float* w, OutT* out, int64_t T, int C, float eps, cudaStream_t st) {
  constexpr int VV = VecOf<InT>::value;
  const bool vec_ok = (C % VV == 0) && aligned16(x) && aligned16(out) && aligned16(w);
  if (vec_ok) {
    const int r = try_fwd_vec<N, InT, OutT, VV>(x, M, hpre, hpost, w, out, T, C, eps, st);
    if (r >= 0) return r;
  }
  return try_fwd_vec<N, InT, OutT, 1>(x, M, hpre, hpost, w, out, T, C, eps, st);
}

// Cluster-split forward (k_fwd_split) for n in {16, 32, 64}; the cluster
// size targets about four CTAs per SM in flight.
template <int N, typename InT, typename OutT>
static int launch_fwd_split(const InT* x, const float* M, const float* hpre, const float* hpost,
                            const float* w, OutT* out, int64_t T, int C, float eps,
                            cudaStream_t st) {
  const int64_t want = 4 * (int64_t)sm_count();
  int cs = 1;
  while (cs < 8 && T * cs < want && C / (2 * cs) >= 256) cs *= 2;
  if (T * cs > 0x7fffffffLL) return -1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(T * cs), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e =
      cudaLaunchKernelEx(&cfg, k_fwd_split<N, InT, OutT>, x, M, hpre, hpost, w, out, T, C, eps);
  if (e != cudaSuccess) return set_error(MHC_ERR_CUDA, "mhc_fwd(split): %s", cudaGetErrorString(e));
  return check_launch("mhc_fwd(split)");
}

template <typename InT, typename OutT>
static int fwd_generic(const InT* x, const float* M, const float* hpre, const float* hpost,
                       const float* w, OutT* out, int64_t T, int n, int C, float eps,
                       cudaStream_t st) {
  if (n <= 16) {
    auto kern = k_fwd_generic<16, InT, OutT>;
    const int grid = persistent_grid(kern, 256, 0, T, 1 << 30);
    kern<<<grid, 256, 0, st>>>(x, M, hpre, hpost, w, out, T, n, C, eps);
  } else {
    auto kern = k_fwd_generic<64, InT, OutT>;
    const int grid = persistent_grid(kern, 256, 0, T, 1 << 30);
    kern<<<grid, 256, 0, st>>>(x, M, hpre, hpost, w, out, T, n, C, eps);
  }
  return check_launch("mhc_fwd(generic)");
}

template <typename InT, typename OutT>
static int fwd_typed(const void* xv, const float* M, const float* hpre, const float* hpost,
                     const float* w, void* ov, int64_t T, int n, int C, float eps,
                     cudaStream_t st) {
  const InT* x = static_cast<const InT*>(xv);
  OutT* out = static_cast<OutT*>(ov);
  if (!env_int("MHC_B200_GENERIC", 0)) {
    int r = -1;
    switch (n) {
      case 1: r = fwd_fast<1, InT, OutT>(x, M, hpre, hpost, w, out, T, C, eps, st); break;
      case 2: r = fwd_fast<2, InT, OutT>(x, M, hpre, hpost, w, out, T, C, eps, st); break;
      case 4: r = fwd_fast<4, InT, OutT>(x, M, hpre, hpost, w, out, T, C, eps, st); break;
      case 8: r = fwd_fast<8, InT, OutT>(x, M, hpre, hpost, w, out, T, C, eps, st); break;
      case 16: r = fwd_fast<16, InT, OutT>(x, M, hpre, hpost, w, out, T, C, eps, st); break;
      case 32: r = fwd_fast<32, InT, OutT>(x, M, hpre, hpost, w, out, T, C, eps, st); break;
      default: break;
    }
    if (r >= 0) return r;
    if (env_int("MHC_B200_SPLIT", 1)) {
      switch (n) {
        case 16: r = launch_fwd_split<16, InT, OutT>(x, M, hpre, hpost, w, out, T, C, eps, st); break;
        case 32: r = launch_fwd_split<32, InT, OutT>(x, M, hpre, hpost, w, out, T, C, eps, st); break;
        case 64: r = launch_fwd_split<64, InT, OutT>(x, M, hpre, hpost, w, out, T, C, eps, st); break;
        default: break;
      }
      if (r >= 0) return r;
    }
  }
  return fwd_generic<InT, OutT>(x, M, hpre, hpost, w, out, T, n, C, eps, st);
}

int launch_fwd(const void* x, int xdt, const float* M, const float* hpre, const float* hpost,
               const float* w, void* out, int odt, int64_t T, int n, int C, float eps,
               cudaStream_t st) {
  if (T == 0) return MHC_OK;
  if (xdt == MHC_F32 && odt == MHC_F32)
    return fwd_typed<float, float>(x, M, hpre, hpost, w, out, T, n, C, eps, st);
  if (xdt == MHC_BF16 && odt == MHC_F32)
    return fwd_typed<bf16, float>(x, M, hpre, hpost, w, out, T, n, C, eps, st);
  if (xdt == MHC_BF16 && odt == MHC_BF16)
    return fwd_typed<bf16, bf16>(x, M, hpre, hpost, w, out, T, n, C, eps, st);
  if (xdt == MHC_F16 && odt == MHC_F32)
    return fwd_typed<f16, float>(x, M, hpre, hpost, w, out, T, n, C, eps, st);
  if (xdt == MHC_F16 && odt == MHC_F16)
    return fwd_typed<f16, f16>(x, M, hpre, hpost, w, out, T, n, C, eps, st);
  return set_error(MHC_ERR_UNSUPPORTED, "mhc_fwd: unsupported dtype pair x=%d out=%d", xdt, odt);
}

// ---- backward dispatch ------------------------------------------------------
size_t bwd_ws_bytes(int64_t T, int n, int C) {
  return WsLayout::bytes(max_partial_rows(T), n, C);
}

struct BwdPtrs {
  float* p;
  float* c;
  int* hdr;
};

static BwdPtrs ws_ptrs(void* ws, int G, int n) {
  char* b = static_cast<char*>(ws);
  return {reinterpret_cast<float*>(b + WsLayout::params_off()),
          reinterpret_cast<float*>(b + WsLayout::cols_off(G, n)), reinterpret_cast<int*>(b)};
}

// Full-row 16-bit backward (k_bwd_rows) for C = 8 * BD, BD in {128, 256,
// 512}.  Returns -1 when the shape has no instantiation.
template <int N, typename T, int BD>
static int launch_bwd_rows(const T* x, const T* d, const float* M, const float* hpre,
                           const float* hpost, const float* w, T* dx, int64_t T_, float eps,
                           void* ws, cudaStream_t st) {
  constexpr bool kMma = N == 4;
  auto go = [&](auto kern, size_t dyn) -> int {
    cudaError_t e = allow_dyn_smem(kern, dyn);
    if (e != cudaSuccess) return set_error(MHC_ERR_CUDA, "mhc_bwd: %s", cudaGetErrorString(e));
    const int G = persistent_grid(kern, BD, dyn, T_, max_partial_rows(T_));
    BwdPtrs p = ws_ptrs(ws, G, N);
    kern<<<G, BD, dyn, st>>>(x, d, M, hpre, hpost, w, dx, T_, eps, p.p, p.c, p.hdr);
    return check_launch("mhc_bwd");
  };
  // w (2 float4 per thread), then NBUF buffers of 2N staged rows
  const size_t wb = (size_t)BD * 32, row = 16;
  const bool two = env_int("MHC_B200_NBUF", 1) == 2;
  if constexpr (kMma) {
    if (env_int("MHC_B200_MMA", 1)) {
      const size_t rows = (size_t)2 * N * (BD + 1) * row;
      // bulk-copy staging, three buffers by default (MHC_B200_BULK = 0
      // selects the per-thread cp.async staging, 2 or 3 the number of
      // bulk-copy buffers).  B200, n = 4, C = 4096, T = 65536 bf16:
      // cp.async 1132-1288 us, 2 buffers 1017 us, 3 buffers 990 us.
      const int bulk = env_int("MHC_B200_BULK", 3);
      if (bulk == 3 && wb + 3 * rows + 4096 <= (size_t)max_smem_optin())
        return go(k_bwd_rows<N, T, BD, true, 3, true>, wb + 3 * rows);
      if (bulk >= 2) return go(k_bwd_rows<N, T, BD, true, 2, true>, wb + 2 * rows);
      if (two) return go(k_bwd_rows<N, T, BD, true, 2>, wb + 2 * rows);
      return go(k_bwd_rows<N, T, BD, true, 1>, wb + rows);
    }
  }
  const size_t rows = (size_t)2 * N * BD * row;
  if (two) return go(k_bwd_rows<N, T, BD, false, 2>, wb + 2 * rows);
  return go(k_bwd_rows<N, T, BD, false, 1>, wb + rows);
}

// fp32 full-row backward with bulk-copy half-token staging (k_bwd_rows32) for
// n = 4, C = 8 * BD, BD in {128, 256, 512}.  Returns -1 when not applicable.
template <int BD>
static int launch_bwd_rows32(const float* x, const float* d, const float* M, const float* hpre,
                             const float* hpost, const float* w, float* dx, int64_t T_,
                             float eps, void* ws, cudaStream_t st) {
  constexpr int C = 8 * BD;
  const size_t dyn = (size_t)BD * 32 + (size_t)3 * 2 * 4 * (C / 2) * sizeof(float);
  if (dyn + 4096 > (size_t)max_smem_optin()) return -1;
  auto kern = k_bwd_rows32<4, BD>;
  cudaError_t e = allow_dyn_smem(kern, dyn);
  if (e != cudaSuccess) return set_error(MHC_ERR_CUDA, "mhc_bwd: %s", cudaGetErrorString(e));
  const int G = persistent_grid(kern, BD, dyn, T_, max_partial_rows(T_));
  BwdPtrs p = ws_ptrs(ws, G, 4);
  kern<<<G, BD, dyn, st>>>(x, d, M, hpre, hpost, w, dx, T_, eps, p.p, p.c, p.hdr);
  return check_launch("mhc_bwd");
}

static int bwd_rows32(const float* x, const float* d, const float* M, const float* hpre,
                      const float* hpost, const float* w, float* dx, int64_t T_, int C,
                      float eps, void* ws, cudaStream_t st) {
  // MHC_B200_BULK32=0 keeps the per-thread cp.async backward (A/B measurement)
  if (!env_int("MHC_B200_BULK32", 1) || !env_int("MHC_B200_FULL", 1)) return -1;
  if (!(aligned16(x) && aligned16(d) && aligned16(dx) && aligned16(w))) return -1;
  switch (C) {
    case 1024: return launch_bwd_rows32<128>(x, d, M, hpre, hpost, w, dx, T_, eps, ws, st);
    case 2048: return launch_bwd_rows32<256>(x, d, M, hpre, hpost, w, dx, T_, eps, ws, st);
    case 4096: return launch_bwd_rows32<512>(x, d, M, hpre, hpost, w, dx, T_, eps, ws, st);
    default: return -1;
  }
}

template <int N, typename T>
static int bwd_rows(const T* x, const T* d, const float* M, const float* hpre, const float* hpost,
                    const float* w, T* dx, int64_t T_, int C, float eps, void* ws,
                    cudaStream_t st) {
  if (!env_int("MHC_B200_FULL", 1) || !env_int("MHC_B200_PIPE", 1)) return -1;
  if (!(aligned16(x) && aligned16(d) && aligned16(dx) && aligned16(w))) return -1;
  switch (C) {
    case 1024: return launch_bwd_rows<N, T, 128>(x, d, M, hpre, hpost, w, dx, T_, eps, ws, st);
    case 2048: return launch_bwd_rows<N, T, 256>(x, d, M, hpre, hpost, w, dx, T_, eps, ws, st);
    case 4096: return launch_bwd_rows<N, T, 512>(x, d, M, hpre, hpost, w, dx, T_, eps, ws, st);
    default: return -1;
  }
}

template <int N, typename XT, typename DT, typename DXT, int VEC, int ITEMS>
static int try_bwd_items(const XT* x, const DT* d, const float* M, const float* hpre,
                         const float* hpost, const float* w, DXT* dx, int64_t T, int C, float eps,
                         void* ws, cudaStream_t st) {
  constexpr int d2 = 2 * N * VEC * ITEMS;
  if constexpr (d2 > 64) {
    return -1;
  } else {
    constexpr int MAXT = d2 <= 16 ? 1024 : 512;
    const int groups = (C + VEC - 1) / VEC;
    const int threads = round32((groups + ITEMS - 1) / ITEMS);
    if (threads > MAXT) return -1;
    constexpr bool kCanPipe = VEC * sizeof(XT) == 16 && VEC * sizeof(DT) == 16;
    const size_t smem = (size_t)2 * ITEMS * N * 16 * threads;
    const bool pipe = kCanPipe && env_int("MHC_B200_PIPE", 1) && smem <= (size_t)max_smem_optin();
    auto launch = [&](auto kern, size_t dyn) -> int {
      cudaError_t e = allow_dyn_smem(kern, dyn);
      if (e != cudaSuccess) return set_error(MHC_ERR_CUDA, "mhc_bwd: %s", cudaGetErrorString(e));
      const int G = persistent_grid(kern, threads, dyn, T, max_partial_rows(T));
      BwdPtrs p = ws_ptrs(ws, G, N);
      kern<<<G, threads, dyn, st>>>(x, d, M, hpre, hpost, w, dx, T, C, eps, p.p, p.c, p.hdr);
      return check_launch("mhc_bwd");
    };
    if constexpr (kCanPipe) {
      if (pipe) return launch(k_bwd_fast<N, XT, DT, DXT, VEC, ITEMS, MAXT, true>, smem);
    }
    return launch(k_bwd_fast<N, XT, DT, DXT, VEC, ITEMS, MAXT, false>, 0);
  }
}

template <int N, typename XT, typename DT, typename DXT, int VEC>
static int try_bwd_vec(const XT* x, const DT* d, const float* M, const float* hpre,
                       const float* hpost, const float* w, DXT* dx, int64_t T, int C, float eps,
                       void* ws, cudaStream_t st) {
  const int forced = env_int("MHC_B200_BWD_ITEMS", 0);
  const int groups = (C + VEC - 1) / VEC;
  const int order[4] = {1, 2, 4, 8};
  for (int k = 0; k < 4; ++k) {
    const int items = order[k];
    if (forced && items != forced) continue;
    if (!forced && round32((groups + items - 1) / items) > 512 && items != 8) continue;
    int r = -1;
    switch (items) {
      case 1: r = try_bwd_items<N, XT, DT, DXT, VEC, 1>(x, d, M, hpre, hpost, w, dx, T, C, eps, ws, st); break;
      case 2: r = try_bwd_items<N, XT, DT, DXT, VEC, 2>(x, d, M, hpre, hpost, w, dx, T, C, eps, ws, st); break;
      case 4: r = try_bwd_items<N, XT, DT, DXT, VEC, 4>(x, d, M, hpre, hpost, w, dx, T, C, eps, ws, st); break;
      case 8: r = try_bwd_items<N, XT, DT, DXT, VEC, 8>(x, d, M, hpre, hpost, w, dx, T, C, eps, ws, st); break;
    }
    if (r >= 0) return r;
  }
  return -1;
}

template <int N, typename XT, typename DT, typename DXT>
static int bwd_fast(const XT* x, const DT* d, const float* M, const float* hpre,
                    const float* hpost, const float* w, DXT* dx, int64_t T, int C, float eps,
                    void* ws, cudaStream_t st) {
  constexpr int VX = VecOf<XT>::value, VD = VecOf<DT>::value;
  // one vector width for both streams: the wider element count is used
  // only if both dtypes share it (f32/f32 -> 4, 16-bit/16-bit -> 8)
  if constexpr (sizeof(XT) == 2 && std::is_same<XT, DT>::value && std::is_same<XT, DXT>::value &&
                N <= 4) {
    const int r = bwd_rows<N, XT>(x, d, M, hpre, hpost, w, dx, T, C, eps, ws, st);
    if (r >= 0) return r;
  }
  if constexpr (N == 4 && std::is_same<XT, float>::value && std::is_same<DT, float>::value &&
                std::is_same<DXT, float>::value) {
    const int r = bwd_rows32(x, d, M, hpre, hpost, w, dx, T, C, eps, ws, st);
    if (r >= 0) return r;
  }
  if constexpr (VX == VD && VecOf<DXT>::value == VX) {
    const bool vec_ok = (C % VX == 0) && aligned16(x) && aligned16(d) && aligned16(dx) &&
                        aligned16(w);
    if (vec_ok) {
      const int r = try_bwd_vec<N, XT, DT, DXT, VX>(x, d, M, hpre, hpost, w, dx, T, C, eps, ws, st);
      if (r >= 0) return r;
    }
  }
  return try_bwd_vec<N, XT, DT, DXT, 1>(x, d, M, hpre, hpost, w, dx, T, C, eps, ws, st);
}

template <typename XT, typename DT, typename DXT>
static int bwd_typed(const void* xv, const void* dv, const float* M, const float* hpre,
                     const float* hpost, const float* w, void* dxv, int64_t T, int n, int C,
                     float eps, void* ws, cudaStream_t st) {
  const XT* x = static_cast<const XT*>(xv);
  const DT* d = static_cast<const DT*>(dv);
  DXT* dx = static_cast<DXT*>(dxv);
  if (!env_int("MHC_B200_GENERIC", 0)) {
    int r = -1;
    switch (n) {
      case 1: r = bwd_fast<1, XT, DT, DXT>(x, d, M, hpre, hpost, w, dx, T, C, eps, ws, st); break;
      case 2: r = bwd_fast<2, XT, DT, DXT>(x, d, M, hpre, hpost, w, dx, T, C, eps, ws, st); break;
      case 4: r = bwd_fast<4, XT, DT, DXT>(x, d, M, hpre, hpost, w, dx, T, C, eps, ws, st); break;
      case 8: r = bwd_fast<8, XT, DT, DXT>(x, d, M, hpre, hpost, w, dx, T, C, eps, ws, st); break;
      default: break;
    }
    if (r >= 0) return r;
  }
  // Cluster launch shared by the wide and generic kernels: split each
  // token's columns over cs CTAs while there are few tokens per resident
  // CTA slot; Q clusters loop over the tokens.
  auto launch_clusters = [&](auto kern, size_t smem, int cs_min, const char* what,
                             auto... tail) -> int {
    {
      cudaError_t e = allow_dyn_smem(kern, smem);
      if (e != cudaSuccess) return set_error(MHC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    }
    const int rows = max_partial_rows(T);
    const int resident = persistent_grid(kern, kGenBD, smem, 1 << 30, 1 << 30);
    auto clusters = [&](int c) -> int64_t {
      int64_t q = resident / c;
      if (q > rows / c) q = rows / c;
      if (q > T) q = T;
      return q < 1 ? 1 : q;
    };
    // cluster size with the least work for the busiest CTA: token rounds
    // ceil(T / Q) times slice width ceil(C / cs); the smaller cs on ties
    int cs = cs_min;
    if (env_int("MHC_B200_SPLIT", 1)) {
      int64_t best = -1;
      for (int c = cs_min; c <= 8; c *= 2) {
        if (c > cs_min && (C / c < kGenBD || c > rows)) break;
        const int64_t q = clusters(c);
        const int64_t work = ((T + q - 1) / q) * ((C + c - 1) / c);
        if (best < 0 || work < best) { best = work; cs = c; }
      }
    }
    const int64_t Q = clusters(cs);
    const int G = (int)(Q * cs);
    BwdPtrs p = ws_ptrs(ws, G, n);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)G, 1, 1);
    cfg.blockDim = dim3(kGenBD, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, x, d, M, hpre, hpost, w, dx, T, tail...,
                                             p.p, p.c, p.hdr);
    if (e != cudaSuccess) return set_error(MHC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return check_launch(what);
  };
  static_assert(kWideBD == kGenBD, "one cluster launch shape");
  // the wide kernel keeps y and dyn of its column slice in shared memory: at
  // most kWideSlice columns per CTA, so wider rows need a cluster split
  int wide_cs = 1;
  while (wide_cs <= 8 && ((((C + wide_cs - 1) / wide_cs) + 3) & ~3) > kWideSlice) wide_cs *= 2;
  if (!env_int("MHC_B200_GENERIC", 0) && (n == 16 || n == 32) && T > 0 && wide_cs <= 8 &&
      wide_cs <= max_partial_rows(T)) {
    // dx rows as 4-element vectors when every row start is aligned for them
    const int vec_dx =
        (C % 4 == 0) && ((reinterpret_cast<uintptr_t>(dx) & (4 * sizeof(DXT) - 1)) == 0);
    // fp32 rows staged with cp.async when every row start is 16-byte aligned
    if constexpr (std::is_same<XT, float>::value && std::is_same<DT, float>::value) {
      if (C % 4 == 0 && aligned16(x) && aligned16(d) && env_int("MHC_B200_PIPE", 1)) {
        if (n == 16)
          return launch_clusters(k_bwd_wide<16, XT, DT, DXT, true>, wide_smem_bytes(16, 2),
                                 wide_cs, "mhc_bwd(wide)", C, eps, vec_dx);
        return launch_clusters(k_bwd_wide<32, XT, DT, DXT, true>, wide_smem_bytes(32, 2),
                               wide_cs, "mhc_bwd(wide)", C, eps, vec_dx);
      }
    }
    if (n == 16)
      return launch_clusters(k_bwd_wide<16, XT, DT, DXT, false>, wide_smem_bytes(16, 1), wide_cs,
                             "mhc_bwd(wide)", C, eps, vec_dx);
    return launch_clusters(k_bwd_wide<32, XT, DT, DXT, false>, wide_smem_bytes(32, 1), wide_cs,
                           "mhc_bwd(wide)", C, eps, vec_dx);
  }
  const size_t smem = ((size_t)n * n + 2 * n + 2 * (size_t)(n + 1) * kGenLD) * sizeof(float);
  return launch_clusters(k_bwd_generic<XT, DT, DXT>, smem, 1, "mhc_bwd(generic)", n, C, eps);
}

int launch_bwd(const void* x, int xdt, const void* dout, int ddt, const float* M,
               const float* hpre, const float* hpost, const float* w, void* dx, int dxdt,
               int64_t T, int n, int C, float eps, void* ws, size_t ws_bytes, cudaStream_t st) {
  const size_t need = bwd_ws_bytes(T, n, C);
  if (ws_bytes < need || !ws)
    return set_error(MHC_ERR_WORKSPACE, "mhc_bwd: workspace %zu < %zu bytes", ws_bytes, need);
  if (dxdt != xdt)
    return set_error(MHC_ERR_UNSUPPORTED, "mhc_bwd: dx dtype must equal x dtype");
  if (ddt != MHC_F32 && ddt != xdt)
    return set_error(MHC_ERR_UNSUPPORTED, "mhc_bwd: d_out dtype must be fp32 or x's dtype");
  // T == 0 still launches one CTA so that the workspace holds zero partials.
  const int64_t Te = T;
  if (xdt == MHC_F32)
    return bwd_typed<float, float, float>(x, dout, M, hpre, hpost, w, dx, Te, n, C, eps, ws, st);
  if (xdt == MHC_BF16 && ddt == MHC_F32)
    return bwd_typed<bf16, float, bf16>(x, dout, M, hpre, hpost, w, dx, Te, n, C, eps, ws, st);
  if (xdt == MHC_BF16)
    return bwd_typed<bf16, bf16, bf16>(x, dout, M, hpre, hpost, w, dx, Te, n, C, eps, ws, st);
  if (xdt == MHC_F16 && ddt == MHC_F32)
    return bwd_typed<f16, float, f16>(x, dout, M, hpre, hpost, w, dx, Te, n, C, eps, ws, st);
  return bwd_typed<f16, f16, f16>(x, dout, M, hpre, hpost, w, dx, Te, n, C, eps, ws, st);
}

int launch_finalize(const void* ws, int n, int C, float* dM, float* dhpre, float* dhpost,
                    float* dw, const float* hpre_raw, const float* hpost_raw,
                    const float* hres_raw, const float* tape, int iters, float eps,
                    float* dhpre_raw, float* dhpost_raw, float* dhres_raw, cudaStream_t st) {
  const int nbc = (C + 31) / 32;
  // Stage the Sinkhorn tape and logits in shared memory when they fit.
  size_t smem = 0;
  if (hres_raw && dhres_raw && tape) {
    const size_t b = sk_stage_floats(n, iters) * sizeof(float);
    if (b <= 160 * 1024) smem = b;
  }
  auto go = [&](auto kern, int bd) {
    if (allow_dyn_smem(kern, smem) != cudaSuccess) smem = 0;
    kern<<<nbc + 1, bd, smem, st>>>(static_cast<const char*>(ws), n, C, dM, dhpre, dhpost, dw,
                                    hpre_raw, hpost_raw, hres_raw, tape, iters, eps, dhpre_raw,
                                    dhpost_raw, dhres_raw, smem > 0);
    return check_launch("mhc_bwd_finalize");
  };
  if (n == 32) return go(k_finalize<1024>, 1024);
  return go(k_finalize<256>, 256);
}

}  // namespace mhc
