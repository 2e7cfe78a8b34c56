// Block-level Sinkhorn-Knopp forward/backward for one n x n matrix (n <= 64),
// shared by the parameter kernels, the batched fallback and the backward
// finalize kernel.
//
// Forward (reference.py:20-48, :58-69):
//   P0 = exp(H - rowmax(H));  repeat iters: rows scaled by 1/sum (if > eps,
//   else 1), then columns scaled by 1/sum (if > eps, else 0).
// Backward: reverse-mode through the recorded iterations; the tape holds,
// per iteration k, the matrix before the row step (n*n), the row sums (n)
// and the column sums (n).  The row-scaled matrix is recomputed bit-exactly
// from them (same fp32 multiply as the forward).  The max shift contributes
// -(rowsum of dS) split evenly over the row's maxima, as autodiff of max does.
#pragma once

#include "mhc_common.cuh"

namespace mhc {

// Shared-memory matrices use a padded leading dimension so that both the
// thread-per-row and thread-per-column sweeps are bank-conflict free.
__host__ __device__ constexpr int sk_ld(int n) { return n + 1; }

__host__ __device__ inline size_t sk_tape_stride(int n) { return (size_t)n * n + 2 * (size_t)n; }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block version, any n <= 64, blockDim a multiple of 32: one warp per row
// (row step) or per column (column step); lanes cover the line's entries and
// reduce with a warp butterfly.  P: shared [n][ld] with ld = n + 1, so row
// and column sweeps are both conflict-free.  tape (global, nullable) uses
// the pitch-n layout [k][n*n | n row sums | n column sums].  Writes M
// (global, nullable).
__device__ inline void sk_forward_block(const float* __restrict__ H, int n, int iters, float eps,
                                        float* P, float* __restrict__ tape,
                                        float* __restrict__ M) {
  const int tid = threadIdx.x, bd = blockDim.x, ld = sk_ld(n), nn = n * n;
  const int lane = tid & 31, warp = tid >> 5, nw = bd >> 5;
  for (int e = tid; e < nn; e += bd) P[(e / n) * ld + e % n] = H[e];
  __syncthreads();
  for (int i = warp; i < n; i += nw) {
    float m = -INFINITY;
    for (int j = lane; j < n; j += 32) m = fmaxf(m, P[i * ld + j]);
    m = warp_max(m);
    for (int j = lane; j < n; j += 32) P[i * ld + j] = expf(P[i * ld + j] - m);
  }
  __syncthreads();
  for (int k = 0; k < iters; ++k) {
    float* tk = tape ? tape + (size_t)k * sk_tape_stride(n) : nullptr;
    if (tk)
      for (int e = tid; e < nn; e += bd) tk[e] = P[(e / n) * ld + e % n];
    for (int i = warp; i < n; i += nw) {
      float s = 0.f;
      for (int j = lane; j < n; j += 32) s += P[i * ld + j];
      s = warp_sum(s);
      const float sc = row_scale(s, eps);
      for (int j = lane; j < n; j += 32) P[i * ld + j] *= sc;
      if (tk && lane == 0) tk[nn + i] = s;
    }
    __syncthreads();
    for (int j = warp; j < n; j += nw) {
      float s = 0.f;
      for (int i = lane; i < n; i += 32) s += P[i * ld + j];
      s = warp_sum(s);
      const float sc = col_scale(s, eps);
      for (int i = lane; i < n; i += 32) P[i * ld + j] *= sc;
      if (tk && lane == 0) tk[nn + n + j] = s;
    }
    __syncthreads();
  }
  if (M)
    for (int e = tid; e < nn; e += bd) M[e] = P[(e / n) * ld + e % n];
}

// Tape view: matrix pitch `tp` (n for the global layout, n + 1 when staged in
// shared memory to keep column reads conflict-free) and iteration stride.
struct SkTape {
  const float* base;
  int tp;
  size_t stride;
  __device__ const float* it(int k) const { return base + (size_t)k * stride; }
};

// Copy the pitch-n global tape into shared memory with pitch n + 1.
__device__ inline SkTape sk_stage_tape(const float* __restrict__ tape, int n, int iters,
                                       float* smem) {
  const int nn = n * n, ld = sk_ld(n);
  const size_t gs = sk_tape_stride(n), ss = (size_t)n * ld + 2 * n;
#pragma unroll 8
  for (size_t e = threadIdx.x; e < (size_t)iters * gs; e += blockDim.x) {
    const size_t k = e / gs, r = e - k * gs;
    const size_t dst = r < (size_t)nn ? (r / n) * ld + r % n : (size_t)n * ld + (r - nn);
    smem[k * ss + dst] = tape[e];
  }
  return SkTape{smem, ld, ss};
}

__host__ __device__ inline size_t sk_staged_tape_floats(int n, int iters) {
  return (size_t)iters * ((size_t)n * sk_ld(n) + 2 * (size_t)n);
}

// D: shared [n][ld] holding dM on entry (caller fills it and syncs).
// H: logits (global or shared).  Writes dH (global).  Same warp-per-line
// mapping as the forward.
__device__ inline void sk_backward_block(const float* __restrict__ H, SkTape tape, int n,
                                         int iters, float eps, float* D, float* __restrict__ dH) {
  const int tid = threadIdx.x, bd = blockDim.x, ld = sk_ld(n);
  const int lane = tid & 31, warp = tid >> 5, nw = bd >> 5;
  const int tp = tape.tp, rofs = n * tp, cofs = n * tp + n;
  for (int k = iters - 1; k >= 0; --k) {
    const float* tk = tape.it(k);
    // column step: out = Pb * cs_j, c_j = sum_i Pb_ij
    for (int j = warp; j < n; j += nw) {
      const float c = tk[cofs + j];
      const float cs = col_scale(c, eps);
      float dcs = 0.f;
      for (int i = lane; i < n; i += 32)
        dcs += D[i * ld + j] * (tk[i * tp + j] * row_scale(tk[rofs + i], eps));
      dcs = warp_sum(dcs);
      const float dc = recip_grad(dcs, c, cs, eps);
      for (int i = lane; i < n; i += 32) D[i * ld + j] = D[i * ld + j] * cs + dc;
    }
    __syncthreads();
    // row step: Pb = Pa * rs_i, r_i = sum_j Pa_ij
    for (int i = warp; i < n; i += nw) {
      const float r = tk[rofs + i];
      const float rs = row_scale(r, eps);
      float drs = 0.f;
      for (int j = lane; j < n; j += 32) drs += D[i * ld + j] * tk[i * tp + j];
      drs = warp_sum(drs);
      const float dr = recip_grad(drs, r, rs, eps);
      for (int j = lane; j < n; j += 32) D[i * ld + j] = D[i * ld + j] * rs + dr;
    }
    __syncthreads();
  }
  // exp and the row-max shift
  for (int i = warp; i < n; i += nw) {
    float m = -INFINITY;
    for (int j = lane; j < n; j += 32) m = fmaxf(m, H[i * n + j]);
    m = warp_max(m);
    float S = 0.f, cnt = 0.f;
    for (int j = lane; j < n; j += 32) {
      const float h = H[i * n + j];
      const float ds = D[i * ld + j] * expf(h - m);
      D[i * ld + j] = ds;
      S += ds;
      cnt += (h == m) ? 1.f : 0.f;
    }
    S = warp_sum(S);
    cnt = warp_sum(cnt);
    const float share = S / cnt;
    for (int j = lane; j < n; j += 32) {
      const float h = H[i * n + j];
      dH[i * n + j] = D[i * ld + j] - ((h == m) ? share : 0.f);
    }
  }
}

// ---------------------------------------------------------------------------
// Warp-level single matrix, n divides 32: lane i (< n) holds row i in
// registers; column sums are butterfly shuffles over the n lanes of the
// group (identical bits on every lane).  Other lane groups compute on a copy
// and write nothing.  Same arithmetic and tape layout as the block versions,
// but a half-step is a few dependent instructions instead of shared-memory
// round trips and barriers -- this matters because the kernels that run it
// are one-CTA latency chains.
template <int N>
__device__ __forceinline__ void sk_forward_warp(const float* __restrict__ H, int iters, float eps,
                                                float* __restrict__ tape, float* __restrict__ M) {
  const int lane = threadIdx.x & 31, row = lane % N;
  const bool w = lane < N;
  constexpr int nn = N * N;
  float p[N];
#pragma unroll
  for (int j = 0; j < N; ++j) p[j] = H[row * N + j];
  float m = p[0];
#pragma unroll
  for (int j = 1; j < N; ++j) m = fmaxf(m, p[j]);
#pragma unroll
  for (int j = 0; j < N; ++j) p[j] = expf(p[j] - m);
  for (int k = 0; k < iters; ++k) {
    float* tk = tape ? tape + (size_t)k * (nn + 2 * N) : nullptr;
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) {
      if (tk && w) tk[row * N + j] = p[j];
      s += p[j];
    }
    if (tk && w) tk[nn + row] = s;
    const float rs = row_scale(s, eps);
#pragma unroll
    for (int j = 0; j < N; ++j) p[j] *= rs;
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const float c = group_sum<N>(p[j]);
      if (tk && w && j == row) tk[nn + N + j] = c;
      p[j] *= col_scale(c, eps);
    }
  }
  if (M && w)
#pragma unroll
    for (int j = 0; j < N; ++j) M[row * N + j] = p[j];
}

// d: this lane's row of dM on entry, of dH_res on exit.  tape: the record
// of sk_forward_* (global or shared memory).
template <int N>
__device__ __forceinline__ void sk_backward_warp(const float* __restrict__ H,
                                                 const float* __restrict__ tape, int iters,
                                                 float eps, float (&d)[N]) {
  const int lane = threadIdx.x & 31, row = lane % N, gbase = lane & ~(N - 1);
  constexpr int nn = N * N;
  for (int k = iters - 1; k >= 0; --k) {
    const float* tk = tape + (size_t)k * (nn + 2 * N);
    float pa[N];
#pragma unroll
    for (int j = 0; j < N; ++j) pa[j] = tk[row * N + j];
    const float r = tk[nn + row];
    const float cown = tk[nn + N + row];
    const float rs = row_scale(r, eps);
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const float c = __shfl_sync(0xffffffffu, cown, gbase + j);
      const float dcs = group_sum<N>(d[j] * (pa[j] * rs));
      const float cs = col_scale(c, eps);
      d[j] = d[j] * cs + recip_grad(dcs, c, cs, eps);
    }
    float drs = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) drs += d[j] * pa[j];
    const float dr = recip_grad(drs, r, rs, eps);
#pragma unroll
    for (int j = 0; j < N; ++j) d[j] = d[j] * rs + dr;
  }
  float h[N];
#pragma unroll
  for (int j = 0; j < N; ++j) h[j] = H[row * N + j];
  float m = h[0];
#pragma unroll
  for (int j = 1; j < N; ++j) m = fmaxf(m, h[j]);
  float S = 0.f, cnt = 0.f;
#pragma unroll
  for (int j = 0; j < N; ++j) {
    d[j] *= expf(h[j] - m);
    S += d[j];
    cnt += (h[j] == m) ? 1.f : 0.f;
  }
  const float share = S / cnt;
#pragma unroll
  for (int j = 0; j < N; ++j) d[j] -= (h[j] == m) ? share : 0.f;
}

// ---------------------------------------------------------------------------
// Element-per-lane Sinkhorn for n in {1, 2, 4}: lane L < n^2 of one warp holds
// entry (i, j) = (L / n, L % n).  A row sum is a butterfly over the n
// consecutive lanes of the row (xor 1 .. n/2), a column sum one over the lanes
// n apart (xor n .. n^2/2), so a half-step is one butterfly, one reciprocal
// and one multiply per lane: the 2 * iters long dependency chain carries a
// few instructions per half-step instead of a loop over a whole row.  Lanes
// >= n^2 run the same steps on their own (unused) values, which keeps every
// shuffle full-warp.  Tape layout as sk_forward_warp: per iteration the n^2
// values before the row scaling (row-major = lane order), the n row sums,
// the n column sums.
__host__ __device__ inline bool sk_lane_ok(int n) { return n == 1 || n == 2 || n == 4; }

template <int N>
__device__ __forceinline__ float sk_col_sum(float v) {
#pragma unroll
  for (int o = N * N / 2; o >= N; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int N>
__device__ __forceinline__ float sk_row_max(float v) {
#pragma unroll
  for (int o = N / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

template <int N>
__device__ __forceinline__ void sk_forward_lane(const float* __restrict__ H, int iters, float eps,
                                                float* __restrict__ tape, float* __restrict__ M) {
  constexpr int NN = N * N, TS = NN + 2 * N;
  const int lane = threadIdx.x & 31;
  const bool act = lane < NN;
  const int i = (lane / N) % N, j = lane % N;
  const float h = act ? H[lane] : 0.f;
  float p = expf(h - sk_row_max<N>(h));
  for (int k = 0; k < iters; ++k) {
    float* tk = tape ? tape + (size_t)k * TS : nullptr;
    const float s = group_sum<N>(p);
    if (tk && act) {
      tk[lane] = p;
      if (j == 0) tk[NN + i] = s;
    }
    p *= row_scale(s, eps);
    const float c = sk_col_sum<N>(p);
    if (tk && act && i == 0) tk[NN + N + j] = c;
    p *= col_scale(c, eps);
  }
  if (M && act) M[lane] = p;
}

// d: this lane's entry of dM on entry, of dH_res on exit.  The next
// iteration's tape entries are loaded before the current one is processed.
// PACKED: every lane group of NN lanes runs its own cotangent on entry le =
// lane % NN (the reductions already stay inside a group), and the tape was
// written by the same kernel: l2 = read it through L2 (global memory), else
// it is in shared memory (sk_jacobian_lane).
template <int N, bool PACKED = false>
__device__ __forceinline__ float sk_backward_lane(const float* __restrict__ H,
                                                  const float* __restrict__ tape, int iters,
                                                  float eps, float d, bool l2 = false) {
  constexpr int NN = N * N, TS = NN + 2 * N;
  const int lane = threadIdx.x & 31;
  const int le = PACKED ? lane % NN : lane;
  const bool act = PACKED || lane < NN;
  const int i = (lane / N) % N, j = lane % N;
  auto ld = [&](int k, float& pa, float& r, float& c) {
    const float* tk = tape + (size_t)k * TS;
    if constexpr (PACKED) {
      if (l2) {
        pa = __ldcg(tk + le);
        r = __ldcg(tk + NN + i);
        c = __ldcg(tk + NN + N + j);
      } else {
        pa = tk[le];
        r = tk[NN + i];
        c = tk[NN + N + j];
      }
    } else {
      pa = act ? tk[lane] : 0.f;
      r = tk[NN + i];
      c = tk[NN + N + j];
    }
  };
  float pa = 0.f, r = 0.f, c = 0.f;
  if (iters > 0) ld(iters - 1, pa, r, c);
  for (int k = iters - 1; k >= 0; --k) {
    float pn = 0.f, rn = 0.f, cn = 0.f;
    if (k > 0) ld(k - 1, pn, rn, cn);
    const float rs = row_scale(r, eps), cs = col_scale(c, eps);
    const float dcs = sk_col_sum<N>(d * (pa * rs));
    d = d * cs + recip_grad(dcs, c, cs, eps);
    const float drs = group_sum<N>(d * pa);
    d = d * rs + recip_grad(drs, r, rs, eps);
    pa = pn;
    r = rn;
    c = cn;
  }
  // exp and the row-max shift (the max's gradient is split over ties)
  const float h = act ? H[le] : 0.f;
  const float m = sk_row_max<N>(h);
  d *= expf(h - m);
  const float S = group_sum<N>(d);
  const float cnt = group_sum<N>(h == m ? 1.f : 0.f);
  return d - (h == m ? S / cnt : 0.f);
}

// Transposed Jacobian of the lane-path Sinkhorn at H (n in {1, 2, 4}), from
// the tape this kernel wrote (visible to the block: the caller syncs first;
// l2: the tape is in global memory, else in shared memory -- the latter
// matters when other blocks saturate DRAM, since every iteration's loads sit
// on the chain).
// The backward is linear in dM, so running it on the unit cotangents e_u
// gives A[u][e] = d(M_u)/d(H_e) and, later, dH_res = sum_u dM[u] A[u][:] as
// a dot product instead of a reverse sweep (a latency chain of 2 iters
// dependent reductions).  Lane group g of warp w takes u = w (32 / NN) + g:
// for n = 4 the 16 cotangents are one pass of 8 warps.
template <int N>
__device__ __forceinline__ void sk_jacobian_lane(const float* __restrict__ H,
                                                 const float* tape, int iters, float eps,
                                                 float* __restrict__ A, bool l2) {
  constexpr int NN = N * N, GPW = 32 / NN;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int u0 = warp * GPW; u0 < NN; u0 += nw * GPW) {  // warp-uniform
    const int u = u0 + lane / NN, le = lane % NN;
    const float d = sk_backward_lane<N, true>(H, tape, iters, eps, le == u ? 1.f : 0.f, l2);
    if (u < NN) A[u * NN + le] = d;
  }
}
__host__ __device__ inline size_t sk_jacobian_floats(int n) {
  return sk_lane_ok(n) ? (size_t)n * n * n * n : 0;
}

// Expand BODY with SK_N = n for the element-per-lane path (n in {1, 2, 4}).
#define MHC_SK_LANE_SWITCH(n, BODY)                    \
  switch (n) {                                         \
    case 1: { constexpr int SK_N = 1; BODY; } break;   \
    case 2: { constexpr int SK_N = 2; BODY; } break;   \
    case 4: { constexpr int SK_N = 4; BODY; } break;   \
    default: break;                                    \
  }

// ---------------------------------------------------------------------------
// Element-per-thread Sinkhorn for n in {16, 32} with BD threads (R = n^2 / BD
// entries per thread, e = tid + BD * r).  Row phase: entry e is (e / n, e % n),
// so a row is n consecutive e and its sum a butterfly within one warp.  Column
// phase: entry e is (e % n, e / n), so a column is n consecutive e.  Between
// the phases the values go through the padded shared buffer P [n][n + 1]:
// every thread writes exactly the slots it read last, so one barrier per
// transpose orders all reads and writes.  Compile-time n: no loops over a
// runtime line length and no integer division on the chain.
__host__ __device__ inline bool sk_elem_ok(int n) { return n == 16 || n == 32; }

template <int N, int BD>
__device__ __forceinline__ void sk_elem_to_col(float (&v)[N * N / BD], float* P) {
  constexpr int R = N * N / BD, LD = N + 1;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int e = threadIdx.x + BD * r;
    P[(e / N) * LD + e % N] = v[r];
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int e = threadIdx.x + BD * r;
    v[r] = P[(e % N) * LD + e / N];
  }
}

template <int N, int BD>
__device__ __forceinline__ void sk_elem_to_row(float (&v)[N * N / BD], float* P) {
  constexpr int R = N * N / BD, LD = N + 1;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int e = threadIdx.x + BD * r;
    P[(e % N) * LD + e / N] = v[r];
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int e = threadIdx.x + BD * r;
    v[r] = P[(e / N) * LD + e % N];
  }
}

// P: shared [N][N + 1] scratch.  Requires blockDim.x == BD.  TAPE: record
// the tape (tape non-null); the variant without it has no tape code at all.
template <int N, int BD, bool TAPE>
__device__ __forceinline__ void sk_forward_elem(const float* __restrict__ H, int iters, float eps,
                                                float* P, float* __restrict__ tape,
                                                float* __restrict__ M) {
  constexpr int R = N * N / BD, NN = N * N, TS = NN + 2 * N;
  static_assert(R * BD == NN && N <= 32 && 32 % N == 0, "rows within one warp");
  float p[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const float h = H[threadIdx.x + BD * r];
    p[r] = expf(h - sk_row_max<N>(h));
  }
  for (int k = 0; k < iters; ++k) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int e = threadIdx.x + BD * r;
      const float s = group_sum<N>(p[r]);
      if constexpr (TAPE) {
        float* tk = tape + (size_t)k * TS;
        tk[e] = p[r];
        if (e % N == 0) tk[NN + e / N] = s;
      }
      p[r] *= row_scale(s, eps);
    }
    sk_elem_to_col<N, BD>(p, P);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int e = threadIdx.x + BD * r;
      const float c = group_sum<N>(p[r]);
      if constexpr (TAPE) {
        if (e % N == 0) tape[(size_t)k * TS + NN + N + e / N] = c;
      }
      p[r] *= col_scale(c, eps);
    }
    sk_elem_to_row<N, BD>(p, P);
  }
  if (M)
#pragma unroll
    for (int r = 0; r < R; ++r) M[threadIdx.x + BD * r] = p[r];
}

// dM (row-major, global or shared) in, dH (global) out; P: shared [N][N + 1]
// scratch.  Same phases in reverse: per iteration the column step (column
// phase), then the row step (row phase).
template <int N, int BD>
__device__ __forceinline__ void sk_backward_elem(const float* __restrict__ H, SkTape tape,
                                                 int iters, float eps, const float* dM, float* P,
                                                 float* __restrict__ dH) {
  constexpr int R = N * N / BD, NN = N * N;
  static_assert(R * BD == NN && N <= 32 && 32 % N == 0, "rows within one warp");
  const int tp = tape.tp, rofs = N * tp, cofs = N * tp + N;
  float d[R];
#pragma unroll
  for (int r = 0; r < R; ++r) d[r] = dM[threadIdx.x + BD * r];
  for (int k = iters - 1; k >= 0; --k) {
    const float* tk = tape.it(k);
    sk_elem_to_col<N, BD>(d, P);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int e = threadIdx.x + BD * r, i = e % N, j = e / N;
      const float rs = row_scale(tk[rofs + i], eps);
      const float c = tk[cofs + j], cs = col_scale(c, eps);
      const float dcs = group_sum<N>(d[r] * (tk[i * tp + j] * rs));
      d[r] = d[r] * cs + recip_grad(dcs, c, cs, eps);
    }
    sk_elem_to_row<N, BD>(d, P);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int e = threadIdx.x + BD * r, i = e / N, j = e % N;
      const float rr = tk[rofs + i], rs = row_scale(rr, eps);
      const float drs = group_sum<N>(d[r] * tk[i * tp + j]);
      d[r] = d[r] * rs + recip_grad(drs, rr, rs, eps);
    }
  }
  // exp and the row-max shift (the max's gradient is split over ties)
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int e = threadIdx.x + BD * r;
    const float h = H[e];
    const float m = sk_row_max<N>(h);
    float v = d[r] * expf(h - m);
    const float S = group_sum<N>(v);
    const float cnt = group_sum<N>(h == m ? 1.f : 0.f);
    dH[e] = v - (h == m ? S / cnt : 0.f);
  }
}

// sk_stage_tape with n a compile-time constant: the index arithmetic of the
// copy is constant division (multiply-shift), not 64-bit division by a
// runtime n, which dominated the staging of a 32 x 32 tape.
template <int N>
__device__ __forceinline__ SkTape sk_stage_tape_fixed(const float* __restrict__ tape, int iters,
                                                     float* smem) {
  constexpr int NN = N * N, LD = N + 1, GS = NN + 2 * N, SS = N * LD + 2 * N;
  const int total = iters * GS;
#pragma unroll 8
  for (int e = threadIdx.x; e < total; e += blockDim.x) {
    const int k = e / GS, r = e - k * GS;
    const int dst = r < NN ? (r / N) * LD + r % N : N * LD + (r - NN);
    smem[k * SS + dst] = tape[e];
  }
  return SkTape{smem, LD, (size_t)SS};
}

// Expand BODY with SK_N = n for the element-per-thread path (n in {16, 32}).
#define MHC_SK_ELEM_SWITCH(n, BODY)                     \
  switch (n) {                                          \
    case 16: { constexpr int SK_N = 16; BODY; } break;  \
    case 32: { constexpr int SK_N = 32; BODY; } break;  \
    default: break;                                     \
  }

// Expand BODY with the compile-time constant SK_N equal to n (n | 32).
#define MHC_SK_WARP_SWITCH(n, BODY)                 \
  switch (n) {                                      \
    case 1: { constexpr int SK_N = 1; BODY; } break;   \
    case 2: { constexpr int SK_N = 2; BODY; } break;   \
    case 4: { constexpr int SK_N = 4; BODY; } break;   \
    case 8: { constexpr int SK_N = 8; BODY; } break;   \
    default: break;                                 \
  }

// The one-lane-per-row register path pays off for small n; from n = 16 on a
// lane would walk n^2 / 32 entries per step, so the warp-per-line block
// version is used instead.
__host__ __device__ inline bool sk_warp_ok(int n) {
  return n == 1 || n == 2 || n == 4 || n == 8;
}

// Shared-memory floats a one-CTA Sinkhorn backward stages: the pitch-n tape
// plus the logits for the register path (n <= 8), the padded tape for the
// warp-per-line path.  Threads per CTA for the single-matrix kernels.
__host__ __device__ inline size_t sk_stage_floats(int n, int iters) {
  return sk_warp_ok(n) ? (size_t)iters * sk_tape_stride(n) + (size_t)n * n
                       : sk_staged_tape_floats(n, iters);
}
__host__ __device__ inline int sk_threads(int n) {
  return sk_warp_ok(n) ? 32 : sk_elem_ok(n) ? n * n : 32 * (n < 32 ? n : 32);
}

// ---------------------------------------------------------------------------
// Raw-parameter gradients at the end of a one-CTA backward finalize, from the
// activation gradients G = [dM (n*n) | dH_pre_act (n) | dH_post_act (n)] in
// shared memory (filled and synced by the caller):
//   dH_pre_raw  = dH_pre_act sigma' (H_pre_act = sigmoid(H_pre_raw))
//   dH_post_raw = 2 dH_post_act sigma' (H_post_act = 2 sigmoid(H_post_raw))
//   dH_res_raw  = Sinkhorn backward of dM: with jac (n <= 4, written by
//                 sk_jacobian_lane) the dot products sum_u dM[u] jac[u][:],
//                 else the reverse sweep through the tape.
// Every one of the BD threads calls it (the sweeps synchronise the block);
// sk_tail_ok(n, BD) must hold.  stage_sk: copy [tape | logits] into s_fin
// (dynamic shared memory of sk_stage_floats(n, iters) floats) first.  D:
// shared [n][sk_ld(n)] scratch.  Null outputs are skipped.
__host__ __device__ inline bool sk_tail_ok(int n, int bd) { return !sk_elem_ok(n) || n * n >= bd; }

template <int BD>
__device__ inline void sk_params_bwd_tail(const float* G, int n, const float* __restrict__ hpre_raw,
                                          const float* __restrict__ hpost_raw,
                                          const float* __restrict__ hres_raw,
                                          const float* __restrict__ tape,
                                          const float* __restrict__ jac, int iters, float eps,
                                          int stage_sk, float* s_fin, float* D,
                                          float* __restrict__ dhpre_raw,
                                          float* __restrict__ dhpost_raw,
                                          float* __restrict__ dhres_raw) {
  const int tid = threadIdx.x;
  if (tid < n) {
    // d/da sigmoid(a) = s (1 - s)
    if (hpre_raw && dhpre_raw) {
      const float s = sigmoidf_(hpre_raw[tid]);
      dhpre_raw[tid] = G[n * n + tid] * (1.0f - s) * s;
    }
    if (hpost_raw && dhpost_raw) {
      const float s = sigmoidf_(hpost_raw[tid]);
      dhpost_raw[tid] = (2.0f * G[n * n + n + tid]) * (1.0f - s) * s;
    }
  }
  if (!hres_raw || !dhres_raw) return;
  if (jac) {
    const int nn = n * n;
    for (int e = tid; e < nn; e += BD) {
      float s = 0.f;
      for (int u = 0; u < nn; ++u) s = fmaf(G[u], jac[u * nn + e], s);
      dhres_raw[e] = s;
    }
    return;
  }
  if (!tape && iters > 0) return;
  if (sk_warp_ok(n)) {
    // one call site per address space of the tape (shared when staged,
    // global otherwise), so its loads are not generic
    auto run = [&](const float* Hs, const float* Ts) {
      if (sk_lane_ok(n)) {
        if (tid < 32) {
          MHC_SK_LANE_SWITCH(n, ({
            const bool act = tid < SK_N * SK_N;
            const float d = sk_backward_lane<SK_N>(Hs, Ts, iters, eps, act ? G[tid] : 0.f);
            if (act) dhres_raw[tid] = d;
          }))
        }
        return;
      }
      if (tid < 32) {
        const int row = tid % n;
        MHC_SK_WARP_SWITCH(n, ({
          float d[SK_N];
          for (int j = 0; j < SK_N; ++j) d[j] = G[row * SK_N + j];
          sk_backward_warp<SK_N>(Hs, Ts, iters, eps, d);
          if (tid < SK_N)
            for (int j = 0; j < SK_N; ++j) dhres_raw[row * SK_N + j] = d[j];
        }))
      }
    };
    if (stage_sk) {  // s_fin holds [tape | logits]
      const size_t tf = (size_t)iters * sk_tape_stride(n);
#pragma unroll 8
      for (size_t e = tid; e < tf; e += BD) s_fin[e] = tape[e];
      for (int e = tid; e < n * n; e += BD) s_fin[tf + e] = hres_raw[e];
      __syncthreads();
      run(s_fin + tf, s_fin);
    } else {
      run(hres_raw, tape);
    }
    return;
  }
  if (sk_elem_ok(n)) {  // BD threads: n^2 / BD entries per thread
    MHC_SK_ELEM_SWITCH(n, ({
      if constexpr (SK_N * SK_N >= BD) {
        if (stage_sk) {
          const SkTape tp = sk_stage_tape_fixed<SK_N>(tape, iters, s_fin);
          __syncthreads();  // staged tape complete
          sk_backward_elem<SK_N, BD>(hres_raw, tp, iters, eps, G, D, dhres_raw);
        } else {
          sk_backward_elem<SK_N, BD>(hres_raw, SkTape{tape, SK_N, sk_tape_stride(SK_N)}, iters,
                                     eps, G, D, dhres_raw);
        }
      }
    }))
    return;
  }
  const SkTape tp = stage_sk ? sk_stage_tape(tape, n, iters, s_fin)
                             : SkTape{tape, n, sk_tape_stride(n)};
  const int ld = sk_ld(n);
  for (int e = tid; e < n * n; e += BD) D[(e / n) * ld + e % n] = G[e];
  __syncthreads();
  sk_backward_block(hres_raw, tp, n, iters, eps, D, dhres_raw);
}

}  // namespace mhc
