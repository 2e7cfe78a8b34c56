// Parameter kernels: sigmoid activations + single-matrix Sinkhorn-Knopp
// forward/backward, and the batched [batch, n, n] Sinkhorn kernels.
//
// Reference: reference.py:20-69 (math), metal.py:1525-1577 and
// kernels/sinkhorn_knopp.metal (single-matrix forward launcher),
// metal.py:1978-2016 and kernels/sinkhorn_knopp_backward.metal (backward).
#include "mhc_sinkhorn.cuh"
#include "mhc_internal.h"

namespace mhc {

size_t sk_tape_floats(int n, int iters) { return (size_t)iters * sk_tape_stride(n); }

// ---------------------------------------------------------------------------
// Single matrix: one CTA computes H_pre_act, H_post_act and M (+ tape).
__global__ void __launch_bounds__(1024)
k_params_fwd(const float* __restrict__ hpre_raw, const float* __restrict__ hpost_raw,
             const float* __restrict__ hres_raw, int n, int iters, float eps,
             float* __restrict__ hpre, float* __restrict__ hpost, float* __restrict__ M,
             float* __restrict__ tape) {
  __shared__ float P[kMaxN * (kMaxN + 1)];
  const int tid = threadIdx.x;
  if (tid < n) {
    if (hpre_raw) hpre[tid] = sigmoidf_(hpre_raw[tid]);
    if (hpost_raw) hpost[tid] = 2.0f * sigmoidf_(hpost_raw[tid]);
  }
  if (!hres_raw) return;
  if (sk_lane_ok(n)) {
    if (tid < 32) MHC_SK_LANE_SWITCH(n, (sk_forward_lane<SK_N>(hres_raw, iters, eps, tape, M)))
    return;
  }
  if (sk_warp_ok(n)) {
    if (threadIdx.x < 32) MHC_SK_WARP_SWITCH(n, (sk_forward_warp<SK_N>(hres_raw, iters, eps, tape, M)))
    return;
  }
  if (sk_elem_ok(n)) {
    if (tape)
      MHC_SK_ELEM_SWITCH(n, (sk_forward_elem<SK_N, SK_N * SK_N, true>(hres_raw, iters, eps, P, tape, M)))
    else
      MHC_SK_ELEM_SWITCH(n, (sk_forward_elem<SK_N, SK_N * SK_N, false>(hres_raw, iters, eps, P, tape, M)))
    return;
  }
  sk_forward_block(hres_raw, n, iters, eps, P, tape, M);
}

__global__ void __launch_bounds__(1024)
k_params_bwd(const float* __restrict__ hpre_raw, const float* __restrict__ hpost_raw,
             const float* __restrict__ hres_raw, const float* __restrict__ tape, int n,
             int iters, float eps, const float* __restrict__ dhpre,
             const float* __restrict__ dhpost, const float* __restrict__ dM,
             float* __restrict__ dhpre_raw, float* __restrict__ dhpost_raw,
             float* __restrict__ dhres_raw, int stage) {
  __shared__ float D[kMaxN * (kMaxN + 1)];
  extern __shared__ float s_stage_sk[];  // optional [tape | logits]
  const int tid = threadIdx.x, ld = sk_ld(n);
  if (tid < n) {
    // d/da sigmoid(a) = s (1 - s); H_post_act = 2 sigmoid(b)
    if (hpre_raw && dhpre) {
      const float s = sigmoidf_(hpre_raw[tid]);
      dhpre_raw[tid] = dhpre[tid] * (1.0f - s) * s;
    }
    if (hpost_raw && dhpost) {
      const float s = sigmoidf_(hpost_raw[tid]);
      dhpost_raw[tid] = (2.0f * dhpost[tid]) * (1.0f - s) * s;
    }
  }
  if (hres_raw && dM) {
    if (sk_warp_ok(n)) {
      // one call site per address space of the tape (shared when staged,
      // global otherwise), so its loads are not generic
      auto run = [&](const float* Hs, const float* Ts) {
        if (sk_lane_ok(n)) {
          if (tid < 32) {
            MHC_SK_LANE_SWITCH(n, ({
              const bool act = tid < SK_N * SK_N;
              const float d = sk_backward_lane<SK_N>(Hs, Ts, iters, eps, act ? dM[tid] : 0.f);
              if (act) dhres_raw[tid] = d;
            }))
          }
          return;
        }
        if (tid < 32) {
          const int row = tid % n;
          MHC_SK_WARP_SWITCH(n, ({
            float d[SK_N];
            for (int j = 0; j < SK_N; ++j) d[j] = dM[row * SK_N + j];
            sk_backward_warp<SK_N>(Hs, Ts, iters, eps, d);
            if (tid < SK_N)
              for (int j = 0; j < SK_N; ++j) dhres_raw[row * SK_N + j] = d[j];
          }))
        }
      };
      if (stage) {
        const size_t tf = (size_t)iters * sk_tape_stride(n);
#pragma unroll 8
        for (size_t e = tid; e < tf; e += blockDim.x) s_stage_sk[e] = tape[e];
        for (int e = tid; e < n * n; e += blockDim.x) s_stage_sk[tf + e] = hres_raw[e];
        __syncthreads();
        run(s_stage_sk + tf, s_stage_sk);
      } else {
        run(hres_raw, tape);
      }
      return;
    }
    if (sk_elem_ok(n)) {  // launched with n^2 threads
      MHC_SK_ELEM_SWITCH(n, ({
        if (stage) {
          const SkTape tp = sk_stage_tape_fixed<SK_N>(tape, iters, s_stage_sk);
          __syncthreads();  // staged tape complete
          sk_backward_elem<SK_N, SK_N * SK_N>(hres_raw, tp, iters, eps, dM, D, dhres_raw);
        } else {
          sk_backward_elem<SK_N, SK_N * SK_N>(hres_raw, SkTape{tape, SK_N, sk_tape_stride(SK_N)},
                                              iters, eps, dM, D, dhres_raw);
        }
      }))
      return;
    }
    const SkTape tp = stage ? sk_stage_tape(tape, n, iters, s_stage_sk)
                            : SkTape{tape, n, sk_tape_stride(n)};
    for (int e = tid; e < n * n; e += blockDim.x) D[(e / n) * ld + e % n] = dM[e];
    __syncthreads();
    sk_backward_block(hres_raw, tp, n, iters, eps, D, dhres_raw);
  }
}

int launch_params_fwd(const float* hpre_raw, const float* hpost_raw, const float* hres_raw,
                      int n, int iters, float eps, float* hpre, float* hpost, float* M,
                      float* tape, cudaStream_t st) {
  const int threads = sk_threads(n);
  k_params_fwd<<<1, threads, 0, st>>>(hpre_raw, hpost_raw, hres_raw, n, iters, eps, hpre,
                                      hpost, M, tape);
  return check_launch("params_fwd");
}

__global__ void k_selftest_reciprocal(const float* __restrict__ x, float* __restrict__ y,
                                      int64_t count) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = rcp_nr(x[i]);
}

int launch_selftest_reciprocal(const float* x, float* y, int64_t count, cudaStream_t st) {
  const int64_t blocks = (count + 255) / 256;
  const int grid = (int)(blocks < 4096 ? blocks : 4096);
  k_selftest_reciprocal<<<grid, 256, 0, st>>>(x, y, count);
  return check_launch("selftest_reciprocal");
}

int launch_params_bwd(const float* hpre_raw, const float* hpost_raw, const float* hres_raw,
                      const float* tape, int n, int iters, float eps, const float* dhpre,
                      const float* dhpost, const float* dM, float* dhpre_raw,
                      float* dhpost_raw, float* dhres_raw, cudaStream_t st) {
  const int threads = sk_threads(n);
  size_t smem = 0;
  if (hres_raw && dM && tape) {
    const size_t b = sk_stage_floats(n, iters) * sizeof(float);
    if (b <= 160 * 1024) smem = b;
  }
  if (allow_dyn_smem(k_params_bwd, smem) != cudaSuccess) smem = 0;
  k_params_bwd<<<1, threads, smem, st>>>(hpre_raw, hpost_raw, hres_raw, tape, n, iters, eps,
                                         dhpre, dhpost, dM, dhpre_raw, dhpost_raw, dhres_raw,
                                         smem > 0);
  return check_launch("params_bwd");
}

// ---------------------------------------------------------------------------
// Batched, n divides 32: one thread per matrix row, a matrix occupies n
// consecutive lanes; row sums are per-thread, column sums are butterfly
// shuffles across the n lanes (identical bits on every lane of the group).
template <int N>
__device__ __forceinline__ void sk_row_load(const float* __restrict__ src, float (&p)[N]) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int j = 0; j < N; j += 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(src) + j / 4);
      p[j] = v.x; p[j + 1] = v.y; p[j + 2] = v.z; p[j + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < N; ++j) p[j] = __ldg(src + j);
  }
}
template <int N>
__device__ __forceinline__ void sk_row_store(float* __restrict__ dst, const float (&p)[N]) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int j = 0; j < N; j += 4)
      reinterpret_cast<float4*>(dst)[j / 4] = make_float4(p[j], p[j + 1], p[j + 2], p[j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < N; ++j) dst[j] = p[j];
  }
}

template <int N>
__global__ void __launch_bounds__(256)
k_sk_batched_fwd(const float* __restrict__ H, int64_t batch, int iters, float eps,
                 float* __restrict__ M) {
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t m = gid / N;
  const int row = (int)(gid % N);
  const bool valid = m < batch;
  float p[N];
  if (valid) sk_row_load<N>(H + (m * N + row) * N, p);
  else
#pragma unroll
    for (int j = 0; j < N; ++j) p[j] = 0.f;
  float mx = p[0];
#pragma unroll
  for (int j = 1; j < N; ++j) mx = fmaxf(mx, p[j]);
#pragma unroll
  for (int j = 0; j < N; ++j) p[j] = expf(p[j] - mx);
  for (int k = 0; k < iters; ++k) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) s += p[j];
    const float rs = row_scale(s, eps);
#pragma unroll
    for (int j = 0; j < N; ++j) p[j] *= rs;
#pragma unroll
    for (int j = 0; j < N; ++j) p[j] *= col_scale(group_sum<N>(p[j]), eps);
  }
  if (valid) sk_row_store<N>(M + (m * N + row) * N, p);
}

// Backward: replays the forward into a shared-memory tape that keeps only
// each thread's row before every row step, [iters][N][blockDim] (thread index
// fastest: conflict-free).  The row sum and the column sums of an iteration
// are recomputed from it in the backward with the forward's own operations
// in the same order (sequential row sum; product by the row scale, then the
// same butterfly), so they are bit-identical to the forward's.  Storing N
// floats per iteration instead of N + 2 lets more threads stay resident.
template <int N>
__global__ void __launch_bounds__(256)
k_sk_batched_bwd(const float* __restrict__ H, const float* __restrict__ dM, int64_t batch,
                 int iters, float eps, float* __restrict__ dH) {
  extern __shared__ float s_tape[];
  const int bd = blockDim.x, tid = threadIdx.x;
  const int64_t gid = (int64_t)blockIdx.x * bd + tid;
  const int64_t m = gid / N;
  const int row = (int)(gid % N);
  const bool valid = m < batch;
  auto TP = [&](int k, int j) -> float& { return s_tape[((size_t)k * N + j) * bd + tid]; };

  float h[N], p[N];
  if (valid) sk_row_load<N>(H + (m * N + row) * N, h);
  else
#pragma unroll
    for (int j = 0; j < N; ++j) h[j] = 0.f;
  float mx = h[0];
#pragma unroll
  for (int j = 1; j < N; ++j) mx = fmaxf(mx, h[j]);
#pragma unroll
  for (int j = 0; j < N; ++j) p[j] = expf(h[j] - mx);
  for (int k = 0; k < iters; ++k) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) { TP(k, j) = p[j]; s += p[j]; }
    const float rs = row_scale(s, eps);
#pragma unroll
    for (int j = 0; j < N; ++j) p[j] *= rs;
#pragma unroll
    for (int j = 0; j < N; ++j) p[j] *= col_scale(group_sum<N>(p[j]), eps);
  }

  float d[N];
  if (valid) sk_row_load<N>(dM + (m * N + row) * N, d);
  else
#pragma unroll
    for (int j = 0; j < N; ++j) d[j] = 0.f;
  for (int k = iters - 1; k >= 0; --k) {
    float pa[N], pb[N];
    float r = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) { pa[j] = TP(k, j); r += pa[j]; }
    const float rs = row_scale(r, eps);
#pragma unroll
    for (int j = 0; j < N; ++j) {
      pb[j] = pa[j] * rs;
      const float c = group_sum<N>(pb[j]);
      const float dcs = group_sum<N>(d[j] * pb[j]);
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
  float S = 0.f, cnt = 0.f;
#pragma unroll
  for (int j = 0; j < N; ++j) {
    d[j] *= expf(h[j] - mx);
    S += d[j];
    cnt += (h[j] == mx) ? 1.f : 0.f;
  }
  const float share = S / cnt;
#pragma unroll
  for (int j = 0; j < N; ++j) d[j] -= (h[j] == mx) ? share : 0.f;
  if (valid) sk_row_store<N>(dH + (m * N + row) * N, d);
}

// ---------------------------------------------------------------------------
// Batched, n in {1, 2, 4}: one thread per matrix, the whole n x n matrix in
// registers.  Row sums are sequential and column sums follow the butterfly
// order of group_sum<N> ((p0 + p2) + (p1 + p3) for n = 4), so every value is
// bit-identical to the lane kernels above, without lane exchanges; the n
// independent rows and columns of a half-step give the instruction-level
// parallelism.  VEC: H, dM and the output are 16-byte aligned (float4 I/O).
template <int N>
__device__ __forceinline__ float sk_tree_sum(float (&t)[N]) {
#pragma unroll
  for (int o = N / 2; o > 0; o >>= 1)
#pragma unroll
    for (int i = 0; i < o; ++i) t[i] = t[i] + t[i + o];
  return t[0];
}

template <int N, bool VEC>
__device__ __forceinline__ void sk_mat_load(const float* __restrict__ src, float (&p)[N][N]) {
  if constexpr (VEC) {
#pragma unroll
    for (int q = 0; q < N * N / 4; ++q) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(src) + q);
      const int e = 4 * q;
      p[e / N][e % N] = v.x; p[(e + 1) / N][(e + 1) % N] = v.y;
      p[(e + 2) / N][(e + 2) % N] = v.z; p[(e + 3) / N][(e + 3) % N] = v.w;
    }
  } else {
#pragma unroll
    for (int e = 0; e < N * N; ++e) p[e / N][e % N] = __ldg(src + e);
  }
}
template <int N, bool VEC>
__device__ __forceinline__ void sk_mat_store(float* __restrict__ dst, const float (&p)[N][N]) {
  if constexpr (VEC) {
#pragma unroll
    for (int q = 0; q < N * N / 4; ++q) {
      const int e = 4 * q;
      reinterpret_cast<float4*>(dst)[q] =
          make_float4(p[e / N][e % N], p[(e + 1) / N][(e + 1) % N],
                      p[(e + 2) / N][(e + 2) % N], p[(e + 3) / N][(e + 3) % N]);
    }
  } else {
#pragma unroll
    for (int e = 0; e < N * N; ++e) dst[e] = p[e / N][e % N];
  }
}

// exp(h - rowmax) (reference.py:67), row maxima kept for the backward.
template <int N>
__device__ __forceinline__ void sk_mat_exp(const float (&h)[N][N], float (&p)[N][N],
                                           float (&mx)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) {
    mx[i] = h[i][0];
#pragma unroll
    for (int j = 1; j < N; ++j) mx[i] = fmaxf(mx[i], h[i][j]);
#pragma unroll
    for (int j = 0; j < N; ++j) p[i][j] = expf(h[i][j] - mx[i]);
  }
}

// One Sinkhorn iteration (reference.py:36-46): row step, then column step.
template <int N>
__device__ __forceinline__ void sk_mat_iter(float (&p)[N][N], float eps) {
#pragma unroll
  for (int i = 0; i < N; ++i) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) s += p[i][j];
    const float rs = row_scale(s, eps);
#pragma unroll
    for (int j = 0; j < N; ++j) p[i][j] *= rs;
  }
#pragma unroll
  for (int j = 0; j < N; ++j) {
    float t[N];
#pragma unroll
    for (int i = 0; i < N; ++i) t[i] = p[i][j];
    const float cs = col_scale(sk_tree_sum<N>(t), eps);
#pragma unroll
    for (int i = 0; i < N; ++i) p[i][j] *= cs;
  }
}

template <int N, bool VEC>
__global__ void __launch_bounds__(128)
k_sk_mat_fwd(const float* __restrict__ H, int64_t batch, int iters, float eps,
             float* __restrict__ M) {
  const int64_t m = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= batch) return;
  float h[N][N], p[N][N], mx[N];
  sk_mat_load<N, VEC>(H + m * N * N, h);
  sk_mat_exp<N>(h, p, mx);
  for (int k = 0; k < iters; ++k) sk_mat_iter<N>(p, eps);
  sk_mat_store<N, VEC>(M + m * N * N, p);
}

// Backward with checkpoints: the forward replay stores P before every S-th
// iteration in shared memory ([ceil(iters / S)][N * N][blockDim], thread
// index fastest: conflict-free); the reverse sweep then re-runs each segment
// of S iterations from its checkpoint into a register tape and reverses it.
// Every recomputed P_k is bit-identical to the forward's (same operations in
// the same order).  Shared memory per thread is ceil(iters / S) * N * N * 4
// bytes instead of iters * N * N * 4, which keeps a whole 65,536-matrix batch
// resident at once; the price is a second forward replay.
template <int N, int S, bool VEC>
__global__ void __launch_bounds__(128, 4)
k_sk_mat_bwd(const float* __restrict__ H, const float* __restrict__ dM, int64_t batch,
             int iters, float eps, float* __restrict__ dH) {
  extern __shared__ float s_ck[];
  const int bd = blockDim.x, tid = threadIdx.x;
  const int64_t m = (int64_t)blockIdx.x * bd + tid;
  if (m >= batch) return;  // no block-wide synchronisation below
  auto CK = [&](int seg, int e) -> float& { return s_ck[((size_t)seg * N * N + e) * bd + tid]; };

  float p[N][N], mx[N];
  {
    float h[N][N];
    sk_mat_load<N, VEC>(H + m * N * N, h);
    sk_mat_exp<N>(h, p, mx);
  }
  for (int k = 0; k < iters; ++k) {
    if (k % S == 0) {
#pragma unroll
      for (int e = 0; e < N * N; ++e) CK(k / S, e) = p[e / N][e % N];
    }
    sk_mat_iter<N>(p, eps);
  }

  float d[N][N];
  sk_mat_load<N, VEC>(dM + m * N * N, d);
  for (int seg = (iters + S - 1) / S - 1; seg >= 0; --seg) {
    const int k0 = seg * S, len = min(S, iters - k0);
    float tp[S][N][N];
#pragma unroll
    for (int e = 0; e < N * N; ++e) p[e / N][e % N] = CK(seg, e);
#pragma unroll
    for (int s = 0; s < S; ++s) {
      if (s < len) {
#pragma unroll
        for (int i = 0; i < N; ++i)
#pragma unroll
          for (int j = 0; j < N; ++j) tp[s][i][j] = p[i][j];
        if (s + 1 < len) sk_mat_iter<N>(p, eps);
      }
    }
#pragma unroll
    for (int s = S - 1; s >= 0; --s) {
      if (s >= len) continue;
      // reverse of iteration k0 + s; tp[s] = P before its row step
      float r[N], rs[N], pb[N][N];
#pragma unroll
      for (int i = 0; i < N; ++i) {
        r[i] = 0.f;
#pragma unroll
        for (int j = 0; j < N; ++j) r[i] += tp[s][i][j];
        rs[i] = row_scale(r[i], eps);
#pragma unroll
        for (int j = 0; j < N; ++j) pb[i][j] = tp[s][i][j] * rs[i];
      }
#pragma unroll
      for (int j = 0; j < N; ++j) {
        float tc[N], td[N];
#pragma unroll
        for (int i = 0; i < N; ++i) { tc[i] = pb[i][j]; td[i] = d[i][j] * pb[i][j]; }
        const float c = sk_tree_sum<N>(tc);
        const float dcs = sk_tree_sum<N>(td);
        const float cs = col_scale(c, eps);
        const float g = recip_grad(dcs, c, cs, eps);
#pragma unroll
        for (int i = 0; i < N; ++i) d[i][j] = d[i][j] * cs + g;
      }
#pragma unroll
      for (int i = 0; i < N; ++i) {
        float drs = 0.f;
#pragma unroll
        for (int j = 0; j < N; ++j) drs += d[i][j] * tp[s][i][j];
        const float dr = recip_grad(drs, r[i], rs[i], eps);
#pragma unroll
        for (int j = 0; j < N; ++j) d[i][j] = d[i][j] * rs[i] + dr;
      }
    }
  }
  // through exp(h - rowmax): the max's gradient is split over ties
  float h[N][N];
  sk_mat_load<N, VEC>(H + m * N * N, h);
#pragma unroll
  for (int i = 0; i < N; ++i) {
    float Ssum = 0.f, cnt = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) {
      d[i][j] *= expf(h[i][j] - mx[i]);
      Ssum += d[i][j];
      cnt += (h[i][j] == mx[i]) ? 1.f : 0.f;
    }
    const float share = Ssum / cnt;
#pragma unroll
    for (int j = 0; j < N; ++j) d[i][j] -= (h[i][j] == mx[i]) ? share : 0.f;
  }
  sk_mat_store<N, VEC>(dH + m * N * N, d);
}

// Batched fallback for n that does not divide 32 (or a tape too large for
// shared memory): persistent CTAs, one matrix at a time, tape in the
// workspace (one tape region per CTA).
__global__ void __launch_bounds__(64)
k_sk_batched_generic(const float* __restrict__ H, const float* __restrict__ dM, int64_t batch,
                     int n, int iters, float eps, float* __restrict__ out,
                     float* __restrict__ tapes, int backward) {
  __shared__ float P[kMaxN * (kMaxN + 1)];
  const int ld = sk_ld(n), nn = n * n;
  float* tape = backward ? tapes + (size_t)blockIdx.x * (size_t)iters * sk_tape_stride(n) : nullptr;
  for (int64_t m = blockIdx.x; m < batch; m += gridDim.x) {
    const float* Hm = H + m * nn;
    if (!backward) {
      sk_forward_block(Hm, n, iters, eps, P, nullptr, out + m * nn);
    } else {
      sk_forward_block(Hm, n, iters, eps, P, tape, nullptr);
      __syncthreads();
      for (int e = threadIdx.x; e < nn; e += blockDim.x) P[(e / n) * ld + e % n] = dM[m * nn + e];
      __syncthreads();
      sk_backward_block(Hm, SkTape{tape, n, sk_tape_stride(n)}, n, iters, eps, P, out + m * nn);
    }
    __syncthreads();
  }
}

static bool sk_small_path(int n) { return n == 1 || n == 2 || n == 4 || n == 8 || n == 16 || n == 32; }

// Threads per CTA for the shared-memory-tape backward: the size that keeps
// the most threads resident per SM given the per-thread tape; 0 if even one
// warp's tape does not fit in a CTA.
static int sk_bwd_threads(int n, int iters) {
  const size_t per_thread = (size_t)iters * n * sizeof(float);
  const size_t cta_cap = (size_t)max_smem_optin();
  const size_t sm_cap = 227 * 1024;
  int best = 0, best_resident = 0;
  for (int t = 32; t <= 256; t += 32) {
    const size_t b = per_thread * t;
    if (b > cta_cap) break;
    int ctas = b ? (int)(sm_cap / b) : 64;
    if (ctas > 2048 / t) ctas = 2048 / t;
    if (ctas * t >= best_resident) { best_resident = ctas * t; best = t; }
  }
  return best;
}

static int sk_generic_grid(int64_t batch) {
  int64_t g = (int64_t)sm_count() * 8;
  if (g > batch) g = batch;
  return (int)(g < 1 ? 1 : g);
}

size_t sk_batched_ws_bytes(int64_t batch, int n, int iters) {
  if (sk_small_path(n) && sk_bwd_threads(n, iters) > 0) return 0;
  return (size_t)sk_generic_grid(batch) * sk_tape_floats(n, iters) * sizeof(float);
}

template <int N>
static int sk_fwd_small(const float* H, int64_t batch, int iters, float eps, float* M,
                        cudaStream_t st) {
  const int threads = 256;
  const int64_t blocks = (batch * N + threads - 1) / threads;
  k_sk_batched_fwd<N><<<(unsigned)blocks, threads, 0, st>>>(H, batch, iters, eps, M);
  return check_launch("sinkhorn_batched_fwd");
}

template <int N>
static int sk_bwd_small(const float* H, const float* dM, int64_t batch, int iters, float eps,
                        float* dH, cudaStream_t st) {
  const int threads = sk_bwd_threads(N, iters);
  const size_t smem = (size_t)iters * N * threads * sizeof(float);
  {
    cudaError_t e = allow_dyn_smem(k_sk_batched_bwd<N>, smem);
    if (e != cudaSuccess) return set_error(MHC_ERR_CUDA, "sinkhorn_batched_bwd: %s", cudaGetErrorString(e));
  }
  const int64_t blocks = (batch * N + threads - 1) / threads;
  k_sk_batched_bwd<N><<<(unsigned)blocks, threads, smem, st>>>(H, dM, batch, iters, eps, dH);
  return check_launch("sinkhorn_batched_bwd");
}

// One thread per matrix (n in {1, 2, 4}); float4 I/O when every pointer is
// 16-byte aligned (a matrix of n * n floats then starts on a 16-byte boundary
// for n in {2, 4}).
constexpr int kSkMatThreads = 128;
template <int N> constexpr int sk_mat_seg() { return N == 4 ? 4 : (N == 2 ? 10 : 20); }
static size_t sk_mat_ck_bytes(int n, int iters) {
  const int S = n == 4 ? sk_mat_seg<4>() : (n == 2 ? sk_mat_seg<2>() : sk_mat_seg<1>());
  return (size_t)((iters + S - 1) / S) * n * n * sizeof(float) * kSkMatThreads;
}
// The checkpoint path keeps its checkpoints within 96 KB of shared memory
// per CTA (iters <= 48 for n = 4, two CTAs per SM still resident); longer
// chains use the lane kernels' full tape or the workspace path.
static bool sk_mat_bwd_ok(int n, int iters) {
  return (n == 1 || n == 2 || n == 4) && sk_mat_ck_bytes(n, iters) <= 96 * 1024;
}
static bool aligned16(const void* a, const void* b, const void* c) {
  return ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
           reinterpret_cast<uintptr_t>(c)) & 15) == 0;
}

template <int N>
static int sk_mat_fwd(const float* H, int64_t batch, int iters, float eps, float* M,
                      cudaStream_t st) {
  const int64_t blocks = (batch + kSkMatThreads - 1) / kSkMatThreads;
  if (N > 1 && aligned16(H, M, M))
    k_sk_mat_fwd<N, N != 1><<<(unsigned)blocks, kSkMatThreads, 0, st>>>(H, batch, iters, eps, M);
  else
    k_sk_mat_fwd<N, false><<<(unsigned)blocks, kSkMatThreads, 0, st>>>(H, batch, iters, eps, M);
  return check_launch("sinkhorn_batched_fwd");
}

template <int N>
static int sk_mat_bwd(const float* H, const float* dM, int64_t batch, int iters, float eps,
                      float* dH, cudaStream_t st) {
  constexpr int S = sk_mat_seg<N>();
  const size_t smem = sk_mat_ck_bytes(N, iters);
  const int64_t blocks = (batch + kSkMatThreads - 1) / kSkMatThreads;
  const bool vec = N > 1 && aligned16(H, dM, dH);
  {
    const cudaError_t e = vec ? allow_dyn_smem(k_sk_mat_bwd<N, S, N != 1>, smem)
                              : allow_dyn_smem(k_sk_mat_bwd<N, S, false>, smem);
    if (e != cudaSuccess)
      return set_error(MHC_ERR_CUDA, "sinkhorn_batched_bwd: %s", cudaGetErrorString(e));
  }
  if (vec)
    k_sk_mat_bwd<N, S, N != 1><<<(unsigned)blocks, kSkMatThreads, smem, st>>>(H, dM, batch, iters,
                                                                             eps, dH);
  else
    k_sk_mat_bwd<N, S, false><<<(unsigned)blocks, kSkMatThreads, smem, st>>>(H, dM, batch, iters,
                                                                            eps, dH);
  return check_launch("sinkhorn_batched_bwd");
}

int launch_sk_batched_fwd(const float* H, int64_t batch, int n, int iters, float eps, float* M,
                          void* ws, size_t ws_bytes, cudaStream_t st) {
  (void)ws; (void)ws_bytes;
  if (batch == 0) return MHC_OK;
  switch (n) {
    case 1: return sk_mat_fwd<1>(H, batch, iters, eps, M, st);
    case 2: return sk_mat_fwd<2>(H, batch, iters, eps, M, st);
    case 4: return sk_mat_fwd<4>(H, batch, iters, eps, M, st);
    case 8: return sk_fwd_small<8>(H, batch, iters, eps, M, st);
    case 16: return sk_fwd_small<16>(H, batch, iters, eps, M, st);
    case 32: return sk_fwd_small<32>(H, batch, iters, eps, M, st);
    default: break;
  }
  k_sk_batched_generic<<<sk_generic_grid(batch), 64, 0, st>>>(H, nullptr, batch, n, iters, eps, M,
                                                              nullptr, 0);
  return check_launch("sinkhorn_batched_fwd(generic)");
}

int launch_sk_batched_bwd(const float* H, const float* dM, int64_t batch, int n, int iters,
                          float eps, float* dH, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (batch == 0) return MHC_OK;
  if (sk_mat_bwd_ok(n, iters)) {
    switch (n) {
      case 1: return sk_mat_bwd<1>(H, dM, batch, iters, eps, dH, st);
      case 2: return sk_mat_bwd<2>(H, dM, batch, iters, eps, dH, st);
      case 4: return sk_mat_bwd<4>(H, dM, batch, iters, eps, dH, st);
      default: break;
    }
  }
  if (sk_small_path(n) && sk_bwd_threads(n, iters) > 0) {
    switch (n) {
      case 1: return sk_bwd_small<1>(H, dM, batch, iters, eps, dH, st);
      case 2: return sk_bwd_small<2>(H, dM, batch, iters, eps, dH, st);
      case 4: return sk_bwd_small<4>(H, dM, batch, iters, eps, dH, st);
      case 8: return sk_bwd_small<8>(H, dM, batch, iters, eps, dH, st);
      case 16: return sk_bwd_small<16>(H, dM, batch, iters, eps, dH, st);
      case 32: return sk_bwd_small<32>(H, dM, batch, iters, eps, dH, st);
      default: break;
    }
  }
  const size_t need = sk_batched_ws_bytes(batch, n, iters);
  if (ws_bytes < need || (need && !ws))
    return set_error(MHC_ERR_WORKSPACE, "sinkhorn_batched_bwd: workspace %zu < %zu bytes", ws_bytes, need);
  k_sk_batched_generic<<<sk_generic_grid(batch), 64, 0, st>>>(H, dM, batch, n, iters, eps, dH,
                                                              static_cast<float*>(ws), 1);
  return check_launch("sinkhorn_batched_bwd(generic)");
}

}  // namespace mhc
