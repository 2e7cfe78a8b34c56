// Shared device helpers for the mHC sm_100a kernels: dtype conversion,
// 16-byte vector loads/stores, warp/block reductions.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <type_traits>

#include "mhc_b200.h"

namespace mhc {

using bf16 = __nv_bfloat16;
using f16 = __half;

constexpr int kMaxN = 64;  // reference metal.py:71 _MAX_N_ALLOWED

// ---------------------------------------------------------------- dtypes --
__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(f16 v) { return __half2float(v); }
__device__ __forceinline__ float to_f(bf16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ f16 from_f<f16>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ bf16 from_f<bf16>(float v) { return __float2bfloat16_rn(v); }

// Elements per 16-byte vector.
template <typename T> struct VecOf { static constexpr int value = 16 / sizeof(T); };

// ------------------------------------------------------ vector load/store --
// Load V consecutive elements starting at p into fp32 registers.  V is either
// 1 (scalar path, any alignment) or the 16-byte width of T (p 16B-aligned).
// `Stream` selects the evict-first cache policy for data touched once.
template <bool Stream>
__device__ __forceinline__ float4 ld4(const float4* p) {
  if constexpr (Stream) return __ldcs(p);
  else return __ldg(p);
}
template <bool Stream>
__device__ __forceinline__ uint4 ldu4(const uint4* p) {
  if constexpr (Stream) return __ldcs(p);
  else return __ldg(p);
}

// Unpack one 16-byte chunk holding V elements of T into fp32.
// bf16 is the high half of an fp32, so each 32-bit word gives its two values
// with one shift (element 2k, the low half) and one mask (element 2k + 1).
template <typename T, int V>
__device__ __forceinline__ void unpack16(const uint4& u, float (&o)[V]) {
  static_assert(V * sizeof(T) == 16, "one 16-byte chunk");
  if constexpr (std::is_same<T, bf16>::value) {
    const unsigned wd[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      o[2 * k] = __uint_as_float(wd[k] << 16);
      o[2 * k + 1] = __uint_as_float(wd[k] & 0xffff0000u);
    }
  } else {
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int k = 0; k < V; ++k) o[k] = to_f(h[k]);
  }
}

template <typename T, int V, bool Stream = true>
__device__ __forceinline__ void load_vec(const T* __restrict__ p, float (&o)[V]) {
  if constexpr (V == 1) {
    o[0] = to_f(p[0]);
  } else if constexpr (sizeof(T) == 4) {
    static_assert(V % 4 == 0, "fp32 vector width is a multiple of 4");
#pragma unroll
    for (int k = 0; k < V; k += 4) {
      float4 v = ld4<Stream>(reinterpret_cast<const float4*>(p) + k / 4);
      o[k] = v.x; o[k + 1] = v.y; o[k + 2] = v.z; o[k + 3] = v.w;
    }
  } else if constexpr (V == 4) {
    uint2 u = *reinterpret_cast<const uint2*>(p);  // 8-byte aligned
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = to_f(h[k]);
  } else {
    static_assert(V == 8, "16-bit vector width is 4 or 8");
    unpack16<T, 8>(ldu4<Stream>(reinterpret_cast<const uint4*>(p)), o);
  }
}

// Two fp32 values rounded to nearest-even into one packed pair of 16-bit T
// (one paired conversion instead of two single ones; the same bits).
template <typename T>
__device__ __forceinline__ unsigned pack2_16(float a, float b) {
  unsigned u;
  if constexpr (std::is_same<T, bf16>::value) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    u = *reinterpret_cast<unsigned*>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    u = *reinterpret_cast<unsigned*>(&h);
  }
  return u;
}

// Store V fp32 values as T.  For T = float with V = 8 (half input, fp32
// output) two float4 stores are issued.
template <typename T, int V, bool Stream = true>
__device__ __forceinline__ void store_vec(T* __restrict__ p, const float (&v)[V]) {
  if constexpr (V == 1) {
    p[0] = from_f<T>(v[0]);
  } else if constexpr (sizeof(T) == 4) {
    static_assert(V % 4 == 0, "fp32 store width");
#pragma unroll
    for (int k = 0; k < V; k += 4) {
      float4 f = make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]);
      if constexpr (Stream) __stcs(reinterpret_cast<float4*>(p) + k / 4, f);
      else reinterpret_cast<float4*>(p)[k / 4] = f;
    }
  } else if constexpr (V == 2) {
    unsigned u;
    T* h = reinterpret_cast<T*>(&u);
    h[0] = from_f<T>(v[0]);
    h[1] = from_f<T>(v[1]);
    *reinterpret_cast<unsigned*>(p) = u;  // 4-byte aligned
  } else if constexpr (V == 4) {
    uint2 u;
    u.x = pack2_16<T>(v[0], v[1]);
    u.y = pack2_16<T>(v[2], v[3]);
    *reinterpret_cast<uint2*>(p) = u;
  } else {
    static_assert(V == 8, "16-bit store width is 2, 4 or 8");
    uint4 u;
    u.x = pack2_16<T>(v[0], v[1]);
    u.y = pack2_16<T>(v[2], v[3]);
    u.z = pack2_16<T>(v[4], v[5]);
    u.w = pack2_16<T>(v[6], v[7]);
    if constexpr (Stream) __stcs(reinterpret_cast<uint4*>(p), u);
    else *reinterpret_cast<uint4*>(p) = u;
  }
}

// ------------------------------------------------ async global->shared copy --
// 16-byte cp.async (L2 only).  Used to prefetch the next token row into
// thread-private shared-memory slots while the current row is processed;
// completion is awaited with cp.async.wait_all (a hardware wait, no spin).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }
// Wait until at most K of this thread's most recent commit groups are pending.
template <int K>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(K) : "memory");
}

// ------------------------------------------- programmatic dependent launch --
// A kernel launched with the PDL attribute (launch_pdl) may become resident
// while the previous kernel of the stream drains.  pdl_wait() blocks until
// that kernel has completed and its writes are visible, so it precedes every
// access to memory the previous kernel may touch; pdl_trigger() lets the next
// kernel's CTAs launch (they wait in their own pdl_wait()).  Both are no-ops
// for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

// ------------------------------------------------- mbarrier + bulk copies --
// 1-D bulk copies (cp.async.bulk: the TMA unit without a tensor map) from
// this GPU's own global memory into the CTA's shared memory, completing on an
// mbarrier through its transaction count.  Plain loads: no cluster multicast.
// Both addresses and the size must be multiples of 16 bytes.
__device__ __forceinline__ unsigned smem_u32(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
// Makes the mbarrier initialisation visible to the async proxy.
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Orders this thread's earlier generic-proxy shared-memory accesses before
// its later async-proxy (bulk copy) writes.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with parity `parity` to complete: false after
// `limit` tries (each try may suspend the thread for a short hardware-chosen
// time), so a copy that never lands cannot hang the kernel.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity,
                                          unsigned limit = 1u << 22) {
  for (unsigned k = 0; k < limit; ++k)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// ------------------------------------------------ warp-level tensor cores --
// ldmatrix.x4: lanes 8q..8q+7 give the row addresses (16 bytes each) of 8x8
// b16 matrix q; r[q] receives this lane's pair of that matrix: row lane/4,
// elements 2*(lane%4) and 2*(lane%4)+1.
__device__ __forceinline__ void ldmatrix_x4(unsigned (&r)[4], const void* smem_row) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem_row));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s)
               : "memory");
}

// D += A * B for a 16x16 (row) A and a 16x8 (col) B of 16-bit T, fp32
// accumulators.  Products of 16-bit values are exact in fp32.
template <typename T>
__device__ __forceinline__ void mma_16816(float (&d)[4], const unsigned (&a)[4], unsigned b0,
                                          unsigned b1) {
  if constexpr (sizeof(T) == 2 && std::is_same<T, bf16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    static_assert(std::is_same<T, f16>::value, "16-bit operands");
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// Plain fp32 vector load for parameter vectors (w) of width V.
template <int V>
__device__ __forceinline__ void load_f32(const float* __restrict__ p, float (&o)[V]) {
  if constexpr (V % 4 == 0) {
#pragma unroll
    for (int k = 0; k < V; k += 4) {
      float4 f = __ldg(reinterpret_cast<const float4*>(p) + k / 4);
      o[k] = f.x; o[k + 1] = f.y; o[k + 2] = f.z; o[k + 3] = f.w;
    }
  } else {
#pragma unroll
    for (int k = 0; k < V; ++k) o[k] = __ldg(p + k);
  }
}

// ------------------------------------------------------------ reductions --
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum of one value.  `red` is a 32-float shared slot; the caller
// alternates between two slots on consecutive calls so one barrier per call
// suffices.  Every thread gets the same bits (fixed order over warps).
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  float s = 0.f;
  for (int w = 0; w < nw; ++w) s += red[w];
  return s;
}

// Two sums with one barrier; `red` holds 64 floats.
__device__ __forceinline__ float2 block_sum2(float a, float b, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  a = warp_sum(a);
  b = warp_sum(b);
  if (lane == 0) { red[warp] = a; red[32 + warp] = b; }
  __syncthreads();
  const int nw = blockDim.x >> 5;
  float sa = 0.f, sb = 0.f;
  for (int w = 0; w < nw; ++w) { sa += red[w]; sb += red[32 + w]; }
  return make_float2(sa, sb);
}

// block_sum2 for a block of NW <= 32 warps with fewer instructions: after
// the barrier each lane reads one warp partial of each sum (zero above NW)
// and a 32-lane butterfly adds them.  Every lane of every warp ends with the
// same bits (each butterfly step adds the same two values on both lanes of a
// pair).  `red` holds 64 floats.
template <int NW>
__device__ __forceinline__ float2 block_sum2_bfly(float a, float b, float* red) {
  static_assert(NW >= 1 && NW <= 32, "at most 32 warps");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  a = warp_sum(a);
  b = warp_sum(b);
  if (lane == 0) { red[warp] = a; red[32 + warp] = b; }
  __syncthreads();
  float sa = lane < NW ? red[lane] : 0.f;
  float sb = lane < NW ? red[32 + lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sa += __shfl_xor_sync(0xffffffffu, sa, o);
    sb += __shfl_xor_sync(0xffffffffu, sb, o);
  }
  return make_float2(sa, sb);
}

// Sum over a group of G consecutive lanes (G divides 32, G a power of two).
// Butterfly order: every lane of the group gets identical bits.
template <int G>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// d0 += a0 * b0, d1 += a1 * b1 as one packed two-lane fp32 FMA (PTX
// fma.rn.f32x2, sm_100a): each lane rounds exactly like fmaf, so results are
// bit-identical to two fmaf calls, with half the issued instructions.
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b0,
                                     float b1) {
  asm("{\n .reg .b64 ra, rb, rc;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " mov.b64 rc, {%0, %1};\n fma.rn.f32x2 rc, ra, rb, rc;\n mov.b64 {%0, %1}, rc;\n}"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// Reference numerics (reference.py:40,45,104):
//   row scale = row_sum > eps ? 1/row_sum : 1
//   col scale = col_sum > eps ? 1/col_sum : 0
//   inv_rms  = 1 / sqrt(mean + eps)
//
// The Sinkhorn scales are reciprocals on a serial dependency chain of 2*iters
// half-steps.  rcp_nr is branch-free, so independent reciprocals of a
// half-step overlap: the hardware approximation (PTX rcp.approx.f32, at most
// 1 ulp from 1/x) refined by one Newton-Raphson step for 1/x,
// r' = r + r (1 - x r).  Zero, infinite and NaN approximations are returned
// as they are (the step would turn them into NaN).  Checked against 1.0f / x
// by a GPU test through mhc_selftest_reciprocal: within 1 ulp.
__device__ __forceinline__ float rcp_nr(float x) {
  float r;
  asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  const float e = fmaf(-x, r, 1.0f);
  const float q = fmaf(r, e, r);
  return (r == 0.f || isinf(r) || isnan(r)) ? r : q;
}
__device__ __forceinline__ float row_scale(float s, float eps) { return s > eps ? rcp_nr(s) : 1.0f; }
__device__ __forceinline__ float col_scale(float s, float eps) { return s > eps ? rcp_nr(s) : 0.0f; }
// Derivative of the masked reciprocal applied to an upstream g: d(1/s)/ds g =
// -g / s^2 where s > eps (inv = 1/s), 0 where the reference's where() masks.
__device__ __forceinline__ float recip_grad(float g, float s, float inv, float eps) {
  return s > eps ? -g * (inv * inv) : 0.f;
}
__device__ __forceinline__ float inv_rms(float sumsq, int C, float eps) {
  return 1.0f / sqrtf(sumsq / (float)C + eps);
}
__device__ __forceinline__ float sigmoidf_(float v) { return 1.0f / (1.0f + expf(-v)); }

// Layout of the workspace written by the backward kernels:
//   [0, 256)            header: int32 number of partial rows G, then the row
//                       step of the parameter partials (1, or the cluster size
//                       when a cluster's CTAs combined theirs into its first row)
//   params partials     G x P floats (P = n*n + 2n: dM row-major, dH_pre, dH_post)
//   column partials     G x C floats (d_rms_weight)
struct WsLayout {
  static constexpr size_t kHeader = 256;
  static __host__ __device__ size_t P(int n) { return (size_t)n * n + 2 * (size_t)n; }
  static __host__ __device__ size_t params_off() { return kHeader; }
  static __host__ __device__ size_t cols_off(int G, int n) {
    size_t b = kHeader + (size_t)G * P(n) * sizeof(float);
    return (b + 255) & ~size_t(255);
  }
  static __host__ __device__ size_t bytes(int G, int n, int C) {
    return cols_off(G, n) + (size_t)G * (size_t)C * sizeof(float);
  }
};

}  // namespace mhc
