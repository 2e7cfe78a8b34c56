// Quantized linear layer for the wrapped module of MHCRewire: a 4-bit affine
// group-wise quantized weight (the QuantizedLinear the reference wraps,
// tests/test_quantized.py:15, examples/patch_llama_mock.py:90, recognised by
// patching.py:74-80) multiplied on the tensor cores with the weight
// dequantised tile by tile inside the GEMM, so the [out, in] weight is never
// written to memory.
//
//   W[n, k] = scales[n, k / 64] * q[n, k] + biases[n, k / 64]   (q in [0, 15])
//   forward:   y[m, n] = sum_k x[m, k] W[n, k]  (+ bias[n])
//   backward:  dx[m, k] = sum_n dy[m, n] W[n, k]
// q is packed eight to a 32-bit word, code j of a word in bits [4j, 4j + 4)
// (word w of row n holds k = 8w .. 8w + 7).  Each weight is q * scale + bias
// computed with one fused multiply-add in the activations' dtype (bf16 or
// fp16, the tensor-core operand type; one rounding), the scale and bias
// rounded to that dtype first when they are stored in the other 16-bit type;
// products are accumulated in fp32.
//
// One CTA computes a 128 x BN output tile (BN = 256 or 128) with
// tcgen05.mma (kind::f16, fp32 accumulators in tensor memory), looping over
// the reduction in slices of 64:
//   warp 0      one thread issues TMA loads of the activation slice (128 x 64,
//               128-byte swizzled) and of the slice's packed words into a
//               five- or six-stage ring;
//   warp 1      allocates the accumulator columns in tensor memory; one
//               thread issues four 128 x BN x 16 MMAs per slice and commits
//               them to the slice's "empty" barrier;
//   warps 2-9   dequantise the slice's words into the B operand's 128-byte
//               swizzled layout in a three- or four-stage ring in shared
//               memory (K-major for the forward, MN-major for the backward),
//               then read the accumulators back
//               (tcgen05.ld) and write the output tile.
// Every wait is bounded: a barrier that never completes makes the CTA write
// NaN into its output tile and return (after waiting, again bounded, for its
// own copies and MMAs), so a fault shows as NaN instead of a hang.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>

#include "mhc_common.cuh"
#include "mhc_internal.h"

namespace mhc {
namespace {

constexpr int kBM = 128, kBK = 64, kGroup = 64;
constexpr int kThreads = 320, kDqThreads = 256;
constexpr unsigned kWaitLimit = 1u << 22;

// Shared-memory descriptor of a 128-byte-swizzled operand tile (tcgen05
// matrix descriptor): start address, leading / stride byte offsets (in 16-byte
// units), version 1, layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor, kind::f16: fp32 accumulate, A and B of one 16-bit
// type (bf16: 1, fp16: 0), A K-major, B K- or MN-major, M = 128, N = BN.
__host__ __device__ constexpr uint32_t f16_idesc(uint32_t ab, uint32_t b_mn, int M, int N) {
  return (1u << 4) | (ab << 7) | (ab << 10) | (b_mn << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y,
                                       uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}

// 32 consecutive accumulator columns of this thread's row (TMEM lane).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

// Bounded barrier wait that also gives up once another role has aborted.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, unsigned parity,
                                              volatile int* abort_flag) {
  for (unsigned k = 0; k < kWaitLimit; ++k) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((k & 1023u) == 1023u && *abort_flag) return false;
  }
  return false;
}

// Packed pairs of 16-bit floats (the dequantisation runs two values per
// instruction in the scales' dtype ST, then converts to the operand dtype XT).
template <typename T> struct Pair;
template <> struct Pair<f16> {
  using P = __half2;
  static constexpr uint32_t kMagic = 0x64006400u;  // 1024 + q, exactly, for q < 1024
  __device__ static P offset() { return __floats2half2_rn(1024.f, 1024.f); }
  __device__ static P dup(f16 v) { return __halves2half2(v, v); }
  __device__ static float2 to_f2(P v) { return __half22float2(v); }
  __device__ static P from_f2(float2 v) { return __float22half2_rn(v); }
};
template <> struct Pair<bf16> {
  using P = __nv_bfloat162;
  static constexpr uint32_t kMagic = 0x43004300u;  // 128 + q, exactly, for q < 128
  __device__ static P offset() { return __floats2bfloat162_rn(128.f, 128.f); }
  __device__ static P dup(bf16 v) { return __halves2bfloat162(v, v); }
  __device__ static float2 to_f2(P v) { return __bfloat1622float2(v); }
  __device__ static P from_f2(float2 v) { return __float22bfloat162_rn(v); }
};

template <typename P>
__device__ __forceinline__ uint32_t bits_of(P v) {
  return *reinterpret_cast<uint32_t*>(&v);
}
template <typename P>
__device__ __forceinline__ P of_bits(uint32_t u) {
  return *reinterpret_cast<P*>(&u);
}

// Eight codes of one word -> eight XT values (one 16-byte chunk, in k order):
// q * scale + bias as one fused multiply-add in XT (one rounding).  The scale
// and bias arrive already in XT (converted once per slice), so no value is
// converted per weight: the conversion unit is the narrowest pipe of the SM.
template <typename XT>
__device__ __forceinline__ uint4 dequant8(uint32_t w, typename Pair<XT>::P s2,
                                          typename Pair<XT>::P b2) {
  using PX = typename Pair<XT>::P;
  const uint32_t w4 = w >> 4;
  uint32_t o[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    // byte p of w holds codes 2p (low nibble) and 2p + 1 (high nibble)
    const uint32_t t = __byte_perm(w, w4, 0x4400u + 0x1111u * (uint32_t)p);
    uint32_t m;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(m) : "r"(t), "r"(0x000F000Fu), "r"(Pair<XT>::kMagic));
    const PX v = __hsub2(of_bits<PX>(m), Pair<XT>::offset());  // exact codes
    o[p] = bits_of(__hfma2(v, s2, b2));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Two rings in shared memory: SA stages of (activation slice, packed words
// of the slice), filled by TMA and released when the slice's MMAs complete,
// and SB stages of the dequantised B slice, filled by the dequantising warps
// and released the same way.  The activation ring is the deeper one, so the
// TMA runs several slices ahead of the tensor cores.
template <int BN, bool BWD>
struct Layout {
  static constexpr int kA = kBM * kBK * 2;                     // 16 KB
  static constexpr int kB = BN * kBK * 2;                      // BN x 64 16-bit values
  static constexpr int kW = BWD ? (kBK * BN / 2) : (BN * 32);  // packed words of the slice
  static constexpr int kAW = kA + kW;
  static constexpr int kSA = BN == 256 ? 5 : 6;
  static constexpr int kSB = BN == 256 ? 3 : 4;
  static constexpr int kBytes = kSA * kAW + kSB * kB + 1024;   // + alignment slack
  static_assert(kBytes <= 226 * 1024, "shared memory");
};

template <int BN, bool BWD, typename XT, typename ST>
__global__ void __launch_bounds__(kThreads, 1)
k_qlinear(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_w,
          const ST* __restrict__ scales, const ST* __restrict__ biases,
          const XT* __restrict__ bias, XT* __restrict__ out, int M, int N, int K) {
  using L = Layout<BN, BWD>;
  using PX = typename Pair<XT>::P;
  constexpr int SA = L::kSA, SB = L::kSB;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t a_full[SA], a_empty[SA], b_full[SB], b_empty[SB], acc_full;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  auto sA = [&](int s) { return smem + s * L::kAW; };
  auto sW = [&](int s) { return smem + s * L::kAW + L::kA; };
  auto sB = [&](int s) { return smem + SA * L::kAW + s * L::kB; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // forward: output tile (m0, n0), reduction over K; backward: output tile
  // (m0, k0 = n0 here), reduction over N
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * kBM;
  const int RED = BWD ? N : K;  // reduction length
  const int KT = RED / kBK;     // slices
  const int ldo = BWD ? K : N;  // output row length
  volatile int* abort_flag = &s_abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SA; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], 1);
    }
    for (int s = 0; s < SB; ++s) {
      mbar_init(&b_full[s], kDqThreads / 32);
      mbar_init(&b_empty[s], 1);
    }
    mbar_init(&acc_full, 1);
    s_abort = 0;
    mbar_init_fence();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     smem_u32(&s_tmem)),
                 "r"((uint32_t)BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA --
    if (lane == 0) {
      int issued = 0;
      for (int it = 0; it < KT; ++it) {
        const int s = it % SA;
        const unsigned ph = (unsigned)(it / SA) & 1u;
        if (!wait_or_abort(&a_empty[s], ph ^ 1u, abort_flag)) { s_abort = 1; break; }
        mbar_arrive_expect_tx(&a_full[s], (unsigned)L::kAW);
        tma_2d(sA(s), &tmap_a, it * kBK, m0, &a_full[s]);
        if constexpr (BWD) tma_2d(sW(s), &tmap_w, n0 / 8, it * kBK, &a_full[s]);
        else tma_2d(sW(s), &tmap_w, it * (kBK / 8), n0, &a_full[s]);
        issued = it + 1;
      }
      if (*abort_flag) {
        // copies still in flight land before the CTA's shared memory goes away
        for (int it = issued - SA < 0 ? 0 : issued - SA; it < issued; ++it)
          (void)mbar_wait(&a_full[it % SA], (unsigned)(it / SA) & 1u);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA --
    if (lane == 0) {
      constexpr uint32_t ab = std::is_same<XT, bf16>::value ? 1u : 0u;
      constexpr uint32_t idesc = f16_idesc(ab, BWD ? 1u : 0u, kBM, BN);
      for (int it = 0; it < KT; ++it) {
        const int sa = it % SA, sb = it % SB;
        if (!wait_or_abort(&a_full[sa], (unsigned)(it / SA) & 1u, abort_flag) ||
            !wait_or_abort(&b_full[sb], (unsigned)(it / SB) & 1u, abort_flag)) {
          s_abort = 1;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA(sa)), b0 = smem_u32(sB(sb));
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          // A: 128 rows x 128 bytes, 8-row groups 1 KB apart; +32 bytes per 16 k
          const uint64_t ad = sw128_desc(a0 + kk * 32, 16, 1024);
          uint64_t bd;
          if constexpr (BWD) {
            // B MN-major: [k-group of 8 rows][MN block of 64][8 rows][128 bytes];
            // one MMA takes two k-groups
            bd = sw128_desc(b0 + kk * 2 * (BN / 64) * 1024, 1024, (BN / 64) * 1024);
          } else {
            bd = sw128_desc(b0 + kk * 32, 16, 1024);
          }
          umma_f16(tmem, ad, bd, idesc, (it | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&a_empty[sa]);  // both slots free once these MMAs complete
        umma_commit(&b_empty[sb]);
      }
      umma_commit(&acc_full);  // also after an abort: marks the issued MMAs' completion
    }
  } else {
    // -------------------------------------------------------- dequantise --
    // A slice holds 8 * BN packed words (forward: BN weight rows x 8 words;
    // backward: 64 weight rows x BN / 8 words); each of the 256 threads
    // dequantises WPT = BN / 32 consecutive words of one row.
    constexpr int WPT = BN / 32;
    const int dq = threadIdx.x - 64;  // 0..255
    const int G = K / kGroup;         // groups per weight row
    int r, blk, j0;                   // B-tile row, 64-column block (backward), first chunk
    if constexpr (BWD) {
      r = dq >> 2;                    // reduction row 0..63
      blk = ((dq & 3) * WPT) >> 3;
      j0 = ((dq & 3) * WPT) & 7;
    } else {
      r = dq % BN;                    // output feature row of the tile
      blk = 0;
      j0 = (dq / BN) * WPT;
    }
    const int wofs = BWD ? r * (BN / 2) + (dq & 3) * WPT * 4 : r * 32 + j0 * 4;
    // scale / bias of slice it: requested kPre slices ahead into a register
    // ring (the inner loop is unrolled, so the ring index is a constant)
    constexpr int kPre = 4;
    auto sb_index = [&](int it) -> size_t {
      const int row = BWD ? it * kBK + r : n0 + r;   // weight row n
      const int grp = BWD ? n0 / kGroup + blk : it;  // its group of 64 columns
      return (size_t)row * G + grp;
    };
    ST sv[kPre], bv[kPre];
#pragma unroll
    for (int u = 0; u < kPre; ++u) {
      const size_t i = sb_index(u < KT ? u : 0);
      sv[u] = scales[i];
      bv[u] = biases[i];
    }
    bool stop = false;
    for (int it0 = 0; it0 < KT && !stop; it0 += kPre) {
#pragma unroll
      for (int u = 0; u < kPre; ++u) {
        const int it = it0 + u;
        if (it >= KT) break;
        const int sa = it % SA, sb = it % SB;
        // scale / bias in the operand dtype (exact when ST is XT)
        const PX s2 = Pair<XT>::dup(from_f<XT>(to_f(sv[u])));
        const PX b2 = Pair<XT>::dup(from_f<XT>(to_f(bv[u])));
        if (it + kPre < KT) {
          const size_t i = sb_index(it + kPre);
          sv[u] = scales[i];
          bv[u] = biases[i];
        }
        if (!wait_or_abort(&a_full[sa], (unsigned)(it / SA) & 1u, abort_flag) ||
            !wait_or_abort(&b_empty[sb], ((unsigned)(it / SB) & 1u) ^ 1u, abort_flag)) {
          s_abort = 1;
          stop = true;
          break;
        }
        uint32_t wd[WPT];
#pragma unroll
        for (int q = 0; q < WPT; q += 4) {
          const uint4 w = *reinterpret_cast<const uint4*>(sW(sa) + wofs + 4 * q);
          wd[q] = w.x; wd[q + 1] = w.y; wd[q + 2] = w.z; wd[q + 3] = w.w;
        }
        uint8_t* bt = sB(sb);
#pragma unroll
        for (int q = 0; q < WPT; ++q) {
          const uint4 v = dequant8<XT>(wd[q], s2, b2);
          const int j = j0 + q;  // 16-byte chunk within the row's 128 bytes
          uint32_t off;
          if constexpr (BWD) {
            // [k-group][64-column block][8 rows][128 bytes], chunks swizzled by row
            off = (uint32_t)((r >> 3) * (BN / 64) * 1024 + blk * 1024 + (r & 7) * 128 +
                             ((j ^ (r & 7)) << 4));
          } else {
            // [8-row group][8 rows][128 bytes], chunks swizzled by row
            off = (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((j ^ (r & 7)) << 4));
          }
          *reinterpret_cast<uint4*>(bt + off) = v;
        }
        fence_proxy_async_smem();  // the MMA reads these through the async proxy
        __syncwarp();
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(
                                        smem_u32(&b_full[sb]))
                                    : "memory");
      }
    }
    // ---------------------------------------------------------- epilogue --
    const bool ok = wait_or_abort(&acc_full, 0u, abort_flag) && !*abort_flag;
    tc_fence_after();
    const int sp = warp & 3;                 // TMEM lanes 32 sp .. 32 sp + 31
    const int half = (warp - 2) >> 2;        // columns [half BN/2, (half + 1) BN/2)
    const int m = m0 + sp * 32 + lane;
    for (int c0 = half * (BN / 2); c0 < (half + 1) * (BN / 2); c0 += 32) {
      uint32_t r[32];
      tmem_ld32(tmem + ((uint32_t)(sp * 32) << 16) + (uint32_t)c0, r);
      if (m < M) {
        XT* dst = out + (size_t)m * ldo + n0 + c0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t pk[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float2 f = make_float2(__uint_as_float(r[8 * q + 2 * e]),
                                   __uint_as_float(r[8 * q + 2 * e + 1]));
            if (!ok) f = make_float2(__int_as_float(0x7fc00000), __int_as_float(0x7fc00000));
            auto p2 = Pair<XT>::from_f2(f);
            if constexpr (!BWD) {
              if (bias) {
                const int n = n0 + c0 + 8 * q + 2 * e;
                p2 = Pair<XT>::from_f2(make_float2(
                    Pair<XT>::to_f2(p2).x + to_f(bias[n]), Pair<XT>::to_f2(p2).y + to_f(bias[n + 1])));
              }
            }
            pk[e] = bits_of(p2);
          }
          *reinterpret_cast<uint4*>(dst + 8 * q) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                 "r"((uint32_t)BN)
                 : "memory");
  }
}

// ------------------------------------------- forward, weights in TMEM --
// Forward y = x W^T computed transposed, y^T[n, m] = sum_k W[n, k] x[m, k]:
// the dequantised weights are the A operand and live in tensor memory (the
// dequantising threads write them with tcgen05.st straight from registers,
// no shared-memory round trip), the activations are the B operand (TMA,
// 128-byte swizzled, K-major).  A CTA computes 128 features x 256 tokens.
//   warp 0      TMA: activation slice (256 x 64) and the slice's packed words
//               (two 128 x 4-word boxes) into a five-stage ring;
//   warp 1      TMEM allocation; one thread issues the MMAs;
//   warps 2-9   dequantise: warp w owns TMEM lanes 32 (w % 4) .. + 31 (its
//               features) and half of the slice's 64 columns; afterwards
//               they read y^T back and write y (32 consecutive features per
//               warp store: 64 contiguous bytes).
// TMEM columns: [0, 256) accumulators, [256, 384) four A stages of 32.
//
// BWD = true computes the input gradient the same way, dx^T[k, m] =
// sum_n W[n, k] dy[m, n]: the A rows are rows of W^T, so it reads the
// transposed packing of the weight (codes of W^T, eight consecutive n per
// word) and, since a row of W^T crosses N different groups, one scale and
// one bias per element: the transposed scales / biases ([K/64][N], already in
// the activations' dtype) of the slice's 64 n and the tile's two groups are
// staged with the words.
constexpr int kTmTok = 256, kTmFeat = 128, kTmSX = 5, kTmSA = 4;

template <bool BWD>
struct TmLayout {
  static constexpr int kX = kTmTok * kBK * 2;                   // 32 KB activation slice
  static constexpr int kW = kTmFeat * 8 * 4;                    // 4 KB of packed words
  static constexpr int kSB = BWD ? 2 * (2 * kBK * 2) : 0;       // scale + bias boxes
  static constexpr int kStage = (kX + kW + kSB + 1023) / 1024 * 1024;  // swizzle alignment
  static constexpr int kBytes = kTmSX * kStage + 1024;
  static_assert(kBytes <= 226 * 1024, "shared memory");
};

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};\n" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Eight codes of one word with a scale and a bias per pair of values (two
// consecutive codes): four XT pairs of each in s4 / b4.
template <typename XT>
__device__ __forceinline__ uint4 dequant8_pairs(uint32_t w, uint4 s4, uint4 b4) {
  using PX = typename Pair<XT>::P;
  const uint32_t w4 = w >> 4;
  const uint32_t sc[4] = {s4.x, s4.y, s4.z, s4.w}, bc[4] = {b4.x, b4.y, b4.z, b4.w};
  uint32_t o[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t t = __byte_perm(w, w4, 0x4400u + 0x1111u * (uint32_t)p);
    uint32_t m;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(m) : "r"(t), "r"(0x000F000Fu), "r"(Pair<XT>::kMagic));
    const PX v = __hsub2(of_bits<PX>(m), Pair<XT>::offset());
    o[p] = bits_of(__hfma2(v, of_bits<PX>(sc[p]), of_bits<PX>(bc[p])));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

template <bool BWD, typename XT, typename ST>
__global__ void __launch_bounds__(kThreads, 1)
k_qlinear_tm(const __grid_constant__ CUtensorMap tmap_x,
             const __grid_constant__ CUtensorMap tmap_w,
             const __grid_constant__ CUtensorMap tmap_st,
             const __grid_constant__ CUtensorMap tmap_bt, const ST* __restrict__ scales,
             const ST* __restrict__ biases, const XT* __restrict__ bias,
             XT* __restrict__ out, int M, int N, int K) {
  using L = TmLayout<BWD>;
  using PX = typename Pair<XT>::P;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t x_full[kTmSX], x_empty[kTmSX], a_full[kTmSA], a_empty[kTmSA],
      acc_full;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  auto sX = [&](int s) { return smem + s * L::kStage; };
  auto sW = [&](int s, int h) { return smem + s * L::kStage + L::kX + h * (L::kW / 2); };
  auto sS = [&](int s) { return smem + s * L::kStage + L::kX + L::kW; };  // [2][64] scales
  auto sBi = [&](int s) { return sS(s) + 2 * kBK * 2; };                  // [2][64] biases

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // features (rows of W, or of W^T for BWD) and tokens of this tile
  const int f0 = blockIdx.x * kTmFeat, m0 = blockIdx.y * kTmTok;
  const int F = BWD ? K : N;                 // output row length
  const int KT = (BWD ? N : K) / kBK;        // reduction slices
  volatile int* abort_flag = &s_abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTmSX; ++s) { mbar_init(&x_full[s], 1); mbar_init(&x_empty[s], 1); }
    for (int s = 0; s < kTmSA; ++s) {
      mbar_init(&a_full[s], kDqThreads / 32);
      mbar_init(&a_empty[s], 1);
    }
    mbar_init(&acc_full, 1);
    s_abort = 0;
    mbar_init_fence();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     smem_u32(&s_tmem)),
                 "r"(512u)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;             // accumulators: columns [0, 256)
  const uint32_t tmem_a = tmem + kTmTok;    // A stages: 32 columns each

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int it = 0; it < KT; ++it) {
        const int s = it % kTmSX;
        if (!wait_or_abort(&x_empty[s], ((unsigned)(it / kTmSX) & 1u) ^ 1u, abort_flag)) {
          s_abort = 1;
          break;
        }
        mbar_arrive_expect_tx(&x_full[s], (unsigned)(L::kX + L::kW + L::kSB));
        tma_2d(sX(s), &tmap_x, it * kBK, m0, &x_full[s]);
        tma_2d(sW(s, 0), &tmap_w, it * 8, f0, &x_full[s]);
        tma_2d(sW(s, 1), &tmap_w, it * 8 + 4, f0, &x_full[s]);
        if constexpr (BWD) {
          tma_2d(sS(s), &tmap_st, it * kBK, f0 / kGroup, &x_full[s]);
          tma_2d(sBi(s), &tmap_bt, it * kBK, f0 / kGroup, &x_full[s]);
        }
        issued = it + 1;
      }
      if (*abort_flag)
        for (int it = issued - kTmSX < 0 ? 0 : issued - kTmSX; it < issued; ++it)
          (void)mbar_wait(&x_full[it % kTmSX], (unsigned)(it / kTmSX) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ab = std::is_same<XT, bf16>::value ? 1u : 0u;
      constexpr uint32_t idesc = f16_idesc(ab, 0u, kTmFeat, kTmTok);
      for (int it = 0; it < KT; ++it) {
        const int sx = it % kTmSX, sa = it % kTmSA;
        if (!wait_or_abort(&x_full[sx], (unsigned)(it / kTmSX) & 1u, abort_flag) ||
            !wait_or_abort(&a_full[sa], (unsigned)(it / kTmSA) & 1u, abort_flag)) {
          s_abort = 1;
          break;
        }
        tc_fence_after();
        const uint32_t x0 = smem_u32(sX(sx));
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          umma_f16_ts(tmem, tmem_a + sa * 32 + kk * 8, sw128_desc(x0 + kk * 32, 16, 1024), idesc,
                      (it | kk) != 0 ? 1u : 0u);
        umma_commit(&x_empty[sx]);
        umma_commit(&a_empty[sa]);
      }
      umma_commit(&acc_full);
    }
  } else {
    // ---- dequantise: feature row f (TMEM lane), 32 of the slice's 64 columns
    const int sp = warp & 3, half = (warp - 2) >> 2;
    const int f = sp * 32 + lane;
    const int G = K / kGroup;
    const uint32_t lane_base = (uint32_t)(sp * 32) << 16;
    constexpr int kPre = 4;
    ST sv[kPre], bv[kPre];
#pragma unroll
    for (int u = 0; u < kPre; ++u) {
      if constexpr (!BWD) {
        const size_t i = (size_t)(f0 + f) * G + (u < KT ? u : 0);
        sv[u] = scales[i];
        bv[u] = biases[i];
      }
    }
    bool stop = false;
    for (int it0 = 0; it0 < KT && !stop; it0 += kPre) {
#pragma unroll
      for (int u = 0; u < kPre; ++u) {
        const int it = it0 + u;
        if (it >= KT) break;
        const int sx = it % kTmSX, sa = it % kTmSA;
        PX s2, b2;
        if constexpr (!BWD) {
          s2 = Pair<XT>::dup(from_f<XT>(to_f(sv[u])));
          b2 = Pair<XT>::dup(from_f<XT>(to_f(bv[u])));
          if (it + kPre < KT) {
            const size_t i = (size_t)(f0 + f) * G + it + kPre;
            sv[u] = scales[i];
            bv[u] = biases[i];
          }
        }
        if (!wait_or_abort(&x_full[sx], (unsigned)(it / kTmSX) & 1u, abort_flag) ||
            !wait_or_abort(&a_empty[sa], ((unsigned)(it / kTmSA) & 1u) ^ 1u, abort_flag)) {
          s_abort = 1;
          stop = true;
          break;
        }
        tc_fence_after();
        // 4 words = 32 values of row f: [128 rows][4 words] per half, 16 B per row
        const uint4 w = *reinterpret_cast<const uint4*>(sW(sx, half) + f * 16);
        const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
        uint32_t v[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 o;
          if constexpr (BWD) {
            // scales / biases of n = 32 half + 8 q .. + 7 in this row's group
            const int ofs = ((f >> 6) * kBK + 32 * half + 8 * q) * 2;
            o = dequant8_pairs<XT>(wd[q], *reinterpret_cast<const uint4*>(sS(sx) + ofs),
                                   *reinterpret_cast<const uint4*>(sBi(sx) + ofs));
          } else {
            o = dequant8<XT>(wd[q], s2, b2);
          }
          v[4 * q] = o.x; v[4 * q + 1] = o.y; v[4 * q + 2] = o.z; v[4 * q + 3] = o.w;
        }
        tmem_st16(tmem_a + lane_base + (uint32_t)(sa * 32 + half * 16), v);
        asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(
                                        smem_u32(&a_full[sa]))
                                    : "memory");
      }
    }
    // ---- epilogue: y[m, f0 + f] for the warp's 128 tokens
    const bool ok = wait_or_abort(&acc_full, 0u, abort_flag) && !*abort_flag;
    tc_fence_after();
    const bool has_bias = !BWD && bias != nullptr;
    const float bf = has_bias ? to_f(bias[f0 + f]) : 0.f;
    for (int c0 = half * (kTmTok / 2); c0 < (half + 1) * (kTmTok / 2); c0 += 32) {
      uint32_t r[32];
      tmem_ld32(tmem + lane_base + (uint32_t)c0, r);
#pragma unroll
      for (int t = 0; t < 32; ++t) {
        const int m = m0 + c0 + t;
        if (m < M) {
          float y = ok ? __uint_as_float(r[t]) : __int_as_float(0x7fc00000);
          XT yv = from_f<XT>(y);
          if (has_bias) yv = from_f<XT>(to_f(yv) + bf);
          out[(size_t)m * F + f0 + f] = yv;
        }
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                 "r"(512u)
                 : "memory");
  }
}

// Transposed packing of 4-bit codes: wt[k][n / 8] holds the codes of rows
// n .. n + 7 at column k (code j of the word for row n + j), from
// w[n][k / 8] (code k % 8 of row n).  One output word per thread; a one-time
// layout build, so the eight scattered reads per word do not matter.
__global__ void k_transpose_pack4(const uint32_t* __restrict__ w, uint32_t* __restrict__ wt,
                                  int N, int K) {
  const int nwords = N / 8;
  const int64_t total = (int64_t)K * nwords;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int k = (int)(idx / nwords), nw = (int)(idx - (int64_t)k * nwords);
    uint32_t o = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t word = w[(size_t)(nw * 8 + j) * (K / 8) + k / 8];
      o |= ((word >> (4 * (k & 7))) & 0xFu) << (4 * j);
    }
    wt[idx] = o;
  }
}

// ------------------------------------------------------------------ host --
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    else
      (void)cudaGetLastError();
  });
  return fn;
}

int make_map(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
             uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
             CUtensorMapSwizzle sw) {
  auto fn = encode_fn();
  if (!fn) return set_error(MHC_ERR_CUDA, "qlinear: cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(MHC_ERR_CUDA, "qlinear: tensor map encode failed (%d)", (int)r);
  return MHC_OK;
}

template <int BN, bool BWD, typename XT, typename ST>
int run_qlinear(const void* a, const uint32_t* wq, const void* scales, const void* biases,
                const void* bias, void* out, int64_t M, int N, int K, cudaStream_t st) {
  CUtensorMap ma, mw;
  const CUtensorMapDataType adt =
      std::is_same<XT, bf16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int RED = BWD ? N : K;
  int r = make_map(&ma, adt, a, (uint64_t)RED, (uint64_t)M, (uint64_t)RED * 2, kBK, kBM,
                   CU_TENSOR_MAP_SWIZZLE_128B);
  if (r != MHC_OK) return r;
  // packed words: [N rows][K / 8 words]
  if constexpr (BWD)
    r = make_map(&mw, CU_TENSOR_MAP_DATA_TYPE_INT32, wq, (uint64_t)K / 8, (uint64_t)N,
                 (uint64_t)K / 2, BN / 8, kBK, CU_TENSOR_MAP_SWIZZLE_NONE);
  else
    r = make_map(&mw, CU_TENSOR_MAP_DATA_TYPE_INT32, wq, (uint64_t)K / 8, (uint64_t)N,
                 (uint64_t)K / 2, kBK / 8, BN, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (r != MHC_OK) return r;
  auto kern = k_qlinear<BN, BWD, XT, ST>;
  const size_t smem = Layout<BN, BWD>::kBytes;
  const cudaError_t e = allow_dyn_smem(kern, smem);
  if (e != cudaSuccess) return set_error(MHC_ERR_CUDA, "qlinear: %s", cudaGetErrorString(e));
  const int out_cols = BWD ? K : N;
  const dim3 grid(out_cols / BN, (unsigned)((M + kBM - 1) / kBM));
  kern<<<grid, kThreads, smem, st>>>(ma, mw, static_cast<const ST*>(scales),
                                     static_cast<const ST*>(biases), static_cast<const XT*>(bias),
                                     static_cast<XT*>(out), (int)M, N, K);
  return check_launch(BWD ? "qlinear_bwd_dx" : "qlinear_fwd");
}

template <typename XT, typename ST>
int run_qlinear_fwd_tm(const void* x, const uint32_t* wq, const void* scales, const void* biases,
                       const void* bias, void* out, int64_t M, int N, int K, cudaStream_t st) {
  CUtensorMap mx, mw;
  const CUtensorMapDataType xdt =
      std::is_same<XT, bf16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  int r = make_map(&mx, xdt, x, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, kBK, kTmTok,
                   CU_TENSOR_MAP_SWIZZLE_128B);
  if (r != MHC_OK) return r;
  r = make_map(&mw, CU_TENSOR_MAP_DATA_TYPE_INT32, wq, (uint64_t)K / 8, (uint64_t)N,
               (uint64_t)K / 2, 4, kTmFeat, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (r != MHC_OK) return r;
  auto kern = k_qlinear_tm<false, XT, ST>;
  const size_t smem = TmLayout<false>::kBytes;
  const cudaError_t e = allow_dyn_smem(kern, smem);
  if (e != cudaSuccess) return set_error(MHC_ERR_CUDA, "qlinear: %s", cudaGetErrorString(e));
  const dim3 grid(N / kTmFeat, (unsigned)((M + kTmTok - 1) / kTmTok));
  // the scale / bias maps are not read by the forward: pass the weight map
  kern<<<grid, kThreads, smem, st>>>(mx, mw, mw, mw, static_cast<const ST*>(scales),
                                     static_cast<const ST*>(biases), static_cast<const XT*>(bias),
                                     static_cast<XT*>(out), (int)M, N, K);
  return check_launch("qlinear_fwd");
}

template <typename XT>
int run_qlinear_bwd_tm(const void* dy, const uint32_t* wt, const void* scales_t,
                       const void* biases_t, void* dx, int64_t M, int N, int K, cudaStream_t st) {
  CUtensorMap md, mw, ms, mb;
  const CUtensorMapDataType xdt =
      std::is_same<XT, bf16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  int r = make_map(&md, xdt, dy, (uint64_t)N, (uint64_t)M, (uint64_t)N * 2, kBK, kTmTok,
                   CU_TENSOR_MAP_SWIZZLE_128B);
  if (r != MHC_OK) return r;
  // codes of W^T: [K rows][N / 8 words]
  r = make_map(&mw, CU_TENSOR_MAP_DATA_TYPE_INT32, wt, (uint64_t)N / 8, (uint64_t)K,
               (uint64_t)N / 2, 4, kTmFeat, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (r != MHC_OK) return r;
  // scales / biases of W^T: [K / 64][N] in the activations' dtype
  r = make_map(&ms, xdt, scales_t, (uint64_t)N, (uint64_t)K / kGroup, (uint64_t)N * 2, kBK, 2,
               CU_TENSOR_MAP_SWIZZLE_NONE);
  if (r != MHC_OK) return r;
  r = make_map(&mb, xdt, biases_t, (uint64_t)N, (uint64_t)K / kGroup, (uint64_t)N * 2, kBK, 2,
               CU_TENSOR_MAP_SWIZZLE_NONE);
  if (r != MHC_OK) return r;
  auto kern = k_qlinear_tm<true, XT, XT>;
  const size_t smem = TmLayout<true>::kBytes;
  const cudaError_t e = allow_dyn_smem(kern, smem);
  if (e != cudaSuccess) return set_error(MHC_ERR_CUDA, "qlinear: %s", cudaGetErrorString(e));
  const dim3 grid(K / kTmFeat, (unsigned)((M + kTmTok - 1) / kTmTok));
  kern<<<grid, kThreads, smem, st>>>(md, mw, ms, mb, nullptr, nullptr, nullptr,
                                     static_cast<XT*>(dx), (int)M, N, K);
  return check_launch("qlinear_bwd_dx_t");
}

template <bool BWD, typename XT, typename ST>
int dispatch_bn(const void* a, const uint32_t* wq, const void* scales, const void* biases,
                const void* bias, void* out, int64_t M, int N, int K, cudaStream_t st) {
  if constexpr (!BWD) {
    // MHC_B200_QMM_SMEM_B=1 selects the shared-memory-B forward (A/B measurement)
    const char* e = std::getenv("MHC_B200_QMM_SMEM_B");
    if (!e || std::atoi(e) == 0)
      return run_qlinear_fwd_tm<XT, ST>(a, wq, scales, biases, bias, out, M, N, K, st);
  }
  const int out_cols = BWD ? K : N;
  if (out_cols % 256 == 0)
    return run_qlinear<256, BWD, XT, ST>(a, wq, scales, biases, bias, out, M, N, K, st);
  return run_qlinear<128, BWD, XT, ST>(a, wq, scales, biases, bias, out, M, N, K, st);
}

template <bool BWD>
int dispatch(const void* a, int adt, const uint32_t* wq, const void* scales, const void* biases,
             int sdt, const void* bias, void* out, int64_t M, int N, int K, cudaStream_t st) {
  if (adt == MHC_BF16)
    return sdt == MHC_BF16
               ? dispatch_bn<BWD, bf16, bf16>(a, wq, scales, biases, bias, out, M, N, K, st)
               : dispatch_bn<BWD, bf16, f16>(a, wq, scales, biases, bias, out, M, N, K, st);
  return sdt == MHC_BF16
             ? dispatch_bn<BWD, f16, bf16>(a, wq, scales, biases, bias, out, M, N, K, st)
             : dispatch_bn<BWD, f16, f16>(a, wq, scales, biases, bias, out, M, N, K, st);
}

int check_args(const char* fn, const void* a, int adt, const uint32_t* wq, const void* scales,
               const void* biases, int sdt, void* out, int64_t M, int N, int K, int group_size,
               int bits) {
  if (M < 0 || N < 1 || K < 1) return set_error(MHC_ERR_INVALID, "%s: bad shape M=%lld N=%d K=%d", fn, (long long)M, N, K);
  if (adt != MHC_BF16 && adt != MHC_F16)
    return set_error(MHC_ERR_UNSUPPORTED, "%s: activations must be bf16 or fp16", fn);
  if (sdt != MHC_BF16 && sdt != MHC_F16)
    return set_error(MHC_ERR_UNSUPPORTED, "%s: scales/biases must be bf16 or fp16", fn);
  if (bits != 4 || group_size != kGroup)
    return set_error(MHC_ERR_UNSUPPORTED, "%s: the in-kernel dequantisation covers bits=4, group_size=64 (got %d, %d)", fn, bits, group_size);
  if (K % 128 != 0 || N % 128 != 0)
    return set_error(MHC_ERR_UNSUPPORTED, "%s: N and K must be multiples of 128 (N=%d K=%d)", fn, N, K);
  if (M > 0 && (!a || !wq || !scales || !biases || !out))
    return set_error(MHC_ERR_INVALID, "%s: NULL pointer", fn);
  if (M > 0 && (!aligned16(a) || !aligned16(wq) || !aligned16(out)))
    return set_error(MHC_ERR_INVALID, "%s: x/dy, the packed weight and the output must be 16-byte aligned", fn);
  return MHC_OK;
}

}  // namespace

int launch_qlinear_fwd(const void* x, int xdt, const uint32_t* wq, const void* scales,
                       const void* biases, int sdt, const void* bias, void* y, int64_t M, int N,
                       int K, int group_size, int bits, cudaStream_t st) {
  int r = check_args("mhc_qlinear_fwd", x, xdt, wq, scales, biases, sdt, y, M, N, K, group_size, bits);
  if (r != MHC_OK || M == 0) return r;
  return dispatch<false>(x, xdt, wq, scales, biases, sdt, bias, y, M, N, K, st);
}

int launch_qlinear_transpose_pack(const uint32_t* w, uint32_t* wt, int N, int K,
                                  cudaStream_t st) {
  if (N < 8 || K < 8 || N % 8 || K % 8)
    return set_error(MHC_ERR_INVALID, "mhc_qlinear_transpose_pack: N and K must be multiples of 8");
  if (!w || !wt) return set_error(MHC_ERR_INVALID, "mhc_qlinear_transpose_pack: NULL pointer");
  const int64_t total = (int64_t)K * (N / 8);
  int64_t blocks = (total + 255) / 256;
  if (blocks > (int64_t)sm_count() * 16) blocks = (int64_t)sm_count() * 16;
  k_transpose_pack4<<<(int)blocks, 256, 0, st>>>(w, wt, N, K);
  return check_launch("qlinear_transpose_pack");
}

int launch_qlinear_bwd_dx_t(const void* dy, int dydt, const uint32_t* wt, const void* scales_t,
                            const void* biases_t, void* dx, int64_t M, int N, int K,
                            int group_size, int bits, cudaStream_t st) {
  int r = check_args("mhc_qlinear_bwd_dx_t", dy, dydt, wt, scales_t, biases_t, dydt, dx, M, N, K,
                     group_size, bits);
  if (r != MHC_OK || M == 0) return r;
  if (!aligned16(scales_t) || !aligned16(biases_t))
    return set_error(MHC_ERR_INVALID, "mhc_qlinear_bwd_dx_t: scales_t / biases_t must be 16-byte aligned");
  if (dydt == MHC_BF16) return run_qlinear_bwd_tm<bf16>(dy, wt, scales_t, biases_t, dx, M, N, K, st);
  return run_qlinear_bwd_tm<f16>(dy, wt, scales_t, biases_t, dx, M, N, K, st);
}

int launch_qlinear_bwd_dx(const void* dy, int dydt, const uint32_t* wq, const void* scales,
                          const void* biases, int sdt, void* dx, int64_t M, int N, int K,
                          int group_size, int bits, cudaStream_t st) {
  int r = check_args("mhc_qlinear_bwd_dx", dy, dydt, wq, scales, biases, sdt, dx, M, N, K, group_size, bits);
  if (r != MHC_OK || M == 0) return r;
  return dispatch<true>(dy, dydt, wq, scales, biases, sdt, nullptr, dx, M, N, K, st);
}

}  // namespace mhc
