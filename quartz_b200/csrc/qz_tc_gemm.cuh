// qz_tc_gemm.cuh -- batched int8 weight-only GEMM (M > 1) on the 5th-gen tensor
// cores (tcgen05 / TMEM), replacing quartz/kernels/int8.py:66-87 (w8a32_gemm).
//
//   Y[m, n] = scale[n] * sum_k X[m, k] * q[n, k]      (+ residual[m, n])
//
// The weights are used exactly as stored: int8 [N, K], loaded by TMA straight
// into the 128-byte-swizzled shared-memory layout the MMA reads. The fp32
// activations are split once per call (split_x_kernel) into three signed int8
// "limbs" with a per-row scale s_m:
//
//   x[m, k] ~= s_m * (d2 * 2^16 + d1 * 2^8 + d0),   |d2*2^16 + d1*2^8 + d0| <= 2^23 - 2^16
//
// i.e. a 24-bit fixed-point copy of each activation row (error <= s_m / 2 =
// max|x_m| * 2^-24 per element). The three limb tiles of a stage form one
// int8 B operand of 3 * MT rows (tcgen05.mma kind::i8), accumulating exactly in
// int32 in tensor memory, so the only rounding is that of the activation split
// and of the final fp32 scale.
// The weights are never widened and never written back.
//
// Operand roles are swapped: the MMA's 128-row "A" operand is a tile of 128
// weight rows, the "B" operand a tile of MT tokens (MT in {16, 32, 64, 128}),
// so a small batch costs no more MMA padding than MT - M columns and the
// kernel streams the weights at HBM speed; large batches become tensor-bound.
//
// CTA: warp 0 = TMA producer, warp 1 = TMEM allocator + MMA issuer,
// warps 4..7 = epilogue (warp 4+i reads TMEM lanes 32i..32i+31 = weight rows).
// One CTA computes a 128 x MT tile over all of K; every wait is bounded.
#pragma once

#include <cuda.h>

#include "qz_device.cuh"

namespace qz {
namespace tc {

constexpr int kRows = 128;         // weight rows per CTA (MMA M)
constexpr int kKBytes = 128;       // K bytes per stage = one 128-B swizzle row
constexpr int kMmaK = 32;          // K per int8 MMA instruction
constexpr int kLimbs = 3;
constexpr int kThreads = 256;
constexpr int kMaxStages = 8;
constexpr int kEpiWarp0 = 4;
// 2^23 - 2^16: the largest limb-representable magnitude with d2 in [-128, 127].
constexpr float kLimbRange = 8323072.0f;

__host__ __device__ constexpr int stage_bytes(int mt) { return kRows * kKBytes + kLimbs * mt * kKBytes; }

struct TcArgs {
  const float* scale;      // [N] per-row weight scale (ng == 1)
  const float* sx;         // [Mpad] per-row activation scale
  float* Y;                // [M, N]
  const float* residual;   // [M, N] or null
  int32_t* acc;            // split-K: [3][Mpad][N] int32 partial sums (zeroed), else null
  int64_t M, N, K, Mpad;
  int nstages;
  int splits;              // K-splits (gridDim.z)
};

// ---------------------------------------------------------------------------
// activation split: one CTA per (padded) activation row
// ---------------------------------------------------------------------------
constexpr int kSplitThreads = 512;

// One value's three limbs: v = d2 * 2^16 + d1 * 2^8 + d0, each in [-128, 127].
__device__ __forceinline__ void limbs3(float x, float inv, int& d0, int& d1, int& d2) {
  const int v = __float2int_rn(x * inv);
  d0 = ((v + 128) & 255) - 128;
  const int v1 = (v - d0) >> 8;
  d1 = ((v1 + 128) & 255) - 128;
  d2 = (v1 - d1) >> 8;
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 255u) | ((static_cast<uint32_t>(b) & 255u) << 8) |
         ((static_cast<uint32_t>(c) & 255u) << 16) | ((static_cast<uint32_t>(d) & 255u) << 24);
}

// What the split kernel applies to each activation row before splitting it,
// so that the op producing the GEMM's input needs no launch of its own:
//   kActNone     x
//   kActRmsNorm  x / sqrt(mean(x^2) + eps) * w        (quartz/ops.py:24-32)
//   kActSiluMul  silu(g) * u of a [g | u] row of 2K    (quartz/quantize.py:112-114)
// The values are computed with the same expressions and, for the RMSNorm, the
// same order of the sum of squares (512 threads, thread t adding elements
// t, t + 512, ... in turn, then warp and block sums) as dec::rmsnorm_kernel
// and silu_mul_kernel, so they equal what those kernels write.
constexpr int kActNone = 0, kActRmsNorm = 1, kActSiluMul = 2;

struct SplitAct {
  const float* w;   // RMSNorm weight [K]
  float r;          // RMSNorm 1 / rms of the row
  int64_t K;
};

template <int ACT>
__device__ __forceinline__ float act1(const float* xr, const SplitAct& p, int64_t k) {
  if constexpr (ACT == kActRmsNorm) {
    return xr[k] * p.r * p.w[k];
  } else if constexpr (ACT == kActSiluMul) {
    const float g = xr[k], u = xr[p.K + k];
    const float c = fminf(fmaxf(g, -88.0f), 88.0f);
    return g * (1.0f / (1.0f + expf(-c))) * u;
  } else {
    return xr[k];
  }
}

template <int ACT>
__device__ __forceinline__ float4 act4(const float* xr, const SplitAct& p, int64_t k) {
  float4 v = *reinterpret_cast<const float4*>(xr + k);
  if constexpr (ACT == kActRmsNorm) {
    const float4 w = *reinterpret_cast<const float4*>(p.w + k);
    v = make_float4(v.x * p.r * w.x, v.y * p.r * w.y, v.z * p.r * w.z, v.w * p.r * w.w);
  } else if constexpr (ACT == kActSiluMul) {
    const float4 u = *reinterpret_cast<const float4*>(xr + p.K + k);
    auto sm = [](float g, float uu) {
      const float c = fminf(fmaxf(g, -88.0f), 88.0f);
      return g * (1.0f / (1.0f + expf(-c))) * uu;
    };
    v = make_float4(sm(v.x, u.x), sm(v.y, u.y), sm(v.z, u.z), sm(v.w, u.w));
  }
  return v;
}

// One CTA per (padded) activation row; rows are ldx floats apart. K % 4 == 0
// and 16-byte aligned rows (and weights): float4 loads, one 4-byte store per
// limb per 4 activations; otherwise element by element.
template <int ACT>
__global__ void __launch_bounds__(kSplitThreads) split_x_kernel(const float* __restrict__ X,
                                                                int64_t ldx,
                                                                const float* __restrict__ norm_w,
                                                                float eps,
                                                                int8_t* __restrict__ limbs,
                                                                float* __restrict__ sx, int64_t M,
                                                                int64_t Mpad, int64_t K) {
  const int64_t m = blockIdx.x;
  int8_t* l0 = limbs + m * K;
  int8_t* l1 = limbs + (Mpad + m) * K;
  int8_t* l2 = limbs + (2 * Mpad + m) * K;
  if (m >= M) {
    for (int64_t k = threadIdx.x; k < K; k += blockDim.x) { l0[k] = 0; l1[k] = 0; l2[k] = 0; }
    if (threadIdx.x == 0) sx[m] = 0.f;
    return;
  }
  const float* xr = X + m * ldx;
  __shared__ float red[kSplitThreads / 32];
  SplitAct p{norm_w, 1.0f, K};
  if constexpr (ACT == kActRmsNorm) {
    float ss = 0.f;
    for (int64_t i = threadIdx.x; i < K; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float t = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w];
    p.r = 1.0f / sqrtf(t / static_cast<float>(K) + eps);
    __syncthreads();   // red is reused below
  }
  bool vec = (K & 3) == 0 && (reinterpret_cast<uintptr_t>(xr) & 15u) == 0;
  if constexpr (ACT == kActRmsNorm) vec = vec && (reinterpret_cast<uintptr_t>(norm_w) & 15u) == 0;
  float mx = 0.f;
  if (vec) {
    for (int64_t k = threadIdx.x * 4; k < K; k += blockDim.x * 4) {
      const float4 v = act4<ACT>(xr, p, k);
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
  } else {
    for (int64_t k = threadIdx.x; k < K; k += blockDim.x) mx = fmaxf(mx, fabsf(act1<ACT>(xr, p, k)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) mx = fmaxf(mx, red[w]);
  const float s = mx > 0.f ? mx / kLimbRange : 1.0f;
  const float inv = 1.0f / s;
  if (vec) {
    for (int64_t k = threadIdx.x * 4; k < K; k += blockDim.x * 4) {
      const float4 v = act4<ACT>(xr, p, k);
      int a0, a1, a2, b0, b1, b2, c0, c1, c2, e0, e1, e2;
      limbs3(v.x, inv, a0, a1, a2);
      limbs3(v.y, inv, b0, b1, b2);
      limbs3(v.z, inv, c0, c1, c2);
      limbs3(v.w, inv, e0, e1, e2);
      *reinterpret_cast<uint32_t*>(l0 + k) = pack4(a0, b0, c0, e0);
      *reinterpret_cast<uint32_t*>(l1 + k) = pack4(a1, b1, c1, e1);
      *reinterpret_cast<uint32_t*>(l2 + k) = pack4(a2, b2, c2, e2);
    }
  } else {
    for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
      int d0, d1, d2;
      limbs3(act1<ACT>(xr, p, k), inv, d0, d1, d2);
      l0[k] = static_cast<int8_t>(d0);
      l1[k] = static_cast<int8_t>(d1);
      l2[k] = static_cast<int8_t>(d2);
    }
  }
  if (threadIdx.x == 0) sx[m] = s;
}

// Split-K finish: Y = scale_n * sx_m * (A2 * 2^16 + A1 * 2^8 + A0) (+ residual),
// from the int32 sums every split added (exactly, in any order) to acc.
__global__ void __launch_bounds__(256) splitk_finish_kernel(const int32_t* __restrict__ acc,
                                                            const float* __restrict__ scale,
                                                            const float* __restrict__ sx,
                                                            const float* __restrict__ residual,
                                                            float* __restrict__ Y, int64_t M,
                                                            int64_t N, int64_t Mpad) {
  const int64_t total = M * N;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = t / N, n = t - m * N;
    const double v = static_cast<double>(acc[(2 * Mpad + m) * N + n]) * 65536.0 +
                     static_cast<double>(acc[(Mpad + m) * N + n]) * 256.0 +
                     static_cast<double>(acc[m * N + n]);
    float o = static_cast<float>(v * static_cast<double>(sx[m])) * scale[n];
    if (residual) o += residual[t];
    Y[t] = o;
  }
}

// ---------------------------------------------------------------------------
// PTX wrappers (tcgen05, TMA)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrive on `bar` once all tcgen05 operations issued so far by this thread complete.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 16 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows of
// 128 bytes, 8-row core groups 1024 bytes apart (sm_100 descriptor version 1).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);          // start address
  d |= static_cast<uint64_t>(1u) << 16;                       // leading byte offset (unused)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;               // stride byte offset
  d |= static_cast<uint64_t>(1u) << 46;                       // descriptor version
  d |= static_cast<uint64_t>(2u) << 61;                       // SWIZZLE_128B
  return d;
}

// Instruction descriptor: D s32, A/B signed int8, both K-major, M = 128, N = mt.
__host__ __device__ constexpr uint32_t idesc_i8(int mt) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(mt >> 3) << 17) |
         (static_cast<uint32_t>(kRows >> 4) << 24);
}

__host__ __device__ constexpr uint32_t tmem_cols(int mt) {
  // power of two >= 32 holding kLimbs accumulators of mt columns
  return kLimbs * mt <= 32 ? 32 : kLimbs * mt <= 64 ? 64 : kLimbs * mt <= 128 ? 128
       : kLimbs * mt <= 256 ? 256 : 512;
}

template <int MT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmap_q,
                   const __grid_constant__ CUtensorMap tmap_x, const TcArgs a) {
  static_assert(MT % 16 == 0 && MT >= 16 && MT <= 128, "MMA N for M=128 must be 16..128 here");
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms (the host adds the slack)
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = a.nstages;
  constexpr int QB = kRows * kKBytes;       // weight tile bytes
  constexpr int XB = MT * kKBytes;          // one limb tile bytes
  constexpr int SB = QB + kLimbs * XB;
  // The three limb tiles lie back to back in the stage, so together they are
  // one K-major B operand of 3 * MT rows: one MMA of N = 3 * MT covers every
  // limb (N <= 256), two of N = 3 * MT / 2 at MT = 128. TMEM column j of the
  // accumulator is then limb j / MT, token j % MT, as the epilogue reads it.
  // (Three MMAs of N = MT per K step measured slower at small MT: the MMA
  // chain, not the copies, set the stage rate.)
  constexpr int kMmaPerK = kLimbs * MT <= 256 ? 1 : 2;
  constexpr int kMmaN = kLimbs * MT / kMmaPerK;
  static_assert(kMmaN % 16 == 0 && kMmaN <= 256, "MMA N for M = 128");
  uint8_t* tiles = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * SB);
  const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * kMaxStages;
  const uint32_t accum_bar = empty0 + 8 * kMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kMaxStages + 1);
  __shared__ int s_err;

  // grid (token tiles, weight tiles, K splits): the token tiles that share a
  // 128-row weight panel are adjacent in launch order, so they run at the
  // same time and the panel comes from DRAM once and from L2 for the rest
  const int64_t n0 = static_cast<int64_t>(blockIdx.y) * kRows;
  const int64_t m0 = static_cast<int64_t>(blockIdx.x) * MT;
  const int nk_all = static_cast<int>(cdiv(a.K, kKBytes));
  // this CTA's K blocks: [kb0, kb0 + nk)
  const int kb0 = static_cast<int>(static_cast<int64_t>(nk_all) * blockIdx.z / a.splits);
  const int nk = static_cast<int>(static_cast<int64_t>(nk_all) * (blockIdx.z + 1) / a.splits) - kb0;
  constexpr uint32_t kCols = tmem_cols(MT);

  if (tid == 0) {
    s_err = 0;
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    mbar_init(accum_bar, 1);
    fence_mbar_init();
    prefetch_tmap(&tmap_q);
    prefetch_tmap(&tmap_x);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint64_t pol_q = l2_evict_first_policy();
      const uint64_t pol_x = l2_evict_last_policy();
      int issued = 0;
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % S;
        if (kb >= S && !mbar_wait(empty0 + 8 * s, ((kb / S) - 1) & 1)) {
          report_error(ERR_WAIT_EMPTY, 0x300u);
          atomicExch(&s_err, 1);
          break;
        }
        const uint32_t st = smem_u32(tiles + s * SB);
        mbar_arrive_expect_tx(full0 + 8 * s, SB);
        const int kx = (kb0 + kb) * kKBytes;
        tma_load_2d(st, &tmap_q, full0 + 8 * s, kx, static_cast<int>(n0), pol_q);
#pragma unroll
        for (int l = 0; l < kLimbs; ++l)
          tma_load_2d(st + QB + l * XB, &tmap_x, full0 + 8 * s, kx,
                      static_cast<int>(l * a.Mpad + m0), pol_x);
        ++issued;
      }
      // never leave a copy in flight into shared memory we are about to release
      for (int kb = issued > S ? issued - S : 0; kb < issued; ++kb)
        if (!mbar_wait(full0 + 8 * (kb % S), (kb / S) & 1)) {
          report_error(ERR_DRAIN, 0x301u);
          break;
        }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(kMmaN);
      int done = 0;
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % S;
        if (!mbar_wait(full0 + 8 * s, (kb / S) & 1) || *(volatile int*)&s_err) {
          report_error(ERR_WAIT_FULL, 0x302u);
          atomicExch(&s_err, 1);
          break;
        }
        tc_fence_after();
        const uint32_t st = smem_u32(tiles + s * SB);
#pragma unroll
        for (int kk = 0; kk < kKBytes / kMmaK; ++kk) {
          const uint64_t ad = smem_desc_sw128(st + kk * kMmaK);
#pragma unroll
          for (int h = 0; h < kMmaPerK; ++h) {
            const uint64_t bd = smem_desc_sw128(st + QB + h * kMmaN * kKBytes + kk * kMmaK);
            mma_i8(tmem + h * kMmaN, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
        }
        tc_commit(empty0 + 8 * s);   // frees the stage once these MMAs have read it
        ++done;
      }
      tc_commit(accum_bar);          // accumulators complete (or all issued MMAs drained)
      (void)done;
      // TMEM is released below only after every issued MMA has finished.
      if (!mbar_wait(accum_bar, 0)) report_error(ERR_DRAIN, 0x304u);
    }
  } else if (warp >= kEpiWarp0) {
    // ---------------- epilogue ----------------
    const int ew = warp - kEpiWarp0;           // TMEM lanes 32*ew .. 32*ew+31
    bool ok = mbar_wait(accum_bar, 0);
    ok = __all_sync(0xffffffffu, ok && !*(volatile int*)&s_err);   // tcgen05.ld is warp-wide
    if (!ok && lane == 0) report_error(ERR_WAIT_FULL, 0x303u);
    tc_fence_after();
    if (ok) {
      const int64_t n = n0 + 32 * ew + lane;
      const uint32_t lane_addr = tmem + (static_cast<uint32_t>(32 * ew) << 16);
      const float sn = n < a.N ? __ldg(a.scale + n) : 0.f;
#pragma unroll 1
      for (int c = 0; c < MT; c += 16) {
        uint32_t v0[16], v1[16], v2[16];
        tmem_ld16(lane_addr + c, v0);
        tmem_ld16(lane_addr + MT + c, v1);
        tmem_ld16(lane_addr + 2 * MT + c, v2);
        tmem_wait_ld();
        if (a.acc) {
          // split-K: add this split's exact int32 sums; the finish kernel scales
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int64_t m = m0 + c + j;
            if (m < a.M && n < a.N) {
              atomicAdd(a.acc + m * a.N + n, static_cast<int32_t>(v0[j]));
              atomicAdd(a.acc + (a.Mpad + m) * a.N + n, static_cast<int32_t>(v1[j]));
              atomicAdd(a.acc + (2 * a.Mpad + m) * a.N + n, static_cast<int32_t>(v2[j]));
            }
          }
          continue;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int64_t m = m0 + c + j;
          if (m < a.M && n < a.N) {
            const double t = static_cast<double>(static_cast<int32_t>(v2[j])) * 65536.0 +
                             static_cast<double>(static_cast<int32_t>(v1[j])) * 256.0 +
                             static_cast<double>(static_cast<int32_t>(v0[j]));
            float o = static_cast<float>(t * static_cast<double>(__ldg(a.sx + m))) * sn;
            if (a.residual) o += a.residual[m * a.N + n];
            a.Y[m * a.N + n] = o;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
}

}  // namespace tc
}  // namespace qz
