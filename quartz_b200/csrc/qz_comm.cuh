// qz_comm.cuh -- one-shot all-reduce (sum) over the GPUs of one node through
// peer memory (NVLink / NVSwitch), for the small [H] partial sums of a
// tensor-parallel decode step.
//
// Every rank owns a communication buffer (cudaMalloc'd, zeroed once, mapped
// into the other ranks' processes with CUDA IPC):
//
//   words u64 [2 parities][P senders][n_max]   (float bits | tag << 32)
//   epoch u32 [kMaxBlocks]                     calls completed by CTA c
//
// Low-latency protocol: every 8-byte word carries its value and the tag
// epoch + 1 of the call that wrote it, and an aligned 8-byte store is seen
// whole, so a receiver needs no separate flag and no fence: it polls the
// words themselves. CTA c of a call handles the float slice
// [c n / nb, (c + 1) n / nb):
//   1. push: (value, tag) of its slice into slot [parity][rank] of EVERY
//      rank's buffer (plain stores through the peer mapping);
//   2. reduce: for each element, for sender j = 0..P-1 in order, poll slot
//      [parity][j] until the tag matches (bounded by kWaitLimitNs), add the
//      value; every rank gets bit-identical sums.
// Two parities: a rank can start call e + 1 (other parity) while a peer still
// reads call e; it cannot reach call e + 2 before having read every peer's
// call e + 1, which each writes only after finishing call e. No multicast
// objects, no switch reductions: plain peer loads and stores.
#pragma once

#include "qz_decode.cuh"
#include "qz_device.cuh"
#include "qz_peer.cuh"

namespace qz {
namespace comm {

constexpr int kThreads = 256;

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kThreads) allreduce_kernel(const float* in, float* out,
                                                             int64_t n, int64_t n_max,
                                                             Peers peers, int rank, int P) {
  const int c = blockIdx.x, nb = gridDim.x, tid = threadIdx.x;
  // peer pointers are indexed with constants only (loops unrolled over
  // kMaxRanks), so they stay in the parameter space
  float* mine_f = peers.base[0];
#pragma unroll
  for (int j = 1; j < kMaxRanks; ++j)
    if (j == rank) mine_f = peers.base[j];
  const unsigned long long* mine = reinterpret_cast<const unsigned long long*>(mine_f);
  unsigned* my_epoch = reinterpret_cast<unsigned*>(mine_f + epochs_offset(P, n_max)) + c;
  __shared__ unsigned s_e;
  if (tid == 0) s_e = *reinterpret_cast<volatile unsigned*>(my_epoch);
  __syncthreads();
  const unsigned e = s_e;
  const unsigned tag = e + 1u;
  const int par = static_cast<int>(e & 1u);
  const int64_t lo = n * c / nb, hi = n * (c + 1) / nb;
  const int64_t slot0 = (static_cast<int64_t>(par) * P) * n_max;   // slot [par][0]
  // 1. push
  for (int64_t i = lo + tid; i < hi; i += kThreads) {
    const unsigned long long w =
        (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(in[i]);
#pragma unroll
    for (int j = 0; j < kMaxRanks; ++j) {
      if (j >= P) break;
      unsigned long long* dst = reinterpret_cast<unsigned long long*>(peers.base[j]);
      st_relaxed_sys_u64(dst + slot0 + static_cast<int64_t>(rank) * n_max + i, w);
    }
  }
  // 2. poll and reduce in rank order: senders outer, this thread's elements
  //    (kPer per round) inner, so one sender's words are loaded together
  constexpr int kPer = 4;
  bool ok = true;
  for (int64_t i0 = lo + tid; i0 < hi && ok; i0 += kPer * kThreads) {
    float acc[kPer];
    for (int j = 0; j < P && ok; ++j) {
      const unsigned long long* src = mine + slot0 + static_cast<int64_t>(j) * n_max;
      unsigned long long x[kPer];
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int64_t i = i0 + static_cast<int64_t>(k) * kThreads;
        x[k] = i < hi ? ld_relaxed_sys_u64(src + i) : 0ull;
      }
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int64_t i = i0 + static_cast<int64_t>(k) * kThreads;
        if (i >= hi) continue;
        if (static_cast<unsigned>(x[k] >> 32) != tag) {
          const unsigned long long t0 = globaltimer();
          while (static_cast<unsigned>((x[k] = ld_relaxed_sys_u64(src + i)) >> 32) != tag) {
            if (globaltimer() - t0 > kWaitLimitNs) {
              report_error(ERR_PEER_WAIT, 0x400u + static_cast<unsigned>(j));
              ok = false;
              break;
            }
          }
          if (!ok) break;
        }
        const float f = __uint_as_float(static_cast<unsigned>(x[k]));
        acc[k] = j == 0 ? f : acc[k] + f;
      }
    }
    if (!ok) break;
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int64_t i = i0 + static_cast<int64_t>(k) * kThreads;
      if (i < hi) out[i] = acc[k];
    }
  }
  __syncthreads();
  if (tid == 0) *reinterpret_cast<volatile unsigned*>(my_epoch) = tag;
}

// The consumer of a fused producer's rows: h = the sum over ranks (rank
// order) of the rows pushed in this call, n <= kRegRows, then
// xn = RMSNorm(h) * w (quartz/ops.py:24-32). One CTA; waits for the pushes
// (bounded), then advances the fused channel's epoch.
constexpr int kSumThreads = 512;
constexpr int kSumPer = 8;
__global__ void __launch_bounds__(kSumThreads) rmsnorm_peer_sum_kernel(
    float* own, int P, int64_t n_max, float* __restrict__ h, const float* __restrict__ w,
    float* __restrict__ xn, int64_t n, float eps) {
  __shared__ float red[32];
  __shared__ unsigned s_e;
  __shared__ int s_ok;
  unsigned* ep = fused_epoch(own, P, n_max);
  if (threadIdx.x == 0) {
    s_e = *reinterpret_cast<volatile unsigned*>(ep);
    s_ok = 1;
  }
  __syncthreads();
  const unsigned tag = s_e + 1u;
  const int par = static_cast<int>(s_e & 1u);
  const unsigned long long* words =
      reinterpret_cast<const unsigned long long*>(own + fused_words_offset(P, n_max)) +
      static_cast<int64_t>(par) * P * n_max;
  // Senders outer, elements inner: the kSumPer words of one sender are loaded
  // together (one round trip per sender), and the sum runs in rank order.
  float v[kSumPer], wv[kSumPer];
#pragma unroll
  for (int k = 0; k < kSumPer; ++k) {
    const int64_t i = threadIdx.x + static_cast<int64_t>(k) * kSumThreads;
    v[k] = 0.f;
    wv[k] = i < n ? w[i] : 0.f;
  }
  bool ok = true;
  for (int j = 0; j < P && ok; ++j) {
    const unsigned long long* src = words + static_cast<int64_t>(j) * n_max;
    unsigned long long x[kSumPer];
#pragma unroll
    for (int k = 0; k < kSumPer; ++k) {
      const int64_t i = threadIdx.x + static_cast<int64_t>(k) * kSumThreads;
      x[k] = 0ull;
      if (i < n)
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(x[k]) : "l"(src + i) : "memory");
    }
#pragma unroll
    for (int k = 0; k < kSumPer; ++k) {
      const int64_t i = threadIdx.x + static_cast<int64_t>(k) * kSumThreads;
      if (i >= n) continue;
      if (static_cast<unsigned>(x[k] >> 32) != tag) {
        const unsigned long long t0 = globaltimer();
        do {
          asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(x[k]) : "l"(src + i) : "memory");
          if (globaltimer() - t0 > kWaitLimitNs) {
            report_error(ERR_PEER_WAIT, 0x410u + static_cast<unsigned>(j));
            ok = false;
            break;
          }
        } while (static_cast<unsigned>(x[k] >> 32) != tag);
        if (!ok) break;
      }
      const float f = __uint_as_float(static_cast<unsigned>(x[k]));
      v[k] = j == 0 ? f : v[k] + f;
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kSumPer; ++k) {
    const int64_t i = threadIdx.x + static_cast<int64_t>(k) * kSumThreads;
    if (i < n) {
      h[i] = v[k];
      ss = fmaf(v[k], v[k], ss);
    }
  }
  if (!ok) s_ok = 0;
  ss = dec::block_sum(ss, red);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(n) + eps);
#pragma unroll
  for (int k = 0; k < kSumPer; ++k) {
    const int64_t i = threadIdx.x + static_cast<int64_t>(k) * kSumThreads;
    if (i < n) xn[i] = v[k] * r * wv[k];
  }
  __syncthreads();
  if (threadIdx.x == 0 && s_ok) *reinterpret_cast<volatile unsigned*>(ep) = tag;
}

}  // namespace comm
}  // namespace qz
