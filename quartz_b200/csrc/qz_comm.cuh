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

#include "qz_device.cuh"

namespace qz {
namespace comm {

constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 32;
constexpr int kThreads = 256;
constexpr unsigned ERR_PEER_WAIT = 16u;

struct Peers {
  float* base[kMaxRanks];   // every rank's buffer, as mapped in this process
};

__host__ __device__ constexpr int64_t buffer_bytes(int P, int64_t n_max) {
  return 2 * static_cast<int64_t>(P) * n_max * 8 + kMaxBlocks * 4;
}

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
  unsigned* my_epoch = reinterpret_cast<unsigned*>(mine_f + 2 * 2 * static_cast<int64_t>(P) * n_max) + c;
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
  // 2. poll and reduce in rank order
  bool ok = true;
  for (int64_t i = lo + tid; i < hi; i += kThreads) {
    float acc = 0.f;
    for (int j = 0; j < P; ++j) {
      const unsigned long long* src = mine + slot0 + static_cast<int64_t>(j) * n_max + i;
      unsigned long long w = ld_relaxed_sys_u64(src);
      if (static_cast<unsigned>(w >> 32) != tag) {
        const unsigned long long t0 = globaltimer();
        while (static_cast<unsigned>((w = ld_relaxed_sys_u64(src)) >> 32) != tag) {
          if (globaltimer() - t0 > kWaitLimitNs) {
            report_error(ERR_PEER_WAIT, 0x400u + static_cast<unsigned>(j));
            ok = false;
            break;
          }
        }
        if (!ok) break;
      }
      const float v = __uint_as_float(static_cast<unsigned>(w));
      acc = j == 0 ? v : acc + v;
    }
    if (!ok) break;
    out[i] = acc;
  }
  __syncthreads();
  if (tid == 0) *reinterpret_cast<volatile unsigned*>(my_epoch) = tag;
}

}  // namespace comm
}  // namespace qz
