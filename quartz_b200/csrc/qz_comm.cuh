// qz_comm.cuh -- one-shot all-reduce (sum) over the GPUs of one node through
// peer memory (NVLink / NVSwitch), for the small [H] partial sums of a
// tensor-parallel decode step.
//
// Every rank owns a communication buffer (cudaMalloc'd, zeroed once, mapped
// into the other ranks' processes with CUDA IPC):
//
//   data  fp32 [2 parities][P senders][n_max]
//   flags u32  [2 parities][P senders][kMaxBlocks]
//   epoch u32  [kMaxBlocks]        calls completed by CTA c of this rank
//
// CTA c of a call handles the float4 slice [c n4 / nb, (c + 1) n4 / nb):
//   1. push: its slice of the input into slot [parity][rank] of EVERY rank's
//      buffer (plain stores through the peer mapping);
//   2. publish: fence at system scope, then flag[parity][rank][c] = epoch + 1
//      in every rank's buffer (release store);
//   3. wait: until flag[parity][j][c] of its own buffer reached epoch + 1 for
//      every sender j (acquire loads, bounded by kWaitLimitNs);
//   4. reduce: out = sum over j = 0..P-1 of slot [parity][j] (fixed order, so
//      every rank gets bit-identical sums).
// Two parities: a rank can start call e + 1 (other parity) while a peer still
// reads call e; it cannot reach call e + 2 before every peer has pushed call
// e + 1, which each does only after finishing call e. No multicast objects,
// no switch reductions: plain peer loads and stores.
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

__host__ __device__ constexpr int64_t flags_offset(int P, int64_t n_max) {  // in floats
  return 2 * static_cast<int64_t>(P) * n_max;
}
__host__ __device__ constexpr int64_t buffer_bytes(int P, int64_t n_max) {
  return (flags_offset(P, n_max) + 2 * static_cast<int64_t>(P) * kMaxBlocks + kMaxBlocks) * 4;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kThreads) allreduce_kernel(const float* in, float* out,
                                                             int64_t n, int64_t n_max,
                                                             Peers peers, int rank, int P) {
  const int c = blockIdx.x, nb = gridDim.x, tid = threadIdx.x;
  // peer pointers are indexed with constants only (loops unrolled over
  // kMaxRanks), so they stay in the parameter space
  float* mine = peers.base[0];
#pragma unroll
  for (int j = 1; j < kMaxRanks; ++j)
    if (j == rank) mine = peers.base[j];
  unsigned* my_flags = reinterpret_cast<unsigned*>(mine + flags_offset(P, n_max));
  unsigned* my_epoch = my_flags + 2 * P * kMaxBlocks + c;
  __shared__ unsigned s_e, s_ok;
  if (tid == 0) {
    s_e = *reinterpret_cast<volatile unsigned*>(my_epoch);
    s_ok = 1u;
  }
  __syncthreads();
  const unsigned e = s_e;
  const int par = static_cast<int>(e & 1u);
  const int64_t n4 = n / 4;
  const int64_t lo = n4 * c / nb, hi = n4 * (c + 1) / nb;
  const float4* in4 = reinterpret_cast<const float4*>(in);
  // 1. push this slice to every rank
  for (int64_t i = lo + tid; i < hi; i += kThreads) {
    const float4 v = in4[i];
#pragma unroll
    for (int j = 0; j < kMaxRanks; ++j) {
      if (j >= P) break;
      float4* dst = reinterpret_cast<float4*>(peers.base[j] +
                                              (static_cast<int64_t>(par) * P + rank) * n_max);
      dst[i] = v;
    }
  }
  __syncthreads();
  // 2. publish
  if (tid == 0) {
    __threadfence_system();
#pragma unroll
    for (int j = 0; j < kMaxRanks; ++j) {
      if (j >= P) break;
      unsigned* f = reinterpret_cast<unsigned*>(peers.base[j] + flags_offset(P, n_max));
      st_release_sys(f + (par * P + rank) * kMaxBlocks + c, e + 1u);
    }
  }
  // 3. wait for every sender's slice of this call
  if (tid < P) {
    const unsigned* f = my_flags + (par * P + tid) * kMaxBlocks + c;
    if (static_cast<int>(ld_acquire_sys(f) - (e + 1u)) < 0) {
      const unsigned long long t0 = globaltimer();
      while (static_cast<int>(ld_acquire_sys(f) - (e + 1u)) < 0) {
        if (globaltimer() - t0 > kWaitLimitNs) {
          report_error(ERR_PEER_WAIT, 0x400u + static_cast<unsigned>(tid));
          s_ok = 0u;
          break;
        }
      }
    }
  }
  __syncthreads();
  // 4. reduce in rank order (identical on every rank); data written by peers
  //    is read through L2 (ld.global.cg), never a stale L1 line
  const float* slots = mine + static_cast<int64_t>(par) * P * n_max;
  float4* out4 = reinterpret_cast<float4*>(out);
  for (int64_t i = lo + tid; i < hi; i += kThreads) {
    float4 acc = __ldcg(reinterpret_cast<const float4*>(slots) + i);
    for (int j = 1; j < P; ++j) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(slots + j * n_max) + i);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    out4[i] = acc;
  }
  if (tid == 0 && s_ok) *reinterpret_cast<volatile unsigned*>(my_epoch) = e + 1u;
}

}  // namespace comm
}  // namespace qz
