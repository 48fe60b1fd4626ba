// qz_peer.cuh -- peer-memory buffers shared by the all-reduce kernels and by
// the producer kernels (GEMV, fused MLP) that push their rows to the ranks of
// a tensor-parallel group: buffer layout, the push helper.
#pragma once

#include "qz_device.cuh"

namespace qz {
namespace comm {

constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 32;
constexpr unsigned ERR_PEER_WAIT = 16u;

struct Peers {
  float* base[kMaxRanks];   // every rank's buffer, as mapped in this process
};

// Buffer regions (offsets in floats from the buffer's base):
//   A  tagged words of qz_allreduce_sum            [2][P][n_max] u64
//   B  tagged words of the fused producers          [2][P][n_max] u64
//      (GEMV / MLP epilogues push, qz_rmsnorm_peer_sum polls)
//   epochs: A per CTA [kMaxBlocks] u32, then B's one u32 (+ padding)
__host__ __device__ constexpr int64_t region_floats(int P, int64_t n_max) {
  return 2 * 2 * static_cast<int64_t>(P) * n_max;
}
__host__ __device__ constexpr int64_t fused_words_offset(int P, int64_t n_max) {
  return region_floats(P, n_max);
}
__host__ __device__ constexpr int64_t epochs_offset(int P, int64_t n_max) {
  return 2 * region_floats(P, n_max);
}
__host__ __device__ constexpr int64_t buffer_bytes(int P, int64_t n_max) {
  return (epochs_offset(P, n_max) + kMaxBlocks + 4) * 4;
}

// Where a producer kernel sends its output rows instead of storing them:
// every rank's buffer (as mapped in this process), this rank, the rank count
// (0: disabled) and the buffers' n_max.
struct PeerOut {
  float* base[kMaxRanks];
  int rank, P;
  int64_t n_max;
};

__device__ __forceinline__ float* own_base(const PeerOut& po) {
  float* b = po.base[0];
#pragma unroll
  for (int j = 1; j < kMaxRanks; ++j)
    if (j == po.rank) b = po.base[j];
  return b;
}

// The fused channel's epoch: calls completed by this rank's consumer.
__device__ __forceinline__ unsigned* fused_epoch(float* own, int P, int64_t n_max) {
  return reinterpret_cast<unsigned*>(own + epochs_offset(P, n_max)) + kMaxBlocks;
}

// Row `row` of this call's output (tagged `tag` in parity `par`) to every rank.
__device__ __forceinline__ void peer_push(const PeerOut& po, unsigned tag, int par, int64_t row,
                                          float v) {
  const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
  const int64_t off = (static_cast<int64_t>(par) * po.P + po.rank) * po.n_max + row;
#pragma unroll
  for (int j = 0; j < kMaxRanks; ++j) {
    if (j >= po.P) break;
    unsigned long long* dst = reinterpret_cast<unsigned long long*>(
        po.base[j] + fused_words_offset(po.P, po.n_max));
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst + off), "l"(w) : "memory");
  }
}

}  // namespace comm
}  // namespace qz
