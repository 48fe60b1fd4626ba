// qz_stream.cuh -- HBM-streaming int8 weight-only kernels for M = 1 (decode).
//
//   gemv_kernel       y[n] = sum_g scale[n,g] * sum_{k in g} x[k] * q[n,k]  (+ residual[n])
//                     (quartz/kernels/int8.py:24-38 and its serial twin 48-63)
//   fused_mlp_kernel  out = down(silu(gate.x) * (up.x))  (+ residual)
//                     (quartz/kernels/fused.py:27-65)
//
// Structure (chosen by measurement on B200):
//   * every warp owns a balanced, contiguous range of weight rows and walks it
//     in row groups of R rows; a group is cut along K into items of at most
//     1 KB per row;
//   * each lane streams its own 16-byte chunks of an item into a private slot
//     of the warp's shared-memory ring (cp.async.cg, kDepth items deep: bytes
//     in flight cost no registers) and later reads back exactly those bytes,
//     so no intra-warp synchronisation is needed;
//   * activations are staged once per CTA in shared memory in a
//     bank-conflict-free [word][chunk] layout;
//   * int8 -> fp32 widening in registers (qz_device.cuh), packed f32x2 FMAs,
//     one transposed butterfly per group; scale, residual and SiLU gate are
//     fused into the epilogue. No fp32 weight array is ever formed;
//   * weights do not depend on the previous kernel in the stream, so a launch
//     issues its first weight copies before it waits on the programmatic
//     dependency (griddepcontrol.wait) and touches activations or outputs.
#pragma once

#include "qz_device.cuh"
#include "qz_peer.cuh"

namespace qz {

constexpr int kWarps = 8;                  // warps per CTA
constexpr int kThreads = kWarps * 32;
constexpr int kSegBytes = 1024;            // K bytes per row per item (32 lanes x 2 chunks)
constexpr int kDepth = 2;                  // items in flight per warp ring

// How K relates to the 1 KB item width, fixed at compile time so the hot loop
// carries no bounds checks in the common cases.
enum KMode : int {
  K1K = 0,    // K == 1024: one item per row group, activations in registers
  KFULL = 1,  // K % 1024 == 0: every item is a full 1 KB per row
  KANY = 2,   // K % 16 == 0: the last item of a row may be partial
};

__host__ __device__ constexpr int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ constexpr int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }

// Shared memory: [x: kmax floats, 128-aligned][rings: kWarps * kDepth * R * kSegBytes]
__host__ __device__ inline int stream_x_bytes(int64_t kmax) {
  return static_cast<int>(((kmax * 4 + 127) / 128) * 128);
}
__host__ __device__ constexpr int ring_bytes(int R) { return kWarps * kDepth * R * kSegBytes; }
__host__ __device__ inline int stream_smem_bytes(int R, int64_t kmax) {
  return stream_x_bytes(kmax) + ring_bytes(R);
}

struct GemvArgs {
  const int8_t* q;        // [N, K]
  const float* scale;     // [N, ng]
  const float* x;         // [K]
  float* y;               // [N]
  const float* residual;  // [N] or null
  int64_t N, K, ng;
  comm::PeerOut po;       // po.P > 0: push the rows to the ranks instead of writing y
  const float* norm_w;    // non-null: the GEMV reads RMSNorm(x) * norm_w instead of x
  float eps;
};

struct MlpArgs {
  const int8_t* gu_q;     // [2I, H]: gate rows 0..I-1, up rows I..2I-1
  const float* gu_s;      // [2I, ng]
  const float* x;         // [H]
  const int8_t* down_q;   // [H, I]
  const float* down_s;    // [H, ngd]
  float* abuf;            // [I] intermediate (global; read back after the grid barrier)
  float* out;             // [H]
  const float* residual;  // [H] or null
  unsigned int* sync_ws;  // grid barrier words {count, generation}, zero at first use
  int64_t H, I, ng, ngd;
  comm::PeerOut po;       // po.P > 0: push the rows to the ranks instead of writing out
  const float* norm_w;    // non-null: phase 1 reads RMSNorm(x) * norm_w instead of x
  float eps;
};

// ---------------------------------------------------------------------------
// cp.async ring + programmatic dependent launch
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Stage K activations into shared memory as float4 blocks ordered [word j4][chunk c].
// COHERENT: the source was written earlier in this kernel by other CTAs (the
// fused MLP's intermediate, read after the grid barrier): read it from L2
// (ld.global.cg), never through the non-coherent path.
// Four consecutive activations 4q .. 4q + 3 land in four consecutive words,
// so a 16-byte aligned x is staged with float4 loads (four in flight per
// thread) and one float4 store each.
template <bool COHERENT = false>
__device__ __forceinline__ void stage_x(float* xs, const float* x, int64_t K, int tid, int nthr) {
  const int64_t nch = K / 16;
  if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
    const int64_t nq = K / 4;      // K % 16 == 0 on the streaming path
    const float4* x4 = reinterpret_cast<const float4*>(x);
    int64_t q = tid;
    for (; q + 3 * nthr < nq; q += 4 * nthr) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = COHERENT ? __ldcg(x4 + q + u * nthr) : x4[q + u * nthr];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t qq = q + u * nthr;
        *reinterpret_cast<float4*>(xs + (((qq & 3) * nch) + (qq >> 2)) * 4) = v[u];
      }
    }
    for (; q < nq; q += nthr) {
      const float4 v = COHERENT ? __ldcg(x4 + q) : x4[q];
      *reinterpret_cast<float4*>(xs + (((q & 3) * nch) + (q >> 2)) * 4) = v;
    }
    return;
  }
  for (int64_t i = tid; i < K; i += nthr) {
    const int64_t c = i >> 4, j = i & 15;
    xs[((j >> 2) * nch + c) * 4 + (j & 3)] = COHERENT ? __ldcg(x + i) : x[i];
  }
}

// Activations of global chunk gc as 8 fp32 pairs.
__device__ __forceinline__ void load_x16(const uint8_t* xs, int64_t nch, int64_t gc,
                                         f2_t (&xv)[8]) {
#pragma unroll
  for (int j4 = 0; j4 < 4; ++j4) {
    const ulonglong2 p = *reinterpret_cast<const ulonglong2*>(xs + (j4 * nch + gc) * 16);
    xv[2 * j4] = p.x;
    xv[2 * j4 + 1] = p.y;
  }
}

// ---------------------------------------------------------------------------
// A warp's walk over one weight matrix: row groups [0, ngrp) of R rows, each
// cut into nseg K-segments; item (g, seg) is number g * nseg + seg of the walk.
// Items occupy consecutive ring positions starting at pos0, i.e. ring slot
// (pos0 + item) % kDepth, so two walks can share one ring back to back.
// Cursors advance item by item without divisions.
// ---------------------------------------------------------------------------
template <int R, int D = kDepth>
struct Walk {
  const int8_t* q;
  int64_t K;        // row length in bytes
  int64_t ngrp;
  int nseg;
  int64_t pos0;     // ring position of item 0
  __device__ int64_t items() const { return ngrp * nseg; }
};

template <int D>
struct Cursor {
  int64_t g;        // row group
  int seg;          // K segment
  int slot;         // ring slot
  __device__ void next(int nseg) {
    if (++seg == nseg) { seg = 0; ++g; }
    slot = slot + 1 == D ? 0 : slot + 1;
  }
};

template <int R, int D>
__device__ __forceinline__ Cursor<D> cursor_at(const Walk<R, D>& w, int64_t it) {
  Cursor<D> c;
  c.g = it / w.nseg;
  c.seg = static_cast<int>(it - c.g * w.nseg);
  c.slot = static_cast<int>((w.pos0 + it) % D);
  return c;
}

// Issue the copies of the item at cursor c (if it exists), then commit one
// cp.async group. rowfn(g, r) -> global row index, or -1 when absent.
template <int R, int KM, int D, class RowFn>
__device__ __forceinline__ void issue_item(const Walk<R, D>& w, uint32_t ring, const Cursor<D>& c,
                                           int lane, RowFn rowfn) {
  if (c.g < w.ngrp) {
    const int64_t k0 = KM == K1K ? 0 : static_cast<int64_t>(c.seg) * kSegBytes;
    const int64_t slen = KM == KANY ? min64(kSegBytes, w.K - k0) : kSegBytes;
    const uint32_t slot = ring + static_cast<uint32_t>(c.slot * R * kSegBytes);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t row = rowfn(c.g, r);
      if (row >= 0) {
        const int8_t* src = w.q + row * w.K + k0;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int ch = lane + 32 * j;
          if (KM != KANY || ch * 16 < slen)
            cp_async16(slot + r * kSegBytes + ch * 16, src + ch * 16);
        }
      }
    }
  }
  cp_async_commit();
}

// Accumulate the (landed) item at cursor c into the per-row accumulators.
// PER_ROW: one scale per row, applied by the caller; acc holds fp32 pairs.
// Otherwise each 16-element chunk's dot is weighted by its group's scale
// scale_of(g, r, group) (G % 16 == 0, so a chunk never straddles groups).
// K1K: xr holds this lane's 2 chunks of activations (loaded once per walk).
template <int R, bool PER_ROW, int KM, int D, class ScaleFn>
__device__ __forceinline__ void accumulate_item(const Walk<R, D>& w, const uint8_t* ring,
                                                const uint8_t* xs, const f2_t (&xr)[2][8],
                                                const Cursor<D>& c, int lane, int64_t G,
                                                f2_t (&acc)[R], float (&accs)[R],
                                                ScaleFn scale_of) {
  const int64_t k0 = KM == K1K ? 0 : static_cast<int64_t>(c.seg) * kSegBytes;
  const int64_t slen = KM == KANY ? min64(kSegBytes, w.K - k0) : kSegBytes;
  const uint8_t* slot = ring + c.slot * R * kSegBytes;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int ch = lane + 32 * j;
    if (KM != KANY || ch * 16 < slen) {
      const int64_t gc = k0 / 16 + ch;
      f2_t xl[8];
      if constexpr (KM != K1K) load_x16(xs, w.K / 16, gc, xl);
      const f2_t* xv = KM == K1K ? xr[j] : xl;
      if (PER_ROW) {
        uint4 qv[R];
#pragma unroll
        for (int r = 0; r < R; ++r)
          qv[r] = *reinterpret_cast<const uint4*>(slot + r * kSegBytes + ch * 16);
#pragma unroll
        for (int r = 0; r < R; ++r) dot16_acc(qv[r], xv, acc[r]);
      } else {
        const int64_t grp = (gc * 16) / G;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const uint4 qv = *reinterpret_cast<const uint4*>(slot + r * kSegBytes + ch * 16);
          f2_t d = 0ull;
          dot16_acc(qv, xv, d);
          const float2 p = f2_unpack(d);
          accs[r] = fmaf(p.x + p.y, scale_of(c.g, r, grp), accs[r]);
        }
      }
    }
  }
}

// Sum the R per-lane row values over the warp. R > 1: afterwards row
// r = (lane >> 2) & 7 is complete on the lanes with that index. R == 1: every
// lane holds the sum.
template <int R, bool PER_ROW>
__device__ __forceinline__ float reduce_rows(const f2_t (&acc)[R], const float (&accs)[R],
                                             int lane) {
  float v[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) v[r] = 0.f;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (PER_ROW) {
      const float2 p = f2_unpack(acc[r]);
      v[r] = p.x + p.y;
    } else {
      v[r] = accs[r];
    }
  }
  if (R == 1) {
    float s = v[0];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    return s;
  }
  return warp_reduce8(v, lane);
}
// The same for R float partial sums, one per row.
template <int R>
__device__ __forceinline__ float reduce_row_sums(const float (&accs)[R], int lane) {
  float v[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) v[r] = r < R ? accs[r] : 0.f;
  if (R == 1) {
    float s = v[0];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    return s;
  }
  return warp_reduce8(v, lane);
}


// The row (within its group) that this lane holds after reduce_rows, or -1.
template <int R>
__device__ __forceinline__ int reduced_row(int lane) {
  if (R == 1) return lane == 0 ? 0 : -1;
  const int r = (lane >> 2) & 7;
  return ((lane & 3) == 0 && r < R) ? r : -1;
}

// This lane's two chunks of activations (K == 1024) as fp32 pairs, straight
// from global memory (16-byte aligned x) or, unaligned, element by element.
__device__ __forceinline__ void load_x_regs(const float* x, int lane, f2_t (&xr)[2][8]) {
  const bool al = (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const float* xp = x + (lane + 32 * j) * 16;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      float4 v;
      if (al) {
        v = *reinterpret_cast<const float4*>(xp + 4 * t);
      } else {
        v = make_float4(xp[4 * t], xp[4 * t + 1], xp[4 * t + 2], xp[4 * t + 3]);
      }
      xr[j][2 * t] = f2_pack(__float_as_uint(v.x), __float_as_uint(v.y));
      xr[j][2 * t + 1] = f2_pack(__float_as_uint(v.z), __float_as_uint(v.w));
    }
  }
}

// The norm weights are constants: a kernel prefetches the lines its threads
// will read into L1 before it waits for the previous grid, so that applying
// the norm costs no extra memory round trip after the sum of squares.
__device__ __forceinline__ void prefetch_l1(const void* p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// RMSNorm folded into the activation load (quartz/ops.py:24-32):
// x <- x * (1 / sqrt(mean(x^2) + eps)) * w, on x staged in shared memory by
// stage_x (K floats; any permutation of the staged layout sums the same
// squares). Every thread of the CTA calls it after the staging barrier; it
// ends with a barrier.
__device__ __forceinline__ void norm_staged_x(float* xs, const float* __restrict__ w, int64_t K,
                                              float eps, int tid, int nthr) {
  __shared__ float red[32];
  float ss = 0.f;
  const float4* xs4 = reinterpret_cast<const float4*>(xs);   // K % 16 == 0
  for (int64_t q = tid; q < K / 4; q += nthr) {
    const float4 v = xs4[q];
    ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  ss = 0.f;
  for (int i = 0; i < (nthr >> 5); ++i) ss += red[i];
  const float r = 1.0f / sqrtf(ss / static_cast<float>(K) + eps);
  const int64_t nch = K / 16;
  if ((reinterpret_cast<uintptr_t>(w) & 15u) == 0) {
    // activations 4q .. 4q + 3 sit in four consecutive words (see stage_x)
    for (int64_t q = tid; q < K / 4; q += nthr) {
      float4& v = *reinterpret_cast<float4*>(xs + (((q & 3) * nch) + (q >> 2)) * 4);
      const float4 wv = reinterpret_cast<const float4*>(w)[q];
      v = make_float4(v.x * r * wv.x, v.y * r * wv.y, v.z * r * wv.z, v.w * r * wv.w);
    }
  } else {
    for (int64_t i = tid; i < K; i += nthr) {
      const int64_t c = i >> 4, j = i & 15;
      float& v = xs[((j >> 2) * nch + c) * 4 + (j & 3)];
      v = v * r * w[i];
    }
  }
  __syncthreads();
}

// Issue items [from, to) of a walk, one cp.async group each.
template <int R, int KM, int D, class RowFn>
__device__ __forceinline__ void issue_items(const Walk<R, D>& w, uint32_t ring, int64_t from,
                                            int64_t to, int lane, RowFn rowfn) {
  Cursor<D> c = cursor_at(w, from);
  for (int64_t it = from; it < to; ++it, c.next(w.nseg)) issue_item<R, KM>(w, ring, c, lane, rowfn);
}

// One walk through a ring of D slots. Before the call, the positions of items
// 0 .. D-2 have been issued (committed as one group each, empty groups for
// missing items), and item D-1 as well when `ahead_issued` (the whole ring;
// the first step then issues nothing). Each step issues the item D-1 ahead (past the end:
// `beyond()` issues the next walk's item or an empty group), waits for the
// current item and accumulates it; at a group's last segment `done(g, sum)`
// runs on every lane (sum is meaningful on the lanes reduced_row<R>() names).
// K1K walks take their activations from `xg` (global) into registers; the
// others read the CTA's staged copy `xs` item by item.
template <int R, bool PER_ROW, int KM, int D, class RowFn, class ScaleFn, class BeyondFn,
          class DoneFn>
__device__ __forceinline__ void walk(const Walk<R, D>& w, uint32_t ring_s, const uint8_t* ring,
                                     const uint8_t* xs, const float* xg, int lane, int64_t G,
                                     RowFn rowfn, ScaleFn scale_of, BeyondFn beyond,
                                     DoneFn done, bool ahead_issued = false) {
  f2_t xr[2][8];
  if constexpr (KM == K1K) load_x_regs(xg, lane, xr);
  f2_t acc[R];
  float accs[R];
  Cursor<D> cur = cursor_at(w, 0);
  Cursor<D> ahead = cursor_at(w, D - 1);
  for (; cur.g < w.ngrp; cur.next(w.nseg), ahead.next(w.nseg)) {
    if (ahead_issued)
      ahead_issued = false;     // the caller already issued item D-1
    else if (ahead.g < w.ngrp)
      issue_item<R, KM>(w, ring_s, ahead, lane, rowfn);
    else
      beyond();
    cp_async_wait<D - 1>();
    if (cur.seg == 0) {
#pragma unroll
      for (int r = 0; r < R; ++r) { acc[r] = 0ull; accs[r] = 0.f; }
    }
    accumulate_item<R, PER_ROW, KM>(w, ring, xs, xr, cur, lane, G, acc, accs, scale_of);
    if (KM == K1K || cur.seg == w.nseg - 1) done(cur.g, reduce_rows<R, PER_ROW>(acc, accs, lane));
  }
}

// Balanced split of [0, n) into `parts`: the range [b, e) of part p.
__device__ __forceinline__ void split_range(int64_t n, int64_t parts, int64_t p, int64_t& b,
                                            int64_t& e) {
  b = n * p / parts;
  e = n * (p + 1) / parts;
}

// ---------------------------------------------------------------------------
// GEMV
// ---------------------------------------------------------------------------
// D: items in a warp's ring. Four-row groups use kDepth; one-row groups (few
// rows per warp) a deeper ring of 1 KB items, so that a warp keeps as many
// bytes in flight as a four-row walk does.
template <int R, bool PER_ROW, int KM, int MINB, int D = kDepth>
__global__ void __launch_bounds__(kThreads, MINB) gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* xs = reinterpret_cast<float*>(smem);
  const uint8_t* ring =
      smem + (KM == K1K ? 0 : stream_x_bytes(a.K)) + warp * D * R * kSegBytes;
  const uint32_t ring_s = smem_u32(ring);

  const int64_t nw = static_cast<int64_t>(gridDim.x) * kWarps;
  const int64_t wg = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
  int64_t r0, r1;
  split_range(a.N, nw, wg, r0, r1);
  const Walk<R, D> w{a.q, a.K, cdiv(r1 - r0, R), static_cast<int>(cdiv(a.K, kSegBytes)), 0};
  auto rowfn = [&](int64_t g, int r) -> int64_t {
    const int64_t row = r0 + g * R + r;
    return row < r1 ? row : -1;
  };
  // The weights do not depend on the previous grid: fill the whole ring
  // before waiting for it.
  issue_items<R, KM>(w, ring_s, 0, D, lane, rowfn);
  if constexpr (KM != K1K) {
    if (a.norm_w)
      for (int64_t i = tid * 32; i < a.K; i += kThreads * 32) prefetch_l1(a.norm_w + i);
  }
  pdl_trigger();
  pdl_wait();
  if constexpr (KM != K1K) {
    stage_x(xs, a.x, a.K, tid, kThreads);
    __syncthreads();
    if (a.norm_w) norm_staged_x(xs, a.norm_w, a.K, a.eps, tid, kThreads);
  }

  const int64_t G = a.K / a.ng;
  auto scale_of = [&](int64_t g, int r, int64_t grp) -> float {
    const int64_t row = r0 + g * R + r;
    return row < r1 ? __ldg(a.scale + row * a.ng + grp) : 0.f;
  };
  // a fused all-reduce's producer pushes each row, tagged with the call of
  // the channel's epoch (stream-ordered: read after griddepcontrol.wait)
  unsigned ptag = 0u;
  if (a.po.P > 0)
    ptag = *reinterpret_cast<volatile unsigned*>(
        comm::fused_epoch(comm::own_base(a.po), a.po.P, a.po.n_max)) + 1u;
  auto done = [&](int64_t g, float s) {
    const int r = reduced_row<R>(lane);
    const int64_t row = r0 + g * R + r;
    if (r >= 0 && row < r1) {
      float o = PER_ROW ? s * __ldg(a.scale + row) : s;
      if (a.residual) o += a.residual[row];
      if (a.po.P > 0)
        comm::peer_push(a.po, ptag, static_cast<int>((ptag - 1u) & 1u), row, o);
      else
        a.y[row] = o;
    }
  };
  auto beyond = [&]() { cp_async_commit(); };
  walk<R, PER_ROW, KM>(w, ring_s, ring, reinterpret_cast<const uint8_t*>(xs), a.x, lane, G, rowfn,
                       scale_of, beyond, done, true);
  cp_async_wait<0>();
}

// ---------------------------------------------------------------------------
// int4 GEMV (M = 1): rows of K / 2 bytes streamed through a per-warp
// cp.async ring like the int8 kernel's, activations staged once per CTA in the
// conflict-free layout of stage_x, pre-scaled for the subnormal widening of
// dot8_w4_acc. K % 32 == 0, so a lane's 16-byte chunk (32 weights) never
// straddles a scale group.
// ---------------------------------------------------------------------------
// Stage x * 2^(85 - p(j mod 8)) in the layout of stage_x, and the sum of
// each 32-weight chunk's activations into csum[K / 32] (one thread per chunk,
// in index order, so every CTA computes the same sums). Ends with a barrier.
__device__ __forceinline__ void stage_x_w4(float* xs, float* csum, const float* x, int64_t K,
                                           int tid, int nthr) {
  const int64_t nch = K / 16;
  for (int64_t i = tid; i < K; i += nthr) {
    const int64_t c = i >> 4, j = i & 15;
    const float s = __int_as_float((127 + 85 - w4_pos(static_cast<int>(i & 7))) << 23);
    xs[((j >> 2) * nch + c) * 4 + (j & 3)] = x[i] * s;
  }
  for (int64_t c = tid; c < K / 32; c += nthr) {
    float t = 0.f;
#pragma unroll 8
    for (int e = 0; e < 32; ++e) t += x[c * 32 + e];
    csum[c] = t;
  }
  __syncthreads();
}

constexpr float kW4Unscale = 18446744073709551616.0f;   // 2^64

// Rows of K / 2 bytes travel in segments of kW4Seg = 512 bytes (1024 weights),
// R rows per item, so an item is 4 KB at R = 8 like the int8 kernel's 4 x 1 KB
// and every lane copies and reads one 16-byte chunk of each row.
constexpr int kW4Seg = 512;

// Shared memory before the ring: the staged activations, then the chunk sums.
__host__ __device__ inline int w4_x_bytes(int64_t K) {
  return stream_x_bytes(K) + static_cast<int>(((K / 32) * 4 + 127) / 128 * 128);
}

template <int R, int KM, int D, class RowFn>
__device__ __forceinline__ void issue_item_w4(const Walk<R, D>& w, uint32_t ring,
                                              const Cursor<D>& c, int lane, RowFn rowfn) {
  if (c.g < w.ngrp) {
    const int64_t k0 = static_cast<int64_t>(c.seg) * kW4Seg;
    const int64_t slen = KM == KANY ? min64(kW4Seg, w.K - k0) : kW4Seg;
    const uint32_t slot = ring + static_cast<uint32_t>(c.slot * R * kW4Seg);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t row = rowfn(c.g, r);
      if (row >= 0 && (KM != KANY || lane * 16 < slen))
        cp_async16(slot + r * kW4Seg + lane * 16, w.q + row * w.K + k0 + lane * 16);
    }
  }
  cp_async_commit();
}

template <int R, bool PER_ROW, int KM, int D, class ScaleFn>
__device__ __forceinline__ void accumulate_item_w4(const Walk<R, D>& w, const uint8_t* ring,
                                                   const uint8_t* xs, const float* csum,
                                                   int64_t K, const Cursor<D>& c, int lane,
                                                   int64_t G, float (&accs)[R],
                                                   ScaleFn scale_of) {
  const int64_t k0 = static_cast<int64_t>(c.seg) * kW4Seg;
  const int64_t slen = KM == KANY ? min64(kW4Seg, w.K - k0) : kW4Seg;
  if (KM == KANY && lane * 16 >= slen) return;
  const uint8_t* slot = ring + c.slot * R * kW4Seg + lane * 16;
  const int64_t nch = K / 16;
  const int64_t gb = k0 / 16 + lane;            // 16-byte chunk = weights [32 gb, 32 gb + 32)
  // both halves of the chunk's activations, then one row's chunk dot at a time
  f2_t xa[8], xb[8];
  load_x16(xs, nch, 2 * gb, xa);
  load_x16(xs, nch, 2 * gb + 1, xb);
  const int64_t grp = PER_ROW ? 0 : (gb * 32) / G;
  const float off = PER_ROW ? 0.f : 8.f * csum[gb];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const uint4 qv = *reinterpret_cast<const uint4*>(slot + r * kW4Seg);
    f2_t d = 0ull;
    dot8_w4_acc(qv.x, xa[0], xa[1], xa[2], xa[3], d);
    dot8_w4_acc(qv.y, xa[4], xa[5], xa[6], xa[7], d);
    dot8_w4_acc(qv.z, xb[0], xb[1], xb[2], xb[3], d);
    dot8_w4_acc(qv.w, xb[4], xb[5], xb[6], xb[7], d);
    const float2 p = f2_unpack(d);
    if (PER_ROW)
      accs[r] += p.x + p.y;                     // scaled and corrected once per row
    else
      accs[r] = fmaf(fmaf(p.x + p.y, kW4Unscale, -off), scale_of(c.g, r, grp), accs[r]);
  }
}

// y[n] = sum_g scale[n, g] sum_j q4[n, j] x[j] for q4 [N, K / 2] packed
// bytes (a.q), K weights per row (a.K). KM is the mode of the row length in
// bytes: KFULL when K / 2 is a multiple of kW4Seg, else KANY.
template <int R, bool PER_ROW, int KM, int MINB>
__global__ void __launch_bounds__(kThreads, MINB) gemv_w4_kernel(const GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* xs = reinterpret_cast<float*>(smem);
  float* csum = reinterpret_cast<float*>(smem + stream_x_bytes(a.K));
  const uint8_t* ring = smem + w4_x_bytes(a.K) + warp * kDepth * R * kW4Seg;
  const uint32_t ring_s = smem_u32(ring);
  __shared__ float s_off;                       // 8 * sum(x), the per-row correction

  const int64_t nw = static_cast<int64_t>(gridDim.x) * kWarps;
  const int64_t wg = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
  int64_t r0, r1;
  split_range(a.N, nw, wg, r0, r1);
  const int64_t kb = a.K / 2;                   // bytes per row
  const Walk<R> w{a.q, kb, cdiv(r1 - r0, R), static_cast<int>(cdiv(kb, kW4Seg)), 0};
  auto rowfn = [&](int64_t g, int r) -> int64_t {
    const int64_t row = r0 + g * R + r;
    return row < r1 ? row : -1;
  };
  issue_item_w4<R, KM>(w, ring_s, cursor_at(w, 0), lane, rowfn);
  issue_item_w4<R, KM>(w, ring_s, cursor_at(w, kDepth - 1), lane, rowfn);
  pdl_trigger();
  pdl_wait();
  stage_x_w4(xs, csum, a.x, a.K, tid, kThreads);
  if (PER_ROW && warp == 0) {
    float t = 0.f;
    for (int64_t c = lane; c < a.K / 32; c += 32) t += csum[c];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) s_off = 8.f * t;
  }
  __syncthreads();

  const int64_t G = a.K / a.ng;
  auto scale_of = [&](int64_t g, int r, int64_t grp) -> float {
    const int64_t row = r0 + g * R + r;
    return row < r1 ? __ldg(a.scale + row * a.ng + grp) : 0.f;
  };
  float accs[R];
  Cursor<kDepth> cur = cursor_at(w, 0);
  Cursor<kDepth> ahead = cursor_at(w, kDepth - 1);
  bool first = true;
  for (; cur.g < w.ngrp; cur.next(w.nseg), ahead.next(w.nseg)) {
    if (first)
      first = false;                            // item D-1 went out before the wait
    else if (ahead.g < w.ngrp)
      issue_item_w4<R, KM>(w, ring_s, ahead, lane, rowfn);
    else
      cp_async_commit();
    cp_async_wait<kDepth - 1>();
    if (cur.seg == 0) {
#pragma unroll
      for (int r = 0; r < R; ++r) accs[r] = 0.f;
    }
    accumulate_item_w4<R, PER_ROW, KM>(w, ring, reinterpret_cast<const uint8_t*>(xs), csum, a.K,
                                       cur, lane, G, accs, scale_of);
    if (cur.seg == w.nseg - 1) {
      const float sum = reduce_row_sums<R>(accs, lane);
      const int r = reduced_row<R>(lane);
      const int64_t row = r0 + cur.g * R + r;
      if (r >= 0 && row < r1) {
        float o = PER_ROW ? fmaf(sum, kW4Unscale, -s_off) * __ldg(a.scale + row) : sum;
        if (a.residual) o += a.residual[row];
        a.y[row] = o;
      }
    }
  }
  cp_async_wait<0>();
}

// ---------------------------------------------------------------------------
// Fused MLP (M = 1). Phase 1 walks "unit groups" of R/2 intermediate units,
// stored as R/2 gate rows followed by the matching R/2 up rows; its epilogue
// writes abuf[n] = silu(gate_n . x) * (up_n . x). A grid-wide barrier (bounded
// spin on a generation counter; the launch is cooperative so all CTAs are
// resident) separates it from phase 2, the down GEMV over abuf with the
// residual fused. Phase 2's first weight copies go out before the barrier.
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool grid_barrier(unsigned int* ws, int tid, unsigned int site) {
  __shared__ unsigned int s_fail;
  __syncthreads();
  if (tid == 0) {
    s_fail = 0u;
    __threadfence();
    const unsigned int gen = ld_acquire_gpu(ws + 1);
    const unsigned int arrived = atomicAdd(ws, 1u);
    if (arrived == gridDim.x - 1) {
      atomicExch(ws, 0u);
      __threadfence();
      atomicAdd(ws + 1, 1u);
    } else {
      const unsigned long long t0 = globaltimer();
      while (ld_acquire_gpu(ws + 1) == gen) {
        if (globaltimer() - t0 > kWaitLimitNs) {
          report_error(ERR_GRID_BARRIER, site);
          s_fail = 1u;
          break;
        }
        __nanosleep(32);
      }
    }
  }
  __syncthreads();
  return s_fail == 0u;
}

template <int R, bool PER_ROW, int KM1, int KM2, int MINB>
__global__ void __launch_bounds__(kThreads, MINB) fused_mlp_kernel(const MlpArgs a) {
  static_assert(R % 2 == 0, "a unit group holds R/2 gate rows and R/2 up rows");
  constexpr int U = R / 2;
  // Phase 2 walks one down row per group through the same per-warp ring,
  // re-cut into D2 slots of 1 KB; up to D2 - 1 of its items are issued before
  // the grid barrier, so for small layers all of phase 2's weights are in
  // shared memory by the time abuf is ready.
  constexpr int D2 = kDepth * R;
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t H = a.H, I = a.I;
  float* xs = reinterpret_cast<float*>(smem);
  const uint8_t* ring = smem + stream_x_bytes(H > I ? H : I) + warp * kDepth * R * kSegBytes;
  const uint32_t ring_s = smem_u32(ring);

  const int64_t nw = static_cast<int64_t>(gridDim.x) * kWarps;
  const int64_t wg = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
  int64_t u0, u1, h0, h1;
  split_range(I, nw, wg, u0, u1);   // phase 1: intermediate units
  split_range(H, nw, wg, h0, h1);   // phase 2: down rows
  const Walk<R> w1{a.gu_q, H, cdiv(u1 - u0, U), static_cast<int>(cdiv(H, kSegBytes)), 0};
  const Walk<1, D2> w2{a.down_q, I, h1 - h0, static_cast<int>(cdiv(I, kSegBytes)), 0};
  auto row1 = [&](int64_t g, int r) -> int64_t {
    const int64_t unit = u0 + g * U + (r % U);
    if (unit >= u1) return -1;
    return r < U ? unit : I + unit;
  };
  auto row2 = [&](int64_t g, int) -> int64_t { return h0 + g < h1 ? h0 + g : -1; };

  issue_item<R, KM1>(w1, ring_s, cursor_at(w1, 0), lane, row1);
  if (a.norm_w)
    for (int64_t i = tid * 32; i < H; i += kThreads * 32) prefetch_l1(a.norm_w + i);
  pdl_wait();
  stage_x(xs, a.x, H, tid, kThreads);
  __syncthreads();
  if (a.norm_w) norm_staged_x(xs, a.norm_w, H, a.eps, tid, kThreads);

  // ---- phase 1 ----
  auto scale1 = [&](int64_t g, int r, int64_t grp) -> float {
    const int64_t row = row1(g, r);
    return row >= 0 ? __ldg(a.gu_s + row * a.ng + grp) : 0.f;
  };
  auto done1 = [&](int64_t g, float s) {
    // gate row r (< U) sits on lanes 4r..4r+3, its up row r + U on lane + 4U
    const float up = __shfl_down_sync(0xffffffffu, s, 4 * U);
    const int r = reduced_row<R>(lane);
    if (r >= 0 && r < U) {
      const int64_t unit = u0 + g * U + r;
      if (unit < u1) {
        const float ga = PER_ROW ? s * __ldg(a.gu_s + unit) : s;
        const float ua = PER_ROW ? up * __ldg(a.gu_s + I + unit) : up;
        a.abuf[unit] = ga / (1.0f + expf(-ga)) * ua;
      }
    }
  };
  auto empty_group = [&]() { cp_async_commit(); };
  walk<R, PER_ROW, KM1>(w1, ring_s, ring, reinterpret_cast<const uint8_t*>(xs), a.x, lane,
                        H / a.ng, row1, scale1, empty_group, done1);
  // The ring is free again (phase 1 consumed every item): prefetch phase 2.
  cp_async_wait<0>();
  __syncwarp();
  issue_items<1, KM2>(w2, ring_s, 0, D2 - 1, lane, row2);
  pdl_trigger();

  // ---- grid barrier, then phase 2 over abuf ----
  const bool ok = grid_barrier(a.sync_ws, tid, 0x205u);
  if (ok) stage_x<true>(xs, a.abuf, I, tid, kThreads);
  __syncthreads();
  if (!ok) {
    cp_async_wait<0>();
    return;
  }
  auto scale2 = [&](int64_t g, int, int64_t grp) -> float {
    return h0 + g < h1 ? __ldg(a.down_s + (h0 + g) * a.ngd + grp) : 0.f;
  };
  unsigned ptag = 0u;
  if (a.po.P > 0)
    ptag = *reinterpret_cast<volatile unsigned*>(
        comm::fused_epoch(comm::own_base(a.po), a.po.P, a.po.n_max)) + 1u;
  auto done2 = [&](int64_t g, float s) {
    const int64_t row = h0 + g;
    if (lane == 0 && row < h1) {
      float o = PER_ROW ? s * __ldg(a.down_s + row) : s;
      if (a.residual) o += a.residual[row];
      if (a.po.P > 0)
        comm::peer_push(a.po, ptag, static_cast<int>((ptag - 1u) & 1u), row, o);
      else
        a.out[row] = o;
    }
  };
  // phase 2 reads abuf from the staged copy (it was written by other CTAs)
  walk<1, PER_ROW, KM2 == K1K ? KFULL : KM2>(w2, ring_s, ring,
                                             reinterpret_cast<const uint8_t*>(xs), nullptr, lane,
                                             I / a.ngd, row2, scale2, empty_group, done2);
  cp_async_wait<0>();
}

}  // namespace qz
