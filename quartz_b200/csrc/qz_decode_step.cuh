// qz_decode_step.cuh -- every decoder layer of one all-int8 decode token in ONE
// persistent cooperative kernel.
//
// quartz runs a token as a chain of ops (quartz/models/common.py:29-78): per
// layer RMSNorm -> q/k/v -> attention -> o + residual -> RMSNorm -> fused MLP
// + residual. As separate kernels that chain is latency-bound on B200: each
// layer's matrices are 4-15 MB, a few microseconds of HBM time, while every
// kernel boundary costs a launch and a cold start. Here one CTA per SM runs
// all layers; grid-wide barriers separate the five data-dependent phases of a
// layer:
//
//   A  x = RMSNorm(h) (layer 0: h = dequantised embedding row); qkv = Wqkv x
//   B  attention: q/k norm + RoPE, K/V append, split-context softmax, the
//      last CTA per kv head merges the partials -> attn
//   C  h2 = h + Wo attn
//   D  x = RMSNorm(h2); a = silu(Wgate x) * (Wup x)
//   E  h = h2 + Wdown a
//
// Each CTA owns a fixed, balanced, contiguous row range of every matrix (and
// a fixed set of (kv head, context chunk) attention items), so its whole
// token is a static schedule of contiguous byte ranges. A producer warp walks
// that schedule, issuing 1-D bulk copies (the TMA engine) into a ring of
// shared-memory slots; it runs ahead of the consumers across phase
// boundaries, so the next phase's weights and KV rows are already on chip
// while the grid waits at a barrier. Eight consumer warps compute from the
// ring. Nothing but the activations (a few KB, L2-resident) crosses between
// CTAs.
//
// Waits: ring slots (mbarrier) and the grid barrier give up after
// kWaitLimitNs, record ERR_* in the status word, and the CTA drains its copies
// and returns. Requires: one CTA per SM resident for the whole grid
// (cooperative launch), per-row scales, row lengths multiples of 16 bytes and
// at most one ring slot, head_dim 64 or 128.
#pragma once

#include "qz_decode.cuh"
#include "qz_device.cuh"
#include "qz_stream.cuh"

namespace qz {
namespace mk {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = 32 * kConsumerWarps;
// + the producer warp. Nine warps put three on some SM sub-partition (16384
// registers each), so a thread may use at most 168 registers.
constexpr int kThreadsMK = kConsumers + 32;
constexpr int kSlotBytes = 16384;
constexpr int kSlots = 8;
constexpr int kMaxX = 16384;                 // longest staged activation (floats)

struct LayerW {
  const int8_t* qkv_q;  const float* qkv_s;   // [(nq + 2 nkv) hd, H]
  const int8_t* o_q;    const float* o_s;     // [H, nq hd]
  const int8_t* gu_q;   const float* gu_s;    // [2 I, H] gate rows then up rows
  const int8_t* down_q; const float* down_s;  // [H, I]
  const float* in_w;    const float* post_w;  // [H]
  const float* qn_w;    const float* kn_w;    // [hd] or null
  float* kc;            float* vc;            // [nkv, max_ctx, hd]
};

struct StepArgs {
  const LayerW* layers;
  int n_layers;
  const int8_t* embed_q;   // [V, H]
  const float* embed_s;    // [V] (per-row)
  const int64_t* tok;      // device token fed at this step
  const int64_t* pos_dev;  // its position
  const float* inv_freq;   // [hd / 2]
  const float* norm_w;     // final RMSNorm [H]
  float* h;                // [H] residual stream (layer input / output)
  float* h2;               // [H] after attention
  float* qkv;              // [(nq + 2 nkv) hd]
  float* attn;             // [nq hd]
  float* act;              // [I]
  float* x_final;          // [H] RMSNorm(h) of the last layer: the lm_head input
  float* part;             // attention partials [nkv][S][NR][hd + 2]
  unsigned* tickets;       // [nkv], zero between launches
  unsigned long long* bar; // grid-barrier arrival count, zero before the first launch
  unsigned long long* trace;  // null, or [gridDim.x][1 + 10 * n_layers] %globaltimer stamps
  int H, I, nq, nkv, hd;
  int64_t max_ctx, V;
  float eps, scale;
};

// shared-memory carve-up (dynamic)
struct Smem {
  static constexpr int ring = 0;
  static constexpr int xs = ring + kSlots * kSlotBytes;          // kMaxX floats
  static constexpr int misc = xs + kMaxX * 4;                    // see below
  // misc: gbuf [kMaxUnits], qs [8 * 256], sc [8 * 64], kvn [2 * 256], red [64]
  static constexpr int kMaxUnits = 256;
  static constexpr int gbuf = misc;
  static constexpr int qs = gbuf + kMaxUnits * 4;
  static constexpr int sc = qs + 8 * 256 * 4;
  static constexpr int kvn = sc + 8 * 64 * 4;
  static constexpr int red = kvn + 2 * 256 * 4;
  // per-layer row scales and residual slices of this CTA: A | C | gate | up | E | res C | res E
  static constexpr int kMaxPre = 2048;
  static constexpr int pre = red + 64 * 4;
  // constants: RoPE inverse frequencies [128], this layer's q/k norm weights [256] each
  static constexpr int cst = pre + kMaxPre * 4;
  static constexpr int bars = cst + 640 * 4;                     // full[kSlots], empty[kSlots]
  static constexpr int flags = bars + 2 * kSlots * 8;
  static constexpr int total = flags + 64;
};

// A contiguous byte range [src, src + rows * row_bytes) cut into chunks of
// whole rows of at most one slot.
struct Seg {
  const uint8_t* src;
  int64_t rows;
  int row_bytes;
  __device__ int rows_per_chunk() const { return kSlotBytes / row_bytes; }
  __device__ int64_t chunks() const {
    return rows > 0 ? cdiv(rows, static_cast<int64_t>(rows_per_chunk())) : 0;
  }
};

// Attention items of this CTA: item = b + k * gridDim.x over nkv * S items;
// item i -> kv head i % nkv, chunk i / nkv.
struct AttnPlan {
  int64_t T, pos;
  int S, rows;     // chunks per kv head, positions per chunk
};

__device__ __forceinline__ AttnPlan attn_plan(const StepArgs& a) {
  AttnPlan p;
  p.pos = *a.pos_dev;
  p.T = p.pos + 1;
  if (p.T > a.max_ctx) p.T = a.max_ctx;
  if (p.T < 1) p.T = 1;
  p.rows = kSlotBytes / (a.hd * 4);
  p.S = static_cast<int>(cdiv(p.T, p.rows));
  return p;
}

// The static schedule, identical for producer and consumers. Phase callbacks
// receive the segments in order; `each_seg(phase, k, seg)`.
template <class F>
__device__ __forceinline__ void schedule(const StepArgs& a, const AttnPlan& ap, int l, F&& f) {
  const LayerW& L = a.layers[l];
  const int64_t P = gridDim.x, b = blockIdx.x;
  const int H = a.H, I = a.I, hd = a.hd;
  const int64_t nqkv = static_cast<int64_t>(a.nq + 2 * a.nkv) * hd;
  const int Ko = a.nq * hd;
  int64_t r0, r1;
  // A
  split_range(nqkv, P, b, r0, r1);
  f(0, 0, Seg{reinterpret_cast<const uint8_t*>(L.qkv_q) + r0 * H, r1 - r0, H});
  // B: per item, K rows then V rows
  const int64_t items = static_cast<int64_t>(a.nkv) * ap.S;
  int k = 0;
  for (int64_t it = b; it < items; it += P, ++k) {
    const int g = static_cast<int>(it % a.nkv);
    const int64_t c = it / a.nkv;
    const int64_t t0 = c * ap.rows, t1 = min64(ap.T, t0 + ap.rows);
    const int64_t off = (static_cast<int64_t>(g) * a.max_ctx + t0) * hd * 4;
    f(1, 2 * k, Seg{reinterpret_cast<const uint8_t*>(L.kc) + off, t1 - t0, hd * 4});
    f(1, 2 * k + 1, Seg{reinterpret_cast<const uint8_t*>(L.vc) + off, t1 - t0, hd * 4});
  }
  // C
  split_range(H, P, b, r0, r1);
  f(2, 0, Seg{reinterpret_cast<const uint8_t*>(L.o_q) + r0 * Ko, r1 - r0, Ko});
  // D: gate rows then up rows of this CTA's units
  split_range(I, P, b, r0, r1);
  f(3, 0, Seg{reinterpret_cast<const uint8_t*>(L.gu_q) + r0 * H, r1 - r0, H});
  f(3, 1, Seg{reinterpret_cast<const uint8_t*>(L.gu_q) + (I + r0) * H, r1 - r0, H});
  // E
  split_range(H, P, b, r0, r1);
  f(4, 0, Seg{reinterpret_cast<const uint8_t*>(L.down_q) + r0 * I, r1 - r0, I});
}

__device__ __forceinline__ void consumer_sync() { named_bar_sync(1, kConsumers); }

// Grid barrier among the consumer warps of every CTA (the producer never
// joins) on a monotonically increasing 64-bit arrival count: a CTA adds 1 with
// a fire-and-forget reduction and waits until the count reaches
// base + k * P for its k-th barrier (fence.acq_rel + relaxed reduction on
// arrival, acquire loads while waiting). No reset round trips; a launch that
// completes all its barriers leaves the count at a multiple of (barriers per
// launch) * P, which is how the next launch recovers its base. Returns false
// on timeout (status recorded); the count is then out of step and the
// workspace must be zeroed before the next launch.
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_relaxed_add_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

struct GridBar {
  unsigned long long* count;
  unsigned long long target;   // meaningful in consumer thread 0 only
};

__device__ __forceinline__ bool consumer_grid_barrier(GridBar& gb, unsigned* s_flag, int tid,
                                                      unsigned site) {
  consumer_sync();
  if (tid == 0) {
    unsigned ok = 1u;
    gb.target += gridDim.x;
    // the CTA's writes (ordered before by the named barrier) are released at
    // gpu scope by this fence, then the arrival is a relaxed reduction
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    red_relaxed_add_u64(gb.count, 1ull);
    if (ld_acquire_u64(gb.count) < gb.target) {
      const unsigned long long t0 = globaltimer();
      while (ld_acquire_u64(gb.count) < gb.target) {
        if (globaltimer() - t0 > kWaitLimitNs) {
          report_error(ERR_GRID_BARRIER, site);
          ok = 0u;
          break;
        }
      }
    }
    *s_flag = ok;
  }
  consumer_sync();
  return *s_flag != 0u;
}

// Block-wide (consumers) sum; every consumer thread gets the total.
__device__ __forceinline__ float consumer_sum(float v, float* red, int tid) {
  v = dec::warp_sum_f(v);
  if ((tid & 31) == 0) red[tid >> 5] = v;
  consumer_sync();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kConsumerWarps; ++i) s += red[i];
  consumer_sync();
  return s;
}

template <bool COHERENT>
__device__ __forceinline__ float ld_act(const float* p) {
  return COHERENT ? __ldcg(p) : *p;
}

// Activations are staged in shared memory in the layout load_x16 reads,
// float index ((j / 4) * nch + c) * 4 + j % 4 for element 16 c + j (nch =
// n / 16), so that lane-consecutive 16-element chunks are conflict-free.
// The staging walks the DESTINATION in thread order (conflict-free stores):
// destination o = j4 * 4 nch + rem holds element 16 (rem / 4) + 4 j4 + rem % 4.
__device__ __forceinline__ int staged_src(int j4, int rem) {
  return (rem >> 2) * 16 + j4 * 4 + (rem & 3);
}

// xs = src (n floats written by other CTAs earlier in this kernel: L2 reads)
__device__ __forceinline__ void stage_act(float* xs, const float* src, int n, int tid) {
  const int nch4 = n / 4;
#pragma unroll
  for (int j4 = 0; j4 < 4; ++j4)
    for (int rem = tid; rem < nch4; rem += kConsumers)
      xs[j4 * nch4 + rem] = __ldcg(src + staged_src(j4, rem));
}

// xs = RMSNorm(src) * w (quartz/ops.py:24-32), src and w read in ONE round of
// loads (values held in registers) when n <= 4 kRegX kConsumers.
constexpr int kRegX = 2;   // per j4
__device__ __forceinline__ void stage_rmsnorm(float* xs, const float* src, const float* w, int n,
                                              float eps, float* red, int tid) {
  const int nch4 = n / 4;
  if (nch4 <= kRegX * kConsumers) {
    float v[4][kRegX], wv[4][kRegX];
    float ss = 0.f;
#pragma unroll
    for (int j4 = 0; j4 < 4; ++j4)
#pragma unroll
      for (int k = 0; k < kRegX; ++k) {
        const int rem = tid + k * kConsumers;
        const bool in = rem < nch4;
        const int i = staged_src(j4, rem);
        v[j4][k] = in ? __ldcg(src + i) : 0.f;
        wv[j4][k] = in ? w[i] : 0.f;
        ss = fmaf(v[j4][k], v[j4][k], ss);
      }
    ss = consumer_sum(ss, red, tid);
    const float r = 1.0f / sqrtf(ss / static_cast<float>(n) + eps);
#pragma unroll
    for (int j4 = 0; j4 < 4; ++j4)
#pragma unroll
      for (int k = 0; k < kRegX; ++k) {
        const int rem = tid + k * kConsumers;
        if (rem < nch4) xs[j4 * nch4 + rem] = v[j4][k] * r * wv[j4][k];
      }
    return;
  }
  float ss = 0.f;
  for (int i = tid; i < n; i += kConsumers) {
    const float v = __ldcg(src + i);
    ss = fmaf(v, v, ss);
  }
  ss = consumer_sum(ss, red, tid);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(n) + eps);
#pragma unroll
  for (int j4 = 0; j4 < 4; ++j4)
    for (int rem = tid; rem < nch4; rem += kConsumers) {
      const int i = staged_src(j4, rem);
      xs[j4 * nch4 + rem] = __ldcg(src + i) * r * w[i];
    }
}

// One row of K bytes in shared memory against the staged activations.
__device__ __forceinline__ float row_dot(const uint8_t* row, const uint8_t* xs, int K, int lane);

// Two rows at once (the activations are read once for both).
__device__ __forceinline__ void row_dot2(const uint8_t* row0, const uint8_t* row1,
                                         const uint8_t* xs, int K, int lane, float& d0,
                                         float& d1) {
  const int64_t nch = K / 16;
  f2_t a0 = 0ull, a1 = 0ull;
  for (int c = lane; c < K / 16; c += 32) {
    const uint4 q0 = *reinterpret_cast<const uint4*>(row0 + c * 16);
    const uint4 q1 = *reinterpret_cast<const uint4*>(row1 + c * 16);
    f2_t xv[8];
    load_x16(xs, nch, c, xv);
    dot16_acc(q0, xv, a0);
    dot16_acc(q1, xv, a1);
  }
  const float2 s0 = f2_unpack(a0), s1 = f2_unpack(a1);
  float v0 = s0.x + s0.y, v1 = s1.x + s1.y;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    v0 += __shfl_xor_sync(0xffffffffu, v0, o);
    v1 += __shfl_xor_sync(0xffffffffu, v1, o);
  }
  d0 = v0;
  d1 = v1;
}

// The rows [0, rows) of a ring slot (row length K) against the staged
// activations: warp w takes rows 2w, 2w + 1, 2w + 16, ...; emit(i, dot) runs
// in lane 0 for every row.
template <class F>
__device__ __forceinline__ void chunk_rows(const uint8_t* slot, int rows, int K, const float* xs,
                                           int warp, int lane, F&& emit) {
  const uint8_t* x8 = reinterpret_cast<const uint8_t*>(xs);
  for (int r = 2 * warp; r < rows; r += 2 * kConsumerWarps) {
    if (r + 1 < rows) {
      float d0, d1;
      row_dot2(slot + r * K, slot + (r + 1) * K, x8, K, lane, d0, d1);
      if (lane == 0) { emit(r, d0); emit(r + 1, d1); }
    } else {
      const float d = row_dot(slot + r * K, x8, K, lane);
      if (lane == 0) emit(r, d);
    }
  }
}

__device__ __forceinline__ float row_dot(const uint8_t* row, const uint8_t* xs, int K, int lane) {
  const int64_t nch = K / 16;
  f2_t acc = 0ull;
  for (int c = lane; c < K / 16; c += 32) {
    const uint4 q = *reinterpret_cast<const uint4*>(row + c * 16);
    f2_t xv[8];
    load_x16(xs, nch, c, xv);
    dot16_acc(q, xv, acc);
  }
  const float2 s = f2_unpack(acc);
  return dec::warp_sum_f(s.x + s.y);
}

// merge_partials for the consumer warps, NR a runtime value (1, 2, 4 or 8).
template <int HD>
__device__ __forceinline__ void merge_group(const float* part_g, int S, int NR, float* out_g,
                                            float* scratch, int tid) {
  auto sync = [] { consumer_sync(); };
  switch (NR) {
    case 1: dec::merge_partials<HD, 1, kConsumers, decltype(sync)&, false>(part_g, S, out_g, scratch, tid, sync); break;
    case 2: dec::merge_partials<HD, 2, kConsumers, decltype(sync)&, false>(part_g, S, out_g, scratch, tid, sync); break;
    case 4: dec::merge_partials<HD, 4, kConsumers, decltype(sync)&, false>(part_g, S, out_g, scratch, tid, sync); break;
    default: dec::merge_partials<HD, 8, kConsumers, decltype(sync)&, false>(part_g, S, out_g, scratch, tid, sync); break;
  }
}

template <int E>
__global__ void __launch_bounds__(kThreadsMK, 1) decode_layers_kernel(const StepArgs a) {
  constexpr int HD = 32 * E;
  extern __shared__ __align__(128) uint8_t smem[];  // 128: the alignment every kernel here declares
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t* ring = smem + Smem::ring;
  float* xs = reinterpret_cast<float*>(smem + Smem::xs);
  float* gbuf = reinterpret_cast<float*>(smem + Smem::gbuf);
  float* qs = reinterpret_cast<float*>(smem + Smem::qs);
  float* sc = reinterpret_cast<float*>(smem + Smem::sc);
  float* kvn = reinterpret_cast<float*>(smem + Smem::kvn);
  float* red = reinterpret_cast<float*>(smem + Smem::red);
  float* pre = reinterpret_cast<float*>(smem + Smem::pre);
  float* invf = reinterpret_cast<float*>(smem + Smem::cst);
  float* qn_s = invf + 128;
  float* kn_s = qn_s + 256;
  const uint32_t bars = smem_u32(smem + Smem::bars);
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (kSlots + s); };
  volatile unsigned* abort_flag = reinterpret_cast<volatile unsigned*>(smem + Smem::flags);
  unsigned* s_flag = reinterpret_cast<unsigned*>(smem + Smem::flags + 4);
  unsigned* s_last = reinterpret_cast<unsigned*>(smem + Smem::flags + 8);

  if (tid == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), kConsumerWarps);
    }
    *abort_flag = 0u;
    fence_mbar_init();
  }
  __syncthreads();
  const AttnPlan ap = attn_plan(a);

  // ------------------------------------------------------------- producer
  if (warp == kConsumerWarps) {
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      int64_t n = 0;   // chunks issued
      bool stop = false;
      for (int l = 0; l < a.n_layers && !stop; ++l) {
        schedule(a, ap, l, [&](int, int, const Seg& sg) {
          const int64_t nc = sg.chunks();
          const int rpc = sg.rows_per_chunk();
          for (int64_t c = 0; c < nc && !stop; ++c, ++n) {
            const int s = static_cast<int>(n % kSlots);
            const int64_t use = n / kSlots;
            if (use > 0 && !mbar_wait(empty_bar(s), static_cast<uint32_t>((use - 1) & 1))) {
              if (!*abort_flag) report_error(ERR_WAIT_EMPTY, 0x301u);
              *abort_flag = 1u;
              stop = true;
              break;
            }
            if (*abort_flag) { stop = true; break; }
            const int64_t r = min64(rpc, sg.rows - c * rpc);
            const uint32_t bytes = static_cast<uint32_t>(r * sg.row_bytes);
            mbar_arrive_expect_tx(full_bar(s), bytes);
            bulk_g2s(smem_u32(ring + s * kSlotBytes), sg.src + c * rpc * sg.row_bytes, bytes,
                     full_bar(s), pol);
          }
        });
      }
      // Drain: every issued copy must land before the CTA may exit. Slots
      // whose last use was consumed already completed; waiting on the last
      // issued use of each slot covers the rest.
      for (int s = 0; s < kSlots; ++s) {
        if (n <= s) break;
        const int64_t last_use = (n - 1 - s) / kSlots;
        if (!mbar_wait(full_bar(s), static_cast<uint32_t>(last_use & 1)))
          report_error(ERR_DRAIN, 0x302u);
      }
    }
    return;
  }

  // ------------------------------------------------------------ consumers
  int64_t n = 0;   // chunks consumed
  bool ok = true;
  // wait for chunk n; returns its slot base or null on failure
  auto acquire = [&]() -> const uint8_t* {
    const int s = static_cast<int>(n % kSlots);
    if (!mbar_wait(full_bar(s), static_cast<uint32_t>((n / kSlots) & 1))) {
      if (lane == 0) report_error(ERR_WAIT_FULL, 0x303u);
      ok = false;
      return nullptr;
    }
    return ring + s * kSlotBytes;
  };
  auto release = [&]() {
    __syncwarp();
    if (lane == 0) mbar_arrive(empty_bar(static_cast<int>(n % kSlots)));
    ++n;
  };

  const int H = a.H, I = a.I, nq = a.nq, nkv = a.nkv;
  constexpr int hd = HD;
  const int NR = nq / nkv;
  const int Ko = nq * hd;
  const int64_t P = gridDim.x, b = blockIdx.x;
  // this launch's barrier base: the count sits at a multiple of
  // (barriers per launch) * P when it starts (see consumer_grid_barrier)
  GridBar gbar{a.bar, 0ull};
  if (tid == 0) {
    const unsigned long long per_launch = 5ull * a.n_layers * gridDim.x;
    gbar.target = ld_acquire_u64(a.bar) / per_launch * per_launch;
  }
  // optional phase trace: stamp k of this CTA (consumer thread 0)
  const int n_stamps = 1 + 10 * a.n_layers;
  auto stamp = [&](int k) {
    if (a.trace && tid == 0) a.trace[static_cast<int64_t>(blockIdx.x) * n_stamps + k] = globaltimer();
  };
  stamp(0);
  int64_t tok = *a.tok;
  tok = tok < 0 ? 0 : (tok >= a.V ? a.V - 1 : tok);   // validated on the host; stay in bounds

  for (int i = tid; i < hd / 2; i += kConsumers) invf[i] = a.inv_freq[i];
  constexpr int KP = kSlotBytes / (HD * 4) / kConsumerWarps;   // K/V rows per warp per chunk
  for (int l = 0; l < a.n_layers && ok; ++l) {
    const LayerW& L = a.layers[l];
    // This CTA's rows of every matrix of the layer (C and E share the
    // H-split). Their scales, the residual rows phase C adds and the q/k norm
    // weights are loaded into shared memory now, beside the activation
    // staging, so that no output row waits on a global load after its dot
    // product.
    int64_t a0, a1, c0, c1, d0, d1;
    split_range(static_cast<int64_t>(nq + 2 * nkv) * hd, P, b, a0, a1);
    split_range(H, P, b, c0, c1);
    split_range(I, P, b, d0, d1);
    const int nA = static_cast<int>(a1 - a0), nC = static_cast<int>(c1 - c0);
    const int nD = static_cast<int>(d1 - d0);
    float* sA = pre;
    float* sC = sA + nA;
    float* sG = sC + nC;
    float* sU = sG + nD;
    float* sE = sU + nD;
    float* rC = sE + nC;
    float* rE = rC + nC;
    {
      const int n_pre = nA + 4 * nC + 2 * nD;   // everything but rE
      for (int i = tid; i < n_pre; i += kConsumers) {
        float v;
        int j = i;
        if (j < nA) v = __ldg(L.qkv_s + a0 + j);
        else if ((j -= nA) < nC) v = __ldg(L.o_s + c0 + j);
        else if ((j -= nC) < nD) v = __ldg(L.gu_s + d0 + j);
        else if ((j -= nD) < nD) v = __ldg(L.gu_s + I + d0 + j);
        else if ((j -= nD) < nC) v = __ldg(L.down_s + c0 + j);
        else {
          j -= nC;   // residual of phase C: h (layer 0: the embedding row)
          v = l == 0 ? static_cast<float>(a.embed_q[tok * H + c0 + j]) * a.embed_s[tok]
                     : __ldcg(a.h + c0 + j);
        }
        pre[i] = v;
      }
      if (L.qn_w)
        for (int i = tid; i < 2 * hd; i += kConsumers)
          (i < hd ? qn_s : kn_s - hd)[i] = i < hd ? L.qn_w[i] : L.kn_w[i - hd];
    }
    // ---------------- A: x = RMSNorm(h); qkv rows
    if (l == 0) {
      // h = dequantised embedding row (quartz/quantize.py:78-80); CTA 0 keeps
      // it as the residual stream
      const int8_t* er = a.embed_q + tok * H;
      const float es = a.embed_s[tok];
      if (b == 0)
        for (int i = tid; i < H; i += kConsumers) a.h[i] = static_cast<float>(er[i]) * es;
      float ss = 0.f;
      for (int i = tid; i < H; i += kConsumers) {
        const float v = static_cast<float>(er[i]) * es;
        ss = fmaf(v, v, ss);
      }
      ss = consumer_sum(ss, red, tid);
      const float r = 1.0f / sqrtf(ss / static_cast<float>(H) + a.eps);
      const int nch4 = H / 4;
#pragma unroll
      for (int j4 = 0; j4 < 4; ++j4)
        for (int rem = tid; rem < nch4; rem += kConsumers) {
          const int i = staged_src(j4, rem);
          xs[j4 * nch4 + rem] = static_cast<float>(er[i]) * es * r * L.in_w[i];
        }
    } else {
      stage_rmsnorm(xs, a.h, L.in_w, H, a.eps, red, tid);
    }
    consumer_sync();
    {
      const Seg sg{nullptr, nA, H};
      const int rpc = sg.rows_per_chunk();
      for (int64_t c = 0; c < sg.chunks() && ok; ++c) {
        const uint8_t* slot = acquire();
        if (!slot) break;
        const int rows = static_cast<int>(min64(rpc, sg.rows - c * rpc));
        float* out = a.qkv + a0 + c * rpc;
        const float* sc_ = sA + c * rpc;
        chunk_rows(slot, rows, H, xs, warp, lane, [&](int r, float d) { out[r] = d * sc_[r]; });
        release();
      }
    }
    stamp(1 + 10 * l + 0);
    if (!ok || !consumer_grid_barrier(gbar, s_flag, tid, 0x310u + l)) { ok = false; break; }
    stamp(2 + 10 * l + 0);

    // ---------------- B: attention items
    {
      const int64_t items = static_cast<int64_t>(nkv) * ap.S;
      const float* qn = L.qn_w ? qn_s : nullptr;
      const float* kn = L.qn_w ? kn_s : nullptr;
      for (int64_t it = b; it < items && ok; it += P) {
        const int g = static_cast<int>(it % nkv);
        const int64_t ci = it / nkv;
        const int64_t t0 = ci * ap.rows, t1 = min64(ap.T, t0 + ap.rows);
        const int nt = static_cast<int>(t1 - t0);
        const bool owner = t0 <= ap.pos && ap.pos < t1 && ap.pos < a.max_ctx;
        // queries of group g (norm + RoPE), and in the owner the new k/v
        for (int r = warp; r < NR; r += kConsumerWarps) {
          float x[E];
          const float* src = a.qkv + static_cast<int64_t>(g * NR + r) * hd + lane * E;
#pragma unroll
          for (int e = 0; e < E; ++e) x[e] = __ldcg(src + e);
          dec::norm_rope<E>(x, qn, invf, ap.pos, a.eps, lane);
#pragma unroll
          for (int e = 0; e < E; ++e) qs[r * hd + lane * E + e] = x[e];
        }
        if (owner && warp == NR % kConsumerWarps) {
          float k[E], v[E];
          const float* ks = a.qkv + static_cast<int64_t>(nq + g) * hd + lane * E;
          const float* vs = a.qkv + static_cast<int64_t>(nq + nkv + g) * hd + lane * E;
#pragma unroll
          for (int e = 0; e < E; ++e) { k[e] = __ldcg(ks + e); v[e] = __ldcg(vs + e); }
          dec::norm_rope<E>(k, kn, invf, ap.pos, a.eps, lane);
          float* kd = L.kc + (static_cast<int64_t>(g) * a.max_ctx + ap.pos) * hd + lane * E;
          float* vd = L.vc + (static_cast<int64_t>(g) * a.max_ctx + ap.pos) * hd + lane * E;
#pragma unroll
          for (int e = 0; e < E; ++e) {
            kd[e] = k[e];
            vd[e] = v[e];
            kvn[lane * E + e] = k[e];
            kvn[hd + lane * E + e] = v[e];
          }
        }
        consumer_sync();
        // K chunk: scores sc[r][t] = (q_r . k_t) * scale. Warp w holds rows
        // w + 8k (k < KP) and reduces their KP dot products together.
        const uint8_t* kslot = acquire();
        if (!kslot) break;
        {
          const float* krows = reinterpret_cast<const float*>(kslot);
          float kr[KP][E];
#pragma unroll
          for (int k = 0; k < KP; ++k) {
            const int t = warp + kConsumerWarps * k;
            const bool fresh = owner && t0 + t == ap.pos;
            const float* src = fresh ? kvn : krows + t * hd;
#pragma unroll
            for (int e = 0; e < E; ++e) kr[k][e] = t < nt ? src[lane * E + e] : 0.f;
          }
          for (int r = 0; r < NR; ++r) {
            float qv[E], d[KP];
#pragma unroll
            for (int e = 0; e < E; ++e) qv[e] = qs[r * hd + lane * E + e];
#pragma unroll
            for (int k = 0; k < KP; ++k) {
              d[k] = 0.f;
#pragma unroll
              for (int e = 0; e < E; ++e) d[k] = fmaf(qv[e], kr[k][e], d[k]);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
              for (int k = 0; k < KP; ++k) d[k] += __shfl_xor_sync(0xffffffffu, d[k], o);
            if (lane == 0)
#pragma unroll
              for (int k = 0; k < KP; ++k) {
                const int t = warp + kConsumerWarps * k;
                if (t < nt) sc[r * 64 + t] = d[k] * a.scale;
              }
          }
        }
        release();
        consumer_sync();
        // softmax statistics per head (warp r), probabilities in place
        for (int r = warp; r < NR; r += kConsumerWarps) {
          float m = -INFINITY;
          for (int t = lane; t < nt; t += 32) m = fmaxf(m, sc[r * 64 + t]);
          m = dec::warp_max_f(m);
          float s = 0.f;
          for (int t = lane; t < nt; t += 32) {
            const float p = expf(sc[r * 64 + t] - m);
            sc[r * 64 + t] = p;
            s += p;
          }
          s = dec::warp_sum_f(s);
          if (lane == 0) { red[32 + 2 * r] = m; red[32 + 2 * r + 1] = s; }
        }
        consumer_sync();
        // V chunk: partial acc[r][d] = sum_t p[r][t] v_t[d]
        const uint8_t* vslot = acquire();
        if (!vslot) break;
        const float* vrows = reinterpret_cast<const float*>(vslot);
        float* pbase = a.part + (static_cast<int64_t>(g) * ap.S + ci) * NR * (hd + 2);
        const int tf = owner ? static_cast<int>(ap.pos - t0) : -1;
        for (int i = tid; i < NR * hd; i += kConsumers) {
          const int r = i / hd, d = i - r * hd;
          float acc = 0.f;
#pragma unroll 8
          for (int t = 0; t < nt; ++t) {
            const float v = t == tf ? kvn[hd + d] : vrows[t * hd + d];
            acc = fmaf(sc[r * 64 + t], v, acc);
          }
          pbase[r * (hd + 2) + d] = acc;
          if (d == 0) { pbase[r * (hd + 2) + hd] = red[32 + 2 * r]; pbase[r * (hd + 2) + hd + 1] = red[32 + 2 * r + 1]; }
        }
        release();
        // ticket: the last item of kv head g merges its S partials
        consumer_sync();
        if (tid == 0) {
          __threadfence();
          *s_last = atomicAdd(a.tickets + g, 1u) == static_cast<unsigned>(ap.S - 1);
        }
        consumer_sync();
        if (*s_last) {
          __threadfence();
          merge_group<HD>(a.part + static_cast<int64_t>(g) * ap.S * NR * (hd + 2), ap.S, NR,
                          a.attn + static_cast<int64_t>(g) * NR * hd, xs, tid);
          if (tid == 0) a.tickets[g] = 0u;
        }
        consumer_sync();
      }
    }
    stamp(1 + 10 * l + 2);
    if (!ok || !consumer_grid_barrier(gbar, s_flag, tid, 0x320u + l)) { ok = false; break; }
    stamp(2 + 10 * l + 2);

    // ---------------- C: h2 = h + Wo attn
    stage_act(xs, a.attn, Ko, tid);
    consumer_sync();
    {
      const Seg sg{nullptr, nC, Ko};
      const int rpc = sg.rows_per_chunk();
      for (int64_t c = 0; c < sg.chunks() && ok; ++c) {
        const uint8_t* slot = acquire();
        if (!slot) break;
        const int rows = static_cast<int>(min64(rpc, sg.rows - c * rpc));
        float* out = a.h2 + c0 + c * rpc;
        const float* sc_ = sC + c * rpc;
        const float* res = rC + c * rpc;
        chunk_rows(slot, rows, Ko, xs, warp, lane,
                   [&](int r, float d) { out[r] = d * sc_[r] + res[r]; });
        release();
      }
    }
    stamp(1 + 10 * l + 4);
    if (!ok || !consumer_grid_barrier(gbar, s_flag, tid, 0x330u + l)) { ok = false; break; }
    stamp(2 + 10 * l + 4);

    // ---------------- D: x = RMSNorm(h2); a = silu(gate x) * (up x)
    for (int i = tid; i < nC; i += kConsumers) rE[i] = __ldcg(a.h2 + c0 + i);   // residual of E
    stage_rmsnorm(xs, a.h2, L.post_w, H, a.eps, red, tid);
    consumer_sync();
    {
      for (int half = 0; half < 2 && ok; ++half) {
        const Seg sg{nullptr, nD, H};
        const int rpc = sg.rows_per_chunk();
        for (int64_t c = 0; c < sg.chunks() && ok; ++c) {
          const uint8_t* slot = acquire();
          if (!slot) break;
          const int rows = static_cast<int>(min64(rpc, sg.rows - c * rpc));
          const int u0 = static_cast<int>(c * rpc);   // unit index within this CTA
          if (half == 0) {
            chunk_rows(slot, rows, H, xs, warp, lane,
                       [&](int r, float d) { gbuf[u0 + r] = d * sG[u0 + r]; });
          } else {
            float* out = a.act + d0 + u0;
            chunk_rows(slot, rows, H, xs, warp, lane, [&](int r, float d) {
              const float gv = gbuf[u0 + r];
              const float uv = d * sU[u0 + r];
              // silu with the unclipped exponent, as the fused decode MLP
              // (quartz/kernels/fused.py:40-54)
              out[r] = gv / (1.0f + expf(-gv)) * uv;
            });
          }
          release();
        }
        consumer_sync();   // gate values visible before the up half reads them
      }
    }
    stamp(1 + 10 * l + 6);
    if (!ok || !consumer_grid_barrier(gbar, s_flag, tid, 0x340u + l)) { ok = false; break; }
    stamp(2 + 10 * l + 6);

    // ---------------- E: h = h2 + Wdown a
    stage_act(xs, a.act, I, tid);
    consumer_sync();
    {
      const Seg sg{nullptr, nC, I};
      const int rpc = sg.rows_per_chunk();
      for (int64_t c = 0; c < sg.chunks() && ok; ++c) {
        const uint8_t* slot = acquire();
        if (!slot) break;
        const int rows = static_cast<int>(min64(rpc, sg.rows - c * rpc));
        float* out = a.h + c0 + c * rpc;
        const float* sc_ = sE + c * rpc;
        const float* res = rE + c * rpc;
        chunk_rows(slot, rows, I, xs, warp, lane,
                   [&](int r, float d) { out[r] = d * sc_[r] + res[r]; });
        release();
      }
    }
    stamp(1 + 10 * l + 8);
    if (!ok || !consumer_grid_barrier(gbar, s_flag, tid, 0x350u + l)) { ok = false; break; }
    stamp(2 + 10 * l + 8);
  }
  if (!ok) {
    *abort_flag = 1u;
    return;
  }
  // final RMSNorm -> the lm_head input
  if (b == 0) {
    float ss = 0.f;
    for (int i = tid; i < H; i += kConsumers) {
      const float v = __ldcg(a.h + i);
      ss = fmaf(v, v, ss);
    }
    ss = consumer_sum(ss, red, tid);
    const float r = 1.0f / sqrtf(ss / static_cast<float>(H) + a.eps);
    for (int i = tid; i < H; i += kConsumers) a.x_final[i] = __ldcg(a.h + i) * r * a.norm_w[i];
  }
}

}  // namespace mk
}  // namespace qz
