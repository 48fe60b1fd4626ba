// qz_stream.cuh -- HBM-streaming int8 weight-only kernels for M = 1 (decode).
//
//   gemv_stream_kernel   y[n] = sum_g scale[n,g] * sum_{k in g} x[k] * q[n,k]  (+ residual[n])
//                        (quartz/kernels/int8.py:24-38 and its serial twin 48-63)
//   fused_mlp_kernel     out = down(silu(gate.x) * (up.x))  (+ residual)
//                        (quartz/kernels/fused.py:27-65)
//
// Shape of both kernels: one persistent CTA per SM, 16 consumer warps and one
// producer warp. The producer's elected lane streams the CTA's slice of the
// weight matrix through a ring of shared-memory stages with 1-D bulk copies
// (cp.async.bulk, the TMA engine) that complete on per-stage mbarriers. A
// stage is a "row group": 8 weight rows x up to 1024 bytes of K. Each consumer
// warp owns whole row groups: lane l takes 16-byte chunks l, l+32, ... of the
// 8 rows, widens int8 -> fp32 in registers (qz_device.cuh), and accumulates
// fp32 pairs; activations sit in shared memory in a bank-conflict-free layout
// and are read once per chunk for all 8 rows. One transposed butterfly
// reduces the 8 row sums; the per-row scale, SiLU gate and residual are fused
// into that epilogue. The fp32 weight array is never formed.
#pragma once

#include "qz_device.cuh"

namespace qz {

constexpr int kRW = 8;                          // weight rows per row group / stage
constexpr int kConsumerWarps = 16;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kSeg = 1024;                      // K bytes per stage row
constexpr int kMaxStages = 32;
constexpr int kStageBytes = kRW * kSeg;
constexpr int kSmemHeader = 2 * kMaxStages * 8 + 128;  // barriers (+ flags), 128-aligned

__host__ __device__ constexpr int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ constexpr int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }

// Layout of dynamic shared memory: [full[32] | empty[32] | flags][x: xfloats][stages]
__host__ __device__ inline int stream_x_bytes(int64_t kmax) {
  return static_cast<int>(((kmax * 4 + 127) / 128) * 128);
}

struct GemvArgs {
  const int8_t* q;        // [N, K]
  const float* scale;     // [N, ng]
  const float* x;         // [K]
  float* y;               // [N]
  const float* residual;  // [N] or null
  int64_t N, K, ng;
  int nstages;
};

struct MlpArgs {
  const int8_t* gu_q;     // [2I, H]: gate rows 0..I-1, up rows I..2I-1
  const float* gu_s;      // [2I, ng]
  const float* x;         // [H]
  const int8_t* down_q;   // [H, I]
  const float* down_s;    // [H, ngd]
  float* abuf;            // [I] intermediate, global (read back after the grid barrier)
  float* out;             // [H]
  const float* residual;  // [H] or null
  unsigned int* sync_ws;  // grid barrier words {count, generation}, zero at first use
  int64_t H, I, ng, ngd;
  int nstages;
};

// Stage the K activations into shared memory as float4 blocks ordered
// [word j4][chunk c] so that lane-consecutive chunks hit consecutive banks.
// COHERENT: the source was written earlier in this kernel by other CTAs (the
// fused MLP's intermediate, read after the grid barrier), so it is read from
// L2 (ld.global.cg), never through the non-coherent path.
template <bool COHERENT = false>
__device__ __forceinline__ void stage_x(float* xs, const float* x, int64_t K, int tid, int nthr) {
  const int64_t nch = K / 16;
  for (int64_t i = tid; i < K; i += nthr) {
    const int64_t c = i >> 4, j = i & 15;
    xs[((j >> 2) * nch + c) * 4 + (j & 3)] = COHERENT ? __ldcg(x + i) : x[i];
  }
}

// Load the 16 activations of global chunk gc as 8 fp32 pairs.
__device__ __forceinline__ void load_x16(uint32_t xs_base, int64_t nch, int64_t gc, f2_t (&xv)[8]) {
#pragma unroll
  for (int j4 = 0; j4 < 4; ++j4)
    lds_f2x2(xs_base + static_cast<uint32_t>((j4 * nch + gc) * 16), xv[2 * j4], xv[2 * j4 + 1]);
}

// ---------------------------------------------------------------------------
// Producer: issue the bulk copies for stage positions [0, total) in order.
// `rows_of(pos)` is the bitmask of stage rows that exist at position pos;
// `src_of(pos, r, k0)` is the global address of stage row r at K offset k0.
// Rows are packed in the stage at r * seglen. With a single K segment, runs
// of rows that are adjacent in global memory go out as one copy.
// Returns the number of positions issued.
// ---------------------------------------------------------------------------
template <class RowsFn, class SrcFn>
__device__ __forceinline__ int produce(uint32_t full0, uint32_t empty0, uint32_t stage0,
                                       int nstages, int total, int nseg, int64_t K,
                                       RowsFn rows_of, SrcFn src_of, unsigned int site) {
  const uint64_t pol = l2_evict_first_policy();
  int pos = 0;
  for (; pos < total; ++pos) {
    const int s = pos % nstages;
    const int use = pos / nstages;
    if (use > 0 && !mbar_wait(empty0 + 8 * s, (use - 1) & 1)) {
      report_error(ERR_WAIT_EMPTY, site);
      break;
    }
    const int seg = pos % nseg;
    const int64_t k0 = static_cast<int64_t>(seg) * kSeg;
    const int sl = static_cast<int>(min64(kSeg, K - k0));
    const uint32_t dst = stage0 + s * kStageBytes;
    const uint32_t mask = rows_of(pos);
    const uint32_t bytes = static_cast<uint32_t>(__popc(mask)) * sl;
    mbar_arrive_expect_tx(full0 + 8 * s, bytes);
    if (nseg == 1) {
      // Whole rows: coalesce runs of adjacent valid rows into one copy.
      int r = 0;
      while (r < kRW) {
        if (!((mask >> r) & 1u)) { ++r; continue; }
        const char* base = static_cast<const char*>(src_of(pos, r, 0));
        int run = 1;
        while (r + run < kRW && ((mask >> (r + run)) & 1u) &&
               static_cast<const char*>(src_of(pos, r + run, 0)) == base + run * K)
          ++run;
        bulk_g2s(dst + r * sl, base, static_cast<uint32_t>(run * sl), full0 + 8 * s, pol);
        r += run;
      }
    } else {
#pragma unroll 1
      for (int r = 0; r < kRW; ++r)
        if ((mask >> r) & 1u)
          bulk_g2s(dst + r * sl, src_of(pos, r, k0), static_cast<uint32_t>(sl), full0 + 8 * s, pol);
    }
  }
  return pos;
}

// Wait (bounded) until every copy issued for positions [issued - nstages, issued)
// has landed, so that no bulk copy is still writing this CTA's shared memory
// when it exits. On the normal path these phases completed long ago.
__device__ __forceinline__ void drain(uint32_t full0, int nstages, int issued, unsigned int site) {
  for (int pos = max(0, issued - nstages); pos < issued; ++pos)
    if (!mbar_wait(full0 + 8 * (pos % nstages), (pos / nstages) & 1)) {
      report_error(ERR_DRAIN, site);
      return;
    }
}

// ---------------------------------------------------------------------------
// Consumer core: one row group (8 rows) over all nseg segments starting at
// stage position pos0. PER_ROW (ng == 1): fp32 pair accumulators, scale applied
// by the caller. Otherwise each 16-element chunk's sum is weighted by the scale
// of its group (G % 16 == 0 so a chunk never straddles two groups).
// Returns false if a wait gave up.
// ---------------------------------------------------------------------------
template <bool PER_ROW, class ScaleFn>
__device__ __forceinline__ bool consume_group(uint32_t full0, uint32_t empty0, uint32_t stage0,
                                              uint32_t xs_base, int nstages, int pos0, int nseg,
                                              int64_t K, int64_t G, int lane, ScaleFn scale_of,
                                              float (&v)[8], unsigned int site) {
  const int64_t nch_all = K / 16;
  f2_t acc[kRW];
  float accs[kRW];
#pragma unroll
  for (int r = 0; r < kRW; ++r) { acc[r] = 0ull; accs[r] = 0.f; }
  bool ok = true;
  for (int seg = 0; seg < nseg; ++seg) {
    const int pos = pos0 + seg;
    const int s = pos % nstages;
    ok = mbar_wait(full0 + 8 * s, (pos / nstages) & 1);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) {
      if (lane == 0) report_error(ERR_WAIT_FULL, site);
      break;
    }
    const int64_t k0 = static_cast<int64_t>(seg) * kSeg;
    const int sl = static_cast<int>(min64(kSeg, K - k0));
    const int nch = sl / 16;
    const int64_t c0 = k0 / 16;
    const uint32_t st = stage0 + s * kStageBytes;
#pragma unroll 1
    for (int c = lane; c < nch; c += 32) {
      f2_t xv[8];
      load_x16(xs_base, nch_all, c0 + c, xv);
      if (PER_ROW) {
#pragma unroll
        for (int r = 0; r < kRW; ++r) {
          const uint4 qv = lds128(st + r * sl + c * 16);
          dot16_acc(qv, xv, acc[r]);
        }
      } else {
        const int64_t g = ((c0 + c) * 16) / G;
#pragma unroll
        for (int r = 0; r < kRW; ++r) {
          const uint4 qv = lds128(st + r * sl + c * 16);
          f2_t d = 0ull;
          dot16_acc(qv, xv, d);
          const float2 p = f2_unpack(d);
          accs[r] = fmaf(p.x + p.y, scale_of(r, g), accs[r]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8 * s);
  }
#pragma unroll
  for (int r = 0; r < kRW; ++r) {
    if (PER_ROW) {
      const float2 p = f2_unpack(acc[r]);
      v[r] = p.x + p.y;
    } else {
      v[r] = accs[r];
    }
  }
  return ok;
}

// ---------------------------------------------------------------------------
// GEMV
// ---------------------------------------------------------------------------
template <bool PER_ROW>
__global__ void __launch_bounds__(kThreads, 1) gemv_stream_kernel(const GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t full0 = smem_u32(smem), empty0 = full0 + 8 * kMaxStages;
  float* xs = reinterpret_cast<float*>(smem + kSmemHeader);
  const uint32_t xs_base = smem_u32(xs);
  const uint32_t stage0 = xs_base + stream_x_bytes(a.K);

  const int64_t n_rg = cdiv(a.N, kRW);
  const int64_t rg_begin = n_rg * blockIdx.x / gridDim.x;
  const int64_t rg_end = n_rg * (blockIdx.x + 1) / gridDim.x;
  const int n_loc = static_cast<int>(rg_end - rg_begin);
  const int nseg = static_cast<int>(cdiv(a.K, kSeg));
  const int64_t G = a.K / a.ng;

  if (tid == 0) {
    for (int s = 0; s < a.nstages; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    fence_mbar_init();
  }
  if (warp < kConsumerWarps) stage_x(xs, a.x, a.K, tid, kConsumerWarps * 32);
  __syncthreads();

  if (warp == kConsumerWarps) {
    if (lane == 0) {
      const int8_t* q = a.q;
      const int64_t N = a.N, K = a.K;
      auto rows_of = [&](int pos) -> uint32_t {
        const int64_t row0 = (rg_begin + pos / nseg) * kRW;
        const int64_t rows = min64(kRW, N - row0);
        return (1u << rows) - 1u;
      };
      auto src_of = [&](int pos, int r, int64_t k0) -> const void* {
        const int64_t row = (rg_begin + pos / nseg) * kRW + r;
        return q + row * K + k0;
      };
      const int issued = produce(full0, empty0, stage0, a.nstages, n_loc * nseg, nseg, K, rows_of,
                                 src_of, 0x100u);
      drain(full0, a.nstages, issued, 0x101u);
    }
    return;
  }

  for (int rgl = warp; rgl < n_loc; rgl += kConsumerWarps) {
    const int64_t row0 = (rg_begin + rgl) * kRW;
    auto scale_of = [&](int r, int64_t g) -> float {
      const int64_t row = row0 + r;
      return row < a.N ? __ldg(a.scale + row * a.ng + g) : 0.f;
    };
    float v[8];
    if (!consume_group<PER_ROW>(full0, empty0, stage0, xs_base, a.nstages, rgl * nseg, nseg, a.K,
                                G, lane, scale_of, v, 0x102u))
      return;
    const float sum = warp_reduce8(v, lane);
    const int64_t row = row0 + ((lane >> 2) & 7);
    if ((lane & 3) == 0 && row < a.N) {
      float o = PER_ROW ? sum * __ldg(a.scale + row) : sum;
      if (a.residual) o += a.residual[row];
      a.y[row] = o;
    }
  }
}

// ---------------------------------------------------------------------------
// Fused MLP (M = 1). Phase 1: a row group is 4 intermediate units = 4 gate rows
// (stage rows 0-3) + the matching 4 up rows (stage rows 4-7); the epilogue
// writes abuf[n] = silu(gate_n . x) * (up_n . x). A grid-wide barrier (bounded
// spin on a generation counter; the launch is cooperative so every CTA is
// resident) separates it from phase 2, the down GEMV over abuf with the
// residual fused. The producer does not wait at the barrier: it keeps
// streaming this CTA's down rows into free stages, so phase 2's weights are
// already in flight while phase 1 drains.
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool grid_barrier(unsigned int* ws, int tid, unsigned int site) {
  __shared__ unsigned int s_fail;
  named_bar_sync(1, kConsumerWarps * 32);
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
      }
    }
  }
  named_bar_sync(1, kConsumerWarps * 32);
  return s_fail == 0u;
}

template <bool PER_ROW>
__global__ void __launch_bounds__(kThreads, 1) fused_mlp_kernel(const MlpArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t full0 = smem_u32(smem), empty0 = full0 + 8 * kMaxStages;
  float* xs = reinterpret_cast<float*>(smem + kSmemHeader);
  const uint32_t xs_base = smem_u32(xs);
  const uint32_t stage0 = xs_base + stream_x_bytes(a.H > a.I ? a.H : a.I);

  const int64_t H = a.H, I = a.I;
  constexpr int kUnits = kRW / 2;
  const int64_t n_ug = cdiv(I, kUnits);
  const int64_t ug_begin = n_ug * blockIdx.x / gridDim.x;
  const int n1 = static_cast<int>(n_ug * (blockIdx.x + 1) / gridDim.x - ug_begin);
  const int64_t n_rg = cdiv(H, kRW);
  const int64_t rg_begin = n_rg * blockIdx.x / gridDim.x;
  const int n2 = static_cast<int>(n_rg * (blockIdx.x + 1) / gridDim.x - rg_begin);
  const int nseg1 = static_cast<int>(cdiv(H, kSeg));
  const int nseg2 = static_cast<int>(cdiv(I, kSeg));
  const int base2 = n1 * nseg1;
  const int64_t G1 = H / a.ng, G2 = I / a.ngd;

  if (tid == 0) {
    for (int s = 0; s < a.nstages; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    fence_mbar_init();
  }
  if (warp < kConsumerWarps) stage_x(xs, a.x, H, tid, kConsumerWarps * 32);
  __syncthreads();

  if (warp == kConsumerWarps) {
    if (lane == 0) {
      // Phase 1 then phase 2 positions in one sequence; each phase's copies
      // use that phase's K (H, then I).
      auto rows1 = [&](int pos) -> uint32_t {
        const int64_t u0 = (ug_begin + pos / nseg1) * kUnits;
        const int64_t units = min64(kUnits, I - u0);
        const uint32_t m = (1u << units) - 1u;
        return m | (m << kUnits);
      };
      auto src1 = [&](int pos, int r, int64_t k0) -> const void* {
        const int64_t u0 = (ug_begin + pos / nseg1) * kUnits;
        const int64_t row = r < kUnits ? u0 + r : I + u0 + (r - kUnits);
        return a.gu_q + row * H + k0;
      };
      int issued = produce(full0, empty0, stage0, a.nstages, base2, nseg1, H, rows1, src1, 0x200u);
      if (issued == base2) {
        // Phase 2 continues the same ring: shift positions by base2.
        auto rows2 = [&](int p) -> uint32_t {
          const int64_t row0 = (rg_begin + p / nseg2) * kRW;
          const int64_t rows = min64(kRW, H - row0);
          return (1u << rows) - 1u;
        };
        auto src2 = [&](int p, int r, int64_t k0) -> const void* {
          const int64_t row = (rg_begin + p / nseg2) * kRW + r;
          return a.down_q + row * I + k0;
        };
        // produce() numbers positions from 0; run it on a shifted ring view.
        const uint64_t pol = l2_evict_first_policy();
        const int total2 = n2 * nseg2;
        for (int p = 0; p < total2; ++p) {
          const int pos = base2 + p;
          const int s = pos % a.nstages;
          const int use = pos / a.nstages;
          if (use > 0 && !mbar_wait(empty0 + 8 * s, (use - 1) & 1)) {
            report_error(ERR_WAIT_EMPTY, 0x203u);
            break;
          }
          const int seg = p % nseg2;
          const int64_t k0 = static_cast<int64_t>(seg) * kSeg;
          const int sl = static_cast<int>(min64(kSeg, I - k0));
          const uint32_t mask = rows2(p);
          const uint32_t dst = stage0 + s * kStageBytes;
          mbar_arrive_expect_tx(full0 + 8 * s, static_cast<uint32_t>(__popc(mask)) * sl);
          if (nseg2 == 1) {
            bulk_g2s(dst, src2(p, 0, 0), static_cast<uint32_t>(__popc(mask) * sl), full0 + 8 * s, pol);
          } else {
#pragma unroll 1
            for (int r = 0; r < kRW; ++r)
              if ((mask >> r) & 1u)
                bulk_g2s(dst + r * sl, src2(p, r, k0), static_cast<uint32_t>(sl), full0 + 8 * s, pol);
          }
          ++issued;
        }
      }
      drain(full0, a.nstages, issued, 0x201u);
    }
    return;
  }

  // ---- phase 1: gate/up GEMV pair + SiLU gate ----
  bool ok = true;
  for (int ugl = warp; ugl < n1; ugl += kConsumerWarps) {
    const int64_t u0 = (ug_begin + ugl) * kUnits;
    auto scale_of = [&](int r, int64_t g) -> float {
      const int64_t unit = u0 + (r & (kUnits - 1));
      if (unit >= I) return 0.f;
      const int64_t row = r < kUnits ? unit : I + unit;
      return __ldg(a.gu_s + row * a.ng + g);
    };
    float v[8];
    if (!consume_group<PER_ROW>(full0, empty0, stage0, xs_base, a.nstages, ugl * nseg1, nseg1, H,
                                G1, lane, scale_of, v, 0x204u)) {
      ok = false;
      break;
    }
    const float sum = warp_reduce8(v, lane);
    const float up = __shfl_down_sync(0xffffffffu, sum, 16);
    const int64_t unit = u0 + (lane >> 2);
    if (lane < 16 && (lane & 3) == 0 && unit < I) {
      const float ga = PER_ROW ? sum * __ldg(a.gu_s + unit) : sum;
      const float ua = PER_ROW ? up * __ldg(a.gu_s + I + unit) : up;
      a.abuf[unit] = ga / (1.0f + expf(-ga)) * ua;
    }
  }
  // A warp that gave up still takes part in the CTA-level barriers below so
  // the others are not left waiting; it just skips phase 2's work.
  if (!grid_barrier(a.sync_ws, tid, 0x205u)) ok = false;
  // ---- phase 2: down GEMV over abuf ----
  stage_x<true>(xs, a.abuf, I, tid, kConsumerWarps * 32);
  named_bar_sync(1, kConsumerWarps * 32);
  if (!ok) return;
  for (int rgl = warp; rgl < n2; rgl += kConsumerWarps) {
    const int64_t row0 = (rg_begin + rgl) * kRW;
    auto scale_of = [&](int r, int64_t g) -> float {
      const int64_t row = row0 + r;
      return row < H ? __ldg(a.down_s + row * a.ngd + g) : 0.f;
    };
    float v[8];
    if (!consume_group<PER_ROW>(full0, empty0, stage0, xs_base, a.nstages, base2 + rgl * nseg2,
                                nseg2, I, G2, lane, scale_of, v, 0x206u))
      return;
    const float sum = warp_reduce8(v, lane);
    const int64_t row = row0 + ((lane >> 2) & 7);
    if ((lane & 3) == 0 && row < H) {
      float o = PER_ROW ? sum * __ldg(a.down_s + row) : sum;
      if (a.residual) o += a.residual[row];
      a.out[row] = o;
    }
  }
}

}  // namespace qz
