// qz_decode.cuh -- the device-side glue of an all-int8 decode step around the
// int8 matmuls: everything quartz's decoder does between its QuantizedLinear
// calls, so a whole token can run on the GPU (and inside one CUDA graph).
//
//   embed_gather_kernel   int8 embedding row gather + dequant    quartz/quantize.py:78-80, 41-48
//   rmsnorm_kernel        x / sqrt(mean(x^2) + eps) * w          quartz/ops.py:24-32
//   qk_rope_kernel        per-head q/k RMSNorm (Qwen3), half-split
//                         RoPE, K/V append to the cache          quartz/models/qwen3.py:31-41,
//                                                                quartz/rope.py:47-78,
//                                                                quartz/cache.py:26-46
//   attn_decode_kernel +  one query per head over the cache,     quartz/attention.py:29-43
//   attn_combine_kernel   context split in chunks, GQA by repeat
//   attn_prefill_kernel   M queries, causal, online softmax       quartz/attention.py:15-43
//   argmax_kernel         greedy token, first index of the max   quartz/sample.py:21-22
//
// All arithmetic is fp32 like the reference. Layouts: activations row-major
// [M, features]; the KV cache of one layer is [n_kv, max_ctx, head_dim].
#pragma once

#include "qz_device.cuh"
#include "qz_stream.cuh"

namespace qz {
namespace dec {

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum for blockDim.x <= 1024 (every thread gets the result).
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum_f(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = (blockDim.x + 31) >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < nw; ++i) s += red[i];
  return s;
}

// out[m, h] = (float)q[id_m, h] * scale[id_m, h / G]
__global__ void embed_gather_kernel(const int8_t* __restrict__ q, const float* __restrict__ scale,
                                    int64_t ng, const int64_t* __restrict__ ids, int64_t V,
                                    int64_t H, float* __restrict__ out) {
  const int64_t m = blockIdx.x;
  int64_t id = ids[m];
  id = id < 0 ? 0 : (id >= V ? V - 1 : id);   // ids are validated on the host; stay in bounds
  const int64_t G = H / ng;
  for (int64_t h = threadIdx.x; h < H; h += blockDim.x)
    out[m * H + h] = static_cast<float>(q[id * H + h]) * scale[id * ng + h / G];
}

// One block per row: y = x * (1 / sqrt(mean(x^2) + eps)) * w. The first
// kNormPer x kNormThreads elements (4096) are loaded in one unrolled round
// (x and w together) and kept in registers, so a row costs one memory round
// trip instead of one per loop iteration.
constexpr int kNormThreads = 512;
constexpr int kNormPer = 8;
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const float* __restrict__ x,
                                                               const float* __restrict__ w,
                                                               float* __restrict__ y, int64_t n,
                                                               float eps) {
  __shared__ float red[32];
  const float* xr = x + blockIdx.x * n;
  float* yr = y + blockIdx.x * n;
  constexpr int64_t kBatch = static_cast<int64_t>(kNormPer) * kNormThreads;
  float v[kNormPer], wv[kNormPer];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kNormPer; ++k) {
    const int64_t i = threadIdx.x + static_cast<int64_t>(k) * kNormThreads;
    v[k] = i < n ? xr[i] : 0.f;
    wv[k] = i < n ? w[i] : 0.f;
    ss = fmaf(v[k], v[k], ss);
  }
  for (int64_t base = kBatch; base < n; base += kBatch) {
#pragma unroll
    for (int k = 0; k < kNormPer; ++k) {
      const int64_t i = base + threadIdx.x + static_cast<int64_t>(k) * kNormThreads;
      const float t = i < n ? xr[i] : 0.f;
      ss = fmaf(t, t, ss);
    }
  }
  ss = block_sum(ss, red);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(n) + eps);
#pragma unroll
  for (int k = 0; k < kNormPer; ++k) {
    const int64_t i = threadIdx.x + static_cast<int64_t>(k) * kNormThreads;
    if (i < n) yr[i] = v[k] * r * wv[k];
  }
  for (int64_t i = kBatch + threadIdx.x; i < n; i += kNormThreads) yr[i] = xr[i] * r * w[i];
}

// qkv: [M, (nq + 2 nkv) * hd] (q heads, k heads, v heads). One block per
// (row m, head): q and k heads get the optional per-head RMSNorm then RoPE at
// position pos0 + m; q goes to q_out [M, nq * hd], k and v to the cache.
// pos_dev (if not null) overrides pos0: the position read from device memory,
// so a captured graph can be replayed at successive positions.
__global__ void qk_rope_kernel(const float* __restrict__ qkv, const float* __restrict__ qn_w,
                               const float* __restrict__ kn_w, const float* __restrict__ inv_freq,
                               float* __restrict__ q_out, float* __restrict__ kc,
                               float* __restrict__ vc, int nq, int nkv, int hd, int64_t max_ctx,
                               int64_t pos0, const int64_t* __restrict__ pos_dev, float eps) {
  extern __shared__ float sh[];   // hd floats
  __shared__ float red[32];
  const int64_t m = blockIdx.x;
  const int head = blockIdx.y;
  const int width = (nq + 2 * nkv) * hd;
  const float* src = qkv + m * width + head * hd;
  const int64_t pos = (pos_dev ? *pos_dev : pos0) + m;
  if (pos < 0 || pos >= max_ctx) return;   // the host checks; never write outside the cache
  const bool is_q = head < nq, is_k = !is_q && head < nq + nkv;
  if (!is_q && !is_k) {   // v head: copy into the cache
    const int vh = head - nq - nkv;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) vc[(vh * max_ctx + pos) * hd + i] = src[i];
    return;
  }
  const float* nw = is_q ? qn_w : kn_w;
  for (int i = threadIdx.x; i < hd; i += blockDim.x) sh[i] = src[i];
  if (nw) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) ss = fmaf(src[i], src[i], ss);
    ss = block_sum(ss, red);
    const float r = 1.0f / sqrtf(ss / static_cast<float>(hd) + eps);
    __syncthreads();
    for (int i = threadIdx.x; i < hd; i += blockDim.x) sh[i] = src[i] * r * nw[i];
  }
  __syncthreads();
  const int d = hd / 2;
  float* dst = is_q ? q_out + (m * nq + head) * hd
                    : kc + ((head - nq) * max_ctx + pos) * hd;
  const float fpos = static_cast<float>(pos);
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    const float ang = fpos * inv_freq[j];
    const float c = cosf(ang), s = sinf(ang);
    const float x1 = sh[j], x2 = sh[j + d];
    dst[j] = x1 * c - x2 * s;
    dst[j + d] = x2 * c + x1 * s;
  }
}

// Decode attention, one query per head. Block (kv head g, chunk c) covers cache
// positions [c*C, min(T, (c+1)*C)) for the n_rep query heads g*n_rep .. g*n_rep
// + n_rep - 1 (quartz repeats each kv head to n_rep adjacent query heads). It
// writes, per query head, the chunk's max score, sum of exp and exp-weighted
// V sum; attn_combine_kernel merges the chunks.
// part layout: [nq][nchunks][hd + 2]  (acc[hd], max, sum)
// T_dev (if not null) overrides T (context length read from device memory);
// chunks at or past T write empty partials.
constexpr int kChunk = 64;
__global__ void __launch_bounds__(256) attn_decode_kernel(
    const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
    float* __restrict__ part, int nq, int nkv, int hd, int64_t max_ctx, int64_t T,
    const int64_t* __restrict__ T_dev, int64_t t_offset, float scale) {
  extern __shared__ float sm[];
  const int g = blockIdx.x, c = blockIdx.y;
  const int n_rep = nq / nkv;
  const int nchunks = gridDim.y;
  float* qs = sm;                        // [n_rep][hd]
  float* ps = qs + n_rep * hd;           // [n_rep][kChunk] scores -> probabilities
  if (T_dev) T = *T_dev + t_offset;
  T = T > max_ctx ? max_ctx : T;
  const int64_t t0 = static_cast<int64_t>(c) * kChunk;
  const int nt = static_cast<int>(min64(kChunk, T - t0));
  if (nt <= 0) {
    for (int i = threadIdx.x; i < n_rep * (hd + 2); i += blockDim.x) {
      const int r = i / (hd + 2), j = i - r * (hd + 2);
      float* pr = part + ((static_cast<int64_t>(g * n_rep + r) * nchunks + c) * (hd + 2));
      pr[j] = j == hd ? -INFINITY : 0.f;
    }
    return;
  }
  for (int i = threadIdx.x; i < n_rep * hd; i += blockDim.x) qs[i] = q[g * n_rep * hd + i];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const float* kg = kc + (static_cast<int64_t>(g) * max_ctx) * hd;
  const float* vg = vc + (static_cast<int64_t>(g) * max_ctx) * hd;
  for (int t = warp; t < nt; t += nw) {
    const float* kr = kg + (t0 + t) * hd;
    for (int r = 0; r < n_rep; ++r) {
      float s = 0.f;
      for (int i = lane; i < hd; i += 32) s = fmaf(qs[r * hd + i], kr[i], s);
      s = warp_sum_f(s);
      if (lane == 0) ps[r * kChunk + t] = s * scale;
    }
  }
  __syncthreads();
  __shared__ float mx_s[32], sum_s[32];
  if (warp < n_rep) {
    float m = -INFINITY;
    for (int t = lane; t < nt; t += 32) m = fmaxf(m, ps[warp * kChunk + t]);
    m = warp_max_f(m);
    float sum = 0.f;
    for (int t = lane; t < nt; t += 32) {
      const float e = expf(ps[warp * kChunk + t] - m);
      ps[warp * kChunk + t] = e;
      sum += e;
    }
    sum = warp_sum_f(sum);
    if (lane == 0) { mx_s[warp] = m; sum_s[warp] = sum; }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n_rep * hd; i += blockDim.x) {
    const int r = i / hd, dd = i - r * hd;
    float acc = 0.f;
    for (int t = 0; t < nt; ++t) acc = fmaf(ps[r * kChunk + t], vg[(t0 + t) * hd + dd], acc);
    float* pr = part + ((static_cast<int64_t>(g * n_rep + r) * nchunks + c) * (hd + 2));
    pr[dd] = acc;
    if (dd == 0) { pr[hd] = mx_s[r]; pr[hd + 1] = sum_s[r]; }
  }
}

// out[h, d] = sum_c exp(m_c - M) acc_c[d] / sum_c exp(m_c - M) l_c  (one block per query head)
__global__ void attn_combine_kernel(const float* __restrict__ part, float* __restrict__ out,
                                    int hd, int nchunks) {
  const int h = blockIdx.x;
  const float* ph = part + static_cast<int64_t>(h) * nchunks * (hd + 2);
  float M = -INFINITY;
  for (int c = 0; c < nchunks; ++c) M = fmaxf(M, ph[c * (hd + 2) + hd]);
  float den = 0.f;
  for (int c = 0; c < nchunks; ++c) {
    const float mc = ph[c * (hd + 2) + hd];
    if (mc != -INFINITY) den += expf(mc - M) * ph[c * (hd + 2) + hd + 1];
  }
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float num = 0.f;
    for (int c = 0; c < nchunks; ++c) {
      const float mc = ph[c * (hd + 2) + hd];
      if (mc != -INFINITY) num += expf(mc - M) * ph[c * (hd + 2) + d];
    }
    out[static_cast<int64_t>(h) * hd + d] = num / den;
  }
}

// Tiled causal prefill attention (fp32 on the CUDA cores, like the reference's
// numpy attention). CTA (row block, kv head g) owns BM query rows of the NR
// query heads of g: 128 threads, TPQ = HD / 32 threads per (row, head) query,
// each holding 32 of its dimensions in registers (q and the accumulator). Key
// tiles of BN rows of K and V are double-buffered in shared memory with
// cp.async (the TPQ slices of a row interleaved float4 by float4, so a
// query's threads hit distinct banks) and read as broadcasts; per tile a thread computes its BN scores
// (four keys at a time, so four dot products are in flight), rescales its
// running accumulator once by e^(m_old - m_new), then adds e^(s - m_new) v.
// Keys after a query's own position get probability 0.
constexpr int kPfThreads = 128;
constexpr int kPfBN = 32;
constexpr int kPfDims = 32;   // dimensions per thread

template <int HD, int NR>
__global__ void __launch_bounds__(kPfThreads) attn_prefill_tiled_kernel(
    const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
    float* __restrict__ out, int64_t M, int nq, int64_t max_ctx, int64_t pos0, float scale) {
  constexpr int DP = kPfDims;
  constexpr int TPQ = HD / DP;
  constexpr int QPC = kPfThreads / TPQ;
  constexpr int BM = QPC / NR;
  constexpr int BN = kPfBN;
  constexpr int TILE = BN * HD;                 // floats per K (or V) tile
  extern __shared__ float4 pf_smem4[];
  float* sm = reinterpret_cast<float*>(pf_smem4);   // [2 stages][K tile | V tile]
  const int g = blockIdx.y;
  const int tid = threadIdx.x;
  const int qi = tid / TPQ, part = tid % TPQ;
  const int rr = qi / BM, i = qi % BM;          // head within the group, row within the block
  const int64_t row = static_cast<int64_t>(blockIdx.x) * BM + i;
  const bool valid = row < M;
  const int h = g * NR + rr;
  const int64_t p = pos0 + (valid ? row : 0);   // this query's position
  const int64_t last_row = min64(M, static_cast<int64_t>(blockIdx.x + 1) * BM) - 1;
  const int64_t t_end = pos0 + last_row + 1;    // keys this CTA needs: [0, t_end)
  const float* kg = kc + static_cast<int64_t>(g) * max_ctx * HD;
  const float* vg = vc + static_cast<int64_t>(g) * max_ctx * HD;

  float qv[DP], acc[DP];
  {
    const float* src = q + (static_cast<int64_t>(valid ? row : 0) * nq + h) * HD + part * DP;
#pragma unroll
    for (int d = 0; d < DP; d += 4) {
      const float4 v = *reinterpret_cast<const float4*>(src + d);
      qv[d] = v.x; qv[d + 1] = v.y; qv[d + 2] = v.z; qv[d + 3] = v.w;
    }
  }
#pragma unroll
  for (int d = 0; d < DP; ++d) acc[d] = 0.f;
  float m = -INFINITY, l = 0.f;

  const int ntiles = static_cast<int>(cdiv(t_end, BN));
  auto load_tile = [&](int tile, int stage) {
    const int64_t t0 = static_cast<int64_t>(tile) * BN;
    float* kd = sm + stage * 2 * TILE;
    float* vd = kd + TILE;
    for (int c = tid; c < TILE / 4; c += kPfThreads) {
      const int j = c / (HD / 4), f = c % (HD / 4);   // row, float4 of the row
      const int64_t t = min64(t0 + j, t_end - 1);   // rows past t_end: any valid row (masked)
      const int64_t off = t * HD + f * 4;
      // float4 f = (slice f / (DP/4), chunk f % (DP/4)) goes to chunk * TPQ + slice, so the
      // TPQ threads of a query read adjacent 16-byte words (distinct banks)
      const int dst = j * HD + ((f % (DP / 4)) * TPQ + f / (DP / 4)) * 4;
      cp_async16(smem_u32(kd + dst), kg + off);
      cp_async16(smem_u32(vd + dst), vg + off);
    }
    cp_async_commit();
  };
  load_tile(0, 0);
  for (int tile = 0; tile < ntiles; ++tile) {
    const int stage = tile & 1;
    if (tile + 1 < ntiles) {
      load_tile(tile + 1, stage ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const float* ks = sm + stage * 2 * TILE + part * 4;   // chunk c of this slice at c * TPQ * 4
    const float* vs = ks + TILE;
    const int64_t t0 = static_cast<int64_t>(tile) * BN;
    float sc[BN];
    float mt = -INFINITY;
#pragma unroll
    for (int j = 0; j < BN; j += 4) {
      float dd[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int d = 0; d < DP; d += 4) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float4 k4 = *reinterpret_cast<const float4*>(ks + (j + u) * HD + d * TPQ);
          dd[u] = fmaf(qv[d], k4.x, dd[u]);
          dd[u] = fmaf(qv[d + 1], k4.y, dd[u]);
          dd[u] = fmaf(qv[d + 2], k4.z, dd[u]);
          dd[u] = fmaf(qv[d + 3], k4.w, dd[u]);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float s = dd[u];
#pragma unroll
        for (int o = 1; o < TPQ; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        s = t0 + j + u <= p ? s * scale : -INFINITY;
        sc[j + u] = s;
        mt = fmaxf(mt, s);
      }
    }
    const float mn = fmaxf(m, mt);
    const float corr = expf(m - mn);   // m = -inf on the first tile: corr = 0
    l *= corr;
#pragma unroll
    for (int d = 0; d < DP; ++d) acc[d] *= corr;
#pragma unroll
    for (int j = 0; j < BN; ++j) {
      const float pj = expf(sc[j] - mn);
      l += pj;
#pragma unroll
      for (int d = 0; d < DP; d += 4) {
        const float4 v4 = *reinterpret_cast<const float4*>(vs + j * HD + d * TPQ);
        acc[d] = fmaf(pj, v4.x, acc[d]);
        acc[d + 1] = fmaf(pj, v4.y, acc[d + 1]);
        acc[d + 2] = fmaf(pj, v4.z, acc[d + 2]);
        acc[d + 3] = fmaf(pj, v4.w, acc[d + 3]);
      }
    }
    m = mn;
    __syncthreads();   // the stage is refilled two tiles later
  }
  if (valid) {
    float* dst = out + (row * nq + h) * HD + part * DP;
    const float inv = 1.0f / l;
#pragma unroll
    for (int d = 0; d < DP; d += 4)
      *reinterpret_cast<float4*>(dst + d) =
          make_float4(acc[d] * inv, acc[d + 1] * inv, acc[d + 2] * inv, acc[d + 3] * inv);
  }
}

template <int HD>
constexpr int prefill_tiled_smem() { return 2 * 2 * kPfBN * HD * 4; }

// Prefill attention: query rows m (position pos0 + m) attend to cache positions
// [0, pos0 + m] (causal). One warp per (row m, query head); online softmax
// over the keys; hd <= 256.
__global__ void __launch_bounds__(256) attn_prefill_kernel(
    const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
    float* __restrict__ out, int64_t M, int nq, int nkv, int hd, int64_t max_ctx, int64_t pos0,
    float scale) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (wid >= M * nq) return;
  const int64_t m = wid / nq;
  const int h = static_cast<int>(wid - m * nq);
  const int g = h / (nq / nkv);
  const int per = (hd + 31) / 32;   // <= 8
  float qv[8], acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int i = lane + 32 * j;
    qv[j] = (j < per && i < hd) ? q[(m * nq + h) * hd + i] : 0.f;
    acc[j] = 0.f;
  }
  const float* kg = kc + static_cast<int64_t>(g) * max_ctx * hd;
  const float* vg = vc + static_cast<int64_t>(g) * max_ctx * hd;
  float mrun = -INFINITY, lrun = 0.f;
  const int64_t T = pos0 + m + 1;
  for (int64_t t = 0; t < T; ++t) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = lane + 32 * j;
      if (j < per && i < hd) s = fmaf(qv[j], kg[t * hd + i], s);
    }
    s = warp_sum_f(s) * scale;
    const float mnew = fmaxf(mrun, s);
    const float corr = expf(mrun - mnew);
    const float p = expf(s - mnew);
    lrun = lrun * corr + p;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = lane + 32 * j;
      if (j < per && i < hd) acc[j] = acc[j] * corr + p * vg[t * hd + i];
    }
    mrun = mnew;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int i = lane + 32 * j;
    if (j < per && i < hd) out[(m * nq + h) * hd + i] = acc[j] / lrun;
  }
}

// ---------------------------------------------------------------------------
// Fused decode attention, one query row: split-context (flash-decoding) with
// the q/k preparation and the KV append folded in and the cross-CTA merge done
// by the last CTA to finish (an atomic ticket per kv head; nothing waits).
//
// Grid (n_kv, S). CTA (g, c) owns the kv head g, its NR = nq / nkv query heads
// g*NR .. g*NR + NR - 1 (quartz repeats each kv head to NR adjacent query
// heads, quartz/attention.py:36-38), and the cache positions
// [c * per, min(T, (c + 1) * per)), per = ceil(T / S) rounded up to 8. The
// context length T is read on the device, so one captured launch serves every
// position.
//
// With QKV the input is the raw projection row [(nq + 2 nkv) hd]: every CTA
// normalises (Qwen3's per-head RMSNorm, quartz/models/qwen3.py:33-34) and
// rotates (half-split RoPE, quartz/rope.py:47-78) its query heads; the CTA
// owning position T - 1 also prepares that position's key and value and
// appends them to the cache before reading it (quartz/cache.py:26-46).
// Without QKV the input is q [nq hd], already rotated, and the cache is read only.
//
// Lane l of a warp holds head elements [l E, l E + E) (hd = 32 E), so the
// RoPE partner of element i < hd/2, element i + hd/2, is in lane l ^ 16.
// Each warp runs an online softmax over every 8th position of the CTA's range,
// U positions per round; the 8 warps merge in shared memory into one partial
// (acc[hd], max, sum) per query head, written to the workspace.
// ---------------------------------------------------------------------------
// Merge S partial softmaxes (acc[HD], max, sum per query head; layout
// [S][NR][HD + 2]) of the NR query heads of one kv head into out [NR][HD]:
// out = sum_c e^(m_c - M) acc_c / sum_c e^(m_c - M) l_c. Threads tid < NT
// take part; sync() is their barrier; scratch holds 2 NR S + NR floats. Two
// dependent rounds of L2 loads: all maxima and sums at once, then the
// accumulators, whose loads are independent of one another so they overlap.
// Splits whose partial accumulators the merge holds in registers.
constexpr int kMergeRegs = 32;

// REGS: with at most kMergeRegs splits and two outputs per thread, every
// thread loads its outputs' partial accumulators together with the maxima and
// sums, one round of L2 loads instead of one per eight splits (off in callers
// whose register budget is tight).
template <int HD, int NR, int NT, class Sync, bool REGS = true>
__device__ __forceinline__ void merge_partials(const float* part_g, int S, float* out_g,
                                               float* scratch, int tid, Sync&& sync) {
  constexpr int NW = NT / 32;
  constexpr int OPT = (NR * HD + NT - 1) / NT;     // outputs per thread
  constexpr bool REG = REGS && OPT <= 2;
  const int warp = tid >> 5, lane = tid & 31;
  float* wf = scratch;                // [NR][S] maxima, then weights
  float* lf = scratch + NR * S;       // [NR][S] sums
  float* dn = scratch + 2 * NR * S;   // [NR]
  constexpr int64_t stride = static_cast<int64_t>(NR) * (HD + 2);
  float acc_v[REG ? OPT : 1][kMergeRegs];
  if constexpr (REG) {
    if (S <= kMergeRegs) {
#pragma unroll
      for (int k = 0; k < OPT; ++k) {
        const int i = tid + k * NT;
        const int r = i / HD, d = i - r * HD;
        const float* pr = part_g + r * (HD + 2) + d;
#pragma unroll
        for (int c = 0; c < kMergeRegs; ++c)
          acc_v[k][c] = (i < NR * HD && c < S) ? __ldcg(pr + c * stride) : 0.f;
      }
    }
  }
  for (int i = tid; i < NR * S; i += NT) {
    const int r = i / S, c = i - r * S;
    const float* pr = part_g + (static_cast<int64_t>(c) * NR + r) * (HD + 2) + HD;
    wf[i] = __ldcg(pr);
    lf[i] = __ldcg(pr + 1);
  }
  sync();
  for (int r = warp; r < NR; r += NW) {
    float M = -INFINITY;
    for (int c = lane; c < S; c += 32) M = fmaxf(M, wf[r * S + c]);
    M = warp_max_f(M);
    float den = 0.f;
    for (int c = lane; c < S; c += 32) {
      const float m = wf[r * S + c];
      const float f = m == -INFINITY ? 0.f : expf(m - M);
      den = fmaf(f, lf[r * S + c], den);
      wf[r * S + c] = f;
    }
    den = warp_sum_f(den);
    if (lane == 0) dn[r] = den;
  }
  sync();
  if constexpr (REG) {
    if (S <= kMergeRegs) {
#pragma unroll
      for (int k = 0; k < OPT; ++k) {
        const int i = tid + k * NT;
        if (i >= NR * HD) continue;
        const int r = i / HD, d = i - r * HD;
        const float* w = wf + r * S;
        float num = 0.f;
#pragma unroll
        for (int c = 0; c < kMergeRegs; ++c)
          if (c < S) num = fmaf(w[c], acc_v[k][c], num);
        out_g[r * HD + d] = num / dn[r];
      }
      return;
    }
  }
  for (int i = tid; i < NR * HD; i += NT) {
    const int r = i / HD, d = i - r * HD;
    const float* pr = part_g + r * (HD + 2) + d;
    const float* w = wf + r * S;
    float num = 0.f;
    int c = 0;
    for (; c + 8 <= S; c += 8) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __ldcg(pr + (c + j) * stride);
#pragma unroll
      for (int j = 0; j < 8; ++j) num = fmaf(w[c + j], v[j], num);
    }
    for (; c < S; ++c) num = fmaf(w[c], __ldcg(pr + c * stride), num);
    out_g[r * HD + d] = num / dn[r];
  }
}

struct AttnArgs {
  const float* in;        // QKV: qkv row [(nq + 2 nkv) hd]; else q [nq hd]
  const float* qn_w;      // [hd] or null
  const float* kn_w;      // [hd] or null
  const float* inv_freq;  // [hd / 2]
  float* kc;              // [nkv, max_ctx, hd] (written only with QKV)
  float* vc;
  float* out;             // [nq hd]
  float* part;            // [nkv][S][NR][hd + 2]
  unsigned* tickets;      // [nkv], zero between launches
  const int64_t* len_dev; // T = (len_dev ? *len_dev : len0) + len_off
  int64_t len0, len_off, max_ctx;
  int nq, nkv;
  float scale, eps;
  // Sequences decoded in lockstep (grid z): sequence b reads in + b * in_bstride,
  // its caches at kc / vc + b * kv_bstride and writes out + b * out_bstride
  // (elements); its partials and tickets follow sequence b-1's. Zero strides
  // with one sequence are the single-sequence launch.
  int64_t in_bstride, kv_bstride, out_bstride;
};

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;

template <int E>
__device__ __forceinline__ void load_vec(const float* p, float (&x)[E]) {
  if constexpr (E == 4) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
  } else if constexpr (E == 2) {
    const float2 v = *reinterpret_cast<const float2*>(p);
    x[0] = v.x; x[1] = v.y;
  } else {
#pragma unroll
    for (int e = 0; e < E; e += 4) {
      const float4 v = *reinterpret_cast<const float4*>(p + e);
      x[e] = v.x; x[e + 1] = v.y; x[e + 2] = v.z; x[e + 3] = v.w;
    }
  }
}

template <int E>
__device__ __forceinline__ void store_vec(float* p, const float (&x)[E]) {
  if constexpr (E == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
  } else if constexpr (E == 2) {
    *reinterpret_cast<float2*>(p) = make_float2(x[0], x[1]);
  } else {
#pragma unroll
    for (int e = 0; e < E; e += 4)
      *reinterpret_cast<float4*>(p + e) = make_float4(x[e], x[e + 1], x[e + 2], x[e + 3]);
  }
}

// Optional per-head RMSNorm, then half-split RoPE at position pos, of the
// head slice x held E elements per lane (whole warp participates).
template <int E>
__device__ __forceinline__ void norm_rope(float (&x)[E], const float* __restrict__ w,
                                          const float* __restrict__ inv_freq, int64_t pos,
                                          float eps, int lane) {
  constexpr int HD = 32 * E, D = HD / 2;
  if (w) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) ss = fmaf(x[e], x[e], ss);
    ss = warp_sum_f(ss);
    const float r = 1.0f / sqrtf(ss / static_cast<float>(HD) + eps);
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = x[e] * r * w[lane * E + e];
  }
  const float fpos = static_cast<float>(pos);
  const bool lower = lane < 16;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float other = __shfl_xor_sync(0xffffffffu, x[e], 16);
    const int j = lane * E + e - (lower ? 0 : D);
    const float ang = fpos * inv_freq[j];
    const float c = cosf(ang), s = sinf(ang);
    // lower: x1 c - x2 s (self x1, partner x2); upper: x2 c + x1 s (self x2, partner x1)
    x[e] = lower ? x[e] * c - other * s : x[e] * c + other * s;
  }
}

// Sum V values (V a power of two <= 32) over the warp at once: each stage
// halves the values a lane holds by trading half of them with the lane `o`
// away, so that afterwards lane l holds the full sum of value l >> log2(32/V)
// (lanes below that granularity finish with plain butterfly steps). V - 1 +
// log2(32/V) shuffles instead of 5 V.
template <int V>
__device__ __forceinline__ float transpose_sum(float (&v)[V], int lane) {
#pragma unroll
  for (int n = V, o = 16; n > 1; n >>= 1, o >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = up ? v[i] : v[i + n / 2];
      const float keep = up ? v[i + n / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  float s = v[0];
#pragma unroll
  for (int o = 16 / V; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}

// Positions per warp per round of the fused attention: a round's K and V rows
// are one cp.async group in the warp's private two-round ring.
template <int E>
__host__ __device__ constexpr int attn_round() { return E >= 8 ? 2 : 4; }

// Copy this lane's E floats of cache row `src` to shared memory `dst` (its own
// bytes of the warp's ring slot; the lane later reads back exactly these).
template <int E>
__device__ __forceinline__ void cp_async_lane(uint32_t dst, const float* src) {
  if constexpr (E % 4 == 0) {
#pragma unroll
    for (int e = 0; e < E; e += 4) cp_async16(dst + 4 * e, src + e);
  } else {
    static_assert(E == 2, "lane slices of 2, 4 or 8 floats");
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
  }
}

template <int E, int NR, bool QKV>
__global__ void __launch_bounds__(kAttnThreads, 1) attn_decode_fused_kernel(AttnArgs a) {
  constexpr int HD = 32 * E;
  constexpr int U = attn_round<E>();   // positions per warp per round
  constexpr int V = U * NR;            // scores per round
  static_assert(V <= 32 && (V & (V - 1)) == 0, "a round's scores fit one transposed butterfly");
  constexpr int SH = V == 32 ? 0 : V == 16 ? 1 : V == 8 ? 2 : V == 4 ? 3 : V == 2 ? 4 : 5;
  extern __shared__ float4 attn_smem4[];
  float* qs = reinterpret_cast<float*>(attn_smem4);   // [NR][HD]
  float* red = qs + NR * HD;                           // [warps][NR][HD + 2]
  // per warp: 2 rounds x U positions x (K row, V row)
  float* ring = red + kAttnWarps * NR * (HD + 2);
  __shared__ unsigned s_last;
  const int g = blockIdx.x, c = blockIdx.y, S = gridDim.y;
  const int64_t b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* in = a.in + b * a.in_bstride;
  float* const kc = a.kc + b * a.kv_bstride;
  float* const vc = a.vc + b * a.kv_bstride;
  const int64_t kv_off = static_cast<int64_t>(g) * a.max_ctx * HD;
  float* const wring = ring + warp * (2 * U * 2 * HD);
  const uint32_t wring_s = smem_u32(wring);

  // This CTA's positions [t0, t1) for context length T; warp w takes positions
  // t0 + w + 8 i, i = 0, 1, ..., U of them per round.
  auto range = [&](int64_t T, int64_t& t0, int64_t& t1) {
    const int64_t per = T > 0 ? (cdiv(T, S) + 7) / 8 * 8 : 0;
    t0 = static_cast<int64_t>(c) * per;
    t1 = min64(T, t0 + per);
  };
  auto ctx = [&]() {
    int64_t T = (a.len_dev ? *a.len_dev : a.len0) + a.len_off;
    return T > a.max_ctx ? a.max_ctx : (T < 0 ? 0 : T);
  };
  // Issue round r's rows among positions [lo, hi), one commit group per call.
  auto issue_round = [&](int64_t r, int64_t t0, int64_t lo, int64_t hi) {
    const uint32_t slot = wring_s + static_cast<uint32_t>((r & 1) * U * 2 * HD * 4);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t t = t0 + warp + static_cast<int64_t>(kAttnWarps) * (r * U + u);
      if (t >= lo && t < hi) {
        const uint32_t d = slot + static_cast<uint32_t>(u * 2 * HD * 4 + lane * E * 4);
        cp_async_lane<E>(d, kc + kv_off + t * HD + lane * E);
        cp_async_lane<E>(d + HD * 4, vc + kv_off + t * HD + lane * E);
      }
    }
    cp_async_commit();
  };

  // Launched as a programmatic dependent of the kernel that writes `in` (and,
  // without QKV, the newest cache row): the next kernel may launch now. Rows
  // before the newest one were written by earlier steps, so the first two
  // rounds of them go in flight before the wait, for the context length read
  // here; after the wait the length is read again and, if it moved, the ring
  // is drained and refilled.
  pdl_trigger();
  const int64_t T_pre = ctx();
  int64_t t0, t1;
  range(T_pre, t0, t1);
  issue_round(0, t0, t0, min64(t1, T_pre - 1));
  issue_round(1, t0, t0, min64(t1, T_pre - 1));
  pdl_wait();
  const int64_t T = ctx();
  const bool moved = T != T_pre;
  if (moved) {
    cp_async_wait<0>();
    range(T, t0, t1);
  }
  const int64_t pos = T - 1;
  // the append happens only for a position inside the cache
  const int64_t t_raw = (a.len_dev ? *a.len_dev : a.len0) + a.len_off;
  const bool append = QKV && t_raw >= 1 && t_raw <= a.max_ctx;
  // this sequence's partials [nkv][S][NR][HD + 2] follow the previous one's
  float* const part = a.part + b * static_cast<int64_t>(a.nkv) * S * NR * (HD + 2);
  float* pbase = part + (static_cast<int64_t>(g) * S + c) * NR * (HD + 2);

  if (t0 < t1) {
    // queries of this group (and, in the owning CTA, the new key/value)
    for (int r = warp; r < NR; r += kAttnWarps) {
      float x[E];
      load_vec<E>(in + static_cast<int64_t>(g * NR + r) * HD + lane * E, x);
      if constexpr (QKV) norm_rope<E>(x, a.qn_w, a.inv_freq, pos, a.eps, lane);
#pragma unroll
      for (int e = 0; e < E; ++e) qs[r * HD + lane * E + e] = x[e];
    }
    if constexpr (QKV) {
      if (append && t0 <= pos && pos < t1 && warp == NR % kAttnWarps) {
        float k[E], v[E];
        load_vec<E>(in + static_cast<int64_t>(a.nq + g) * HD + lane * E, k);
        load_vec<E>(in + static_cast<int64_t>(a.nq + a.nkv + g) * HD + lane * E, v);
        norm_rope<E>(k, a.kn_w, a.inv_freq, pos, a.eps, lane);
        store_vec<E>(kc + kv_off + pos * HD + lane * E, k);
        store_vec<E>(vc + kv_off + pos * HD + lane * E, v);
      }
    }
    __syncthreads();   // queries in shared memory; the appended row visible to the CTA
    if (moved) {
      issue_round(0, t0, t0, t1);
      issue_round(1, t0, t0, t1);
    } else if (T_pre - 1 < t1) {
      // the newest row (and anything after it in this CTA's range) of the
      // first two rounds, now that it is written; then let everything land
      const int64_t lo = T_pre - 1 > t0 ? T_pre - 1 : t0;
      for (int64_t r = 0; r < 2; ++r) {
        const uint32_t slot = wring_s + static_cast<uint32_t>((r & 1) * U * 2 * HD * 4);
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t t = t0 + warp + static_cast<int64_t>(kAttnWarps) * (r * U + u);
          if (t >= lo && t < t1) {
            const uint32_t d = slot + static_cast<uint32_t>(u * 2 * HD * 4 + lane * E * 4);
            cp_async_lane<E>(d, kc + kv_off + t * HD + lane * E);
            cp_async_lane<E>(d + HD * 4, vc + kv_off + t * HD + lane * E);
          }
        }
      }
      cp_async_commit();
      cp_async_wait<0>();
    }

    float q[NR][E], acc[NR][E], m[NR], l[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      m[r] = -INFINITY;
      l[r] = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        q[r][e] = qs[r * HD + lane * E + e];
        acc[r][e] = 0.f;
      }
    }
    const int64_t n_w = t1 - t0 > warp ? (t1 - t0 - warp + kAttnWarps - 1) / kAttnWarps : 0;
    const int64_t rounds = (n_w + U - 1) / U;
    for (int64_t rd = 0; rd < rounds; ++rd) {
      // rounds rd and rd + 1 were issued before; issue rd + 1 into the slot
      // round rd - 1 vacated, then round rd has landed once at most one group
      // is pending
      if (rd >= 1) issue_round(rd + 1, t0, t0, t1);
      cp_async_wait<1>();
      const float* slot = wring + (rd & 1) * U * 2 * HD;
      float kr[U][E], vr[U][E];
      bool ok[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t t = t0 + warp + static_cast<int64_t>(kAttnWarps) * (rd * U + u);
        ok[u] = t < t1;
        if (ok[u]) {
          load_vec<E>(slot + u * 2 * HD + lane * E, kr[u]);
          load_vec<E>(slot + u * 2 * HD + HD + lane * E, vr[u]);
        } else {
#pragma unroll
          for (int e = 0; e < E; ++e) kr[u][e] = vr[u][e] = 0.f;
        }
      }
      // The round's U x NR scores: one transposed butterfly sums all of them
      // over the warp (lane l then holds score v = l >> SH, v = r U + u); the
      // holders take each head's round maximum among themselves and compute
      // the softmax numerators, which are then broadcast for the V update.
      float v[V];
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int r = 0; r < NR; ++r) {
          float d = 0.f;
#pragma unroll
          for (int e = 0; e < E; ++e) d = fmaf(q[r][e], kr[u][e], d);
          v[r * U + u] = d;
        }
      const float s_own = transpose_sum<V>(v, lane) * a.scale;
      const int v_own = lane >> SH;
      const int r_own = v_own / U, u_own = v_own % U;
      const bool ok_own =
          t0 + warp + static_cast<int64_t>(kAttnWarps) * (rd * U + u_own) < t1;
      float mx = ok_own ? s_own : -INFINITY;
#pragma unroll
      for (int o = 1 << SH; o < (U << SH); o <<= 1)
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      float m_own = m[0];
#pragma unroll
      for (int r = 1; r < NR; ++r)
        if (r == r_own) m_own = m[r];
      // every round's first position exists, so each head's maximum is finite
      const float mnew_own = fmaxf(m_own, mx);
      const float p_own = ok_own ? expf(s_own - mnew_own) : 0.f;
#pragma unroll
      for (int r = 0; r < NR; ++r) {
        const float mnew = __shfl_sync(0xffffffffu, mnew_own, (r * U) << SH);
        const float corr = expf(m[r] - mnew);
        l[r] *= corr;
#pragma unroll
        for (int e = 0; e < E; ++e) acc[r][e] *= corr;
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const float pu = __shfl_sync(0xffffffffu, p_own, (r * U + u) << SH);
          l[r] += pu;
#pragma unroll
          for (int e = 0; e < E; ++e) acc[r][e] = fmaf(pu, vr[u][e], acc[r][e]);
        }
        m[r] = mnew;
      }
    }
    cp_async_wait<0>();
    // merge the warps: per-warp (acc, m, l) to shared memory, then one partial per head
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      float* wr = red + (warp * NR + r) * (HD + 2);
#pragma unroll
      for (int e = 0; e < E; ++e) wr[lane * E + e] = acc[r][e];
      if (lane == 0) { wr[HD] = m[r]; wr[HD + 1] = l[r]; }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < NR * HD; i += kAttnThreads) {
      const int r = i / HD, d = i - r * HD;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, red[(w * NR + r) * (HD + 2) + HD]);
      float num = 0.f, den = 0.f;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) {
        const float* wr = red + (w * NR + r) * (HD + 2);
        if (wr[HD] == -INFINITY) continue;
        const float f = expf(wr[HD] - M);
        num = fmaf(f, wr[d], num);
        den = fmaf(f, wr[HD + 1], den);
      }
      pbase[r * (HD + 2) + d] = num;
      if (d == 0) { pbase[r * (HD + 2) + HD] = M; pbase[r * (HD + 2) + HD + 1] = den; }
    }
  } else {
    cp_async_wait<0>();
    for (int r = threadIdx.x; r < NR; r += kAttnThreads) {
      pbase[r * (HD + 2) + HD] = -INFINITY;
      pbase[r * (HD + 2) + HD + 1] = 0.f;
    }
  }

  // the last CTA of kv head g merges the S partials of its query heads
  __syncthreads();
  unsigned* const tickets = a.tickets + b * a.nkv;
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(tickets + g, 1u) == static_cast<unsigned>(S - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const float* gbase = part + static_cast<int64_t>(g) * S * NR * (HD + 2);
  merge_partials<HD, NR, kAttnThreads>(gbase, S, a.out + b * a.out_bstride + static_cast<int64_t>(g) * NR * HD, red,
                                       threadIdx.x, [] { __syncthreads(); });
  if (threadIdx.x == 0) tickets[g] = 0u;
}

template <int E, int NR>
constexpr int attn_fused_smem() {
  return (NR * 32 * E + kAttnWarps * NR * (32 * E + 2) + kAttnWarps * 2 * attn_round<E>() * 2 * 32 * E) * 4;
}

// Greedy argmax of each row of logits [M, V]: a block reduces a slice of a row
// to one packed key (order-preserving float bits << 32 | ~index) and
// atomicMax-es it into keys[m] (zeroed before); larger value wins, then the
// lower index, as np.argmax.
__device__ __forceinline__ unsigned long long pack_key(float v, int64_t idx) {
  const uint32_t b = __float_as_uint(v);
  const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(ord) << 32) |
         (0xFFFFFFFFull - static_cast<unsigned long long>(idx));
}

__global__ void argmax_kernel(const float* __restrict__ logits, int64_t V,
                              unsigned long long* __restrict__ keys) {
  __shared__ unsigned long long red[32];
  const int64_t m = blockIdx.y;
  const float* row = logits + m * V;
  unsigned long long best = 0ull;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < V;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const unsigned long long k = pack_key(row[i], i);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < static_cast<int>(blockDim.x >> 5); ++i) best = red[i] > best ? red[i] : best;
    best = red[0] > best ? red[0] : best;
    atomicMax(keys + m, best);
  }
}

// token[m] = index packed in keys[m]; keys reset to 0 for the next call.
// If pos_dev is set, thread 0 also advances that position counter by `step`.
__global__ void argmax_finish_kernel(unsigned long long* __restrict__ keys,
                                     int64_t* __restrict__ tokens, int64_t M,
                                     int64_t* __restrict__ pos_dev, int64_t step) {
  const int64_t m = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (m < M) {
    tokens[m] = static_cast<int64_t>(0xFFFFFFFFull - (keys[m] & 0xFFFFFFFFull));
    keys[m] = 0ull;
  }
  if (pos_dev && m == 0) *pos_dev += step;
}

}  // namespace dec
}  // namespace qz
