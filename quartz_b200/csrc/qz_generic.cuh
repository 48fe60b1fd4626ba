// qz_generic.cuh -- shape-agnostic kernels for the int8 weight-only path.
//
// These cover every case the streaming kernels' preconditions exclude (K or the
// group size not a multiple of 16, unaligned weight pointers, activations too
// long to stage in shared memory), plus the elementwise SiLU-times-up of the
// M > 1 MLP. They are plain CUDA-core kernels: one warp per weight row, lanes
// striding over K, the group scale folded into each product.
#pragma once

#include "qz_device.cuh"

namespace qz {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Y[m, n] = sum_k X[m, k] * q[n, k] * scale[n, k / G]  (+ residual[m, n])
// (quartz/kernels/int8.py:24-38 for M = 1, 66-87 for M > 1)
__global__ void generic_gemm_kernel(const int8_t* __restrict__ q, const float* __restrict__ scale,
                                    int64_t ng, const float* __restrict__ X, float* __restrict__ Y,
                                    const float* __restrict__ residual, int64_t M, int64_t N,
                                    int64_t K) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t G = ng > 0 ? K / ng : K;
  for (int64_t n = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; n < N;
       n += warps) {
    const int8_t* qr = q + n * K;
    const float* sr = scale + n * ng;
    for (int64_t m = 0; m < M; ++m) {
      const float* xr = X + m * K;
      float acc = 0.f;
      for (int64_t k = lane; k < K; k += 32)
        acc = fmaf(xr[k] * static_cast<float>(qr[k]), __ldg(sr + k / G), acc);
      acc = warp_sum(acc);
      if (lane == 0) {
        if (residual) acc += residual[m * N + n];
        Y[m * N + n] = acc;
      }
    }
  }
}

// abuf[n] = silu(gate_n . x) * (up_n . x), unclipped exp  (quartz/kernels/fused.py:40-54)
__global__ void generic_mlp_gate_kernel(const int8_t* __restrict__ gu_q,
                                        const float* __restrict__ gu_s, int64_t ng,
                                        const float* __restrict__ x, float* __restrict__ abuf,
                                        int64_t H, int64_t I) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t G = H / ng;
  for (int64_t n = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; n < I;
       n += warps) {
    const int8_t* gr = gu_q + n * H;
    const int8_t* ur = gu_q + (n + I) * H;
    const float* gs = gu_s + n * ng;
    const float* us = gu_s + (n + I) * ng;
    float ga = 0.f, ua = 0.f;
    for (int64_t k = lane; k < H; k += 32) {
      const float xv = x[k];
      ga = fmaf(xv * static_cast<float>(gr[k]), __ldg(gs + k / G), ga);
      ua = fmaf(xv * static_cast<float>(ur[k]), __ldg(us + k / G), ua);
    }
    ga = warp_sum(ga);
    ua = warp_sum(ua);
    if (lane == 0) abuf[n] = ga / (1.0f + expf(-ga)) * ua;
  }
}

// a[m, i] = silu(gu[m, i]) * gu[m, I + i] with the exponent clipped to [-88, 88]
// (quartz/ops.py:35-37, used by quartz/quantize.py:112-114 for M > 1).
__global__ void silu_mul_kernel(const float* __restrict__ gu, float* __restrict__ a, int64_t M,
                                int64_t I) {
  const int64_t total = M * I;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = t / I, i = t - m * I;
    const float g = gu[m * 2 * I + i];
    const float u = gu[m * 2 * I + I + i];
    const float c = fminf(fmaxf(g, -88.0f), 88.0f);
    a[t] = g * (1.0f / (1.0f + expf(-c))) * u;
  }
}

}  // namespace qz
