// qz_device.cuh -- sm_100a device helpers shared by the int8 weight-only kernels.
//
// * a device status word that kernels set when a bounded wait gives up;
// * mbarrier / 1-D bulk-copy (TMA engine) wrappers in inline PTX;
// * the int8 -> fp32 widening used by every CUDA-core kernel here.
//
// Widening: a signed byte b becomes an unsigned u = b ^ 0x80 = b + 128; PRMT
// drops u into the low mantissa byte of 2^23 (bits 0x4B0000uu == 8388608 + u),
// and one packed f32x2 subtract of 8388736 (= 2^23 + 128) yields (float)b
// exactly. Per weight byte that is one PRMT and half an FADD2, instead of an
// I2F on the conversion pipe, which runs at a fraction of the FMA rate. The
// products then accumulate with packed fma.rn.f32x2 (sm_100+).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace qz {

// ---------------------------------------------------------------------------
// Device status word. [0]: OR of error bits; [1]: site of the first error;
// [2]: blockIdx.x of the first error; [3]: number of errors reported.
// ---------------------------------------------------------------------------
__device__ unsigned int g_status[4];

enum : unsigned int {
  ERR_WAIT_FULL = 1u,      // consumer gave up waiting for a stage to land
  ERR_WAIT_EMPTY = 2u,     // producer gave up waiting for a stage to drain
  ERR_GRID_BARRIER = 4u,   // grid-wide barrier did not complete in time
  ERR_DRAIN = 8u,          // copies still in flight when a CTA gave up
};

// Every spin in these kernels gives up after this many nanoseconds of
// %globaltimer time (a stage normally lands in about a microsecond).
constexpr unsigned long long kWaitLimitNs = 1000000000ull;

__device__ __forceinline__ void report_error(unsigned int bit, unsigned int site) {
  atomicOr(&g_status[0], bit);
  if (atomicAdd(&g_status[3], 1u) == 0u) {
    g_status[1] = site;
    g_status[2] = blockIdx.x;
  }
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// mbarrier + bulk copy
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Wait until the grids this one depends on have completed and their memory is
// visible (a no-op without a programmatic dependency).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next kernel in the stream to begin launching; it still waits for
// this grid's completion before it reads anything this grid writes.
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0u;
}

// Wait for the phase of parity `parity` to complete; false after kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > kWaitLimitNs) return false;
  }
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 1-D bulk copy global -> this CTA's shared memory, completing `bytes` of
// transaction count on `bar`. dst/src 16-byte aligned, bytes a multiple of 16.
// (No cluster multicast: the destination is always the issuing CTA.)
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

// Per-stage position tags. mbarrier parity waits only tell the current phase
// from the previous one, so a consumer that may run ahead of the ring first
// waits until the producer has published (st.release) the position it wants.
__device__ __forceinline__ void st_release_shared(uint32_t addr, uint32_t v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_shared(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}

// Wait until the word at `addr` equals `want`; false after kWaitLimitNs.
__device__ __forceinline__ bool wait_tag(uint32_t addr, uint32_t want) {
  if (ld_acquire_shared(addr) == want) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 16; ++i) {
      __nanosleep(32);
      if (ld_acquire_shared(addr) == want) return true;
    }
    if (globaltimer() - t0 > kWaitLimitNs) return false;
  }
}

// Named barrier over the first `nthreads` threads of the CTA (id != 0).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ---------------------------------------------------------------------------
// packed fp32 pairs (sm_100: add/sub/fma .f32x2)
// ---------------------------------------------------------------------------
typedef unsigned long long f2_t;

__device__ __forceinline__ f2_t f2_pack(uint32_t lo, uint32_t hi) {
  f2_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}

__device__ __forceinline__ float2 f2_unpack(f2_t v) {
  uint32_t lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=r"(lo), "=r"(hi) : "l"(v));
  return make_float2(__uint_as_float(lo), __uint_as_float(hi));
}

__device__ __forceinline__ f2_t f2_sub(f2_t a, f2_t b) {
  f2_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ f2_t f2_fma(f2_t a, f2_t b, f2_t c) {
  f2_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// (2^23 + 128, 2^23 + 128) as an fp32 pair.
constexpr unsigned long long kMagic2 = 0x4B0000804B000080ull;

// acc += sum_{j<4} x[j] * (float)(int8)byte_j(w), as two fp32 pair lanes.
// x01 = (x0, x1), x23 = (x2, x3).
__device__ __forceinline__ void dot4_acc(uint32_t w, f2_t x01, f2_t x23, f2_t& acc) {
  const uint32_t u = w ^ 0x80808080u;
  const uint32_t f0 = prmt(u, 0x4B000000u, 0x7540u);
  const uint32_t f1 = prmt(u, 0x4B000000u, 0x7541u);
  const uint32_t f2 = prmt(u, 0x4B000000u, 0x7542u);
  const uint32_t f3 = prmt(u, 0x4B000000u, 0x7543u);
  const f2_t q01 = f2_sub(f2_pack(f0, f1), kMagic2);
  const f2_t q23 = f2_sub(f2_pack(f2, f3), kMagic2);
  acc = f2_fma(x01, q01, acc);
  acc = f2_fma(x23, q23, acc);
}

// One 16-byte chunk of weights against 16 activations held as 8 fp32 pairs.
__device__ __forceinline__ void dot16_acc(const uint4& q, const f2_t* x, f2_t& acc) {
  dot4_acc(q.x, x[0], x[1], acc);
  dot4_acc(q.y, x[2], x[3], acc);
  dot4_acc(q.z, x[4], x[5], acc);
  dot4_acc(q.w, x[6], x[7], acc);
}

// ---------------------------------------------------------------------------
// int4 weights (two per byte, element 2i in the low nibble, two's complement,
// symmetric in [-7, 7]). After the bias XOR a nibble holds n + 8 in 0..15.
// Masked where it lies, at bit p(t) = 4t for t < 5 (nibbles 5..7 are shifted
// right by 12 first: p = 8, 12, 16), it is the bit pattern of the subnormal
// float (n + 8) * 2^(p - 149): no magic constant, no subtraction, one AND per
// weight. The activations are staged as x * 2^(85 - p(t)) (|x| < 2^43 stays
// finite), so each product is (n + 8) * x * 2^-64 in one FMA (fma.rn.f32x2
// keeps subnormal inputs); the caller scales the sum by 2^64 and subtracts
// 8 * sum(x) over the same weights. The packed FMA has no .ftz, so the
// subnormal operands are exact.
// ---------------------------------------------------------------------------
__host__ __device__ constexpr int w4_pos(int t) { return t < 5 ? 4 * t : 4 * (t - 3); }

// acc += sum_{t<8} x''[t] * f(nibble t of w); x01..x67 are the staged pairs.
__device__ __forceinline__ void dot8_w4_acc(uint32_t w, f2_t x01, f2_t x23, f2_t x45, f2_t x67,
                                            f2_t& acc) {
  const uint32_t u = w ^ 0x88888888u;
  const uint32_t v = u >> 12;
  acc = f2_fma(x01, f2_pack(u & 0xFu, u & 0xF0u), acc);
  acc = f2_fma(x23, f2_pack(u & 0xF00u, u & 0xF000u), acc);
  acc = f2_fma(x45, f2_pack(u & 0xF0000u, v & 0xF00u), acc);
  acc = f2_fma(x67, f2_pack(v & 0xF000u, v & 0xF0000u), acc);
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

__device__ __forceinline__ void lds_f2x2(uint32_t addr, f2_t& a, f2_t& b) {
  asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "r"(addr));
}

// Sum 8 per-lane values over the warp so that, afterwards, every lane holds the
// full sum of row r = (lane >> 2) & 7. Nine shuffles instead of forty.
__device__ __forceinline__ float warp_reduce8(float (&v)[8], int lane) {
  const unsigned FULL = 0xffffffffu;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool up = lane & 16;
    const float keep = up ? v[i + 4] : v[i];
    const float send = up ? v[i] : v[i + 4];
    v[i] = keep + __shfl_xor_sync(FULL, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const bool up = lane & 8;
    const float keep = up ? v[i + 2] : v[i];
    const float send = up ? v[i] : v[i + 2];
    v[i] = keep + __shfl_xor_sync(FULL, send, 8);
  }
  {
    const bool up = lane & 4;
    const float keep = up ? v[1] : v[0];
    const float send = up ? v[0] : v[1];
    v[0] = keep + __shfl_xor_sync(FULL, send, 4);
  }
  v[0] += __shfl_xor_sync(FULL, v[0], 2);
  v[0] += __shfl_xor_sync(FULL, v[0], 1);
  return v[0];
}

}  // namespace qz
