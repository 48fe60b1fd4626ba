// qz_api.cu -- the extern "C" boundary (include/quartz_b200.h): argument
// checks, kernel selection and launch configuration. One translation unit so
// that the device status word is a single symbol without relocatable code.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>

#include "quartz_b200.h"
#include "qz_generic.cuh"
#include "qz_stream.cuh"
#include "qz_tc_gemm.cuh"
#include "qz_decode.cuh"
#include "qz_decode_step.cuh"
#include "qz_comm.cuh"

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

#define QZ_CUDA(call)                                                                   \
  do {                                                                                  \
    cudaError_t e_ = (call);                                                            \
    if (e_ != cudaSuccess)                                                              \
      return fail(QZ_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_));     \
  } while (0)

constexpr int kMaxDevices = 64;

// Rows per group of the streaming kernels: 4 for tall matrices, 1 when a tall
// grouping would leave SMs idle.
constexpr int kTallRows = 4;
constexpr int kMinBlocks = 3;   // launch bound: CTAs per SM the register budget allows

struct DeviceInfo {
  std::atomic<bool> ready{false};   // set (release) once the fields below are final
  int sms = 0;
  int smem_optin = 0;   // max dynamic shared memory per block (opt-in)
  int coop = 0;         // cooperative launch supported
};

DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

template <class F>
cudaError_t allow_smem(F* fn, int bytes) {
  return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

template <int R, int D = qz::kDepth>
cudaError_t allow_gemv_variants(int smem) {
  cudaError_t e = cudaSuccess;
  auto set = [&](auto fn) { if (e == cudaSuccess) e = allow_smem(fn, smem); };
  set(qz::gemv_kernel<R, true, qz::K1K, kMinBlocks, D>);
  set(qz::gemv_kernel<R, true, qz::KFULL, kMinBlocks, D>);
  set(qz::gemv_kernel<R, true, qz::KANY, kMinBlocks, D>);
  set(qz::gemv_kernel<R, false, qz::K1K, kMinBlocks, D>);
  set(qz::gemv_kernel<R, false, qz::KFULL, kMinBlocks, D>);
  set(qz::gemv_kernel<R, false, qz::KANY, kMinBlocks, D>);
  return e;
}

// Ring depth of one-row GEMV walks when three CTAs per SM still fit: 6 KB in
// flight per warp instead of 2.
constexpr int kDeepRing = 6;

template <int R, bool ANY>
cudaError_t allow_gemv_w4_variants(int smem) {
  cudaError_t e = cudaSuccess;
  auto set = [&](auto fn) { if (e == cudaSuccess) e = allow_smem(fn, smem); };
  set(qz::gemv_w4_kernel<R, true, qz::KFULL, kMinBlocks>);
  set(qz::gemv_w4_kernel<R, false, qz::KFULL, kMinBlocks>);
  if constexpr (ANY) {
    set(qz::gemv_w4_kernel<R, true, qz::KANY, kMinBlocks>);
    set(qz::gemv_w4_kernel<R, false, qz::KANY, kMinBlocks>);
  }
  return e;
}

template <int R>
cudaError_t allow_mlp_variants(int smem) {
  cudaError_t e = cudaSuccess;
  auto set = [&](auto fn) { if (e == cudaSuccess) e = allow_smem(fn, smem); };
  set(qz::fused_mlp_kernel<R, true, qz::KFULL, qz::KFULL, kMinBlocks>);
  set(qz::fused_mlp_kernel<R, true, qz::KANY, qz::KANY, kMinBlocks>);
  set(qz::fused_mlp_kernel<R, false, qz::KFULL, qz::KFULL, kMinBlocks>);
  set(qz::fused_mlp_kernel<R, false, qz::KANY, qz::KANY, kMinBlocks>);
  return e;
}

int kmode(int64_t K) {
  if (K == qz::kSegBytes) return qz::K1K;
  if (K % qz::kSegBytes == 0) return qz::KFULL;
  return qz::KANY;
}

int device_info(DeviceInfo** out) {
  int dev = 0;
  QZ_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(QZ_ERR_UNSUPPORTED, "device index out of range");
  DeviceInfo& d = g_dev[dev];
  if (!d.ready.load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(g_dev_mu);
    if (!d.ready.load(std::memory_order_relaxed)) {
      cudaDeviceProp p;
      QZ_CUDA(cudaGetDeviceProperties(&p, dev));
      if (p.major != 10)
        return fail(QZ_ERR_UNSUPPORTED, std::string("quartz_b200 needs an sm_100 GPU, got ") +
                                            p.name + " sm_" + std::to_string(p.major) +
                                            std::to_string(p.minor));
      d.sms = p.multiProcessorCount;
      d.smem_optin = static_cast<int>(p.sharedMemPerBlockOptin);
      d.coop = p.cooperativeLaunch;
      // Leave room for the kernels' few bytes of static shared memory.
      const int smem = d.smem_optin - 256;
      QZ_CUDA(allow_gemv_variants<kTallRows>(smem));
      QZ_CUDA(allow_gemv_variants<1>(smem));
      QZ_CUDA((allow_gemv_variants<1, kDeepRing>(smem)));
      QZ_CUDA((allow_gemv_w4_variants<2 * kTallRows, false>(smem)));
      QZ_CUDA((allow_gemv_w4_variants<2, true>(smem)));
      QZ_CUDA(allow_mlp_variants<kTallRows>(smem));
      QZ_CUDA(allow_mlp_variants<2>(smem));
      d.ready.store(true, std::memory_order_release);
    }
  }
  *out = &d;
  return QZ_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_weights(const int8_t* q, const float* scale, int64_t ng, int64_t N, int64_t K,
                  const char* what) {
  if (N < 0 || K < 0) return fail(QZ_ERR_INVALID, std::string(what) + ": negative dimension");
  if (ng < 1) return fail(QZ_ERR_INVALID, std::string(what) + ": ng must be >= 1");
  if (K % ng != 0)
    return fail(QZ_ERR_INVALID, std::string(what) + ": scale has " + std::to_string(ng) +
                                    " groups that do not tile K=" + std::to_string(K));
  if (N > 0 && (!scale || (K > 0 && !q)))
    return fail(QZ_ERR_INVALID, std::string(what) + ": null weight pointer");
  return QZ_OK;
}

int launch_generic_gemm(const DeviceInfo& d, const int8_t* q, const float* scale, int64_t ng,
                        const float* X, float* Y, const float* residual, int64_t M, int64_t N,
                        int64_t K, cudaStream_t st) {
  const int threads = 256;
  const int64_t want = qz::cdiv(N, threads / 32);
  const int blocks = static_cast<int>(std::min<int64_t>(want, int64_t(d.sms) * 8));
  qz::generic_gemm_kernel<<<blocks, threads, 0, st>>>(q, scale, ng, X, Y, residual, M, N, K);
  QZ_CUDA(cudaGetLastError());
  return QZ_OK;
}

// Launch `fn` with programmatic stream serialisation (and, for the fused MLP,
// as a cooperative grid too). Kernels launched this way issue their first
// weight copies before griddepcontrol.wait, overlapping the previous kernel's
// tail. If the runtime refuses cooperative + programmatic together, the
// cooperative launch is retried alone and that choice is remembered.
std::atomic<int> g_coop_pdl{1};

template <class... Args>
int launch_ex(void (*fn)(Args...), int grid, int smem, cudaStream_t st, bool cooperative,
              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(qz::kThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  const bool pdl = !cooperative || g_coop_pdl.load(std::memory_order_relaxed);
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cooperative) {
    attr[n].id = cudaLaunchAttributeCooperative;
    attr[n].val.cooperative = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaError_t e = cudaLaunchKernelEx(&cfg, fn, args...);
  if (e != cudaSuccess && cooperative && pdl) {
    (void)cudaGetLastError();
    g_coop_pdl.store(0, std::memory_order_relaxed);
    cfg.attrs = attr + 1;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, fn, args...);
  }
  QZ_CUDA(e);
  return QZ_OK;
}

// CTAs of `fn` that fit on one SM with `smem` bytes of dynamic shared memory.
template <class F>
int blocks_per_sm(F* fn, int smem, int* out) {
  int nb = 0;
  QZ_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, fn, qz::kThreads, smem));
  *out = nb;
  return QZ_OK;
}

template <int R, bool PER_ROW, int KM, int D = qz::kDepth>
int launch_gemv(const DeviceInfo& d, const qz::GemvArgs& a, cudaStream_t st) {
  auto fn = qz::gemv_kernel<R, PER_ROW, KM, kMinBlocks, D>;
  const int ring = qz::kWarps * D * R * qz::kSegBytes;
  const int smem = (KM == qz::K1K ? 0 : qz::stream_x_bytes(a.K)) + ring;
  int nb = 0;
  if (int rc = blocks_per_sm(fn, smem, &nb)) return rc;
  if (nb < 1) return fail(QZ_ERR_UNSUPPORTED, "gemv: shared memory does not fit");
  const int64_t want = qz::cdiv(a.N, int64_t(R) * qz::kWarps);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, int64_t(d.sms) * nb)));
  return launch_ex(fn, grid, smem, st, false, a);
}

template <int R, bool PER_ROW>
int launch_gemv_k(const DeviceInfo& d, const qz::GemvArgs& a, cudaStream_t st) {
  if constexpr (R == 1) {
    // one-row groups: the deep ring when x plus the ring leave room for three
    // CTAs on an SM
    const int x = kmode(a.K) == qz::K1K && !a.norm_w ? 0 : qz::stream_x_bytes(a.K);
    const int deep = x + qz::kWarps * kDeepRing * qz::kSegBytes;
    if (deep * kMinBlocks <= d.smem_optin - 256 * kMinBlocks) {
      switch (kmode(a.K)) {
        case qz::K1K:
          if (a.norm_w) return launch_gemv<1, PER_ROW, qz::KFULL, kDeepRing>(d, a, st);
          return launch_gemv<1, PER_ROW, qz::K1K, kDeepRing>(d, a, st);
        case qz::KFULL: return launch_gemv<1, PER_ROW, qz::KFULL, kDeepRing>(d, a, st);
        default: return launch_gemv<1, PER_ROW, qz::KANY, kDeepRing>(d, a, st);
      }
    }
  }
  switch (kmode(a.K)) {
    case qz::K1K:
      // A folded RMSNorm needs x staged in shared memory (one coalesced pass
      // per CTA). Single-row groups take the staged mode; four-row groups
      // keep x in registers, where the extra 4 KB would cost a CTA per SM, so
      // the caller runs the norm as its own pass.
      if (a.norm_w && R == 1) return launch_gemv<R, PER_ROW, qz::KFULL>(d, a, st);
      if (a.norm_w) return QZ_ERR_UNSUPPORTED;
      return launch_gemv<R, PER_ROW, qz::K1K>(d, a, st);
    case qz::KFULL: return launch_gemv<R, PER_ROW, qz::KFULL>(d, a, st);
    default: return launch_gemv<R, PER_ROW, qz::KANY>(d, a, st);
  }
}

// int4 row groups: twice the int8 kernel's rows per item over half-size
// (512-byte) segments, so an item carries the same bytes.
constexpr int kW4TallRows = 2 * kTallRows;
constexpr int kW4Rows = 2;

int w4_smem_bytes(int R, int64_t K) {
  return qz::w4_x_bytes(K) + qz::kWarps * qz::kDepth * R * qz::kW4Seg;
}

template <int R, bool PER_ROW, int KM>
int launch_gemv_w4(const DeviceInfo& d, const qz::GemvArgs& a, cudaStream_t st) {
  auto fn = qz::gemv_w4_kernel<R, PER_ROW, KM, kMinBlocks>;
  const int smem = w4_smem_bytes(R, a.K);
  int nb = 0;
  if (int rc = blocks_per_sm(fn, smem, &nb)) return rc;
  if (nb < 1) return fail(QZ_ERR_UNSUPPORTED, "qz_gemv_w4: shared memory does not fit");
  const int64_t want = qz::cdiv(a.N, int64_t(R) * qz::kWarps);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, int64_t(d.sms) * nb)));
  return launch_ex(fn, grid, smem, st, false, a);
}

int gemv_impl(const int8_t* q, const float* scale, int64_t ng, const float* x, float* y,
              int64_t N, int64_t K, const float* residual, cudaStream_t st,
              const qz::comm::PeerOut* po = nullptr, const float* norm_w = nullptr,
              float eps = 0.f) {
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  const int64_t G = K / ng;
  const bool fits = qz::stream_smem_bytes(kTallRows, K) <= d->smem_optin - 256;
  const bool fast = K > 0 && K % 16 == 0 && G % 16 == 0 && aligned16(q) && fits;
  if (!fast && (po || norm_w))
    return fail(QZ_ERR_UNSUPPORTED, "gemv variant: shape outside the streaming kernel");
  if (!fast) return launch_generic_gemm(*d, q, scale, ng, x, y, residual, 1, N, K, st);
  qz::GemvArgs a{q, scale, x, y, residual, N, K, ng};
  if (po) a.po = *po;
  a.norm_w = norm_w;
  a.eps = eps;
  // Tall grouping unless it would leave SMs without a CTA.
  const bool tall = qz::cdiv(N, int64_t(kTallRows) * qz::kWarps) >= d->sms;
  if (ng == 1)
    return tall ? launch_gemv_k<kTallRows, true>(*d, a, st) : launch_gemv_k<1, true>(*d, a, st);
  return tall ? launch_gemv_k<kTallRows, false>(*d, a, st) : launch_gemv_k<1, false>(*d, a, st);
}

template <int R, bool PER_ROW, int KM>
int launch_mlp(const DeviceInfo& d, const qz::MlpArgs& a, cudaStream_t st) {
  auto fn = qz::fused_mlp_kernel<R, PER_ROW, KM, KM, kMinBlocks>;
  const int smem = qz::stream_smem_bytes(R, std::max(a.H, a.I));
  int nb = 0;
  if (int rc = blocks_per_sm(fn, smem, &nb)) return rc;
  if (nb < 1) return fail(QZ_ERR_UNSUPPORTED, "fused mlp: shared memory does not fit");
  const int64_t want = std::max(qz::cdiv(a.I, int64_t(R / 2) * qz::kWarps),
                                qz::cdiv(a.H, int64_t(R) * qz::kWarps));
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, int64_t(d.sms) * nb)));
  return launch_ex(fn, grid, smem, st, true, a);
}

template <int R, bool PER_ROW>
int launch_mlp_k(const DeviceInfo& d, const qz::MlpArgs& a, cudaStream_t st) {
  // Both phases without partial items when H and I are whole KB multiples.
  if (a.H % qz::kSegBytes == 0 && a.I % qz::kSegBytes == 0)
    return launch_mlp<R, PER_ROW, qz::KFULL>(d, a, st);
  return launch_mlp<R, PER_ROW, qz::KANY>(d, a, st);
}

// ---------------------------------------------------------------------------
// tcgen05 GEMM (M > 1): TMA descriptors, workspace layout, launch
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_tiled_fn(EncodeTiledFn* out) {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (err == cudaSuccess && q != cudaDriverEntryPointSuccess) err = cudaErrorNotSupported;
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (err != cudaSuccess || !fn)
    return fail(QZ_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled is not available");
  *out = fn;
  return QZ_OK;
}

// 2-D uint8 tensor [rows, cols] (row-major), tiles of box_rows x 128 bytes,
// 128-byte swizzle.
int make_tmap_u8(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows) {
  EncodeTiledFn enc = nullptr;
  if (int rc = encode_tiled_fn(&enc)) return rc;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(qz::tc::kKBytes),
                             static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(QZ_ERR_CUDA, "cuTensorMapEncodeTiled failed with code " + std::to_string(r));
  return QZ_OK;
}

int tc_token_tile(int64_t M) {
  const int64_t m16 = qz::cdiv(M, 16) * 16;
  return m16 >= 128 ? 128 : m16 > 32 ? 64 : static_cast<int>(m16);
}

// Workspace: [3][Mpad][K] int8 limbs | Mpad fp32 row scales | (split-K)
// [3][Mpad][N] int32 partial sums; each part 256-byte aligned.
struct TcLayout {
  int mt;
  int64_t mpad, limb_bytes, sx_bytes, acc_bytes;
  int64_t total() const { return limb_bytes + sx_bytes + acc_bytes; }
};

TcLayout tc_layout(int64_t M, int64_t N, int64_t K) {
  TcLayout l;
  l.mt = tc_token_tile(M);
  l.mpad = qz::cdiv(M, l.mt) * l.mt;
  auto al = [](int64_t b) { return ((b + 255) / 256) * 256; };
  l.limb_bytes = al(qz::tc::kLimbs * l.mpad * K);
  l.sx_bytes = al(l.mpad * 4);
  l.acc_bytes = al(qz::tc::kLimbs * l.mpad * N * 4);
  return l;
}

template <int MT>
int launch_tc(const DeviceInfo& d, const CUtensorMap& tq, const CUtensorMap& tx,
              const qz::tc::TcArgs& a0, int32_t* acc, cudaStream_t st) {
  auto fn = qz::tc::gemm_i8_kernel<MT>;
  constexpr int sb = qz::tc::stage_bytes(MT);
  // dynamic = stages * sb + 1024 (alignment slack) + 512 (barriers, TMEM slot).
  // Small token tiles: size the ring so two CTAs share an SM (one streams
  // while the other runs its prologue/epilogue); large tiles: one CTA, deep ring.
  const int per_cta = MT <= 32 ? d.smem_optin / 2 - 1024 : d.smem_optin - 256;
  const int budget = per_cta - 1024 - 512;
  const int64_t nk = qz::cdiv(a0.K, qz::tc::kKBytes);
  const int stages = static_cast<int>(std::min<int64_t>(
      std::min(qz::tc::kMaxStages, budget / sb), std::max<int64_t>(2, nk)));
  if (stages < 2) return fail(QZ_ERR_UNSUPPORTED, "tc gemm: shared memory does not fit");
  const int smem = stages * sb + 1024 + 512;
  static std::once_flag once[kMaxDevices];
  int dev = 0;
  QZ_CUDA(cudaGetDevice(&dev));
  cudaError_t ae = cudaSuccess;
  std::call_once(once[dev], [&] { ae = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, d.smem_optin - 256); });
  QZ_CUDA(ae);
  qz::tc::TcArgs a = a0;
  a.nstages = stages;
  // Split K when the output tiles alone would leave SMs idle; the splits add
  // exact int32 partial sums, so the result does not depend on their order.
  const int64_t tiles = qz::cdiv(a.N, qz::tc::kRows) * (a.Mpad / MT);
  // About one CTA per SM for small token tiles (two fit) and one per two SMs
  // for large ones: a same-box sweep of this target (x0.25 .. x4 of
  // 2 x SMs / 1 x SMs) gave the best batched decode and prefill here
  // (Llama-1B prefill 7.03 -> 6.48 ms, 16-sequence Qwen3-8B +3 %).
  const int64_t target = MT <= 32 ? int64_t(d.sms) : int64_t(d.sms) / 2;
  a.splits = tiles >= d.sms || !acc
                 ? 1
                 : static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(nk, qz::cdiv(target, tiles))));
  a.acc = a.splits > 1 ? acc : nullptr;
  if (a.acc)
    QZ_CUDA(cudaMemsetAsync(a.acc, 0, sizeof(int32_t) * qz::tc::kLimbs * a.Mpad * a.N, st));
  const dim3 grid(static_cast<unsigned>(a.Mpad / MT),
                  static_cast<unsigned>(qz::cdiv(a.N, qz::tc::kRows)), static_cast<unsigned>(a.splits));
  fn<<<grid, qz::tc::kThreads, smem, st>>>(tq, tx, a);
  QZ_CUDA(cudaGetLastError());
  if (a.acc) {
    const int64_t total = a.M * a.N;
    const int blocks = static_cast<int>(std::min<int64_t>(qz::cdiv(total, 256), d.sms * 8));
    qz::tc::splitk_finish_kernel<<<blocks, 256, 0, st>>>(a.acc, a.scale, a.sx, a.residual, a.Y,
                                                        a.M, a.N, a.Mpad);
    QZ_CUDA(cudaGetLastError());
  }
  return QZ_OK;
}

int tc_gemm(const DeviceInfo& d, const int8_t* q, const float* scale, const float* X, float* Y,
            int64_t M, int64_t N, int64_t K, const float* residual, void* ws, size_t ws_bytes,
            cudaStream_t st, int act = qz::tc::kActNone, const float* norm_w = nullptr,
            float eps = 0.f) {
  const TcLayout L = tc_layout(M, N, K);
  int8_t* limbs = static_cast<int8_t*>(ws);
  float* sx = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + L.limb_bytes);
  int32_t* acc = static_cast<int64_t>(ws_bytes) >= L.total()
                     ? reinterpret_cast<int32_t*>(static_cast<uint8_t*>(ws) + L.limb_bytes +
                                                  L.sx_bytes)
                     : nullptr;
  const dim3 sgrid(static_cast<unsigned>(L.mpad));
  switch (act) {
    case qz::tc::kActRmsNorm:
      qz::tc::split_x_kernel<qz::tc::kActRmsNorm><<<sgrid, qz::tc::kSplitThreads, 0, st>>>(
          X, K, norm_w, eps, limbs, sx, M, L.mpad, K);
      break;
    case qz::tc::kActSiluMul:
      qz::tc::split_x_kernel<qz::tc::kActSiluMul><<<sgrid, qz::tc::kSplitThreads, 0, st>>>(
          X, 2 * K, nullptr, 0.f, limbs, sx, M, L.mpad, K);
      break;
    default:
      qz::tc::split_x_kernel<qz::tc::kActNone><<<sgrid, qz::tc::kSplitThreads, 0, st>>>(
          X, K, nullptr, 0.f, limbs, sx, M, L.mpad, K);
  }
  QZ_CUDA(cudaGetLastError());
  CUtensorMap tq, tx;
  if (int rc = make_tmap_u8(&tq, q, N, K, qz::tc::kRows)) return rc;
  if (int rc = make_tmap_u8(&tx, limbs, qz::tc::kLimbs * L.mpad, K, L.mt)) return rc;
  const qz::tc::TcArgs a{scale, sx, Y, residual, nullptr, M, N, K, L.mpad, 0, 1};
  switch (L.mt) {
    case 16: return launch_tc<16>(d, tq, tx, a, acc, st);
    case 32: return launch_tc<32>(d, tq, tx, a, acc, st);
    case 64: return launch_tc<64>(d, tq, tx, a, acc, st);
    default: return launch_tc<128>(d, tq, tx, a, acc, st);
  }
}

}  // namespace

extern "C" {

int qz_version(void) { return (0 << 16) | (1 << 8) | 0; }

int qz_init(int device) {
  QZ_CUDA(cudaSetDevice(device));
  DeviceInfo* d = nullptr;
  return device_info(&d);
}

int qz_last_error(char* buf, size_t len) {
  if (buf && len) {
    const size_t n = std::min(len - 1, g_err.size());
    std::memcpy(buf, g_err.data(), n);
    buf[n] = '\0';
  }
  return static_cast<int>(g_err.size());
}

int qz_gemv_w8(const int8_t* q, const float* scale, int64_t ng, const float* x, float* y,
               int64_t N, int64_t K, const float* residual, void* stream) {
  if (int rc = check_weights(q, scale, ng, N, K, "qz_gemv_w8")) return rc;
  if (N == 0) return QZ_OK;
  if (!y || (K > 0 && !x)) return fail(QZ_ERR_INVALID, "qz_gemv_w8: null x or y");
  return gemv_impl(q, scale, ng, x, y, N, K, residual, static_cast<cudaStream_t>(stream));
}

namespace {
// Device-to-host copies of y go out in chunks of this size, each followed by
// an event, so the host copy of one chunk into the caller's array overlaps
// the DMA of the next.
constexpr int64_t kHostChunkBytes = 128 * 1024;
constexpr int kHostChunks = 16;
thread_local cudaEvent_t t_copy_ev[kMaxDevices][kHostChunks];

int copy_events(cudaEvent_t** out) {
  int dev = 0;
  QZ_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(QZ_ERR_UNSUPPORTED, "device index out of range");
  cudaEvent_t* ev = t_copy_ev[dev];
  if (!ev[kHostChunks - 1]) {
    // all or nothing: a failed creation leaves the set empty for the next call
    cudaEvent_t fresh[kHostChunks] = {};
    for (int i = 0; i < kHostChunks; ++i) {
      const cudaError_t e = cudaEventCreateWithFlags(&fresh[i], cudaEventDisableTiming);
      if (e != cudaSuccess) {
        for (int j = 0; j < i; ++j) (void)cudaEventDestroy(fresh[j]);
        return fail(QZ_ERR_CUDA, std::string("cudaEventCreateWithFlags: ") + cudaGetErrorString(e));
      }
    }
    for (int i = 0; i < kHostChunks; ++i) ev[i] = fresh[i];
  }
  *out = ev;
  return QZ_OK;
}
}  // namespace

int qz_gemv_w8_host(const int8_t* q, const float* scale, int64_t ng, const float* x_host,
                    float* y_host, int64_t N, int64_t K, float* x_pin, float* y_pin,
                    float* x_dev, float* y_dev, void* stream) {
  if (int rc = check_weights(q, scale, ng, N, K, "qz_gemv_w8_host")) return rc;
  if (N == 0) return QZ_OK;
  if (!y_host || !y_pin || !y_dev || (K > 0 && (!x_host || !x_pin || !x_dev)))
    return fail(QZ_ERR_INVALID, "qz_gemv_w8_host: null host, pinned or device buffer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaEvent_t* ev = nullptr;
  if (int rc = copy_events(&ev)) return rc;
  if (K > 0) {
    std::memcpy(x_pin, x_host, static_cast<size_t>(K) * 4);
    QZ_CUDA(cudaMemcpyAsync(x_dev, x_pin, static_cast<size_t>(K) * 4, cudaMemcpyHostToDevice, st));
  }
  if (int rc = gemv_impl(q, scale, ng, x_dev, y_dev, N, K, nullptr, st)) return rc;
  const int64_t bytes = N * 4;
  const int64_t chunk = std::max<int64_t>(kHostChunkBytes, qz::cdiv(bytes, kHostChunks * 16) * 16);
  const int n = static_cast<int>(qz::cdiv(bytes, chunk));
  for (int i = 0; i < n; ++i) {
    const int64_t off = i * chunk, len = std::min(chunk, bytes - off);
    QZ_CUDA(cudaMemcpyAsync(reinterpret_cast<char*>(y_pin) + off,
                            reinterpret_cast<const char*>(y_dev) + off, static_cast<size_t>(len),
                            cudaMemcpyDeviceToHost, st));
    QZ_CUDA(cudaEventRecord(ev[i], st));
  }
  for (int i = 0; i < n; ++i) {
    const int64_t off = i * chunk, len = std::min(chunk, bytes - off);
    QZ_CUDA(cudaEventSynchronize(ev[i]));
    std::memcpy(reinterpret_cast<char*>(y_host) + off, reinterpret_cast<const char*>(y_pin) + off,
                static_cast<size_t>(len));
  }
  return QZ_OK;
}


int qz_gemv_w4(const uint8_t* q4, const float* scale, int64_t ng, const float* x, float* y,
               int64_t N, int64_t K, const float* residual, void* stream) {
  if (N < 0 || K < 0) return fail(QZ_ERR_INVALID, "qz_gemv_w4: negative dimension");
  if (ng < 1 || K % ng != 0) return fail(QZ_ERR_INVALID, "qz_gemv_w4: ng must be >= 1 and divide K");
  if (K % 32 != 0 || (K / ng) % 32 != 0)
    return fail(QZ_ERR_INVALID, "qz_gemv_w4: K and the group size must be multiples of 32");
  if (N == 0) return QZ_OK;
  if (K == 0) return fail(QZ_ERR_INVALID, "qz_gemv_w4: K must be positive");
  if (!q4 || !scale || !x || !y) return fail(QZ_ERR_INVALID, "qz_gemv_w4: null pointer");
  if (!aligned16(q4)) return fail(QZ_ERR_INVALID, "qz_gemv_w4: q4 must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  if (w4_smem_bytes(kW4TallRows, K) > d->smem_optin - 256)
    return fail(QZ_ERR_UNSUPPORTED, "qz_gemv_w4: K too large for the staged activations");
  qz::GemvArgs a{reinterpret_cast<const int8_t*>(q4), scale, x, y, residual, N, K, ng};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Eight-row groups for tall matrices whose rows are whole 512-byte
  // segments (the lm_head); two-row groups otherwise, including rows with a
  // partial last segment.
  const bool full = (K / 2) % qz::kW4Seg == 0;
  const bool tall = full && qz::cdiv(N, int64_t(kW4TallRows) * qz::kWarps) >= d->sms;
  if (tall)
    return ng == 1 ? launch_gemv_w4<kW4TallRows, true, qz::KFULL>(*d, a, st)
                   : launch_gemv_w4<kW4TallRows, false, qz::KFULL>(*d, a, st);
  if (full)
    return ng == 1 ? launch_gemv_w4<kW4Rows, true, qz::KFULL>(*d, a, st)
                   : launch_gemv_w4<kW4Rows, false, qz::KFULL>(*d, a, st);
  return ng == 1 ? launch_gemv_w4<kW4Rows, true, qz::KANY>(*d, a, st)
                 : launch_gemv_w4<kW4Rows, false, qz::KANY>(*d, a, st);
}

int qz_gemm_w8(const int8_t* q, const float* scale, int64_t ng, const float* X, float* Y,
               int64_t M, int64_t N, int64_t K, const float* residual, void* stream) {
  if (int rc = check_weights(q, scale, ng, N, K, "qz_gemm_w8")) return rc;
  if (M < 0) return fail(QZ_ERR_INVALID, "qz_gemm_w8: negative M");
  if (M == 0 || N == 0) return QZ_OK;
  if (!Y || (K > 0 && !X)) return fail(QZ_ERR_INVALID, "qz_gemm_w8: null X or Y");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (M == 1) return gemv_impl(q, scale, ng, X, Y, N, K, residual, st);
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  return launch_generic_gemm(*d, q, scale, ng, X, Y, residual, M, N, K, st);
}

int qz_gemm_w8_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t* bytes) {
  if (!bytes) return fail(QZ_ERR_INVALID, "qz_gemm_w8_workspace_bytes: null bytes");
  if (M < 0 || N < 0 || K < 0)
    return fail(QZ_ERR_INVALID, "qz_gemm_w8_workspace_bytes: negative size");
  *bytes = M >= 2 ? tc_layout(M, N, K).total() : 0;
  return QZ_OK;
}

int qz_gemm_w8_ws(const int8_t* q, const float* scale, int64_t ng, const float* X, float* Y,
                  int64_t M, int64_t N, int64_t K, const float* residual, void* workspace,
                  size_t workspace_bytes, void* stream) {
  if (int rc = check_weights(q, scale, ng, N, K, "qz_gemm_w8_ws")) return rc;
  if (M < 0) return fail(QZ_ERR_INVALID, "qz_gemm_w8_ws: negative M");
  if (M == 0 || N == 0) return QZ_OK;
  if (!Y || (K > 0 && !X)) return fail(QZ_ERR_INVALID, "qz_gemm_w8_ws: null X or Y");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (M == 1) return gemv_impl(q, scale, ng, X, Y, N, K, residual, st);
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  // The tensor path needs at least the limb + row-scale part of the workspace;
  // with the whole of it, it may also split K.
  const TcLayout L = tc_layout(M, N, K);
  const bool tensor = ng == 1 && K > 0 && K % 16 == 0 && aligned16(q) && workspace &&
                      aligned16(workspace) &&
                      static_cast<int64_t>(workspace_bytes) >= L.limb_bytes + L.sx_bytes;
  if (!tensor) return launch_generic_gemm(*d, q, scale, ng, X, Y, residual, M, N, K, st);
  return tc_gemm(*d, q, scale, X, Y, M, N, K, residual, workspace, workspace_bytes, st);
}

int qz_gemm_w8_act_ws(const int8_t* q, const float* scale, int64_t ng, const float* X, int act,
                      const float* norm_w, float eps, float* Y, int64_t M, int64_t N, int64_t K,
                      const float* residual, void* workspace, size_t workspace_bytes,
                      void* stream) {
  if (act == QZ_ACT_NONE)
    return qz_gemm_w8_ws(q, scale, ng, X, Y, M, N, K, residual, workspace, workspace_bytes,
                         stream);
  if (act != QZ_ACT_RMSNORM && act != QZ_ACT_SILU_MUL)
    return fail(QZ_ERR_INVALID, "qz_gemm_w8_act_ws: unknown act");
  if (int rc = check_weights(q, scale, ng, N, K, "qz_gemm_w8_act_ws")) return rc;
  if (M < 0) return fail(QZ_ERR_INVALID, "qz_gemm_w8_act_ws: negative M");
  if (M == 0 || N == 0) return QZ_OK;
  if (!Y || !X || K < 1) return fail(QZ_ERR_INVALID, "qz_gemm_w8_act_ws: null X or Y, or K < 1");
  if (act == QZ_ACT_RMSNORM && !norm_w)
    return fail(QZ_ERR_INVALID, "qz_gemm_w8_act_ws: RMSNorm needs norm_w");
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  const TcLayout L = tc_layout(M, N, K);
  // only the tensor path has a split kernel to carry the prologue
  const bool tensor = M >= 2 && ng == 1 && K % 16 == 0 && aligned16(q) && workspace &&
                      aligned16(workspace) &&
                      static_cast<int64_t>(workspace_bytes) >= L.limb_bytes + L.sx_bytes;
  if (!tensor)
    return fail(QZ_ERR_UNSUPPORTED,
                "qz_gemm_w8_act_ws: needs M >= 2, per-row scales, K % 16 == 0, aligned weights "
                "and the limb workspace");
  return tc_gemm(*d, q, scale, X, Y, M, N, K, residual, workspace, workspace_bytes,
                 static_cast<cudaStream_t>(stream),
                 act == QZ_ACT_RMSNORM ? qz::tc::kActRmsNorm : qz::tc::kActSiluMul, norm_w, eps);
}

int qz_mlp_workspace_bytes(void) { return 256; }

}  // extern "C"

namespace {
int mlp_impl(const int8_t* gu_q, const float* gu_s, int64_t ng, const float* x,
             const int8_t* down_q, const float* down_s, int64_t ngd, float* abuf, float* out,
             const float* residual, int64_t H, int64_t I, uint32_t* sync_ws, void* stream,
             const qz::comm::PeerOut* po, const float* norm_w = nullptr, float eps = 0.f,
             bool clear_barrier = false) {
  if (int rc = check_weights(gu_q, gu_s, ng, 2 * I, H, "qz_fused_mlp_decode (gate|up)")) return rc;
  if (int rc = check_weights(down_q, down_s, ngd, H, I, "qz_fused_mlp_decode (down)")) return rc;
  if (H == 0) return QZ_OK;
  if ((!out && !po) || (I > 0 && !abuf) || !x)
    return fail(QZ_ERR_INVALID, "qz_fused_mlp_decode: null x, abuf or out");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  const int64_t kmax = std::max(H, I);
  const bool fits = qz::stream_smem_bytes(kTallRows, kmax) <= d->smem_optin - 256;
  const bool fast = I > 0 && H % 16 == 0 && I % 16 == 0 && (H / ng) % 16 == 0 &&
                    (I / ngd) % 16 == 0 && aligned16(gu_q) && aligned16(down_q) && fits &&
                    sync_ws != nullptr && d->coop;
  if (!fast && (po || norm_w))
    return fail(QZ_ERR_UNSUPPORTED, "fused mlp variant: shape outside the fused kernel");
  if (!fast) {
    // Two launches: gate/up + SiLU into abuf, then the down GEMV.
    if (I > 0) {
      const int threads = 256;
      const int blocks = static_cast<int>(std::min<int64_t>(qz::cdiv(I, threads / 32), d->sms * 8));
      qz::generic_mlp_gate_kernel<<<blocks, threads, 0, st>>>(gu_q, gu_s, ng, x, abuf, H, I);
      QZ_CUDA(cudaGetLastError());
    }
    return launch_generic_gemm(*d, down_q, down_s, ngd, abuf, out, residual, 1, H, I, st);
  }
  // clear_barrier: the arrival count is zeroed (stream-ordered) right before
  // the cooperative launch, the only path that uses it
  if (clear_barrier) QZ_CUDA(cudaMemsetAsync(sync_ws, 0, sizeof(uint32_t), st));
  qz::MlpArgs a{gu_q, gu_s, x, down_q, down_s, abuf, out, residual, sync_ws, H, I, ng, ngd};
  if (po) a.po = *po;
  a.norm_w = norm_w;
  a.eps = eps;
  const bool per_row = ng == 1 && ngd == 1;
  // Tall groups (2 units = 4 rows) unless too few units to fill the SMs.
  const bool tall = qz::cdiv(I, int64_t(kTallRows / 2) * qz::kWarps) >= d->sms;
  if (per_row)
    return tall ? launch_mlp_k<kTallRows, true>(*d, a, st) : launch_mlp_k<2, true>(*d, a, st);
  return tall ? launch_mlp_k<kTallRows, false>(*d, a, st) : launch_mlp_k<2, false>(*d, a, st);
}

int peer_out(const qz_peer_sum* ps, int64_t n, qz::comm::PeerOut* po, const char* what) {
  if (!ps || ps->ranks < 1 || ps->ranks > qz::comm::kMaxRanks || ps->rank < 0 ||
      ps->rank >= ps->ranks || ps->n_max % 4 || n > ps->n_max)
    return fail(QZ_ERR_INVALID, std::string(what) + ": bad qz_peer_sum (ranks, rank, n_max)");
  *po = qz::comm::PeerOut{};
  for (int j = 0; j < ps->ranks; ++j) {
    if (!ps->buffers[j] || !aligned16(ps->buffers[j]))
      return fail(QZ_ERR_INVALID, std::string(what) + ": null or unaligned peer buffer");
    po->base[j] = static_cast<float*>(ps->buffers[j]);
  }
  po->rank = ps->rank;
  po->P = ps->ranks;
  po->n_max = ps->n_max;
  return QZ_OK;
}
}  // namespace

extern "C" {

int qz_fused_mlp_decode(const int8_t* gu_q, const float* gu_s, int64_t ng, const float* x,
                        const int8_t* down_q, const float* down_s, int64_t ngd, float* abuf,
                        float* out, const float* residual, int64_t H, int64_t I,
                        uint32_t* sync_ws, void* stream) {
  return mlp_impl(gu_q, gu_s, ng, x, down_q, down_s, ngd, abuf, out, residual, H, I, sync_ws,
                  stream, nullptr);
}

int qz_fused_mlp_decode_peer(const int8_t* gu_q, const float* gu_s, int64_t ng, const float* x,
                             const int8_t* down_q, const float* down_s, int64_t ngd, float* abuf,
                             const float* residual, int64_t H, int64_t I, uint32_t* sync_ws,
                             const qz_peer_sum* ps, void* stream) {
  qz::comm::PeerOut po;
  if (int rc = peer_out(ps, H, &po, "qz_fused_mlp_decode_peer")) return rc;
  return mlp_impl(gu_q, gu_s, ng, x, down_q, down_s, ngd, abuf, nullptr, residual, H, I, sync_ws,
                  stream, &po);
}

int qz_gemv_w8_rmsnorm(const int8_t* q, const float* scale, int64_t ng, const float* x,
                       const float* norm_w, float eps, float* y, int64_t N, int64_t K,
                       const float* residual, float* xn_scratch, void* stream) {
  if (int rc = check_weights(q, scale, ng, N, K, "qz_gemv_w8_rmsnorm")) return rc;
  if (N == 0) return QZ_OK;
  if (!y || !norm_w || (K > 0 && !x))
    return fail(QZ_ERR_INVALID, "qz_gemv_w8_rmsnorm: null x, norm_w or y");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int rc = gemv_impl(q, scale, ng, x, y, N, K, residual, st, nullptr, norm_w, eps);
  if (rc != QZ_ERR_UNSUPPORTED) return rc;
  // other shapes: the norm into the caller's scratch, then the plain GEMV
  if (!xn_scratch) return fail(QZ_ERR_UNSUPPORTED, "qz_gemv_w8_rmsnorm: shape needs xn_scratch");
  if (int rc = qz_rmsnorm(x, norm_w, xn_scratch, 1, K, eps, stream)) return rc;
  return gemv_impl(q, scale, ng, xn_scratch, y, N, K, residual, st);
}

int qz_fused_mlp_decode_rmsnorm(const int8_t* gu_q, const float* gu_s, int64_t ng,
                                const float* x, const float* norm_w, float eps,
                                const int8_t* down_q, const float* down_s, int64_t ngd,
                                float* abuf, float* out, const float* residual, int64_t H,
                                int64_t I, uint32_t* sync_ws, float* xn_scratch, void* stream) {
  if (!norm_w) return fail(QZ_ERR_INVALID, "qz_fused_mlp_decode_rmsnorm: null norm_w");
  const int rc = mlp_impl(gu_q, gu_s, ng, x, down_q, down_s, ngd, abuf, out, residual, H, I,
                          sync_ws, stream, nullptr, norm_w, eps);
  if (rc != QZ_ERR_UNSUPPORTED) return rc;
  if (!xn_scratch)
    return fail(QZ_ERR_UNSUPPORTED, "qz_fused_mlp_decode_rmsnorm: shape needs xn_scratch");
  if (int rc2 = qz_rmsnorm(x, norm_w, xn_scratch, 1, H, eps, stream)) return rc2;
  return mlp_impl(gu_q, gu_s, ng, xn_scratch, down_q, down_s, ngd, abuf, out, residual, H, I,
                  sync_ws, stream, nullptr);
}

int qz_gemv_w8_peer(const int8_t* q, const float* scale, int64_t ng, const float* x, int64_t N,
                    int64_t K, const float* residual, const qz_peer_sum* ps, void* stream) {
  if (int rc = check_weights(q, scale, ng, N, K, "qz_gemv_w8_peer")) return rc;
  if (N == 0) return QZ_OK;
  if (K > 0 && !x) return fail(QZ_ERR_INVALID, "qz_gemv_w8_peer: null x");
  qz::comm::PeerOut po;
  if (int rc = peer_out(ps, N, &po, "qz_gemv_w8_peer")) return rc;
  return gemv_impl(q, scale, ng, x, nullptr, N, K, residual, static_cast<cudaStream_t>(stream),
                   &po);
}

int qz_rmsnorm_peer_sum(const qz_peer_sum* ps, int64_t n, const float* w, float eps, float* h,
                        float* xn, void* stream) {
  qz::comm::PeerOut po;
  if (int rc = peer_out(ps, n, &po, "qz_rmsnorm_peer_sum")) return rc;
  if (n < 1 || n > qz::comm::kSumThreads * qz::comm::kSumPer)
    return fail(QZ_ERR_INVALID, "qz_rmsnorm_peer_sum: n must be in [1, 4096]");
  if (!w || !h || !xn) return fail(QZ_ERR_INVALID, "qz_rmsnorm_peer_sum: null pointer");
  qz::comm::rmsnorm_peer_sum_kernel<<<1, qz::comm::kSumThreads, 0,
                                      static_cast<cudaStream_t>(stream)>>>(
      po.base[po.rank], po.P, po.n_max, h, w, xn, n, eps);
  QZ_CUDA(cudaGetLastError());
  return QZ_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free fused MLP. Its scratch (the [I] intermediate and the grid
// barrier words) lives in this file-scope device array instead of buffers the
// caller allocates. Every GPU that loads the library holds the array
// (kNoAllocMaxI * 4 + 256 bytes = 128.25 KB) until the process exits.
// ---------------------------------------------------------------------------
namespace {
constexpr int64_t kNoAllocMaxI = 32768;      // largest intermediate size accepted
constexpr int64_t kNoAllocBarrierWords = 64; // qz_mlp_workspace_bytes() / 4
}  // namespace

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocMaxI + kNoAllocBarrierWords];

namespace {
struct NoAllocScratch {
  std::once_flag once;
  float* ptr = nullptr;
  cudaError_t err = cudaSuccess;
};
NoAllocScratch g_noalloc[kMaxDevices];

// Device address of the scratch array on the current device, looked up once
// per device (with that device current) on the first call there.
int noalloc_scratch(float** out) {
  int dev = 0;
  QZ_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(QZ_ERR_UNSUPPORTED, "device index out of range");
  NoAllocScratch& s = g_noalloc[dev];
  std::call_once(s.once, [&] {
    s.err = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.ptr), g_noalloc_scratch);
  });
  if (s.err != cudaSuccess)
    return fail(QZ_ERR_CUDA, std::string("cudaGetSymbolAddress(no-alloc scratch): ") +
                                 cudaGetErrorString(s.err));
  *out = s.ptr;
  return QZ_OK;
}
}  // namespace

extern "C" {

int qz_fused_mlp_decode_noalloc(const int8_t* gu_q, const float* gu_s, int64_t ng, const float* x,
                                const int8_t* down_q, const float* down_s, int64_t ngd, float* out,
                                const float* residual, int64_t H, int64_t I, void* stream) {
  if (I < 0 || I > kNoAllocMaxI)
    return fail(QZ_ERR_INVALID,
                "qz_fused_mlp_decode_noalloc: I=" + std::to_string(I) +
                    " is outside the built-in scratch capacity [0, " +
                    std::to_string(kNoAllocMaxI) +
                    "]; call qz_fused_mlp_decode with caller-owned abuf and sync_ws instead");
  float* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  uint32_t* barrier = reinterpret_cast<uint32_t*>(scratch + kNoAllocMaxI);
  // The barrier's arrival count must be zero when the cooperative kernel
  // starts; a call whose wait gave up could have left it otherwise. mlp_impl
  // checks the arguments first and clears it (stream-ordered) only on the
  // path that launches that kernel, so a refused call or the two-launch
  // fallback leaves nothing on the stream beyond its own kernels.
  return mlp_impl(gu_q, gu_s, ng, x, down_q, down_s, ngd, scratch, out, residual, H, I, barrier,
                  stream, nullptr, nullptr, 0.f, /*clear_barrier=*/true);
}


// ---------------------------------------------------------------------------
// decode-step glue (device pointers; stream-ordered)
// ---------------------------------------------------------------------------
int qz_embed_gather(const int8_t* q, const float* scale, int64_t ng, const int64_t* ids,
                    int64_t M, int64_t V, int64_t H, float* out, void* stream) {
  if (int rc = check_weights(q, scale, ng, V, H, "qz_embed_gather")) return rc;
  if (M < 0) return fail(QZ_ERR_INVALID, "qz_embed_gather: negative M");
  if (M == 0 || H == 0) return QZ_OK;
  if (!ids || !out || V < 1) return fail(QZ_ERR_INVALID, "qz_embed_gather: null ids/out or empty table");
  qz::dec::embed_gather_kernel<<<static_cast<unsigned>(M), 256, 0,
                                 static_cast<cudaStream_t>(stream)>>>(q, scale, ng, ids, V, H, out);
  QZ_CUDA(cudaGetLastError());
  return QZ_OK;
}

int qz_rmsnorm(const float* x, const float* w, float* y, int64_t rows, int64_t n, float eps,
               void* stream) {
  if (rows < 0 || n < 0) return fail(QZ_ERR_INVALID, "qz_rmsnorm: negative size");
  if (rows == 0 || n == 0) return QZ_OK;
  if (!x || !w || !y) return fail(QZ_ERR_INVALID, "qz_rmsnorm: null pointer");
  qz::dec::rmsnorm_kernel<<<static_cast<unsigned>(rows), qz::dec::kNormThreads, 0,
                            static_cast<cudaStream_t>(stream)>>>(x, w, y, n, eps);
  QZ_CUDA(cudaGetLastError());
  return QZ_OK;
}

}  // extern "C"

namespace {
int check_heads(int nq, int nkv, int hd, const char* what) {
  if (nq < 1 || nkv < 1 || nq % nkv)
    return fail(QZ_ERR_INVALID, std::string(what) + ": query heads must be a multiple of kv heads");
  if (hd < 2 || hd % 2 || hd > 256)
    return fail(QZ_ERR_INVALID, std::string(what) + ": head_dim must be even and <= 256");
  if (nq / nkv > 8) return fail(QZ_ERR_INVALID, std::string(what) + ": at most 8 query heads per kv head");
  return QZ_OK;
}
}  // namespace

extern "C" {

int qz_qk_rope(const float* qkv, const float* q_norm_w, const float* k_norm_w,
               const float* inv_freq, float* q_out, float* k_cache, float* v_cache, int64_t M,
               int nq, int nkv, int hd, int64_t max_ctx, int64_t pos0, const int64_t* pos_dev,
               float eps, void* stream) {
  if (int rc = check_heads(nq, nkv, hd, "qz_qk_rope")) return rc;
  if (M < 0 || max_ctx < 1) return fail(QZ_ERR_INVALID, "qz_qk_rope: bad M or max_ctx");
  if (M == 0) return QZ_OK;
  if (!qkv || !inv_freq || !q_out || !k_cache || !v_cache)
    return fail(QZ_ERR_INVALID, "qz_qk_rope: null pointer");
  if (!pos_dev && (pos0 < 0 || pos0 + M > max_ctx))
    return fail(QZ_ERR_INVALID, "qz_qk_rope: positions beyond the cache");
  const dim3 grid(static_cast<unsigned>(M), static_cast<unsigned>(nq + 2 * nkv));
  qz::dec::qk_rope_kernel<<<grid, 128, hd * sizeof(float), static_cast<cudaStream_t>(stream)>>>(
      qkv, q_norm_w, k_norm_w, inv_freq, q_out, k_cache, v_cache, nq, nkv, hd, max_ctx, pos0,
      pos_dev, eps);
  QZ_CUDA(cudaGetLastError());
  return QZ_OK;
}

}  // extern "C"

namespace {

// Decode-attention workspace: [tickets: n_kv u32, padded to 256 B]
// [fused partials: n_kv * S * n_rep * (hd + 2) fp32, or the chunked kernels'
// nq * ceil(max_ctx / 64) * (hd + 2), whichever is larger] [q scratch: nq * hd fp32].
struct AttnLayout {
  int S;
  int64_t part_off, q_off, total;
};

// Context splits per kv head: about two CTAs per SM in all, at least 32
// positions per split, at most 32. Since the merge loads every split's
// partials in one round, two CTAs per SM beat one (Qwen3-8B heads, context
// 2048, graph replay: 11.5 vs 12.7 us); before that change one was faster.
// The cap: the last CTA of a kv head merges the splits' partials from L2, so
// a tensor-parallel rank with one or two kv heads would otherwise spend more
// on the merge (66 splits at one kv head and context 2112) than on its share
// of the cache.
constexpr int kMaxAttnSplits = 32;
int attn_splits(const DeviceInfo& d, int nkv, int64_t max_ctx) {
  const int64_t s = std::min<int64_t>(std::min<int64_t>(qz::cdiv(2 * int64_t(d.sms), nkv),
                                                         qz::cdiv(max_ctx, 32)), kMaxAttnSplits);
  return static_cast<int>(std::max<int64_t>(1, s));
}

AttnLayout attn_layout(const DeviceInfo& d, int nq, int nkv, int hd, int64_t max_ctx) {
  AttnLayout l;
  l.S = attn_splits(d, nkv, max_ctx);
  auto al = [](int64_t b) { return ((b + 255) / 256) * 256; };
  const int64_t fused = static_cast<int64_t>(nkv) * l.S * (nq / nkv) * (hd + 2) * 4;
  const int64_t chunked = static_cast<int64_t>(nq) * qz::cdiv(max_ctx, qz::dec::kChunk) * (hd + 2) * 4;
  l.part_off = al(static_cast<int64_t>(nkv) * 4);
  l.q_off = l.part_off + al(std::max(fused, chunked));
  l.total = l.q_off + al(static_cast<int64_t>(nq) * hd * 4);
  return l;
}

template <int E, int NR, bool QKV>
int launch_attn_fused(const qz::dec::AttnArgs& a, int S, cudaStream_t st, int batch = 1) {
  constexpr int smem = qz::dec::attn_fused_smem<E, NR>();
  static_assert(smem <= 200 * 1024, "fused attention shared memory above the opt-in limit");
  // above 48 KB the launch needs the opt-in limit, set once per device
  static std::once_flag once[kMaxDevices];
  int dev = 0;
  QZ_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(QZ_ERR_UNSUPPORTED, "device index out of range");
  cudaError_t ae = cudaSuccess;
  std::call_once(once[dev], [&] {
    ae = cudaFuncSetAttribute(qz::dec::attn_decode_fused_kernel<E, NR, QKV>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  });
  QZ_CUDA(ae);
  // a programmatic dependent launch: the kernel hints its cache rows into L2
  // before griddepcontrol.wait and lets the next kernel launch early
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(a.nkv), static_cast<unsigned>(S),
                     static_cast<unsigned>(batch));
  cfg.blockDim = dim3(qz::dec::kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  QZ_CUDA(cudaLaunchKernelEx(&cfg, qz::dec::attn_decode_fused_kernel<E, NR, QKV>, a));
  return QZ_OK;
}

template <bool QKV>
int dispatch_attn_fused(int hd, int n_rep, const qz::dec::AttnArgs& a, int S, cudaStream_t st,
                        bool* done, int batch = 1) {
  *done = true;
#define QZ_ATTN_CASE(E_, NR_) \
  if (hd == 32 * (E_) && n_rep == (NR_)) return launch_attn_fused<E_, NR_, QKV>(a, S, st, batch);
  QZ_ATTN_CASE(2, 1) QZ_ATTN_CASE(2, 2) QZ_ATTN_CASE(2, 4) QZ_ATTN_CASE(2, 8)
  QZ_ATTN_CASE(4, 1) QZ_ATTN_CASE(4, 2) QZ_ATTN_CASE(4, 4) QZ_ATTN_CASE(4, 8)
  QZ_ATTN_CASE(8, 1) QZ_ATTN_CASE(8, 2) QZ_ATTN_CASE(8, 4)
#undef QZ_ATTN_CASE
  *done = false;
  return QZ_OK;
}

bool aligned_to(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// The chunked kernels (any head_dim <= 256, n_rep <= 8): attention + combine.
int attn_chunked(const float* q, const float* kc, const float* vc, float* out, int nq, int nkv,
                 int hd, int64_t max_ctx, int64_t T, const int64_t* T_dev, int64_t t_offset,
                 float scale, float* part, cudaStream_t st) {
  const int64_t span = T_dev ? max_ctx : T;
  const int64_t nchunks = qz::cdiv(span, qz::dec::kChunk);
  const int n_rep = nq / nkv;
  const int smem = (n_rep * hd + n_rep * qz::dec::kChunk) * 4;
  const dim3 grid(static_cast<unsigned>(nkv), static_cast<unsigned>(nchunks));
  qz::dec::attn_decode_kernel<<<grid, 256, smem, st>>>(q, kc, vc, part, nq, nkv, hd, max_ctx, T,
                                                       T_dev, t_offset, scale);
  QZ_CUDA(cudaGetLastError());
  qz::dec::attn_combine_kernel<<<static_cast<unsigned>(nq), 128, 0, st>>>(
      part, out, hd, static_cast<int>(nchunks));
  QZ_CUDA(cudaGetLastError());
  return QZ_OK;
}
}  // namespace

extern "C" {

int qz_attention_decode_workspace_bytes(int nq, int nkv, int hd, int64_t max_ctx, int64_t* bytes) {
  if (!bytes || nq < 1 || nkv < 1 || nq % nkv || hd < 1 || max_ctx < 1)
    return fail(QZ_ERR_INVALID, "qz_attention_decode_workspace_bytes: bad arguments");
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  *bytes = attn_layout(*d, nq, nkv, hd, max_ctx).total;
  return QZ_OK;
}

int qz_attention_decode(const float* q, const float* k_cache, const float* v_cache, float* out,
                        int nq, int nkv, int hd, int64_t max_ctx, int64_t T, const int64_t* T_dev,
                        int64_t t_offset, float scale, void* ws, size_t ws_bytes, void* stream) {
  if (int rc = check_heads(nq, nkv, hd, "qz_attention_decode")) return rc;
  if (max_ctx < 1) return fail(QZ_ERR_INVALID, "qz_attention_decode: bad max_ctx");
  if (!T_dev && (T < 1 || T > max_ctx))
    return fail(QZ_ERR_INVALID, "qz_attention_decode: context length outside [1, max_ctx]");
  if (!q || !k_cache || !v_cache || !out || !ws)
    return fail(QZ_ERR_INVALID, "qz_attention_decode: null pointer");
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  const AttnLayout L = attn_layout(*d, nq, nkv, hd, max_ctx);
  if (static_cast<int64_t>(ws_bytes) < L.total || !aligned_to(ws, 256))
    return fail(QZ_ERR_INVALID, "qz_attention_decode: workspace too small or not 256-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* w = static_cast<char*>(ws);
  float* part = reinterpret_cast<float*>(w + L.part_off);
  if (aligned16(q) && aligned16(k_cache) && aligned16(v_cache)) {
    qz::dec::AttnArgs a{};
    a.in = q;
    a.kc = const_cast<float*>(k_cache);
    a.vc = const_cast<float*>(v_cache);
    a.out = out;
    a.part = part;
    a.tickets = reinterpret_cast<unsigned*>(w);
    a.len_dev = T_dev;
    a.len0 = T_dev ? 0 : T;
    a.len_off = T_dev ? t_offset : 0;
    a.max_ctx = max_ctx;
    a.nq = nq;
    a.nkv = nkv;
    a.scale = scale;
    bool done = false;
    if (int rc = dispatch_attn_fused<false>(hd, nq / nkv, a, L.S, st, &done)) return rc;
    if (done) return QZ_OK;
  }
  return attn_chunked(q, k_cache, v_cache, out, nq, nkv, hd, max_ctx, T, T_dev, t_offset, scale,
                      part, st);
}

int qz_attention_decode_qkv(const float* qkv, const float* q_norm_w, const float* k_norm_w,
                            const float* inv_freq, float* k_cache, float* v_cache, float* out,
                            int nq, int nkv, int hd, int64_t max_ctx, int64_t pos0,
                            const int64_t* pos_dev, float eps, float scale, void* ws,
                            size_t ws_bytes, void* stream) {
  if (int rc = check_heads(nq, nkv, hd, "qz_attention_decode_qkv")) return rc;
  if (max_ctx < 1) return fail(QZ_ERR_INVALID, "qz_attention_decode_qkv: bad max_ctx");
  if (!pos_dev && (pos0 < 0 || pos0 >= max_ctx))
    return fail(QZ_ERR_INVALID, "qz_attention_decode_qkv: position outside the cache");
  if (!qkv || !inv_freq || !k_cache || !v_cache || !out || !ws)
    return fail(QZ_ERR_INVALID, "qz_attention_decode_qkv: null pointer");
  if ((q_norm_w == nullptr) != (k_norm_w == nullptr))
    return fail(QZ_ERR_INVALID, "qz_attention_decode_qkv: pass both norm weights or neither");
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  const AttnLayout L = attn_layout(*d, nq, nkv, hd, max_ctx);
  if (static_cast<int64_t>(ws_bytes) < L.total || !aligned_to(ws, 256))
    return fail(QZ_ERR_INVALID,
                "qz_attention_decode_qkv: workspace too small or not 256-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* w = static_cast<char*>(ws);
  float* part = reinterpret_cast<float*>(w + L.part_off);
  if (aligned16(qkv) && aligned16(k_cache) && aligned16(v_cache)) {
    qz::dec::AttnArgs a{};
    a.in = qkv;
    a.qn_w = q_norm_w;
    a.kn_w = k_norm_w;
    a.inv_freq = inv_freq;
    a.kc = k_cache;
    a.vc = v_cache;
    a.out = out;
    a.part = part;
    a.tickets = reinterpret_cast<unsigned*>(w);
    a.len_dev = pos_dev;
    a.len0 = pos_dev ? 0 : pos0;
    a.len_off = 1;
    a.max_ctx = max_ctx;
    a.nq = nq;
    a.nkv = nkv;
    a.scale = scale;
    a.eps = eps;
    bool done = false;
    if (int rc = dispatch_attn_fused<true>(hd, nq / nkv, a, L.S, st, &done)) return rc;
    if (done) return QZ_OK;
  }
  // other shapes: rope + append, then the chunked kernels
  float* qs = reinterpret_cast<float*>(w + L.q_off);
  const dim3 grid(1u, static_cast<unsigned>(nq + 2 * nkv));
  qz::dec::qk_rope_kernel<<<grid, 128, hd * sizeof(float), st>>>(
      qkv, q_norm_w, k_norm_w, inv_freq, qs, k_cache, v_cache, nq, nkv, hd, max_ctx, pos0, pos_dev,
      eps);
  QZ_CUDA(cudaGetLastError());
  return attn_chunked(qs, k_cache, v_cache, out, nq, nkv, hd, max_ctx, pos_dev ? 0 : pos0 + 1,
                      pos_dev, 1, scale, part, st);
}

}  // extern "C"

namespace {
// Batched decode attention: context splits per (sequence, kv head) so that
// all sequences together put about three CTAs on every SM (two resident at a
// time), never more than one sequence alone uses. Same-box sweep of the
// multiplier (2, 3, 4, 6, 8, 12 CTAs per SM) at Qwen3-8B heads, context 2048:
// 3 was fastest at 4, 8 and 16 sequences (16: 56.3 us vs 61.8 at 6).
int attn_splits_batch(const DeviceInfo& d, int nkv, int64_t max_ctx, int batch) {
  const int one = attn_splits(d, nkv, max_ctx);
  if (batch <= 1) return one;
  const int64_t s = qz::cdiv(int64_t(3) * d.sms, int64_t(nkv) * batch);
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(s, one)));
}

// [tickets: batch * n_kv u32][the fused partials of every sequence, or, on
// the per-sequence fallback, a whole single-sequence workspace (attn_layout)].
// q_off is unused here.
AttnLayout attn_layout_batch(const DeviceInfo& d, int batch, int nq, int nkv, int hd,
                             int64_t max_ctx) {
  AttnLayout l;
  l.S = attn_splits_batch(d, nkv, max_ctx, batch);
  auto al = [](int64_t b) { return ((b + 255) / 256) * 256; };
  const int64_t fused = int64_t(batch) * nkv * l.S * (nq / nkv) * (hd + 2) * 4;
  const AttnLayout one = attn_layout(d, nq, nkv, hd, max_ctx);
  l.part_off = al(int64_t(batch) * nkv * 4);
  l.q_off = l.part_off;
  l.total = l.part_off + std::max(al(fused), one.total);
  return l;
}
}  // namespace

extern "C" {

int qz_attention_decode_batch_workspace_bytes(int batch, int nq, int nkv, int hd, int64_t max_ctx,
                                              int64_t* bytes) {
  if (!bytes || batch < 1 || nq < 1 || nkv < 1 || nq % nkv || hd < 1 || max_ctx < 1)
    return fail(QZ_ERR_INVALID, "qz_attention_decode_batch_workspace_bytes: bad arguments");
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  *bytes = attn_layout_batch(*d, batch, nq, nkv, hd, max_ctx).total;
  return QZ_OK;
}

int qz_attention_decode_qkv_batch(const float* qkv, int64_t qkv_stride, const float* q_norm_w,
                                  const float* k_norm_w, const float* inv_freq, float* k_cache,
                                  float* v_cache, int64_t cache_stride, float* out,
                                  int64_t out_stride, int batch, int nq, int nkv, int hd,
                                  int64_t max_ctx, int64_t pos0, const int64_t* pos_dev,
                                  float eps, float scale, void* ws, size_t ws_bytes,
                                  void* stream) {
  if (int rc = check_heads(nq, nkv, hd, "qz_attention_decode_qkv_batch")) return rc;
  if (batch < 1 || max_ctx < 1) return fail(QZ_ERR_INVALID, "qz_attention_decode_qkv_batch: bad batch or max_ctx");
  const int64_t rows = static_cast<int64_t>(nq + 2 * nkv) * hd;
  if (qkv_stride < rows || out_stride < static_cast<int64_t>(nq) * hd ||
      cache_stride < static_cast<int64_t>(nkv) * max_ctx * hd)
    return fail(QZ_ERR_INVALID, "qz_attention_decode_qkv_batch: a stride is shorter than its row");
  if (!pos_dev && (pos0 < 0 || pos0 >= max_ctx))
    return fail(QZ_ERR_INVALID, "qz_attention_decode_qkv_batch: position outside the cache");
  if (!qkv || !inv_freq || !k_cache || !v_cache || !out || !ws)
    return fail(QZ_ERR_INVALID, "qz_attention_decode_qkv_batch: null pointer");
  if ((q_norm_w == nullptr) != (k_norm_w == nullptr))
    return fail(QZ_ERR_INVALID, "qz_attention_decode_qkv_batch: pass both norm weights or neither");
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  const AttnLayout L = attn_layout_batch(*d, batch, nq, nkv, hd, max_ctx);
  if (static_cast<int64_t>(ws_bytes) < L.total || !aligned_to(ws, 256))
    return fail(QZ_ERR_INVALID,
                "qz_attention_decode_qkv_batch: workspace too small or not 256-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* w = static_cast<char*>(ws);
  const bool strides16 = qkv_stride % 4 == 0 && cache_stride % 4 == 0;
  if (aligned16(qkv) && aligned16(k_cache) && aligned16(v_cache) && strides16) {
    qz::dec::AttnArgs a{};
    a.in = qkv;
    a.qn_w = q_norm_w;
    a.kn_w = k_norm_w;
    a.inv_freq = inv_freq;
    a.kc = k_cache;
    a.vc = v_cache;
    a.out = out;
    a.part = reinterpret_cast<float*>(w + L.part_off);
    a.tickets = reinterpret_cast<unsigned*>(w);
    a.len_dev = pos_dev;
    a.len0 = pos_dev ? 0 : pos0;
    a.len_off = 1;
    a.max_ctx = max_ctx;
    a.nq = nq;
    a.nkv = nkv;
    a.scale = scale;
    a.eps = eps;
    a.in_bstride = qkv_stride;
    a.kv_bstride = cache_stride;
    a.out_bstride = out_stride;
    bool done = false;
    if (int rc = dispatch_attn_fused<true>(hd, nq / nkv, a, L.S, st, &done, batch)) return rc;
    if (done) return QZ_OK;
  }
  // other shapes: one sequence after the other through the single-sequence
  // path (stream-ordered, so they share one single-sequence workspace placed
  // after the batched tickets, which stay zero)
  void* ws1 = w + L.part_off;
  const size_t ws1_bytes = ws_bytes - static_cast<size_t>(L.part_off);
  for (int b = 0; b < batch; ++b) {
    if (int rc = qz_attention_decode_qkv(qkv + b * qkv_stride, q_norm_w, k_norm_w, inv_freq,
                                         k_cache + b * cache_stride, v_cache + b * cache_stride,
                                         out + b * out_stride, nq, nkv, hd, max_ctx, pos0, pos_dev,
                                         eps, scale, ws1, ws1_bytes, stream))
      return rc;
  }
  return QZ_OK;
}

}  // extern "C"

namespace {

static_assert(sizeof(qz_decoder_layer) == sizeof(qz::mk::LayerW),
              "qz_decoder_layer must match the kernel's layer record");

// decode_layers workspace: [barrier count u64, tickets nkv u32, padded to 256 B]
// [attention partials nkv * S_max * n_rep * (hd + 2) fp32] [activations
// h, h2, qkv, attn, act fp32]
struct StepLayout {
  int64_t part_off, act_off, total;
  int64_t h, h2, qkv, attn, act;   // float offsets within the activation block
};

StepLayout step_layout(int H, int I, int nq, int nkv, int hd, int64_t max_ctx) {
  StepLayout l;
  auto al = [](int64_t b) { return ((b + 255) / 256) * 256; };
  const int64_t rows = qz::mk::kSlotBytes / (hd * 4);
  const int64_t smax = qz::cdiv(max_ctx, rows);
  l.part_off = al(8 + static_cast<int64_t>(nkv) * 4);
  l.act_off = l.part_off + al(static_cast<int64_t>(nkv) * smax * (nq / nkv) * (hd + 2) * 4);
  auto a64 = [](int64_t f) { return ((f + 63) / 64) * 64; };
  l.h = 0;
  l.h2 = l.h + a64(H);
  l.qkv = l.h2 + a64(H);
  l.attn = l.qkv + a64(static_cast<int64_t>(nq + 2 * nkv) * hd);
  l.act = l.attn + a64(static_cast<int64_t>(nq) * hd);
  l.total = l.act_off + (l.act + a64(I)) * 4;
  return l;
}

int check_step_shape(const DeviceInfo& d, int H, int I, int nq, int nkv, int hd, int64_t max_ctx,
                     const char* what) {
  if (int rc = check_heads(nq, nkv, hd, what)) return rc;
  if (H < 16 || I < 16 || max_ctx < 1) return fail(QZ_ERR_INVALID, std::string(what) + ": bad sizes");
  const int64_t Ko = static_cast<int64_t>(nq) * hd;
  if (hd != 64 && hd != 128)
    return fail(QZ_ERR_UNSUPPORTED, std::string(what) + ": head_dim must be 64 or 128");
  for (int64_t k : {static_cast<int64_t>(H), static_cast<int64_t>(I), Ko})
    if (k % 16 || k > qz::mk::kMaxX || k > qz::mk::kSlotBytes)
      return fail(QZ_ERR_UNSUPPORTED, std::string(what) +
                                          ": row lengths must be multiples of 16 up to 16384");
  const int n_rep = nq / nkv;
  if (n_rep != 1 && n_rep != 2 && n_rep != 4 && n_rep != 8)
    return fail(QZ_ERR_UNSUPPORTED, std::string(what) + ": query heads per kv head must be 1, 2, 4 or 8");
  const int64_t smax = qz::cdiv(max_ctx, qz::mk::kSlotBytes / (hd * 4));
  if (2 * smax * n_rep + n_rep > qz::mk::kMaxX)
    return fail(QZ_ERR_UNSUPPORTED, std::string(what) + ": context too long");
  const int64_t nA = qz::cdiv(static_cast<int64_t>(nq + 2 * nkv) * hd, d.sms);
  if (nA + 5 * qz::cdiv(H, d.sms) + 2 * qz::cdiv(I, d.sms) > qz::mk::Smem::kMaxPre)
    return fail(QZ_ERR_UNSUPPORTED, std::string(what) + ": layer too large for the row caches");
  if (qz::cdiv(I, d.sms) > qz::mk::Smem::kMaxUnits)
    return fail(QZ_ERR_UNSUPPORTED, std::string(what) + ": intermediate size too large");
  if (!d.coop) return fail(QZ_ERR_UNSUPPORTED, std::string(what) + ": no cooperative launch");
  if (d.smem_optin < qz::mk::Smem::total)
    return fail(QZ_ERR_UNSUPPORTED, std::string(what) + ": not enough shared memory");
  return QZ_OK;
}

template <int HD, int NR>
int launch_prefill_t(const float* q, const float* kc, const float* vc, float* out, int64_t M,
                     int nq, int nkv, int64_t max_ctx, int64_t pos0, float scale,
                     cudaStream_t st) {
  auto fn = qz::dec::attn_prefill_tiled_kernel<HD, NR>;
  constexpr int smem = qz::dec::prefill_tiled_smem<HD>();
  static std::once_flag once[kMaxDevices];
  int dev = 0;
  QZ_CUDA(cudaGetDevice(&dev));
  cudaError_t ae = cudaSuccess;
  std::call_once(once[dev], [&] {
    ae = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  });
  QZ_CUDA(ae);
  constexpr int BM = qz::dec::kPfThreads / (HD / qz::dec::kPfDims) / NR;
  const dim3 grid(static_cast<unsigned>(qz::cdiv(M, BM)), static_cast<unsigned>(nkv));
  fn<<<grid, qz::dec::kPfThreads, smem, st>>>(q, kc, vc, out, M, nq, max_ctx, pos0, scale);
  QZ_CUDA(cudaGetLastError());
  return QZ_OK;
}

// The tiled prefill attention for head_dim 64 / 128 and 1, 2, 4 or 8 query
// heads per kv head; *done = false for other shapes.
int launch_prefill_tiled(int hd, int n_rep, const float* q, const float* kc, const float* vc,
                         float* out, int64_t M, int nq, int nkv, int64_t max_ctx, int64_t pos0,
                         float scale, cudaStream_t st, bool* done) {
  *done = true;
#define QZ_PF_CASE(HD_, NR_) \
  if (hd == (HD_) && n_rep == (NR_)) \
    return launch_prefill_t<HD_, NR_>(q, kc, vc, out, M, nq, nkv, max_ctx, pos0, scale, st);
  QZ_PF_CASE(64, 1) QZ_PF_CASE(64, 2) QZ_PF_CASE(64, 4) QZ_PF_CASE(64, 8)
  QZ_PF_CASE(128, 1) QZ_PF_CASE(128, 2) QZ_PF_CASE(128, 4) QZ_PF_CASE(128, 8)
#undef QZ_PF_CASE
  *done = false;
  return QZ_OK;
}

template <int E>
int launch_step(const DeviceInfo& d, const qz::mk::StepArgs& a, cudaStream_t st) {
  auto fn = qz::mk::decode_layers_kernel<E>;
  static std::atomic<int> attr_done{0};
  if (!attr_done.load()) {
    QZ_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 qz::mk::Smem::total));
    attr_done.store(1);
  }
  int nb = 0;
  QZ_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, fn, qz::mk::kThreadsMK,
                                                        qz::mk::Smem::total));
  if (nb < 1) return fail(QZ_ERR_UNSUPPORTED, "qz_decode_layers: kernel does not fit on an SM");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(d.sms));
  cfg.blockDim = dim3(qz::mk::kThreadsMK);
  cfg.dynamicSmemBytes = qz::mk::Smem::total;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  QZ_CUDA(cudaLaunchKernelEx(&cfg, fn, a));
  return QZ_OK;
}

}  // namespace

extern "C" {

int qz_decode_step_workspace_bytes(int H, int I, int nq, int nkv, int hd, int64_t max_ctx,
                                   int64_t* bytes) {
  if (!bytes) return fail(QZ_ERR_INVALID, "qz_decode_step_workspace_bytes: null bytes");
  if (int rc = check_heads(nq, nkv, hd, "qz_decode_step_workspace_bytes")) return rc;
  if (H < 1 || I < 1 || max_ctx < 1)
    return fail(QZ_ERR_INVALID, "qz_decode_step_workspace_bytes: bad sizes");
  *bytes = step_layout(H, I, nq, nkv, hd, max_ctx).total;
  return QZ_OK;
}

int qz_decode_layers_supported(int H, int I, int nq, int nkv, int hd, int64_t max_ctx) {
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  return check_step_shape(*d, H, I, nq, nkv, hd, max_ctx, "qz_decode_layers");
}

int qz_decode_layers(const qz_decoder_layer* layers, int n_layers, const int8_t* embed_q,
                     const float* embed_s, int64_t vocab, const int64_t* token,
                     const int64_t* pos_dev, const float* inv_freq, const float* norm_w,
                     float* x_final, int H, int I, int nq, int nkv, int hd, int64_t max_ctx,
                     float eps, float scale, void* ws, size_t ws_bytes, uint64_t* trace,
                     void* stream) {
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  if (int rc = check_step_shape(*d, H, I, nq, nkv, hd, max_ctx, "qz_decode_layers")) return rc;
  if (n_layers < 1 || !layers || !embed_q || !embed_s || !token || !pos_dev || !inv_freq ||
      !norm_w || !x_final || !ws || vocab < 1)
    return fail(QZ_ERR_INVALID, "qz_decode_layers: null pointer or empty model");
  const StepLayout L = step_layout(H, I, nq, nkv, hd, max_ctx);
  if (static_cast<int64_t>(ws_bytes) < L.total || !aligned_to(ws, 256))
    return fail(QZ_ERR_INVALID, "qz_decode_layers: workspace too small or not 256-byte aligned");
  char* w = static_cast<char*>(ws);
  float* act = reinterpret_cast<float*>(w + L.act_off);
  qz::mk::StepArgs a{};
  a.layers = reinterpret_cast<const qz::mk::LayerW*>(layers);
  a.n_layers = n_layers;
  a.embed_q = embed_q;
  a.embed_s = embed_s;
  a.tok = token;
  a.pos_dev = pos_dev;
  a.inv_freq = inv_freq;
  a.norm_w = norm_w;
  a.h = act + L.h;
  a.h2 = act + L.h2;
  a.qkv = act + L.qkv;
  a.attn = act + L.attn;
  a.act = act + L.act;
  a.x_final = x_final;
  a.part = reinterpret_cast<float*>(w + L.part_off);
  a.bar = reinterpret_cast<unsigned long long*>(w);
  a.tickets = reinterpret_cast<unsigned*>(w + 8);
  a.H = H;
  a.I = I;
  a.nq = nq;
  a.nkv = nkv;
  a.hd = hd;
  a.max_ctx = max_ctx;
  a.V = vocab;
  a.eps = eps;
  a.scale = scale;
  a.trace = reinterpret_cast<unsigned long long*>(trace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return hd == 64 ? launch_step<2>(*d, a, st) : launch_step<4>(*d, a, st);
}

// ---------------------------------------------------------------------------
// peer-memory all-reduce for tensor-parallel decoding
// ---------------------------------------------------------------------------
static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");

int qz_comm_buffer_bytes(int ranks, int64_t n_max, int64_t* bytes) {
  if (!bytes || ranks < 1 || ranks > qz::comm::kMaxRanks || n_max < 4 || n_max % 4)
    return fail(QZ_ERR_INVALID, "qz_comm_buffer_bytes: 1..8 ranks and n_max a positive multiple of 4");
  *bytes = qz::comm::buffer_bytes(ranks, n_max);
  return QZ_OK;
}

int qz_comm_alloc(int64_t bytes, void** ptr) {
  if (!ptr || bytes <= 0) return fail(QZ_ERR_INVALID, "qz_comm_alloc: bad arguments");
  void* p = nullptr;
  QZ_CUDA(cudaMalloc(&p, static_cast<size_t>(bytes)));
  const cudaError_t e = cudaMemset(p, 0, static_cast<size_t>(bytes));
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(QZ_ERR_CUDA, std::string("qz_comm_alloc: cudaMemset: ") + cudaGetErrorString(e));
  }
  *ptr = p;
  return QZ_OK;
}

int qz_comm_free(void* ptr) {
  if (ptr) QZ_CUDA(cudaFree(ptr));
  return QZ_OK;
}

int qz_ipc_handle(const void* ptr, void* handle64) {
  if (!ptr || !handle64) return fail(QZ_ERR_INVALID, "qz_ipc_handle: null pointer");
  cudaIpcMemHandle_t h;
  QZ_CUDA(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)));
  std::memcpy(handle64, &h, sizeof(h));
  return QZ_OK;
}

int qz_ipc_open(const void* handle64, void** ptr) {
  if (!handle64 || !ptr) return fail(QZ_ERR_INVALID, "qz_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof(h));
  QZ_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return QZ_OK;
}

int qz_ipc_close(void* ptr) {
  if (ptr) QZ_CUDA(cudaIpcCloseMemHandle(ptr));
  return QZ_OK;
}

int qz_allreduce_sum(const float* in, float* out, int64_t n, int64_t n_max,
                     void* const* peer_buffers, int rank, int ranks, void* stream) {
  if (ranks < 1 || ranks > qz::comm::kMaxRanks || rank < 0 || rank >= ranks)
    return fail(QZ_ERR_INVALID, "qz_allreduce_sum: bad rank / rank count");
  if (n < 0 || n > n_max || n_max % 4)
    return fail(QZ_ERR_INVALID, "qz_allreduce_sum: n must be at most n_max (a multiple of 4)");
  if (n == 0) return QZ_OK;
  if (!in || !out || !peer_buffers)
    return fail(QZ_ERR_INVALID, "qz_allreduce_sum: null pointer");
  qz::comm::Peers peers{};
  for (int j = 0; j < ranks; ++j) {
    if (!peer_buffers[j] || !aligned16(peer_buffers[j]))
      return fail(QZ_ERR_INVALID, "qz_allreduce_sum: null or unaligned peer buffer");
    peers.base[j] = static_cast<float*>(peer_buffers[j]);
  }
  // one CTA per 1024 elements, at most kMaxBlocks
  const int nb = static_cast<int>(std::max<int64_t>(
      1, std::min<int64_t>(qz::comm::kMaxBlocks, qz::cdiv(n, 1024))));
  qz::comm::allreduce_kernel<<<nb, qz::comm::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      in, out, n, n_max, peers, rank, ranks);
  QZ_CUDA(cudaGetLastError());
  return QZ_OK;
}

int qz_attention_prefill(const float* q, const float* k_cache, const float* v_cache, float* out,
                         int64_t M, int nq, int nkv, int hd, int64_t max_ctx, int64_t pos0,
                         float scale, void* stream) {
  if (int rc = check_heads(nq, nkv, hd, "qz_attention_prefill")) return rc;
  if (M < 0 || pos0 < 0 || pos0 + M > max_ctx)
    return fail(QZ_ERR_INVALID, "qz_attention_prefill: positions beyond the cache");
  if (M == 0) return QZ_OK;
  if (!q || !k_cache || !v_cache || !out) return fail(QZ_ERR_INVALID, "qz_attention_prefill: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (aligned16(q) && aligned16(k_cache) && aligned16(v_cache) && aligned16(out)) {
    bool done = false;
    if (int rc = launch_prefill_tiled(hd, nq / nkv, q, k_cache, v_cache, out, M, nq, nkv, max_ctx,
                                      pos0, scale, st, &done))
      return rc;
    if (done) return QZ_OK;
  }
  const int64_t warps = M * nq;
  const unsigned blocks = static_cast<unsigned>(qz::cdiv(warps * 32, 256));
  qz::dec::attn_prefill_kernel<<<blocks, 256, 0, st>>>(q, k_cache, v_cache, out, M, nq, nkv, hd,
                                                       max_ctx, pos0, scale);
  QZ_CUDA(cudaGetLastError());
  return QZ_OK;
}

int qz_argmax(const float* logits, int64_t M, int64_t V, uint64_t* keys, int64_t* tokens,
              int64_t* pos_dev, int64_t pos_step, void* stream) {
  if (M < 0 || V < 1 || V > 0xFFFFFFFFll) return fail(QZ_ERR_INVALID, "qz_argmax: bad sizes");
  if (M == 0) return QZ_OK;
  if (!logits || !keys || !tokens) return fail(QZ_ERR_INVALID, "qz_argmax: null pointer");
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned bx = static_cast<unsigned>(std::min<int64_t>(qz::cdiv(V, 1024), d->sms));
  qz::dec::argmax_kernel<<<dim3(bx, static_cast<unsigned>(M)), 256, 0, st>>>(
      logits, V, reinterpret_cast<unsigned long long*>(keys));
  QZ_CUDA(cudaGetLastError());
  qz::dec::argmax_finish_kernel<<<static_cast<unsigned>(qz::cdiv(M, 128)), 128, 0, st>>>(
      reinterpret_cast<unsigned long long*>(keys), tokens, M, pos_dev, pos_step);
  QZ_CUDA(cudaGetLastError());
  return QZ_OK;
}

int qz_silu_mul(const float* gu, float* a, int64_t M, int64_t I, void* stream) {
  if (M < 0 || I < 0) return fail(QZ_ERR_INVALID, "qz_silu_mul: negative dimension");
  if (M == 0 || I == 0) return QZ_OK;
  if (!gu || !a) return fail(QZ_ERR_INVALID, "qz_silu_mul: null pointer");
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  const int threads = 256;
  const int blocks = static_cast<int>(std::min<int64_t>(qz::cdiv(M * I, threads), d->sms * 8));
  qz::silu_mul_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(gu, a, M, I);
  QZ_CUDA(cudaGetLastError());
  return QZ_OK;
}

int qz_device_status(uint32_t* words, int clear) {
  if (!words) return fail(QZ_ERR_INVALID, "qz_device_status: null words");
  QZ_CUDA(cudaDeviceSynchronize());
  QZ_CUDA(cudaMemcpyFromSymbol(words, qz::g_status, sizeof(unsigned int) * 4));
  if (clear) {
    const unsigned int zero[4] = {0u, 0u, 0u, 0u};
    QZ_CUDA(cudaMemcpyToSymbol(qz::g_status, zero, sizeof(zero)));
  }
  return QZ_OK;
}

int qz_sync(void* stream) {
  QZ_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  return QZ_OK;
}

}  // extern "C"
