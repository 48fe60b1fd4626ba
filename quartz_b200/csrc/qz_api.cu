// qz_api.cu -- the extern "C" boundary (include/quartz_b200.h): argument
// checks, kernel selection and launch configuration. One translation unit so
// that the device status word is a single symbol without relocatable code.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "quartz_b200.h"
#include "qz_generic.cuh"
#include "qz_stream.cuh"

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

struct DeviceInfo {
  bool ready = false;
  int sms = 0;
  int smem_optin = 0;   // max dynamic shared memory per block (opt-in)
  int coop = 0;         // cooperative launch supported
};

DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

int device_info(DeviceInfo** out) {
  int dev = 0;
  QZ_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(QZ_ERR_UNSUPPORTED, "device index out of range");
  DeviceInfo& d = g_dev[dev];
  if (!d.ready) {
    std::lock_guard<std::mutex> lock(g_dev_mu);
    if (!d.ready) {
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
      QZ_CUDA(cudaFuncSetAttribute(qz::gemv_stream_kernel<true>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      QZ_CUDA(cudaFuncSetAttribute(qz::gemv_stream_kernel<false>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      QZ_CUDA(cudaFuncSetAttribute(qz::fused_mlp_kernel<true>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      QZ_CUDA(cudaFuncSetAttribute(qz::fused_mlp_kernel<false>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      d.ready = true;
    }
  }
  *out = &d;
  return QZ_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Stages that fit next to an x region of xbytes; 0 when fewer than 2 fit.
int stream_stages(const DeviceInfo& d, int64_t kmax) {
  const int64_t avail = static_cast<int64_t>(d.smem_optin) - qz::kSmemHeader -
                        qz::stream_x_bytes(kmax) - 256 /* static shared */;
  if (avail < 2 * qz::kStageBytes) return 0;
  return static_cast<int>(std::min<int64_t>(qz::kMaxStages, avail / qz::kStageBytes));
}

int stream_smem(int64_t kmax, int nstages) {
  return qz::kSmemHeader + qz::stream_x_bytes(kmax) + nstages * qz::kStageBytes;
}

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

int gemv_impl(const int8_t* q, const float* scale, int64_t ng, const float* x, float* y,
              int64_t N, int64_t K, const float* residual, cudaStream_t st) {
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  const int64_t G = K / ng;
  const int nst = stream_stages(*d, K);
  const bool fast = K > 0 && K % 16 == 0 && G % 16 == 0 && aligned16(q) && nst >= 2;
  if (!fast) return launch_generic_gemm(*d, q, scale, ng, x, y, residual, 1, N, K, st);
  qz::GemvArgs a{q, scale, x, y, residual, N, K, ng, nst};
  const int64_t n_rg = qz::cdiv(N, qz::kRW);
  const int grid = static_cast<int>(std::min<int64_t>(n_rg, d->sms));
  const int smem = stream_smem(K, nst);
  if (ng == 1)
    qz::gemv_stream_kernel<true><<<grid, qz::kThreads, smem, st>>>(a);
  else
    qz::gemv_stream_kernel<false><<<grid, qz::kThreads, smem, st>>>(a);
  QZ_CUDA(cudaGetLastError());
  return QZ_OK;
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

int qz_mlp_workspace_bytes(void) { return 256; }

int qz_fused_mlp_decode(const int8_t* gu_q, const float* gu_s, int64_t ng, const float* x,
                        const int8_t* down_q, const float* down_s, int64_t ngd, float* abuf,
                        float* out, const float* residual, int64_t H, int64_t I,
                        uint32_t* sync_ws, void* stream) {
  if (int rc = check_weights(gu_q, gu_s, ng, 2 * I, H, "qz_fused_mlp_decode (gate|up)")) return rc;
  if (int rc = check_weights(down_q, down_s, ngd, H, I, "qz_fused_mlp_decode (down)")) return rc;
  if (H == 0) return QZ_OK;
  if (!out || (I > 0 && !abuf) || !x)
    return fail(QZ_ERR_INVALID, "qz_fused_mlp_decode: null x, abuf or out");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  const int64_t kmax = std::max(H, I);
  const int nst = stream_stages(*d, kmax);
  const bool fast = I > 0 && H % 16 == 0 && I % 16 == 0 && (H / ng) % 16 == 0 &&
                    (I / ngd) % 16 == 0 && aligned16(gu_q) && aligned16(down_q) && nst >= 2 &&
                    sync_ws != nullptr && d->coop;
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
  qz::MlpArgs a{gu_q, gu_s, x, down_q, down_s, abuf, out, residual, sync_ws, H, I, ng, ngd, nst};
  const int64_t work = std::max(qz::cdiv(I, qz::kRW / 2), qz::cdiv(H, qz::kRW));
  const int grid = static_cast<int>(std::min<int64_t>(work, d->sms));
  const int smem = stream_smem(kmax, nst);
  void* args[] = {&a};
  const void* fn = (ng == 1 && ngd == 1)
                       ? reinterpret_cast<const void*>(qz::fused_mlp_kernel<true>)
                       : reinterpret_cast<const void*>(qz::fused_mlp_kernel<false>);
  QZ_CUDA(cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(qz::kThreads), args, smem, st));
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
