/*
 * quartz_b200.h -- C ABI of the B200 (sm_100a) int8 weight-only matmul path.
 *
 * Replaces the native kernels behind quartz's `quartz.kernels` package (a Numba
 * JIT, CPU only in the reference). Pointers are DEVICE pointers; host<->device
 * copies and the device-resident weight cache live in the Python layer
 * (quartz_b200.kernels), which keeps the reference's numpy signatures.
 *
 * Conventions
 *   - Every entry point returns an int status (QZ_OK == 0). On failure,
 *     qz_last_error() returns a message for the calling thread. No C++
 *     exception crosses this boundary.
 *   - All work is stream-ordered on `stream` (a cudaStream_t; NULL = the
 *     legacy default stream). Nothing here synchronises except qz_sync().
 *   - Layouts are C-contiguous. q is int8 [N, K]; scale is fp32 [N, ng] with
 *     K % ng == 0 and group size G = K / ng (ng == 1: one scale per row).
 *   - Any N, K, M >= 0 is accepted. The streaming kernels run when q is
 *     16-byte aligned, K % 16 == 0 and G % 16 == 0; other shapes take a generic
 *     kernel with the same results (within fp32 reassociation).
 *   - Kernels that wait (mbarrier stages, the fused MLP's grid barrier) give
 *     up after about one second, record the failure in a device status word
 *     and return; qz_device_status() reads it.
 */
#ifndef QUARTZ_B200_H_
#define QUARTZ_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  QZ_OK = 0,
  QZ_ERR_INVALID = 1,     /* bad argument: shape, null pointer, group tiling */
  QZ_ERR_CUDA = 2,        /* a CUDA runtime call failed */
  QZ_ERR_UNSUPPORTED = 3, /* device is not sm_100 / missing capability */
};

/* Library version, (major << 16) | (minor << 8) | patch. */
int qz_version(void);

/* Select `device`, check it is an sm_100 part, and prepare kernel attributes.
 * Optional: the first call on a device does the same. */
int qz_init(int device);

/* Copy the calling thread's last error message into buf (NUL-terminated,
 * truncated to len). Returns the full message length. */
int qz_last_error(char* buf, size_t len);

/*
 * y[n] = sum_g scale[n, g] * sum_{j < G} x[g*G + j] * q[n, g*G + j]  (+ residual[n])
 * Replaces w8a32_gemv and w8a32_gemv_serial
 * (quartz/kernels/int8.py:24-38 and :48-63): the reference's size-based
 * serial/parallel choice (int8.py:45,101-105) becomes a launch-shape choice
 * here. residual may be NULL.
 */
int qz_gemv_w8(const int8_t* q, const float* scale, int64_t ng, const float* x, float* y,
               int64_t N, int64_t K, const float* residual, void* stream);

/*
 * The whole numpy-signature call of w8a32_gemv (quartz/kernels/int8.py:24-38:
 * x and y in host memory, y complete on return) in one call: x_host is
 * copied into x_pin (pinned, K floats) and on to x_dev, the GEMV writes y_dev,
 * and y comes back through y_pin (pinned, N floats) into y_host in chunks, the
 * host copy of one chunk overlapping the transfer of the next. q and scale
 * are device pointers. Synchronises with the stream. Allocates no memory;
 * the first call on a thread and device creates the 16 events it reuses
 * for the chunked copy.
 */
int qz_gemv_w8_host(const int8_t* q, const float* scale, int64_t ng, const float* x_host,
                    float* y_host, int64_t N, int64_t K, float* x_pin, float* y_pin,
                    float* x_dev, float* y_dev, void* stream);

/*
 * int4 weight GEMV: y[n] = sum_g scale[n, g] * sum_{j < G} x[g*G + j] * q[n, g*G + j]
 * (+ residual[n]) with q stored two weights per byte, q4 [N, K / 2]: element
 * 2i in the low nibble, 2i + 1 in the high one, two's complement, symmetric
 * in [-7, 7] (quartz_b200.quantize.quantize_symmetric_int4). No counterpart
 * in the reference: quartz keeps a `bits` field for 4-bit weights as future
 * work (quartz/config.py:98). K and the group size G = K / ng must be
 * multiples of 32 and q4 16-byte aligned; other shapes return
 * QZ_ERR_INVALID. residual may be NULL. The kernel stages x scaled by up to
 * 2^85, so it is exact for |x| < 2^43 (activations beyond that overflow).
 */
int qz_gemv_w4(const uint8_t* q4, const float* scale, int64_t ng, const float* x, float* y,
               int64_t N, int64_t K, const float* residual, void* stream);

/*
 * Y[m, n] = the same reduction for each of M rows of X [M, K]  (+ residual[m, n])
 * Replaces w8a32_gemm (quartz/kernels/int8.py:66-87). Y is [M, N]; residual,
 * if not NULL, is [M, N]. M == 1 runs the GEMV.
 */
int qz_gemm_w8(const int8_t* q, const float* scale, int64_t ng, const float* X, float* Y,
               int64_t M, int64_t N, int64_t K, const float* residual, void* stream);

/*
 * Bytes of device workspace qz_gemm_w8_ws can use for an [M, K] x [N, K]^T
 * product (0 when M < 2), written to *bytes: the activation limbs and row
 * scales, plus int32 partial sums for splitting K across CTAs when the output
 * has too few 128-row tiles to fill the GPU.
 */
int qz_gemm_w8_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t* bytes);

/*
 * qz_gemm_w8 on the tensor cores. With ng == 1, K % 16 == 0, q 16-byte
 * aligned and a 16-byte aligned workspace of qz_gemm_w8_workspace_bytes(M, N, K)
 * bytes, M > 1 runs the tcgen05 kernel: X is split into three int8 limbs with
 * a per-row scale (a 24-bit fixed-point copy, error <= max|X[m,:]| * 2^-24 per
 * element) and every limb is multiplied by the int8 weights with exact int32
 * accumulation in tensor memory (split-K partials add exactly, so results do
 * not depend on the split). Otherwise it behaves as qz_gemm_w8. Calls sharing
 * one workspace must not overlap on the GPU.
 * Replaces w8a32_gemm (quartz/kernels/int8.py:66-87) for batched rows.
 */
int qz_gemm_w8_ws(const int8_t* q, const float* scale, int64_t ng, const float* X, float* Y,
                  int64_t M, int64_t N, int64_t K, const float* residual, void* workspace,
                  size_t workspace_bytes, void* stream);

/* Activation prologues of qz_gemm_w8_act_ws. */
#define QZ_ACT_NONE 0
#define QZ_ACT_RMSNORM 1
#define QZ_ACT_SILU_MUL 2

/*
 * qz_gemm_w8_ws on an activation computed inside the GEMM's limb split, so
 * the op that produces the GEMM's input needs no kernel of its own:
 *   QZ_ACT_RMSNORM   the rows are RMSNorm(X[m, :K]) with weight norm_w [K] and
 *                    eps (quartz/ops.py:24-32), X is [M, K];
 *   QZ_ACT_SILU_MUL  the rows are silu(g) * u with the clipped exp of
 *                    quartz/quantize.py:112-114, X is [M, 2K] holding [g | u];
 *   QZ_ACT_NONE      qz_gemm_w8_ws itself.
 * The activations equal what qz_rmsnorm / qz_silu_mul write (same
 * expressions, same order of the RMSNorm sum), so the result equals the
 * unfused sequence. Needs the tensor path: M >= 2, ng == 1, K % 16 == 0,
 * 16-byte aligned q and the workspace of qz_gemm_w8_workspace_bytes;
 * otherwise QZ_ERR_UNSUPPORTED and nothing is queued. Replaces the RMSNorm +
 * matmul_int8 and silu-mul + matmul_int8 pairs of quartz's batched decode
 * (quartz/models/common.py:79-88, quartz/quantize.py:112-114).
 */
int qz_gemm_w8_act_ws(const int8_t* q, const float* scale, int64_t ng, const float* X, int act,
                      const float* norm_w, float eps, float* Y, int64_t M, int64_t N, int64_t K,
                      const float* residual, void* workspace, size_t workspace_bytes,
                      void* stream);

/*
 * out[h] = sum down[h, :] * abuf * down_s  (+ residual[h]),
 *   abuf[n] = silu(gate_n . x) * (up_n . x)     (silu with unclipped exp)
 * Replaces fused_mlp_decode (quartz/kernels/fused.py:27-65).
 *   gu_q [2I, H] int8 (gate rows 0..I-1, up rows I..2I-1), gu_s [2I, ng];
 *   x [H]; down_q [H, I] int8, down_s [H, ngd]; abuf [I] (written, as in the
 *   reference); out [H]; residual [H] or NULL.
 * sync_ws: qz_mlp_workspace_bytes() bytes of device memory, zeroed once before
 * its first use; the kernel leaves it ready for the next call. Calls that
 * share one sync_ws must not overlap on the GPU.
 */
int qz_fused_mlp_decode(const int8_t* gu_q, const float* gu_s, int64_t ng, const float* x,
                        const int8_t* down_q, const float* down_s, int64_t ngd, float* abuf,
                        float* out, const float* residual, int64_t H, int64_t I,
                        uint32_t* sync_ws, void* stream);

/* Bytes of device workspace qz_fused_mlp_decode needs for its grid barrier. */
int qz_mlp_workspace_bytes(void);

/*
 * qz_fused_mlp_decode without caller-provided scratch. No counterpart in the
 * reference: the reference's fused_mlp_decode takes its abuf from the caller.
 *
 * For callers that cannot allocate device memory: a host engine or plugin
 * whose device memory is owned by another allocator (a fixed pool or a
 * framework's caching allocator) and that must not call cudaMalloc behind its
 * back, or a caller with no allocation rights at all after start-up. This
 * entry point allocates nothing (no cudaMalloc, cudaFree or allocating
 * library call): the [I] intermediate and the grid-barrier words live in a
 * file-scope __device__ array of 128.25 KB that every GPU loading the library
 * holds until the process exits.
 *
 *   - I must be at most 32768; larger I returns QZ_ERR_INVALID.
 *   - The first call on a device looks up the array's device address with
 *     cudaGetSymbolAddress (with that device current). Make that first call
 *     before any stream capture.
 *   - All calls share the one array, which keeps the last call's intermediate.
 *     The barrier count is cleared (cudaMemsetAsync on `stream`) after the
 *     arguments are checked and before the one-launch kernel that uses it;
 *     a refused call queues nothing. Calls that overlap on the GPU
 *     (different streams, or concurrent host threads) race on the array:
 *     serialise them.
 * Arguments and results are those of qz_fused_mlp_decode minus abuf/sync_ws.
 */
int qz_fused_mlp_decode_noalloc(const int8_t* gu_q, const float* gu_s, int64_t ng, const float* x,
                                const int8_t* down_q, const float* down_s, int64_t ngd, float* out,
                                const float* residual, int64_t H, int64_t I, void* stream);

/*
 * a[m, i] = silu(gu[m, i]) * gu[m, I + i], exponent clipped to [-88, 88].
 * The elementwise step of the M > 1 MLP (quartz/quantize.py:112-114 with
 * quartz/ops.py:35-37). gu is [M, 2I], a is [M, I].
 */
int qz_silu_mul(const float* gu, float* a, int64_t M, int64_t I, void* stream);

/*
 * qz_gemv_w8 of RMSNorm(x) * norm_w (quartz/ops.py:24-32 followed by the
 * projection, quartz/models/common.py:37-38): the streaming kernel normalises
 * x as it stages it in shared memory (no separate launch). Shapes where the
 * kernel keeps x in registers instead (K == 1024 and N > 36 * (SMs - 1), such
 * as an lm_head) and shapes outside the streaming kernel
 * normalise into xn_scratch ([K] device floats) first; NULL there makes such
 * shapes return QZ_ERR_UNSUPPORTED.
 */
int qz_gemv_w8_rmsnorm(const int8_t* q, const float* scale, int64_t ng, const float* x,
                       const float* norm_w, float eps, float* y, int64_t N, int64_t K,
                       const float* residual, float* xn_scratch, void* stream);

/* qz_fused_mlp_decode of RMSNorm(x) * norm_w, normalised in the kernel's
 * activation staging; xn_scratch ([H]) as above. */
int qz_fused_mlp_decode_rmsnorm(const int8_t* gu_q, const float* gu_s, int64_t ng,
                                const float* x, const float* norm_w, float eps,
                                const int8_t* down_q, const float* down_s, int64_t ngd,
                                float* abuf, float* out, const float* residual, int64_t H,
                                int64_t I, uint32_t* sync_ws, float* xn_scratch, void* stream);

/* ------------------------------------------------------------------------
 * Decode-step glue: the fp32 work quartz's decoder does around its int8
 * matmuls, so a whole token can run on the device (and in one CUDA graph).
 * ------------------------------------------------------------------------ */

/* out[m, :] = dequant(q[ids[m], :]) -- the int8 embedding gather
 * (quartz/quantize.py:78-80 with dequantize_symmetric, 41-48). ids: device int64 [M]. */
int qz_embed_gather(const int8_t* q, const float* scale, int64_t ng, const int64_t* ids,
                    int64_t M, int64_t V, int64_t H, float* out, void* stream);

/* y[r, :] = x[r, :] / sqrt(mean(x[r, :]^2) + eps) * w  (quartz/ops.py:24-32). */
int qz_rmsnorm(const float* x, const float* w, float* y, int64_t rows, int64_t n, float eps,
               void* stream);

/*
 * qkv [M, (nq + 2 nkv) * hd] -> q_out [M, nq * hd] and the KV cache
 * ([nkv, max_ctx, hd] per layer) at positions pos0 + m: optional per-head
 * RMSNorm of q and k (Qwen3, quartz/models/qwen3.py:33-34; pass NULL weights
 * for Llama), half-split RoPE with the given inverse frequencies
 * (quartz/rope.py:47-78), K/V append (quartz/cache.py:26-46). pos_dev, if
 * not NULL, is a device int64 that replaces pos0 (for graph replay).
 */
int qz_qk_rope(const float* qkv, const float* q_norm_w, const float* k_norm_w,
               const float* inv_freq, float* q_out, float* k_cache, float* v_cache, int64_t M,
               int nq, int nkv, int hd, int64_t max_ctx, int64_t pos0, const int64_t* pos_dev,
               float eps, void* stream);

/* Workspace bytes the decode attention entry points need for contexts up to
 * max_ctx on the current device. The workspace must be 256-byte aligned and
 * zeroed once before its first use (the kernels leave it ready for the next
 * call); calls sharing one workspace must not overlap on the GPU.
 *
 * The decode attention kernels launch as programmatic dependents of the
 * previous kernel in the stream and start copying cache rows 0 .. T-2 before
 * they wait for it (row T-1, the newest, only after): those rows must have
 * been written by work that completed before the previous kernel started --
 * host copies, or kernels with an ordinary (non-programmatic) launch after
 * them, like the per-token embedding gather and argmax of a decode loop. */
int qz_attention_decode_workspace_bytes(int nq, int nkv, int hd, int64_t max_ctx, int64_t* bytes);

/*
 * One query row per head over the first T cache positions:
 * out[h] = softmax(q[h] . K^T * scale) V, kv head h / (nq / nkv) (GQA by
 * repeat, quartz/attention.py:29-43). T_dev, if not NULL, replaces T with
 * *T_dev + t_offset (for graph replay). The context is split across CTAs and
 * the last CTA of each kv head merges the partial softmaxes.
 */
int qz_attention_decode(const float* q, const float* k_cache, const float* v_cache, float* out,
                        int nq, int nkv, int hd, int64_t max_ctx, int64_t T, const int64_t* T_dev,
                        int64_t t_offset, float scale, void* ws, size_t ws_bytes, void* stream);

/*
 * The whole attention block of one decode token after the q/k/v projections,
 * in one launch: from the projection row qkv [(nq + 2 nkv) hd] (q heads, k
 * heads, v heads), optional per-head q/k RMSNorm (Qwen3,
 * quartz/models/qwen3.py:33-34; NULL weights for Llama), RoPE at position
 * pos (quartz/rope.py:47-78), append of k/v at pos (quartz/cache.py:26-46),
 * then qz_attention_decode over positions [0, pos]. pos = *pos_dev when
 * pos_dev is not NULL (graph replay), else pos0.
 */
int qz_attention_decode_qkv(const float* qkv, const float* q_norm_w, const float* k_norm_w,
                            const float* inv_freq, float* k_cache, float* v_cache, float* out,
                            int nq, int nkv, int hd, int64_t max_ctx, int64_t pos0,
                            const int64_t* pos_dev, float eps, float scale, void* ws,
                            size_t ws_bytes, void* stream);

/* Workspace bytes of qz_attention_decode_qkv_batch for `batch` sequences
 * (256-byte aligned, zeroed once before first use, left ready for the next
 * call; calls sharing it must not overlap on the GPU). */
int qz_attention_decode_batch_workspace_bytes(int batch, int nq, int nkv, int hd, int64_t max_ctx,
                                              int64_t* bytes);

/*
 * qz_attention_decode_qkv for `batch` sequences decoded in lockstep, the
 * reference's batched decode step (quartz/models/common.py:79-88 with ids
 * [B, 1]; quartz/attention.py:29-43 per batch row over its own cache,
 * quartz/cache.py:26-46 appending each row's k/v). Sequence b reads its
 * projection row at qkv + b * qkv_stride, appends to and attends over its
 * caches at k_cache / v_cache + b * cache_stride ([n_kv, max_ctx, hd] each,
 * cache_stride >= n_kv * max_ctx * hd) and writes out + b * out_stride
 * (elements). All sequences share the position (pos0, or *pos_dev for graph
 * replay). One launch for all sequences.
 */
int qz_attention_decode_qkv_batch(const float* qkv, int64_t qkv_stride, const float* q_norm_w,
                                  const float* k_norm_w, const float* inv_freq, float* k_cache,
                                  float* v_cache, int64_t cache_stride, float* out,
                                  int64_t out_stride, int batch, int nq, int nkv, int hd,
                                  int64_t max_ctx, int64_t pos0, const int64_t* pos_dev,
                                  float eps, float scale, void* ws, size_t ws_bytes, void* stream);

/* M query rows at positions pos0 .. pos0 + M - 1, each attending causally to
 * cache positions 0 .. its own (the additive mask of quartz/attention.py:15-26). */
int qz_attention_prefill(const float* q, const float* k_cache, const float* v_cache, float* out,
                         int64_t M, int nq, int nkv, int hd, int64_t max_ctx, int64_t pos0,
                         float scale, void* stream);

/*
 * tokens[m] = argmax of logits[m, :V], first index on ties (np.argmax,
 * quartz/sample.py:21-22). keys: device uint64 [M], zero before the first
 * call (left zero afterwards). pos_dev, if not NULL, is advanced by pos_step.
 */
int qz_argmax(const float* logits, int64_t M, int64_t V, uint64_t* keys, int64_t* tokens,
              int64_t* pos_dev, int64_t pos_step, void* stream);

/* ------------------------------------------------------------------------
 * Every decoder layer of one decode token in one persistent kernel.
 * ------------------------------------------------------------------------ */

/* Device pointers of one decoder layer (an array of these lives in device
 * memory). int8 matrices are row-major with one fp32 scale per row; every
 * pointer 16-byte aligned. qkv: q rows, k rows, v rows stacked; gu: gate rows
 * then up rows (quartz/quantize.py:95-96). Norm weights fp32; q/k norms NULL
 * for architectures without them (Llama). Caches [n_kv, max_ctx, head_dim]. */
typedef struct {
  const int8_t* qkv_q;   const float* qkv_s;    /* [(nq + 2 nkv) hd, H] */
  const int8_t* o_q;     const float* o_s;      /* [H, nq hd] */
  const int8_t* gu_q;    const float* gu_s;     /* [2 I, H] */
  const int8_t* down_q;  const float* down_s;   /* [H, I] */
  const float* in_norm_w;  const float* post_norm_w;   /* [H] */
  const float* q_norm_w;   const float* k_norm_w;      /* [hd] or NULL */
  float* k_cache;        float* v_cache;
} qz_decoder_layer;

/* Workspace bytes of qz_decode_layers (256-byte aligned, zeroed once before
 * first use; calls sharing it must not overlap on the GPU). A call whose
 * kernel reported a failed wait (qz_device_status) leaves it inconsistent:
 * zero it again before the next call. */
int qz_decode_step_workspace_bytes(int H, int I, int nq, int nkv, int hd, int64_t max_ctx,
                                   int64_t* bytes);

/* QZ_OK when qz_decode_layers runs these shapes on the current device (per-row
 * scales, head_dim 64 or 128, 1/2/4/8 query heads per kv head, rows of at most
 * 16 KB, ...), else QZ_ERR_UNSUPPORTED (use the per-op entry points instead). */
int qz_decode_layers_supported(int H, int I, int nq, int nkv, int hd, int64_t max_ctx);

/*
 * One decode token through all n_layers layers of a Qwen3/Llama decoder
 * (quartz/models/common.py:29-78, qwen3.py:31-45, llama.py:29-41) in one
 * cooperative launch of one CTA per SM: embedding row of *token (per-row int8
 * table, quartz/quantize.py:78-80), per layer RMSNorm -> q/k/v -> per-head
 * q/k RMSNorm (if given) -> RoPE at position *pos_dev -> K/V append ->
 * attention over positions [0, *pos_dev] -> o + residual -> RMSNorm -> fused
 * SwiGLU MLP + residual; then the final RMSNorm into x_final [H], the
 * lm_head input. The kernel waits at grid barriers between phases; each wait
 * gives up after about a second (status word) instead of hanging.
 * trace: NULL, or device uint64 [n_SMs][1 + 10 n_layers] that receives
 * %globaltimer stamps per CTA: launch start, then per layer and phase
 * (qkv, attention, o, gate/up, down) the end of its work and the end of the
 * grid barrier that follows.
 */
int qz_decode_layers(const qz_decoder_layer* layers, int n_layers, const int8_t* embed_q,
                     const float* embed_s, int64_t vocab, const int64_t* token,
                     const int64_t* pos_dev, const float* inv_freq, const float* norm_w,
                     float* x_final, int H, int I, int nq, int nkv, int hd, int64_t max_ctx,
                     float eps, float scale, void* ws, size_t ws_bytes, uint64_t* trace,
                     void* stream);

/* ------------------------------------------------------------------------
 * Peer-memory all-reduce for tensor-parallel decoding (one process per GPU,
 * GPUs of one node with peer access over NVLink). quartz has no counterpart:
 * it is single-process.
 * ------------------------------------------------------------------------ */

/* Bytes of one rank's communication buffer for `ranks` ranks and sums of at
 * most n_max floats (n_max a multiple of 4). */
int qz_comm_buffer_bytes(int ranks, int64_t n_max, int64_t* bytes);

/* cudaMalloc + zero a communication buffer on the current device / free it.
 * (Its own allocation, so that its IPC handle maps exactly this range.) */
int qz_comm_alloc(int64_t bytes, void** ptr);
int qz_comm_free(void* ptr);

/* 64-byte CUDA IPC handle of a qz_comm_alloc buffer; open a peer's handle in
 * this process (peer access enabled lazily); close it again. */
int qz_ipc_handle(const void* ptr, void* handle64);
int qz_ipc_open(const void* handle64, void** ptr);
int qz_ipc_close(void* ptr);

/*
 * out[i] = sum over ranks of their in[i], i < n, identical on every rank (the
 * sum runs in rank order). peer_buffers: host array of the `ranks` buffers as
 * mapped in this process (this rank's own at [rank]). Every rank must make
 * the same sequence of calls on its buffer; a call waits for its peers' pushes
 * for at most about a second (then the status word records it). in may equal
 * out. Each value travels with the call's tag in one 8-byte word, so a
 * receiver polls the data itself (no separate flag, no fence).
 */
int qz_allreduce_sum(const float* in, float* out, int64_t n, int64_t n_max,
                     void* const* peer_buffers, int rank, int ranks, void* stream);

/* Fused all-reduce: a producer kernel (qz_gemv_w8_peer,
 * qz_fused_mlp_decode_peer) sends its output rows, tagged with the call, to
 * every rank's buffer (region B of qz_comm_buffer_bytes) from its epilogue,
 * instead of writing them; qz_rmsnorm_peer_sum on each rank then sums the
 * ranks' rows in rank order as it reads them and applies an RMSNorm. The
 * partial sums of a row-parallel projection are reduced without a separate
 * collective launch. Producers and consumers must alternate, in the same order
 * on every rank. */
typedef struct {
  void* buffers[8];   /* every rank's qz_comm_alloc buffer as mapped in this process */
  int rank;
  int ranks;          /* 1..8 */
  int64_t n_max;      /* the buffers' n_max (qz_comm_buffer_bytes) */
} qz_peer_sum;

/* qz_gemv_w8 whose rows y[n] (+ residual[n]) go to the ranks (no local y). */
int qz_gemv_w8_peer(const int8_t* q, const float* scale, int64_t ng, const float* x, int64_t N,
                    int64_t K, const float* residual, const qz_peer_sum* ps, void* stream);

/* qz_fused_mlp_decode whose output rows (+ residual) go to the ranks. */
int qz_fused_mlp_decode_peer(const int8_t* gu_q, const float* gu_s, int64_t ng, const float* x,
                             const int8_t* down_q, const float* down_s, int64_t ngd, float* abuf,
                             const float* residual, int64_t H, int64_t I, uint32_t* sync_ws,
                             const qz_peer_sum* ps, void* stream);

/* h[i] = sum over ranks (rank order) of the rows the last producer pushed,
 * i < n (n <= 4096); xn = h / sqrt(mean(h^2) + eps) * w (quartz/ops.py:24-32).
 * Waits for the pushes for at most about a second (status word). */
int qz_rmsnorm_peer_sum(const qz_peer_sum* ps, int64_t n, const float* w, float eps, float* h,
                        float* xn, void* stream);

/* Read the device status word of the current device into words[0..3]
 * ({error bits, first error site, block of first error, error count}); when
 * clear != 0 reset it to zero afterwards. Synchronises the device. */
int qz_device_status(uint32_t* words, int clear);

/* cudaStreamSynchronize(stream) with the error mapped to a status. */
int qz_sync(void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QUARTZ_B200_H_ */
