/*
 * qz_oracle.c -- CPU restatement of quartz's fused int8 weight-only kernels.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker the CUDA path is compared
 * against (and the timed CPU baseline). Nothing in the shipped library links,
 * loads or calls it.
 *
 * Each function restates one Numba kernel of the reference, loop for loop:
 *   qzo_w8a32_gemv        quartz/kernels/int8.py:24-38   (w8a32_gemv; the serial
 *                         twin int8.py:48-63 computes the same rows)
 *   qzo_w8a32_gemm        quartz/kernels/int8.py:66-87   (w8a32_gemm)
 *   qzo_fused_mlp_decode  quartz/kernels/fused.py:27-65  (fused_mlp_decode)
 *
 * Arithmetic follows the reference: int8 weights are widened to fp32 in
 * register, products accumulate in fp32 per group of G = K / ng elements, and
 * each group sum is weighted by its fp32 scale. The reference compiles with
 * fastmath, which lets LLVM reassociate the inner fp32 sum; dot_i8f32 takes the
 * same freedom on the same loop (and only there). Rows are split over OpenMP
 * threads as the reference splits them over its prange pool: one output row
 * per iteration.
 */
#include <math.h>
#include <stdint.h>
#include <omp.h>

static int g_threads = 0; /* 0 = OpenMP default */

void qzo_set_threads(int n) { g_threads = n; }

int qzo_get_threads(void) {
    return g_threads > 0 ? g_threads : omp_get_max_threads();
}

/*
 * sum_{j<n} x[j] * (float)q[j] in fp32 with four independent vector partial
 * sums: the reassociation the reference's fastmath grants its LLVM vectoriser,
 * which interleaves its reduction the same way. (Explicit intrinsics: gcc
 * scalarises the int8 -> fp32 widening otherwise.)
 */
#if defined(__AVX512F__)
#include <immintrin.h>
static inline __m512 q16(const int8_t *p) {
    return _mm512_cvtepi32_ps(_mm512_cvtepi8_epi32(_mm_loadu_si128((const __m128i *)p)));
}
static inline float dot_i8f32(const int8_t *q, const float *x, int64_t n) {
    __m512 a0 = _mm512_setzero_ps(), a1 = a0, a2 = a0, a3 = a0;
    int64_t j = 0;
    for (; j + 64 <= n; j += 64) {
        a0 = _mm512_fmadd_ps(_mm512_loadu_ps(x + j), q16(q + j), a0);
        a1 = _mm512_fmadd_ps(_mm512_loadu_ps(x + j + 16), q16(q + j + 16), a1);
        a2 = _mm512_fmadd_ps(_mm512_loadu_ps(x + j + 32), q16(q + j + 32), a2);
        a3 = _mm512_fmadd_ps(_mm512_loadu_ps(x + j + 48), q16(q + j + 48), a3);
    }
    for (; j + 16 <= n; j += 16)
        a0 = _mm512_fmadd_ps(_mm512_loadu_ps(x + j), q16(q + j), a0);
    float s = _mm512_reduce_add_ps(_mm512_add_ps(_mm512_add_ps(a0, a1), _mm512_add_ps(a2, a3)));
    for (; j < n; ++j)
        s += x[j] * (float)q[j];
    return s;
}
#elif defined(__AVX2__) && defined(__FMA__)
#include <immintrin.h>
static inline __m256 q8(const int8_t *p) {
    return _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i *)p)));
}
static inline float dot_i8f32(const int8_t *q, const float *x, int64_t n) {
    __m256 a0 = _mm256_setzero_ps(), a1 = a0, a2 = a0, a3 = a0;
    int64_t j = 0;
    for (; j + 32 <= n; j += 32) {
        a0 = _mm256_fmadd_ps(_mm256_loadu_ps(x + j), q8(q + j), a0);
        a1 = _mm256_fmadd_ps(_mm256_loadu_ps(x + j + 8), q8(q + j + 8), a1);
        a2 = _mm256_fmadd_ps(_mm256_loadu_ps(x + j + 16), q8(q + j + 16), a2);
        a3 = _mm256_fmadd_ps(_mm256_loadu_ps(x + j + 24), q8(q + j + 24), a3);
    }
    for (; j + 8 <= n; j += 8)
        a0 = _mm256_fmadd_ps(_mm256_loadu_ps(x + j), q8(q + j), a0);
    const __m256 a = _mm256_add_ps(_mm256_add_ps(a0, a1), _mm256_add_ps(a2, a3));
    float t[8];
    _mm256_storeu_ps(t, a);
    float s = ((t[0] + t[1]) + (t[2] + t[3])) + ((t[4] + t[5]) + (t[6] + t[7]));
    for (; j < n; ++j)
        s += x[j] * (float)q[j];
    return s;
}
#else
static inline float dot_i8f32(const int8_t *q, const float *x, int64_t n) {
    float s = 0.0f;
    for (int64_t j = 0; j < n; ++j)
        s += x[j] * (float)q[j];
    return s;
}
#endif

/* One row: sum_g scale[g] * sum_{j<G} x[gG+j] * (float)q[gG+j]  (int8.py:31-38). */
static inline float row_dot(const int8_t *qr, const float *sr, const float *x,
                            int64_t ng, int64_t G) {
    float acc = 0.0f;
    for (int64_t gi = 0; gi < ng; ++gi) {
        const int64_t base = gi * G;
        const float gs = dot_i8f32(qr + base, x + base, G);
        acc += gs * sr[gi];
    }
    return acc;
}

/* y[n] for n < N. q: [N,K] int8 row-major; scale: [N,ng]; x: [K]; y: [N]. */
void qzo_w8a32_gemv(const int8_t *q, const float *scale, int64_t N, int64_t K,
                    int64_t ng, const float *x, float *y) {
    const int64_t G = K / ng;
#pragma omp parallel for schedule(static) num_threads(qzo_get_threads())
    for (int64_t n = 0; n < N; ++n)
        y[n] = row_dot(q + n * K, scale + n * ng, x, ng, G);
}

/* Y[m,n] for m < M, n < N: rows parallel, tokens serial (int8.py:77-87). */
void qzo_w8a32_gemm(const int8_t *q, const float *scale, int64_t N, int64_t K,
                    int64_t ng, const float *X, int64_t M, float *Y) {
    const int64_t G = K / ng;
#pragma omp parallel for schedule(static) num_threads(qzo_get_threads())
    for (int64_t n = 0; n < N; ++n)
        for (int64_t m = 0; m < M; ++m)
            Y[m * N + n] = row_dot(q + n * K, scale + n * ng, X + m * K, ng, G);
}

/*
 * out[H] = down( silu(gate . x) * (up . x) )      (fused.py:27-65)
 * gu_q: [2I, H] int8 (rows 0..I-1 gate, I..2I-1 up); gu_s: [2I, ng];
 * down_q: [H, I] int8; down_s: [H, ngd]; abuf: [I] scratch; out: [H].
 * silu is ga / (1 + exp(-ga)) with no clipping (fused.py:53).
 */
void qzo_fused_mlp_decode(const int8_t *gu_q, const float *gu_s, int64_t I,
                          int64_t H, int64_t ng, const float *x,
                          const int8_t *down_q, const float *down_s, int64_t ngd,
                          float *abuf, float *out) {
    const int64_t G = H / ng;
#pragma omp parallel for schedule(static) num_threads(qzo_get_threads())
    for (int64_t n = 0; n < I; ++n) {
        float ga = 0.0f, ua = 0.0f;
        for (int64_t gi = 0; gi < ng; ++gi) {
            float gg, uu;
            const int64_t base = gi * G;
            const int8_t *gr = gu_q + n * H + base;
            const int8_t *ur = gu_q + (n + I) * H + base;
            gg = dot_i8f32(gr, x + base, G);
            uu = dot_i8f32(ur, x + base, G);
            ga += gg * gu_s[n * ng + gi];
            ua += uu * gu_s[(n + I) * ng + gi];
        }
        const float s = ga / (1.0f + expf(-ga));
        abuf[n] = s * ua;
    }
    const int64_t Gd = I / ngd;
#pragma omp parallel for schedule(static) num_threads(qzo_get_threads())
    for (int64_t h = 0; h < H; ++h)
        out[h] = row_dot(down_q + h * I, down_s + h * ngd, abuf, ngd, Gd);
}
