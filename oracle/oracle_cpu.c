/*
 * oracle_cpu.c -- plain-C restatement of the reference's W8A8 arithmetic. TEST
 * INFRASTRUCTURE ONLY: used by tests/ as a second, independent checker and by bench.py's
 * CPU-baseline / reference legs as the host-core implementation of the reference path.
 * Nothing in the product (mica_b200/) loads it.
 *
 *   oracle_quant_act  per-token int8 quantiser, both rounding modes:
 *     mode 0 = the reference GPU kernel  v0.5/serving/kernel_src/kernels.py:15-38
 *              (s = max(amax, 1e-8)/127, v = x/s, q = trunc(fl(v +- 0.5)), clamp +-127)
 *     mode 1 = the reference torch path  v0.5/serving/lib/int8_quant.py:64-74 (round half even)
 *   oracle_int_gemm   exact int8 x int8 -> int32 products, C[m,n] = sum_k A[m,k] B[n,k]
 *                     (int8_quant.int_gemm_exact / torch_int_mm, lib/int8_quant.py:88-97)
 *   oracle_dequant    y = (float)acc * sa[m] * sb[n] (+ bias[n]) in fp32, left to right, then
 *                     round-to-nearest-even to bf16 bits (ksrc/kernels.py:63-66,
 *                     lib/int8_runtime.py:186-192)
 *
 * Build (oracle/Makefile): gcc -O3 -mavx2 -fopenmp -ffp-contract=off -shared -fPIC.
 * -ffp-contract=off keeps every product and sum separately rounded, as the reference's fp32
 * math is; -mavx2 lets the compiler vectorise the int8 dot products (int16 multiply-adds).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

int oracle_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void oracle_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

void oracle_quant_act(const float* x, const float* inv, long M, long K, int mode, int8_t* q, float* s) {
#pragma omp parallel for schedule(static)
    for (long m = 0; m < M; ++m) {
        const float* xr = x + m * K;
        float amax = 0.0f;
        for (long k = 0; k < K; ++k) {
            const float v = inv ? xr[k] * inv[k] : xr[k];
            const float a = fabsf(v);
            if (a > amax) amax = a;
        }
        const float scale = (amax > 1e-8f ? amax : 1e-8f) / 127.0f;
        s[m] = scale;
        for (long k = 0; k < K; ++k) {
            const float v = (inv ? xr[k] * inv[k] : xr[k]) / scale;
            float r;
            if (mode == 1) {
                r = nearbyintf(v);                       /* default rounding mode: half to even */
            } else {
                const float t = v >= 0.0f ? v + 0.5f : v - 0.5f;
                r = truncf(t);
            }
            if (r > 127.0f) r = 127.0f;
            if (r < -127.0f) r = -127.0f;
            q[m * K + k] = (int8_t)r;
        }
    }
}

static int32_t dot_i8(const int8_t* a, const int8_t* b, long K) {
    int32_t acc = 0;
    for (long k = 0; k < K; ++k) acc += (int16_t)a[k] * (int16_t)b[k];
    return acc;
}

#if defined(__AVX2__)
#include <immintrin.h>
static inline int32_t hsum8(__m256i v) {
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4E));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xB1));
    return _mm_cvtsi128_si32(s);
}
/* 2 rows of A x 4 rows of B over the first Kv (multiple of 16) columns: sign-extend 16 int8
 * to int16, multiply-add adjacent pairs into int32 (exact: |a*b + a*b| < 2^15), accumulate in
 * 8 int32 vectors (8 accumulators + 6 operands fit AVX2's 16 registers). */
static void block2x4(const int8_t* A, const int8_t* B, long K, long Kv, int32_t out[2][4]) {
    __m256i acc[2][4];
    for (int i = 0; i < 2; ++i)
        for (int j = 0; j < 4; ++j) acc[i][j] = _mm256_setzero_si256();
    for (long k = 0; k < Kv; k += 16) {
        const __m256i a0 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(A + k)));
        const __m256i a1 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(A + K + k)));
        for (int j = 0; j < 4; ++j) {
            const __m256i b = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(B + j * K + k)));
            acc[0][j] = _mm256_add_epi32(acc[0][j], _mm256_madd_epi16(a0, b));
            acc[1][j] = _mm256_add_epi32(acc[1][j], _mm256_madd_epi16(a1, b));
        }
    }
    for (int i = 0; i < 2; ++i)
        for (int j = 0; j < 4; ++j) {
            int32_t t = hsum8(acc[i][j]);
            for (long k = Kv; k < K; ++k) t += (int16_t)A[i * K + k] * (int16_t)B[j * K + k];
            out[i][j] = t;
        }
}
#endif

void oracle_int_gemm(const int8_t* A, const int8_t* B, long M, long N, long K, int32_t* C) {
    /* 2 x 4 register blocks over (m, n) */
    const long MB = 2, NB = 4;
#pragma omp parallel for collapse(2) schedule(dynamic, 4)
    for (long m0 = 0; m0 < M; m0 += MB) {
        for (long n0 = 0; n0 < N; n0 += NB) {
            const long me = m0 + MB < M ? m0 + MB : M;
            const long ne = n0 + NB < N ? n0 + NB : N;
#if defined(__AVX2__)
            if (me - m0 == 2 && ne - n0 == 4) {
                int32_t o[2][4];
                block2x4(A + m0 * K, B + n0 * K, K, K & ~15L, o);
                for (int i = 0; i < 2; ++i)
                    for (int j = 0; j < 4; ++j) C[(m0 + i) * N + n0 + j] = o[i][j];
                continue;
            }
#endif
            for (long m = m0; m < me; ++m)
                for (long n = n0; n < ne; ++n) C[m * N + n] = dot_i8(A + m * K, B + n * K, K);
        }
    }
}

static uint16_t bf16_rne(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40u);   /* quiet NaN */
    u += ((u >> 16) & 1u) + 0x7FFFu;
    return (uint16_t)(u >> 16);
}

void oracle_dequant(const int32_t* acc, const float* sa, const float* sb, const float* bias, long M, long N,
                    uint16_t* out) {
#pragma omp parallel for schedule(static)
    for (long m = 0; m < M; ++m) {
        for (long n = 0; n < N; ++n) {
            float y = (float)acc[m * N + n] * sa[m];
            y = y * sb[n];
            if (bias) y = y + bias[n];
            out[m * N + n] = bf16_rne(y);
        }
    }
}
