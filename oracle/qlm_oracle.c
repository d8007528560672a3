/*
 * TEST INFRASTRUCTURE ONLY — a plain-C restatement of QuickLM's int8 path,
 * used as the parity checker for the CUDA kernels. The product never links,
 * loads or calls this file; only tests/, the smoke check and bench.py's CPU
 * baseline do. Built by oracle/Makefile into oracle/_build/libqlm_oracle.so.
 *
 * Pinned: tests/test_oracle.py checks every function here bit-for-bit against
 * the reference's own implementation (compiled from its sources into
 * oracle/_ref/) and against the committed fixtures in tests/golden/.
 *
 * Must be compiled WITHOUT floating-point contraction (-ffp-contract=off) and
 * without -ffast-math: every multiply and add below is one IEEE-754 binary32
 * operation rounded to nearest-even, as in the reference's AVX2 intrinsics.
 *
 * Reference citations are paths inside the QuickLM source tree.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define QLMO_BLOCK 32 /* Tensor::INT8_BLOCK_SIZE (tensor/tensor.hpp:32) */

/* x86 MAXPS / MAXSS lane semantics: dest = (a > b) ? a : b, so an unordered
 * compare returns the SECOND operand (io/safetensors.cpp:308,360 use
 * _mm256_max_ps(vmax, |v|); the NaN behaviour follows from that). */
static inline float maxps(float a, float b) { return (a > b) ? a : b; }

/* std::max(a, b) == (a < b) ? b : a (io/safetensors.cpp:315,364). */
static inline float stdmax(float a, float b) { return (a < b) ? b : a; }

/* _mm256_round_ps(.., NEAREST) followed by _mm256_cvtps_epi32: RN-even, and
 * the x86 "integer indefinite" 0x80000000 for NaN / out-of-range
 * (io/safetensors.cpp:325-327, 374-376). */
static inline int32_t cvt_rne_indefinite(float v) {
    float r = rintf(v); /* default rounding mode: to nearest, ties to even */
    if (!(fabsf(r) < 2147483648.0f)) return INT32_MIN;
    return (int32_t)r;
}

/* static_cast<int>(std::lround(v)) for the scalar tail (io/safetensors.cpp:340,
 * 386): ties away from zero; glibc returns (long)v == LONG_MIN for NaN/Inf/huge,
 * and the narrowing cast keeps the low 32 bits. */
static inline int32_t cvt_lround_int(float v) {
    if (isnan(v) || !(fabsf(v) < 9.2233720368547758e18f)) return 0; /* (int)LONG_MIN */
    float r = roundf(v);
    long long l = (long long)r;
    return (int32_t)(uint32_t)(unsigned long long)l;
}

static inline int8_t clamp127(int32_t q) { return (int8_t)(q < -127 ? -127 : (q > 127 ? 127 : q)); }
/* int4: clamp to [-8, 7] (io/safetensors.cpp:436-437, 452-453). */
static inline int8_t clamp_q4(int32_t q) { return (int8_t)(q < -8 ? -8 : (q > 7 ? 7 : q)); }

static inline float bf16_to_f32(uint16_t h) {
    uint32_t bits = (uint32_t)h << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* One block [k0, k1) of a row, values supplied by get(i). Restates the loop
 * body of st_quantize_row_f32 / st_quantize_row_bf16 (io/safetensors.cpp:
 * 353-390 / 301-344). */
#define QLMO_QUANT_BLOCK(GET) QLMO_QUANT_BLOCK_T(GET, 127.0f, clamp127)
#define QLMO_QUANT_BLOCK_T(GET, DIV, CLAMP)                                            \
    do {                                                                               \
        float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0}; /* vmax = _mm256_setzero_ps() */   \
        int k = k0;                                                                    \
        for (; k + 8 <= k1; k += 8)                                                    \
            for (int i = 0; i < 8; ++i) lane[i] = maxps(lane[i], fabsf(GET(k + i)));  \
        /* st_hmax (io/safetensors.cpp:283-290) */                                     \
        float m0 = maxps(lane[0], lane[4]), m1 = maxps(lane[1], lane[5]);             \
        float m2 = maxps(lane[2], lane[6]), m3 = maxps(lane[3], lane[7]);             \
        m0 = maxps(m0, m2);                                                            \
        m1 = maxps(m1, m3);                                                            \
        float max_abs = maxps(m0, m1);                                                 \
        for (; k < k1; ++k) max_abs = stdmax(max_abs, fabsf(GET(k)));                 \
        float scale = (max_abs > 0.0f) ? (max_abs / (DIV)) : 1.0f;                     \
        scales[blk] = scale;                                                           \
        float inv = 1.0f / scale;                                                      \
        k = k0;                                                                        \
        for (; k + 8 <= k1; k += 8)                                                    \
            for (int i = 0; i < 8; ++i) out[k + i] = CLAMP(cvt_rne_indefinite(GET(k + i) * inv)); \
        for (; k < k1; ++k) out[k] = CLAMP(cvt_lround_int(GET(k) * inv));             \
    } while (0)

/* st_quantize_row_f32 (io/safetensors.cpp:348-391). */
void qlmo_quantize_row_f32(const float* row, int K, int8_t* out, float* scales) {
    int nb = (K + QLMO_BLOCK - 1) / QLMO_BLOCK;
    for (int blk = 0; blk < nb; ++blk) {
        int k0 = blk * QLMO_BLOCK;
        int k1 = k0 + QLMO_BLOCK < K ? k0 + QLMO_BLOCK : K;
#define QLMO_GET_F32(i) (row[(i)])
        QLMO_QUANT_BLOCK(QLMO_GET_F32);
#undef QLMO_GET_F32
    }
}

/* st_quantize_row_bf16 (io/safetensors.cpp:296-345). */
void qlmo_quantize_row_bf16(const uint16_t* row, int K, int8_t* out, float* scales) {
    int nb = (K + QLMO_BLOCK - 1) / QLMO_BLOCK;
    for (int blk = 0; blk < nb; ++blk) {
        int k0 = blk * QLMO_BLOCK;
        int k1 = k0 + QLMO_BLOCK < K ? k0 + QLMO_BLOCK : K;
#define QLMO_GET_BF16(i) (bf16_to_f32(row[(i)]))
        QLMO_QUANT_BLOCK(QLMO_GET_BF16);
#undef QLMO_GET_BF16
    }
}

/* get_tensor_keep_int8 over a whole [n, k] matrix (io/safetensors.cpp:517-585);
 * dtype 0 = F32, 1 = BF16. The row split across threads does not change bits. */
void qlmo_quantize(const void* w, int dtype, int n, int k, int8_t* q, float* s) {
    int nb = (k + QLMO_BLOCK - 1) / QLMO_BLOCK;
    for (int r = 0; r < n; ++r) {
        if (dtype == 1)
            qlmo_quantize_row_bf16((const uint16_t*)w + (size_t)r * k, k, q + (size_t)r * k, s + (size_t)r * nb);
        else
            qlmo_quantize_row_f32((const float*)w + (size_t)r * k, k, q + (size_t)r * k, s + (size_t)r * nb);
    }
}

void qlmo_quantize_row_f32_q4(const float* row, int K, int8_t* out, float* scales);
void qlmo_quantize_row_bf16_q4(const uint16_t* row, int K, int8_t* out, float* scales);

/* get_tensor_keep_int4 over a whole [n, k] matrix (io/safetensors.cpp, the
 * int4 loader); q receives signed values in [-8, 7]. */
void qlmo_quantize_q4(const void* w, int dtype, int n, int k, int8_t* q, float* s) {
    int nb = (k + QLMO_BLOCK - 1) / QLMO_BLOCK;
    for (int r = 0; r < n; ++r) {
        if (dtype == 1)
            qlmo_quantize_row_bf16_q4((const uint16_t*)w + (size_t)r * k, k, q + (size_t)r * k, s + (size_t)r * nb);
        else
            qlmo_quantize_row_f32_q4((const float*)w + (size_t)r * k, k, q + (size_t)r * k, s + (size_t)r * nb);
    }
}

/* One output element y = a . dequant(b) with per-32-block scales. Restates
 * dot_avx2_int8 (ops/math_ops.cpp:414-444); dot8_avx2_int8 (448-494) and
 * dot4_avx2_int8 (498-553) perform the identical per-row sequence:
 *   lane l in [0,8), block b ascending:
 *     p_j  = a[32b+8j+l] * (float)q[32b+8j+l]          j = 0..3
 *     bs   = (p_0 + p_1) + (p_2 + p_3)
 *     t_l  = fmaf(bs, s[b], t_l)                        t_l starts at +0
 *   u_i = t_i + t_{i+4} (i = 0..3); y = (u_0 + u_1) + (u_2 + u_3)
 *   K % 32 tail: acc = sum_k a[k]*q[k] in k order from 0, y += acc * s[last].
 */
float qlmo_dot_int8(const float* a, const int8_t* b, const float* scales, int K) {
    float t[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int k = 0, blk = 0;
    for (; k + QLMO_BLOCK <= K; k += QLMO_BLOCK, ++blk) {
        for (int l = 0; l < 8; ++l) {
            float p0 = a[k + l] * (float)b[k + l];
            float p1 = a[k + 8 + l] * (float)b[k + 8 + l];
            float p2 = a[k + 16 + l] * (float)b[k + 16 + l];
            float p3 = a[k + 24 + l] * (float)b[k + 24 + l];
            float bs = (p0 + p1) + (p2 + p3);
            t[l] = fmaf(bs, scales[blk], t[l]);
        }
    }
    /* hsum: lo+hi, then two hadd (ops/math_ops.cpp:429-434, 477-484) */
    float u0 = t[0] + t[4], u1 = t[1] + t[5], u2 = t[2] + t[6], u3 = t[3] + t[7];
    float result = (u0 + u1) + (u2 + u3);
    if (k < K) { /* ops/math_ops.cpp:436-442 */
        float tail = 0.0f;
        for (int kk = k; kk < K; ++kk) tail += a[kk] * (float)b[kk];
        result += tail * scales[blk];
    }
    return result;
}

/* math::matmul with an int8 B (ops/math_ops.cpp:820-900): every output row m
 * and column n is one qlmo_dot_int8 — independent of M, thread count and the
 * 64-row tiling. C has row stride ldc. */
void qlmo_matmul_int8(const float* A, int M, int K, const int8_t* q, const float* s, int N, float* C, int ldc) {
    int nb = (K + QLMO_BLOCK - 1) / QLMO_BLOCK;
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n)
            C[(size_t)m * ldc + n] = qlmo_dot_int8(A + (size_t)m * K, q + (size_t)n * K, s + (size_t)n * nb, K);
}

/* st_quantize_row_f32_int4 / st_quantize_row_bf16_int4 (io/safetensors.cpp:
 * 393-515): the same block loop with scale = max|v| / 8 and values clamped to
 * [-8, 7]. out receives the SIGNED values (one per element); the reference
 * stores value + 8 two per byte (low nibble = even column), which the caller
 * packs. Its scalar tail defaults a missing odd partner to nibble 8 (value 0). */
void qlmo_quantize_row_f32_q4(const float* row, int K, int8_t* out, float* scales) {
    int nb = (K + QLMO_BLOCK - 1) / QLMO_BLOCK;
    for (int blk = 0; blk < nb; ++blk) {
        int k0 = blk * QLMO_BLOCK;
        int k1 = k0 + QLMO_BLOCK < K ? k0 + QLMO_BLOCK : K;
#define QLMO_GET_F32(i) (row[(i)])
        QLMO_QUANT_BLOCK_T(QLMO_GET_F32, 8.0f, clamp_q4);
#undef QLMO_GET_F32
    }
}

void qlmo_quantize_row_bf16_q4(const uint16_t* row, int K, int8_t* out, float* scales) {
    int nb = (K + QLMO_BLOCK - 1) / QLMO_BLOCK;
    for (int blk = 0; blk < nb; ++blk) {
        int k0 = blk * QLMO_BLOCK;
        int k1 = k0 + QLMO_BLOCK < K ? k0 + QLMO_BLOCK : K;
#define QLMO_GET_BF16(i) (bf16_to_f32(row[(i)]))
        QLMO_QUANT_BLOCK_T(QLMO_GET_BF16, 8.0f, clamp_q4);
#undef QLMO_GET_BF16
    }
}
