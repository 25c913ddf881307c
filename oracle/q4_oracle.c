/*
 * CPU oracle for the int4-dequant GEMM/GEMV + LoRA hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links, loads or
 * calls this file: only the test suite, the smoke check and the benchmark's
 * CPU-baseline leg use it, and only as the checker.
 *
 * It is a restatement in plain C of the reference algorithm
 * (cpntodd/Spaceslug-main).  Each function cites the reference lines it
 * follows.  The restatement is pinned against outputs of the reference's own
 * code (compiled from its sources by oracle/Makefile into oracle/_ref/) via
 * the fixtures in tests/golden/.
 *
 * Weight layout (vulkan-runtime/shaders/q4gemm.comp:7-19):
 *   - int4 v in [-8,7] stored as the nibble v & 0xF;
 *   - packed byte pb = n*(K/2) + k/2; even k -> low nibble, odd k -> high;
 *   - 4 bytes per little-endian uint32 word (byte pb -> word pb>>2, lane pb&3);
 *   - scale for (k, n) = scales[n*(K/32) + k/32];
 *   - dequant w = float(v) * scale.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#define OQ4_LCG_A 1664525u
#define OQ4_LCG_C 1013904223u

/* LCG uniform floats in [lo, hi).
 * Follows vulkan-runtime/tests/test_q4gemm.cpp:58-68: s = s*1664525+1013904223,
 * u = float(s>>8) * 2^-24, v = lo + u*(hi-lo), all in fp32. */
void oq4_lcg_floats(size_t n, uint32_t seed, float lo, float hi, float* out) {
    uint32_t s = seed;
    for (size_t i = 0; i < n; ++i) {
        s = s * OQ4_LCG_A + OQ4_LCG_C;
        float u = (float)(s >> 8) * (1.0f / 16777216.0f);
        out[i] = lo + u * (hi - lo); /* built with -ffp-contract=off: no FMA */
    }
}

/* LCG int4 values in [-8, 7].
 * Follows vulkan-runtime/tests/test_q4gemm.cpp:71-80: v = ((s>>8) % 16) - 8. */
void oq4_lcg_int4(size_t n, uint32_t seed, int8_t* out) {
    uint32_t s = seed;
    for (size_t i = 0; i < n; ++i) {
        s = s * OQ4_LCG_A + OQ4_LCG_C;
        out[i] = (int8_t)((int)((s >> 8) % 16u) - 8);
    }
}

/* Pack logical int4 b[k*N + n] into the reference layout.
 * Follows vulkan-runtime/tests/test_q4gemm.cpp:84-99.  packed must hold
 * K*N/8 words; it is cleared here.  Returns 0, or 1 when K is odd. */
int oq4_pack(const int8_t* b_kn, uint32_t K, uint32_t N, uint32_t* packed) {
    if (K % 2u) return 1;
    const uint32_t k_half = K / 2u;
    const size_t words = ((size_t)k_half * N + 3u) / 4u;
    memset(packed, 0, words * sizeof(uint32_t));
    for (uint32_t n = 0; n < N; ++n) {
        for (uint32_t k = 0; k < K; ++k) {
            uint32_t nib = (uint32_t)(uint8_t)b_kn[(size_t)k * N + n] & 0xFu;
            uint32_t shift = (k & 1u) * 4u;
            size_t pb = (size_t)n * k_half + (k >> 1u);
            packed[pb >> 2u] |= nib << (shift + (uint32_t)(pb & 3u) * 8u);
        }
    }
    return 0;
}

/* Nibble unpack of one (k, n) element, sign-extended to [-8, 7].
 * Follows vulkan-runtime/shaders/q4gemm.comp:104-116. */
static inline int oq4_nibble(const uint32_t* packed, uint32_t K, uint32_t k, uint32_t n) {
    size_t pb = (size_t)n * (K / 2u) + (k >> 1u);
    uint32_t byte = (packed[pb >> 2u] >> ((uint32_t)(pb & 3u) * 8u)) & 0xFFu;
    uint32_t nib = (k & 1u) ? (byte >> 4u) : (byte & 0xFu);
    return nib >= 8u ? (int)nib - 16 : (int)nib;
}

/* Unpack packed words back to logical int8 b[k*N + n] (inverse of oq4_pack). */
void oq4_unpack(const uint32_t* packed, uint32_t K, uint32_t N, int8_t* b_kn) {
    for (uint32_t k = 0; k < K; ++k)
        for (uint32_t n = 0; n < N; ++n)
            b_kn[(size_t)k * N + n] = (int8_t)oq4_nibble(packed, K, k, n);
}

/* Dequantised weights w[k*N + n] = float(v) * scale (fp32, one rounding).
 * Follows vulkan-runtime/shaders/q4gemm.comp:104-122. */
void oq4_dequant(const uint32_t* packed, const float* scales, uint32_t K, uint32_t N, float* w_kn) {
    const uint32_t groups = K / 32u;
    for (uint32_t k = 0; k < K; ++k)
        for (uint32_t n = 0; n < N; ++n) {
            float s = scales[(size_t)n * groups + k / 32u];
            w_kn[(size_t)k * N + n] = (float)oq4_nibble(packed, K, k, n) * s;
        }
}

/* Double-precision reference GEMM  C = A * dequant(B), loop order m, k, n.
 * Follows vulkan-runtime/tests/test_q4gemm.cpp:102-119.  Rows [m0, m1) only
 * (so callers can sample rows of large problems); c is [(m1-m0) x N]. */
void oq4_gemm_ref_rows(const float* a, const int8_t* b_kn, const float* scales,
                       uint32_t M, uint32_t N, uint32_t K, uint32_t m0, uint32_t m1,
                       double* c) {
    const uint32_t groups = K / 32u;
    (void)M;
    memset(c, 0, sizeof(double) * (size_t)(m1 - m0) * N);
    for (uint32_t m = m0; m < m1; ++m) {
        double* crow = c + (size_t)(m - m0) * N;
        for (uint32_t k = 0; k < K; ++k) {
            double av = (double)a[(size_t)m * K + k];
            const int8_t* brow = b_kn + (size_t)k * N;
            for (uint32_t n = 0; n < N; ++n) {
                double bv = (double)brow[n] * (double)scales[(size_t)n * groups + k / 32u];
                crow[n] += av * bv;
            }
        }
    }
}

/* Same oracle, reading the packed layout instead of the logical int8 matrix
 * (identical values: unpack is exact). */
void oq4_gemm_ref_packed_rows(const float* a, const uint32_t* packed, const float* scales,
                              uint32_t N, uint32_t K, uint32_t m0, uint32_t m1, double* c) {
    const uint32_t groups = K / 32u;
    memset(c, 0, sizeof(double) * (size_t)(m1 - m0) * N);
    for (uint32_t m = m0; m < m1; ++m) {
        double* crow = c + (size_t)(m - m0) * N;
        for (uint32_t n = 0; n < N; ++n) {
            double acc = 0.0;
            for (uint32_t k = 0; k < K; ++k) {
                double bv = (double)oq4_nibble(packed, K, k, n) *
                            (double)scales[(size_t)n * groups + k / 32u];
                acc += (double)a[(size_t)m * K + k] * bv;
            }
            crow[n] = acc;
        }
    }
}

/* LoRA term in double: out[m][n] = (alpha/rank) * sum_r (sum_k x[m][k]*A[k][r]) * B[r][n].
 * Restates vulkan-runtime/tests/test_lora_delta_api.cpp:14 (the X*A*B loop)
 * generalised from hidden 64 to K x N, with the alpha/rank scale of
 * python/spaceslug/lora.py:21-23.  Rows [m0, m1); out is [(m1-m0) x N] and is
 * ADDED to (so it composes with oq4_gemm_ref_rows). */
void oq4_lora_ref_rows(const float* x, const float* lora_a, const float* lora_b,
                       uint32_t K, uint32_t N, uint32_t rank, float alpha,
                       uint32_t m0, uint32_t m1, double* out) {
    const double scale = (double)alpha / (double)rank;
    for (uint32_t m = m0; m < m1; ++m) {
        double* orow = out + (size_t)(m - m0) * N;
        for (uint32_t r = 0; r < rank; ++r) {
            double t = 0.0;
            for (uint32_t k = 0; k < K; ++k)
                t += (double)x[(size_t)m * K + k] * (double)lora_a[(size_t)k * rank + r];
            for (uint32_t n = 0; n < N; ++n)
                orow[n] += scale * t * (double)lora_b[(size_t)r * N + n];
        }
    }
}

/* fp32 LoRA delta with the shader's own accumulation order, hidden fixed at 64:
 * y[row][col] = sum_r (sum_k x[row][k]*a[k][r]) * b[r][col].
 * Follows vulkan-runtime/shaders/lora_delta.comp:10-21 (no alpha/rank inside;
 * the caller pre-scales B, python/spaceslug/backend.py:666). */
void oq4_lora_delta_f32(const float* x, const float* a, const float* b, float* y,
                        uint32_t m, uint32_t rank) {
    for (uint32_t id = 0; id < m * 64u; ++id) {
        uint32_t row = id / 64u, column = id % 64u;
        float value = 0.0f;
        for (uint32_t r = 0; r < rank; ++r) {
            float reduced = 0.0f;
            for (uint32_t k = 0; k < 64u; ++k) reduced += x[row * 64u + k] * a[k * rank + r];
            value += reduced * b[r * 64u + column];
        }
        y[id] = value;
    }
}

/* vector add of the existing runtime ABI (native/runtime_abi.cpp:3-7). */
int oq4_vector_add(const float* left, const float* right, float* output, size_t count) {
    if (!left || !right || !output) return 1;
    for (size_t i = 0; i < count; ++i) output[i] = left[i] + right[i];
    return 0;
}
