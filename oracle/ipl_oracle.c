/*
 * CPU oracle (TEST INFRASTRUCTURE ONLY: used by tests/, the smoke check and the CPU-baseline leg
 * of bench.py as the checker; never by the product path).
 *
 * Plain-C restatement of the reference's fp32 oracle,
 * src/inference_performance_lab/kernels/reference.py of sreeganeshji/inference-performance-lab:
 *
 *   fused_add_rms_norm_reference (reference.py:7-23):
 *     residual_out_fp32 = x.float() + residual.float()                       (:18)
 *     inverse_rms = rsqrt(residual_out_fp32.square().mean(-1) + epsilon)     (:19)
 *     output = residual_out_fp32 * inverse_rms * weight.float()              (:21)
 *     return output.to(bf16), residual_out_fp32.to(bf16)                     (:23)
 *
 *   plain RMSNorm (no counterpart in the reference; its arithmetic with no residual term):
 *     v = x.float(); output = v * rsqrt(v.square().mean(-1) + epsilon) * weight.float()
 *
 *   silu_and_mul_reference (reference.py:26-35):
 *     gate, up = x.float().chunk(2, -1); output = silu(gate) * up; output.to(bf16)  (:32-35)
 *
 * Rounding: every fp32 operation rounds to nearest (compile with -ffp-contract=off so no FMA
 * contraction changes a product). bf16 narrowing is round-to-nearest-even with NaN -> 0x7FC0,
 * as c10::BFloat16 does. The mean of squares is accumulated in double and rounded once to fp32,
 * which is at least as accurate as torch's fp32 cascade sum; the normalised output can therefore
 * differ from torch's by one bf16 ulp in rare elements (within the tests' tolerance), while the
 * residual output is exact.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline float bf16_to_f32(uint16_t bits) {
    uint32_t u = (uint32_t)bits << 16;
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

static inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, sizeof u);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)0x7fc0u;
    const uint32_t bias = 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)((u + bias) >> 16);
}

/* fp32 -> OCP e4m3 (E4M3FN: sign, 4 exponent bits with bias 7, 3 mantissa bits, max 448, no
 * infinities, NaN = S.1111.111), round to nearest even, saturating to +-448; NaN -> 0x7F.
 * Written from the format definition: q = rne(|f| * 2^(3 - e)) for the binade 2^e of |f|
 * (q in [8, 16]), or rne(|f| * 2^9) below the smallest normal 2^-6, so that (E << 3) | M
 * follows from q with the subnormal/normal boundary falling out of the carry. */
static inline uint8_t f32_to_e4m3(float f) {
    if (isnan(f)) return 0x7Fu;
    const uint8_t sign = signbit(f) ? 0x80u : 0x00u;
    const float a = fabsf(f);
    if (a >= 448.0f) return (uint8_t)(sign | 0x7Eu);
    if (a < 0.015625f) { /* below 2^-6: subnormal grid of 2^-9 */
        const float q = nearbyintf(a * 512.0f); /* 0..8; 8 is the smallest normal (E = 1, M = 0) */
        return (uint8_t)(sign | (uint8_t)q);
    }
    int exponent;
    frexpf(a, &exponent); /* a = m * 2^exponent, m in [0.5, 1): binade e = exponent - 1 */
    int e = exponent - 1;
    float q = nearbyintf(ldexpf(a, 3 - e)); /* 8..16 */
    if (q >= 16.0f) {
        q = 8.0f;
        e += 1;
    }
    const int code = ((e + 7) << 3) | ((int)q - 8);
    return (uint8_t)(sign | (code > 0x7E ? 0x7E : code));
}

uint16_t oracle_f32_to_bf16(float f) { return f32_to_bf16(f); }
uint8_t oracle_f32_to_e4m3(float f) { return f32_to_e4m3(f); }
float oracle_bf16_to_f32(uint16_t b) { return bf16_to_f32(b); }

/* Returns 0, or -1 if the scratch row could not be allocated. */
int oracle_fused_add_rms_norm_bf16(const uint16_t* x, const uint16_t* residual, const uint16_t* weight,
                                   int64_t rows, int64_t hidden, double epsilon, uint16_t* out,
                                   uint16_t* residual_out) {
    if (rows <= 0 || hidden <= 0) return 0;
    float* v = (float*)malloc(sizeof(float) * (size_t)hidden);
    if (v == NULL) return -1;
    const float eps = (float)epsilon;
    for (int64_t r = 0; r < rows; ++r) {
        const uint16_t* xr = x + r * hidden;
        const uint16_t* rr = residual + r * hidden;
        double acc = 0.0;
        for (int64_t c = 0; c < hidden; ++c) {
            const float value = bf16_to_f32(xr[c]) + bf16_to_f32(rr[c]);
            const float square = value * value;
            v[c] = value;
            residual_out[r * hidden + c] = f32_to_bf16(value);
            acc += (double)square;
        }
        const float mean = (float)(acc / (double)hidden);
        const float inverse_rms = 1.0f / sqrtf(mean + eps);
        for (int64_t c = 0; c < hidden; ++c) {
            const float scaled = v[c] * inverse_rms;
            out[r * hidden + c] = f32_to_bf16(scaled * bf16_to_f32(weight[c]));
        }
    }
    free(v);
    return 0;
}

/* add+RMSNorm with a static fp8 output: reference.py:18-21 up to the fp32 product, then
 * e4m3(product * (1 / scale)). residual_out as in oracle_fused_add_rms_norm_bf16. */
int oracle_fused_add_rms_norm_static_fp8_quant(const uint16_t* x, const uint16_t* residual, const uint16_t* weight,
                                               int64_t rows, int64_t hidden, double epsilon, float scale,
                                               uint8_t* out, uint16_t* residual_out) {
    if (rows <= 0 || hidden <= 0) return 0;
    float* v = (float*)malloc(sizeof(float) * (size_t)hidden);
    if (v == NULL) return -1;
    const float eps = (float)epsilon;
    const float scale_inv = 1.0f / scale;
    for (int64_t r = 0; r < rows; ++r) {
        double acc = 0.0;
        for (int64_t c = 0; c < hidden; ++c) {
            const float value = bf16_to_f32(x[r * hidden + c]) + bf16_to_f32(residual[r * hidden + c]);
            const float square = value * value;
            v[c] = value;
            residual_out[r * hidden + c] = f32_to_bf16(value);
            acc += (double)square;
        }
        const float mean = (float)(acc / (double)hidden);
        const float inverse_rms = 1.0f / sqrtf(mean + eps);
        for (int64_t c = 0; c < hidden; ++c) {
            const float normed = (v[c] * inverse_rms) * bf16_to_f32(weight[c]);
            out[r * hidden + c] = f32_to_e4m3(normed * scale_inv);
        }
    }
    free(v);
    return 0;
}

/* Plain RMSNorm: reference.py:19-23 applied to x itself (no residual add, no residual output). */
int oracle_rms_norm_bf16(const uint16_t* x, const uint16_t* weight, int64_t rows, int64_t hidden, double epsilon,
                         uint16_t* out) {
    if (rows <= 0 || hidden <= 0) return 0;
    const float eps = (float)epsilon;
    for (int64_t r = 0; r < rows; ++r) {
        const uint16_t* xr = x + r * hidden;
        double acc = 0.0;
        for (int64_t c = 0; c < hidden; ++c) {
            const float value = bf16_to_f32(xr[c]);
            const float square = value * value;
            acc += (double)square;
        }
        const float mean = (float)(acc / (double)hidden);
        const float inverse_rms = 1.0f / sqrtf(mean + eps);
        for (int64_t c = 0; c < hidden; ++c) {
            const float scaled = bf16_to_f32(xr[c]) * inverse_rms;
            out[r * hidden + c] = f32_to_bf16(scaled * bf16_to_f32(weight[c]));
        }
    }
    return 0;
}

void oracle_silu_and_mul_bf16(const uint16_t* input, int64_t rows, int64_t intermediate, uint16_t* out) {
    for (int64_t r = 0; r < rows; ++r) {
        const uint16_t* gate = input + r * 2 * intermediate;
        const uint16_t* up = gate + intermediate;
        for (int64_t c = 0; c < intermediate; ++c) {
            const float g = bf16_to_f32(gate[c]);
            const float silu = g / (1.0f + expf(-g));
            out[r * intermediate + c] = f32_to_bf16(silu * bf16_to_f32(up[c]));
        }
    }
}
