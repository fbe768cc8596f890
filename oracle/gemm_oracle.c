/*
 * CPU oracle for the GEMM hot path, plain C (TEST INFRASTRUCTURE ONLY).
 *
 * This file is a second, independent restatement of the reference's numerical
 * contract (chudinovAI/matrix-multiplication, src/precision.py), used by the
 * test suite to cross-check the numpy oracle in precision_oracle.py.  It is
 * never linked into the product library and the product never calls it.
 *
 *   oracle_quantize      -- src/precision.py:53-76  (RNE to TF32/BF16 by integer
 *                           rounding of the FP32 bit pattern; FP16 by IEEE RNE
 *                           with subnormals; ties-away option for TF32;
 *                           infinities/NaNs pass through unchanged)
 *   oracle_gemm_rows     -- src/precision.py:79-86  (FP64 product of the rounded
 *                           inputs, restricted to a list of output rows)
 *   oracle_verify_rows   -- src/precision.py:99-161 (gamma_K bound with
 *                           u = 2^-23, atol = rtol = 5e-4; returns the largest
 *                           tolerance ratio)
 *
 * Build: oracle/Makefile (target "oracle") -> oracle/_lib/liboracle.so.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

enum { ORACLE_FP32 = 0, ORACLE_TF32 = 1, ORACLE_FP16 = 2, ORACLE_BF16 = 3 };

static uint32_t bits_of(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static float float_of(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }

/* Round an FP32 value to the nearest FP16 value (ties to even) and return it
 * widened back to FP32.  Overflow gives +-inf, underflow keeps subnormals. */
static float round_to_half(float x)
{
    uint32_t u = bits_of(x);
    uint32_t sign = u & 0x80000000u;
    uint32_t mag = u & 0x7fffffffu;
    if (mag >= 0x7f800000u)                 /* inf / nan unchanged */
        return x;
    double v = fabs((double)x);
    /* FP16: 10 fraction bits, min normal 2^-14, subnormal step 2^-24, max 65504 */
    double step;
    int e;
    frexp(v, &e);                           /* v = f * 2^e, f in [0.5,1) */
    if (v == 0.0)
        return x;
    if (e - 1 < -14)
        step = ldexp(1.0, -24);
    else
        step = ldexp(1.0, e - 1 - 10);
    double q = v / step;
    double fl = floor(q);
    double rem = q - fl;
    double r;
    if (rem > 0.5) r = fl + 1;
    else if (rem < 0.5) r = fl;
    else r = fmod(fl, 2.0) == 0.0 ? fl : fl + 1;
    double out = r * step;
    /* 65520 is the midpoint between 65504 and 65536 (the first overflow value) */
    if (out > 65504.0)
        out = INFINITY;
    float f = (float)out;
    return float_of(bits_of(f) | sign);
}

void oracle_quantize(const float *in, float *out, size_t count, int precision, int ties_away)
{
    for (size_t i = 0; i < count; ++i) {
        float x = in[i];
        uint32_t u = bits_of(x);
        if (precision == ORACLE_FP32 || (u & 0x7f800000u) == 0x7f800000u) {
            out[i] = x;
            continue;
        }
        if (precision == ORACLE_FP16) {
            out[i] = round_to_half(x);
            continue;
        }
        unsigned dropped = precision == ORACLE_TF32 ? 13u : 16u;
        uint64_t half = 1ull << (dropped - 1);
        uint64_t add = ties_away ? half : half - 1 + ((u >> dropped) & 1u);
        uint64_t r = ((uint64_t)u + add) & (0xffffffffull & ~((1ull << dropped) - 1));
        out[i] = float_of((uint32_t)r);
    }
}

/* out[r*n + j] = sum_k qa[rows[r]*k + kk] * qb[kk*n + j] in FP64, where qa/qb are
 * the rounded inputs (already quantized by the caller). */
void oracle_gemm_rows(const float *qa, const float *qb, double *out, const int64_t *rows,
                      int64_t row_count, int64_t k, int64_t n)
{
    for (int64_t r = 0; r < row_count; ++r) {
        double *dst = out + r * n;
        for (int64_t j = 0; j < n; ++j)
            dst[j] = 0.0;
        const float *arow = qa + rows[r] * k;
        for (int64_t kk = 0; kk < k; ++kk) {
            double av = (double)arow[kk];
            const float *brow = qb + kk * n;
            for (int64_t j = 0; j < n; ++j)
                dst[j] += av * (double)brow[j];
        }
    }
}

/* Largest |actual - ref| / (atol + rtol*|ref| + gamma_K * (|A||B|)) over the
 * given rows; actual holds the full M x N FP32 output. */
double oracle_verify_rows(const float *qa, const float *qb, const float *actual,
                          const int64_t *rows, int64_t row_count, int64_t k, int64_t n)
{
    const double u = ldexp(1.0, -23);
    const double ku = (double)k * u;
    const double g = ku < 1.0 ? ku / (1.0 - ku) : expm1((double)k * log1p(u));
    double worst = 0.0;
    for (int64_t r = 0; r < row_count; ++r) {
        const float *arow = qa + rows[r] * k;
        for (int64_t j = 0; j < n; ++j) {
            double ref = 0.0, mag = 0.0;
            for (int64_t kk = 0; kk < k; ++kk) {
                double av = (double)arow[kk], bv = (double)qb[kk * n + j];
                ref += av * bv;
                mag += fabs(av) * fabs(bv);
            }
            double got = (double)actual[rows[r] * n + j];
            if (!isfinite(got))
                return INFINITY;
            double ratio = fabs(got - ref) / (5e-4 + 5e-4 * fabs(ref) + g * mag);
            if (ratio > worst)
                worst = ratio;
        }
    }
    return worst;
}
