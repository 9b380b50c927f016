/* Oracle: plain-C restatement of lowbit's reference arithmetic.
 * TEST INFRASTRUCTURE ONLY: used by tests/ and bench.py's CPU-baseline leg as
 * the checker, never by the lowbit_b200 product. Built by oracle/Makefile into
 * oracle/_build/liblbref.so. Pinned against the golden vectors generated from
 * the reference (tests/test_oracle.py).
 *
 * GEMMs accumulate in double (the reference's numpy oracle is float64,
 * src/lowbit/reference.py:9-34); the activation quantizer and the group
 * accumulators are exact (src/lowbit/csrc/dispatch.c:231-257,
 * src/lowbit/csrc/kern_scalar.c:49-59,86-99). */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define G128 128
#define B32 32

static double e2m1_f64(unsigned c) {
    /* sign bit 3, exponent bits 2..1 (bias 1), mantissa bit 0 */
    const double sign = (c & 8u) ? -1.0 : 1.0;
    const unsigned ex = (c >> 1) & 3u, man = c & 1u;
    const double mag = ex == 0 ? 0.5 * man : ldexp(1.0 + 0.5 * man, (int)ex - 1);
    return sign * mag;
}

static double e8m0_f64(unsigned e) { return e == 255u ? NAN : ldexp(1.0, (int)e - 127); }

/* code of element k (0..Kp-1) of a packed row, for a block size `blk` */
static unsigned code_at(const uint8_t *row, int k, int blk) {
    const int b = k / blk, j = k % blk, half = blk / 2;
    const uint8_t byte = row[b * half + (j < half ? j : j - half)];
    return j < half ? (byte & 15u) : (byte >> 4);
}

void lbref_gemm_w4a16(const float *x, int M, int Kp, const uint8_t *qw, const float *scales,
                      const uint8_t *zeros, int N, double *y) {
    const int G = Kp / G128;
    for (int m = 0; m < M; m++)
        for (int n = 0; n < N; n++) {
            const uint8_t *row = qw + (size_t)n * (Kp / 2);
            double acc = 0.0;
            for (int k = 0; k < Kp; k++) {
                const int g = k / G128;
                const double z = zeros ? zeros[(size_t)n * G + g] : 8.0;
                /* (q - z) * s rounded to fp32, as the reference dequantizes */
                const float w = ((float)code_at(row, k, G128) - (float)z) * scales[(size_t)n * G + g];
                acc += (double)w * x[(size_t)m * Kp + k];
            }
            y[(size_t)m * N + n] = acc;
        }
}

void lbref_gemm_mxfp4(const float *x, int M, int Kp, const uint8_t *qw, const uint8_t *e8m0,
                      int N, double *y) {
    const int NB = Kp / B32;
    for (int m = 0; m < M; m++)
        for (int n = 0; n < N; n++) {
            const uint8_t *row = qw + (size_t)n * (Kp / 2);
            double acc = 0.0;
            for (int k = 0; k < Kp; k++)
                acc += e2m1_f64(code_at(row, k, B32)) * e8m0_f64(e8m0[(size_t)n * NB + k / B32]) *
                       x[(size_t)m * Kp + k];
            y[(size_t)m * N + n] = acc;
        }
}

/* bit-exact per-token int8 quantizer: fp32 division, round half to even */
void lbref_quant_act_int8(const float *x, int M, int Kp, int8_t *xq, float *xs, int32_t *asum) {
    const int G = Kp / G128;
    for (int m = 0; m < M; m++) {
        const float *r = x + (size_t)m * Kp;
        float amax = 0.0f;
        for (int k = 0; k < Kp; k++) {
            const float a = fabsf(r[k]);
            if (a > amax) amax = a;
        }
        const volatile float sc = amax > 0.0f ? amax / 127.0f : 1.0f;
        xs[m] = sc;
        for (int g = 0; g < G; g++) {
            int32_t s = 0;
            for (int k = g * G128; k < (g + 1) * G128; k++) {
                const volatile float v = r[k] / sc;
                float q = rintf(v);
                if (q > 127.0f) q = 127.0f;
                if (q < -127.0f) q = -127.0f;
                xq[(size_t)m * Kp + k] = (int8_t)q;
                s += (int8_t)q;
            }
            asum[(size_t)m * G + g] = s;
        }
    }
}

/* exact acc[m,n,g] = sum_{k in g} q*xq - z*asum[m,g] */
void lbref_w4a8_group_acc(const int8_t *xq, const int32_t *asum, int M, int Kp, const uint8_t *qw,
                          const uint8_t *zeros, int N, int32_t *out) {
    const int G = Kp / G128;
    for (int m = 0; m < M; m++)
        for (int n = 0; n < N; n++) {
            const uint8_t *row = qw + (size_t)n * (Kp / 2);
            for (int g = 0; g < G; g++) {
                int64_t acc = 0;
                for (int k = g * G128; k < (g + 1) * G128; k++)
                    acc += (int64_t)code_at(row, k, G128) * xq[(size_t)m * Kp + k];
                const int64_t z = zeros ? zeros[(size_t)n * G + g] : 8;
                out[((size_t)m * N + n) * G + g] = (int32_t)(acc - z * asum[(size_t)m * G + g]);
            }
        }
}
