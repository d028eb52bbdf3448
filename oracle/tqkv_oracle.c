/*
 * tqkv_oracle.c — CPU restatement of the reference's INT8 KV decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the GPU kernels
 * are compared against; only the tests, the smoke check and bench.py's CPU
 * baseline leg may load it.  The product never calls it.
 *
 * Plain C99, IEEE-754 binary32/binary64 arithmetic (build without
 * -ffast-math), scalar loops.  Each function cites the reference code it
 * restates (paths relative to the reference project).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

/* ---- binary16 <-> binary32, from the IEEE-754 definitions ---- */

/* Exact value of a binary16 bit pattern. */
float oracle_half_to_float(uint16_t h) {
    const int sign = (h >> 15) & 1;
    const int exp = (h >> 10) & 0x1f;
    const int man = h & 0x3ff;
    float v;
    if (exp == 0) {
        v = ldexpf((float)man, -24); /* zero or subnormal: man * 2^-24 */
    } else if (exp == 31) {
        v = man ? NAN : INFINITY;
    } else {
        v = ldexpf((float)(man | 0x400), exp - 25); /* 1.man * 2^(exp-15) */
    }
    return sign ? -v : v;
}

/* binary32 -> binary16, round to nearest, ties to even (the conversion
 * __float2half / cvt.rn.f16.f32 performs; reference src/kv_compress.cu:87). */
uint16_t oracle_float_to_half(float f) {
    uint32_t bits;
    memcpy(&bits, &f, sizeof bits);
    const uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    if (isnan(f)) return (uint16_t)(sign | 0x7e00u);
    const float a = fabsf(f);
    if (a >= 65520.0f) return (uint16_t)(sign | 0x7c00u); /* halfway to 2^16 and above -> inf */
    if (a < 6.103515625e-05f) {                           /* below 2^-14: quantum 2^-24 */
        const double q = (double)a * 16777216.0;          /* exact */
        return (uint16_t)(sign | (uint16_t)rint(q));      /* rint: ties to even */
    }
    int e2;
    frexpf(a, &e2); /* a = frac * 2^e2, frac in [0.5, 1) */
    const int E = e2 - 1;
    const double q = ldexp((double)a, 10 - E); /* in [1024, 2048), exact */
    const uint32_t m = (uint32_t)rint(q);      /* 2048 carries into the exponent */
    return (uint16_t)(sign | (((uint32_t)(E + 15) << 10) + (m - 1024u)));
}

/* cvt.rni.s32.f32: round to nearest even, NaN -> 0, saturating. */
static int round_half_even_to_int(float t) {
    if (isnan(t)) return 0;
    if (t >= 2147483647.0f) return 2147483647;
    if (t <= -2147483648.0f) return (-2147483647 - 1);
    return (int)nearbyintf(t);
}

/* fmaxf as CUDA defines it: a NaN operand is ignored unless both are NaN. */
static float max_ignore_nan(float a, float b) {
    if (isnan(a)) return b;
    if (isnan(b)) return a;
    return a > b ? a : b;
}

/*
 * Kernel A rule (reference src/kv_compress.cu:41-95), IEEE arithmetic:
 *   m = max|x| over the block; s = m / 127.0f; s = 1 if s == 0;
 *   scale = fp16(s) (RNE); code = clamp(rni(x / s), -127, 127) with fp32 s.
 * x: binary16 [rows][D]; q: int8 [rows][D]; scales: binary16 [rows][D/bs].
 */
void oracle_kv_compress(const uint16_t* x, int8_t* q, uint16_t* scales, long long rows, int D,
                        int bs) {
    const int nsub = D / bs;
    for (long long r = 0; r < rows; ++r) {
        for (int b = 0; b < nsub; ++b) {
            const uint16_t* xb = x + r * D + (long long)b * bs;
            float m = fabsf(oracle_half_to_float(xb[0]));
            for (int i = 1; i < bs; ++i) m = max_ignore_nan(m, fabsf(oracle_half_to_float(xb[i])));
            volatile float s = m / 127.0f;
            if (s == 0.0f) s = 1.0f;
            scales[r * nsub + b] = oracle_float_to_half(s);
            for (int i = 0; i < bs; ++i) {
                volatile float t = oracle_half_to_float(xb[i]) / s;
                int qi = round_half_even_to_int(t);
                if (qi > 127) qi = 127;
                if (qi < -127) qi = -127;
                q[r * D + (long long)b * bs + i] = (int8_t)qi;
            }
        }
    }
}

/*
 * Marks the "tie class" of Kernel A: elements whose exact quotient
 * 127 * x / m is a half-integer (254 * x / m an odd integer).  Only there can
 * two division implementations that are each within 2 ulp of x / s round to
 * different codes: for every other element the exact quotient lies farther
 * from a rounding boundary than those errors can reach (the distance is at
 * least |x/s| / (254 * 2047), the errors at most |x/s| * 3e-7), and the fp16
 * scales never differ (m / 127 stays at least 1/254 of an fp16 ulp away from
 * an fp16 rounding midpoint).  Returns the number of marked elements.
 */
long long oracle_kv_tie_mask(const uint16_t* x, uint8_t* mask, long long rows, int D, int bs) {
    const int nsub = D / bs;
    long long n = 0;
    for (long long r = 0; r < rows; ++r) {
        for (int b = 0; b < nsub; ++b) {
            const uint16_t* xb = x + r * D + (long long)b * bs;
            uint8_t* mb = mask + r * D + (long long)b * bs;
            float m = fabsf(oracle_half_to_float(xb[0]));
            for (int i = 1; i < bs; ++i) m = max_ignore_nan(m, fabsf(oracle_half_to_float(xb[i])));
            for (int i = 0; i < bs; ++i) {
                mb[i] = 0;
                if (!(m > 0.0f) || isinf(m)) continue;
                const double xv = (double)oracle_half_to_float(xb[i]);
                if (!isfinite(xv)) continue;
                const double t = 254.0 * xv / (double)m; /* exact when it is an integer */
                if (t == floor(t) && fmod(fabs(t), 2.0) == 1.0) {
                    mb[i] = 1;
                    ++n;
                }
            }
        }
    }
    return n;
}

/* Kernel B (reference src/kv_reconstruct.cu:30-33): fp16(float(code) * float(scale)). */
void oracle_kv_reconstruct(const int8_t* q, const uint16_t* scales, uint16_t* y, long long rows,
                           int D, int bs) {
    const int nsub = D / bs;
    for (long long r = 0; r < rows; ++r)
        for (int d = 0; d < D; ++d) {
            const float s = oracle_half_to_float(scales[r * nsub + d / bs]);
            y[r * D + d] = oracle_float_to_half((float)q[r * D + d] * s);
        }
}

/* The dequantised K/V the reference's Python check feeds to its attention
 * (python/check_correctness.py:47-56): fp16(float32(code) * float32(scale)),
 * returned as float. */
void oracle_dequantize_f32(const int8_t* q, const uint16_t* scales, float* out, long long rows,
                           int D, int bs) {
    const int nsub = D / bs;
    for (long long r = 0; r < rows; ++r)
        for (int d = 0; d < D; ++d) {
            const float s = oracle_half_to_float(scales[r * nsub + d / bs]);
            out[r * D + d] = oracle_half_to_float(oracle_float_to_half((float)q[r * D + d] * s));
        }
}

void oracle_half_array_to_float(const uint16_t* h, float* f, long long n) {
    for (long long i = 0; i < n; ++i) f[i] = oracle_half_to_float(h[i]);
}

void oracle_float_array_to_half(const float* f, uint16_t* h, long long n) {
    for (long long i = 0; i < n; ++i) h[i] = oracle_float_to_half(f[i]);
}

/*
 * Decode attention (python/check_correctness.py:38-44):
 *   scores = (q . k_t) / sqrt(D); p = softmax(scores); out = sum_t p_t v_t
 * evaluated in binary64 (the reference evaluates it in fp32; binary64 is the
 * more exact restatement of the same function).
 *   q [BH][D], k, v [BH][S][D] (float), out [BH][D] (double precision result
 * rounded to float).  S == 0 gives NaN (0 / 0).
 */
void oracle_attention(const float* q, const float* k, const float* v, float* out, long long BH,
                      int S, int D) {
    const double scale = 1.0 / sqrt((double)D);
    for (long long h = 0; h < BH; ++h) {
        const float* qh = q + h * D;
        const float* kh = k + h * (long long)S * D;
        const float* vh = v + h * (long long)S * D;
        double m = -INFINITY;
        /* pass 1: max score */
        for (int t = 0; t < S; ++t) {
            double s = 0.0;
            for (int d = 0; d < D; ++d) s += (double)qh[d] * (double)kh[(long long)t * D + d];
            s *= scale;
            if (s > m) m = s;
        }
        double l = 0.0;
        double acc[128];
        for (int d = 0; d < D; ++d) acc[d] = 0.0;
        for (int t = 0; t < S; ++t) {
            double s = 0.0;
            for (int d = 0; d < D; ++d) s += (double)qh[d] * (double)kh[(long long)t * D + d];
            const double p = exp(s * scale - m);
            l += p;
            for (int d = 0; d < D; ++d) acc[d] += p * (double)vh[(long long)t * D + d];
        }
        for (int d = 0; d < D; ++d) out[h * D + d] = (float)(acc[d] / l);
    }
}

/*
 * Split-S partial record of one slice (the format of tqkv_decode_int8_partial):
 * rec[0..D-1] = sum_t exp(s_t - m) v_t, rec[D] = m, rec[D+1] = sum_t exp(s_t - m),
 * natural-log units; an empty slice gives m = -inf, l = 0, acc = 0.
 */
void oracle_attention_partial(const float* q, const float* k, const float* v, double* rec,
                              long long BH, int S, int D) {
    const double scale = 1.0 / sqrt((double)D);
    for (long long h = 0; h < BH; ++h) {
        const float* qh = q + h * D;
        const float* kh = k + h * (long long)S * D;
        const float* vh = v + h * (long long)S * D;
        double* rh = rec + h * (D + 2);
        double m = -INFINITY;
        for (int t = 0; t < S; ++t) {
            double s = 0.0;
            for (int d = 0; d < D; ++d) s += (double)qh[d] * (double)kh[(long long)t * D + d];
            s *= scale;
            if (s > m) m = s;
        }
        double l = 0.0;
        for (int d = 0; d < D; ++d) rh[d] = 0.0;
        for (int t = 0; t < S; ++t) {
            double s = 0.0;
            for (int d = 0; d < D; ++d) s += (double)qh[d] * (double)kh[(long long)t * D + d];
            const double p = exp(s * scale - m);
            l += p;
            for (int d = 0; d < D; ++d) rh[d] += p * (double)vh[(long long)t * D + d];
        }
        rh[D] = m;
        rh[D + 1] = l;
    }
}
