/*
 * bnn_oracle.c - CPU restatement of the reference W1A8 contraction.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker that the B200 kernels
 * are compared against; only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg may load it. The product path never calls it.
 *
 * It restates, function by function, the arithmetic of the reference soft
 * backend (bnn-accelerator/soft-bnn-accelerator.c) so that results are
 * bit-identical:
 *   oracle_half_to_float  <- HalfToFloat           soft-bnn-accelerator.c:92-121
 *   oracle_quantize_row   <- QuantizeRow           soft-bnn-accelerator.c:175-211
 *   oracle_compute_rows   <- ComputeRow            soft-bnn-accelerator.c:219-276
 *   oracle_validate_f32   <- ValidateF32Input      soft-bnn-accelerator.c:294-308
 *   oracle_validate_i8    <- ValidateI8Input       soft-bnn-accelerator.c:278-292
 * Every output element is independent, so the loop over output channels is
 * split across OpenMP threads without changing any rounding.
 *
 * Pinned against the reference's golden vectors (bnn-hw-v2/simple_test/
 * tests/case/golden_*.hex) and against the compiled soft backend by
 * tests/test_oracle.py.
 *
 * Build: oracle/Makefile (gcc -O2 -std=c11 -fno-fast-math -ffp-contract=off).
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef __FAST_MATH__
#error "the oracle must be compiled without fast-math"
#endif

#define ORACLE_GROUP 128u

/* binary16 bit pattern -> binary32, subnormals kept (soft :92-121). */
float oracle_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t mant = h & 0x03ffu;
    int exp = (int)((h >> 10) & 0x1fu);
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            /* normalise the subnormal: shift until the implicit bit appears */
            int e = 1;
            while ((mant & 0x0400u) == 0) {
                mant <<= 1;
                --e;
            }
            bits = sign | ((uint32_t)(e + 112) << 23) | ((mant & 0x03ffu) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else {
        bits = sign | ((uint32_t)(exp + 112) << 23) | (mant << 13);
    }
    float out;
    memcpy(&out, &bits, sizeof out);
    return out;
}

/* Full-row absmax int8 quantisation (soft :175-211). Returns the row scale. */
float oracle_quantize_row(const float* x, uint32_t count, int8_t* q) {
    float absmax = 0.0f;
    for (uint32_t i = 0; i < count; ++i) {
        float a = fabsf(x[i]);
        if (a > absmax)
            absmax = a;
    }
    float s;
    if (absmax == 0.0f) {
        s = 1.0f;
    } else {
        s = absmax / 127.0f;
        if (s == 0.0f)
            s = FLT_TRUE_MIN;
    }
    for (uint32_t i = 0; i < count; ++i) {
        float r = roundf(x[i] / s); /* half away from zero */
        if (r > 127.0f)
            r = 127.0f;
        else if (r < -127.0f)
            r = -127.0f;
        q[i] = (int8_t)r;
    }
    return s;
}

/* 1 if every value is finite (soft :294-308). */
int oracle_validate_f32(const float* x, uint64_t count) {
    for (uint64_t i = 0; i < count; ++i)
        if (!isfinite(x[i]))
            return 0;
    return 1;
}

/* 1 if no value is -128 (soft :278-292). */
int oracle_validate_i8(const int8_t* x, uint64_t count) {
    for (uint64_t i = 0; i < count; ++i)
        if (x[i] == INT8_MIN)
            return 0;
    return 1;
}

/*
 * Contraction of M quantised rows against one W1 matrix (soft :219-276).
 *   mode 0: DOT_GROUPS, out is int16 [M][N][K/128]
 *   mode 1: scaled, out is float [M][N]; row_scale == NULL returns Z
 *           (I8 GEMV/GEMM), otherwise Y = fl(Z * row_scale[m]) (F32 ops).
 * bits: [N][K/8]; scales: [N][K/128] binary16 patterns; q: [M][K].
 */
void oracle_compute_rows(uint32_t k, uint32_t n, uint32_t m_rows, const uint8_t* bits,
                         const uint16_t* scales, const int8_t* q, const float* row_scale,
                         int mode, void* out) {
    const uint32_t groups = k / ORACLE_GROUP;
    const size_t row_bytes = k / 8u;
    for (uint32_t m = 0; m < m_rows; ++m) {
        const int8_t* x = q + (size_t)m * k;
        int32_t totals[1024];
        for (uint32_t g = 0; g < groups; ++g) {
            int32_t t = 0;
            for (uint32_t i = g * ORACLE_GROUP; i < (g + 1) * ORACLE_GROUP; ++i)
                t += x[i];
            totals[g] = t;
        }
#pragma omp parallel for schedule(static)
        for (int64_t nn = 0; nn < (int64_t)n; ++nn) {
            const uint8_t* w = bits + (size_t)nn * row_bytes;
            float acc = 0.0f;
            for (uint32_t g = 0; g < groups; ++g) {
                int32_t pos = 0;
                for (uint32_t i = g * ORACLE_GROUP; i < (g + 1) * ORACLE_GROUP; ++i)
                    if ((w[i >> 3] >> (i & 7u)) & 1u)
                        pos += x[i];
                int32_t dot = 2 * pos - totals[g];
                size_t idx = (size_t)nn * groups + g;
                if (mode == 0) {
                    ((int16_t*)out)[(size_t)m * n * groups + idx] = (int16_t)dot;
                } else {
                    float term = oracle_half_to_float(scales[idx]) * (float)dot;
                    acc = acc + term;
                }
            }
            if (mode != 0) {
                float y = row_scale ? acc * row_scale[m] : acc;
                ((float*)out)[(size_t)m * n + (size_t)nn] = y;
            }
        }
    }
}

/* F32 job: quantise each row then contract (soft :589-600). q_out/s_out
 * receive the quantised rows and scales so tests can compare them too. */
void oracle_gemm_f32(uint32_t k, uint32_t n, uint32_t m_rows, const uint8_t* bits,
                     const uint16_t* scales, const float* x, int8_t* q_out, float* s_out,
                     float* y) {
    for (uint32_t m = 0; m < m_rows; ++m)
        s_out[m] = oracle_quantize_row(x + (size_t)m * k, k, q_out + (size_t)m * k);
    oracle_compute_rows(k, n, m_rows, bits, scales, q_out, s_out, 1, y);
}
