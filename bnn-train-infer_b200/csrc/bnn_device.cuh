// bnn_device.cuh - small device helpers shared by the W1A8 kernels.
//
// Everything FP32 here is written with explicit round-to-nearest intrinsics
// (__fmul_rn/__fadd_rn/__fdiv_rn) so no multiply-add is ever contracted,
// matching the reference's "-ffp-contract=off, volatile per-op rounding"
// rule (bnn-accelerator/soft-bnn-accelerator.c:123-140). The library is
// compiled without fast-math and with -ftz=false, so subnormals survive.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace bnn {

constexpr uint32_t kGroup = 128;        // weights per binary16 scale
constexpr uint32_t kRowBlock = 8;       // output rows per repacked weight block
constexpr uint32_t kWordsPerGroup = 32; // sliced activation words per group
constexpr uint32_t kActStride = 36;     // smem words per group (144 B: bank spread)

// binary16 bit pattern -> binary32. cvt.f32.f16 is exact for every binary16
// value including subnormals and signed zero (HalfToFloat, soft :92-121).
__device__ __forceinline__ float h2f(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

// d = c + sum_i a.u8[i] * b.s8[i]: unsigned weight-mask bytes times signed
// activation bytes, exact in int32.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ float load_f32_any(const unsigned char* p) {
    if ((reinterpret_cast<uintptr_t>(p) & 3u) == 0)
        return *reinterpret_cast<const float*>(p);
    uint32_t v = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) |
                 ((uint32_t)p[3] << 24);
    return __uint_as_float(v);
}

__device__ __forceinline__ void store_f32_any(unsigned char* p, float f) {
    if ((reinterpret_cast<uintptr_t>(p) & 3u) == 0) {
        *reinterpret_cast<float*>(p) = f;
        return;
    }
    uint32_t v = __float_as_uint(f);
    p[0] = (unsigned char)v;
    p[1] = (unsigned char)(v >> 8);
    p[2] = (unsigned char)(v >> 16);
    p[3] = (unsigned char)(v >> 24);
}

__device__ __forceinline__ void store_i16_any(unsigned char* p, int16_t x) {
    if ((reinterpret_cast<uintptr_t>(p) & 1u) == 0) {
        *reinterpret_cast<int16_t*>(p) = x;
        return;
    }
    uint16_t v = (uint16_t)x;
    p[0] = (unsigned char)v;
    p[1] = (unsigned char)(v >> 8);
}

// Programmatic dependent launch. launch_dependents lets the next kernel of
// the stream be scheduled as soon as every CTA of this one has started;
// wait blocks until the preceding kernel has completed and its writes are
// visible. Both are no-ops for kernels launched without the PDL attribute.
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Smallest positive binary32 subnormal (FLT_TRUE_MIN).
__device__ __forceinline__ float flt_true_min() { return __uint_as_float(1u); }

// Row scale of the full-row absmax quantiser (QuantizeRow, soft :187-195).
__device__ __forceinline__ float row_scale_from_absmax(float absmax) {
    if (absmax == 0.0f)
        return 1.0f;
    float s = __fdiv_rn(absmax, 127.0f);
    return s == 0.0f ? flt_true_min() : s;
}

// One element of QuantizeRow (soft :197-208): RN division, round half away
// from zero, clamp to [-127, 127].
__device__ __forceinline__ int8_t quantize_one(float x, float s) {
    float r = roundf(__fdiv_rn(x, s));
    r = fminf(fmaxf(r, -127.0f), 127.0f);
    return (int8_t)(int)r;
}

// The same, kept out of line: the rare exact path of RowQuantizer.
static __device__ __noinline__ int8_t quantize_one_slow(float x, float s) { return quantize_one(x, s); }

// Quantiser for one row with a known scale s, exactly equal to quantize_one
// but without a division per element in the common case.
// y = fl(x * fl(1/s)) differs from fl(x/s) by less than 2e-5 when |x/s| <= 127
// (two RN steps of relative error 2^-24 on a value below 128, plus half an
// ulp of fl(x/s) there); round() of the two can only differ if a half-integer
// lies within that distance of y, which the test below excludes, falling back
// to the exact division. Scales below 2^-125 (whose reciprocal overflows)
// always take the exact path.
struct RowQuantizer {
    float s, rcp;
    bool exact_only;
    __device__ __forceinline__ explicit RowQuantizer(float scale) : s(scale) {
        exact_only = !(scale >= 0x1p-125f);
        rcp = exact_only ? 0.0f : __frcp_rn(scale);
    }
    __device__ __forceinline__ int8_t operator()(float x) const {
        if (!exact_only) {
            const float y = __fmul_rn(x, rcp);
            // t = fl(1.5 * 2^23 + y) holds RNE(y) as an integer (|y| < 2^22);
            // y - RNE(y) is exact. Away from half-integers RNE equals the
            // reference's round-half-away-from-zero.
            const float t = __fadd_rn(y, 12582912.0f);
            const float r = __fsub_rn(t, 12582912.0f);
            if (fabsf(__fsub_rn(y, r)) < 0.49997f) {  // farther than 3e-5 from a half-integer
                const int v = (int)(__float_as_uint(t) - 0x4b400000u);
                return (int8_t)min(max(v, -127), 127);
            }
        }
        return quantize_one_slow(x, s);
    }
};

// x / d correctly rounded, given rd = RN(1/d) (one reciprocal per divisor):
// q = RN(x * rd) is within an ulp of x / d, so r = x - q d is exact by FMA,
// and q1 = RN(q + r rd) is Markstein's corrected quotient (P. Markstein,
// "IA-64 and Elementary Functions", 2000). q1 is then PROVED correct here:
// its own remainder r1 = x - q1 d (exact by FMA whenever q1 is faithful) must
// be below half the spacing of floats around q1, times |d| (a quarter ulp at
// a power of two, where the spacing below halves); binary division has no
// exact ties. Operands outside [2^-40, 2^40] (divisor) or quotients outside
// [2^-60, 2^60], where those scalings could leave the normal range, and any
// failed proof take __fdiv_rn. The result always equals __fdiv_rn(x, d).
__device__ __forceinline__ float div_cr(float x, float d, float rd) {
    const float q = __fmul_rn(x, rd);
    const float r = __fmaf_rn(-q, d, x);
    const float q1 = __fmaf_rn(r, rd, q);
    const float r1 = __fmaf_rn(-q1, d, x);
    const uint32_t qb = __float_as_uint(q1);
    const uint32_t eq = (qb >> 23) & 0xffu;
    const uint32_t ed = (__float_as_uint(d) >> 23) & 0xffu;
    const uint32_t down = (qb & 0x7fffffu) == 0 ? 1u : 0u;  // a power of two: the spacing below is half
    const float bound = __fmul_rn(fabsf(d), __uint_as_float((eq - 24u - down) << 23));
    if (eq >= 127u - 60u && eq <= 127u + 60u && ed >= 127u - 40u && ed <= 127u + 40u && fabsf(r1) < bound)
        return q1;
    return __fdiv_rn(x, d);
}

// Correctly rounded binary32 exp: the double-precision exp rounded once to
// float. (glibc's expf, which the reference links, is faithfully but not
// correctly rounded: it differs from this on about 0.004% of inputs.)
__device__ __forceinline__ float expf_cr(float x) { return __double2float_rn(exp((double)x)); }

// Pack four activation bytes for one (group, word t, bit slice j): byte i is
// q[32t + 8i + j] of the group, the activation that meets bit (8i + j) of the
// group's 32-bit weight word t.
__device__ __forceinline__ uint32_t pack_slice(const int8_t* qg, uint32_t t, uint32_t j) {
    const int8_t* b = qg + 32u * t + j;
    return (uint32_t)(uint8_t)b[0] | ((uint32_t)(uint8_t)b[8] << 8) |
           ((uint32_t)(uint8_t)b[16] << 16) | ((uint32_t)(uint8_t)b[24] << 24);
}

}  // namespace bnn
