// w1a8_prep.cuh - input pass of BNN_Execute.
//
//   w1a8_prep_kernel  validate one logical input row, quantise it (F32 ops)
//                     and re-slice it for the contraction
//                     (QuantizeRow/Validate*, soft-bnn-accelerator.c:175-211, 278-308)
// The contraction itself is w1a8_gemv_kernel (w1a8_gemv.cuh).
//
#pragma once

#include <cstdint>
#include <cfloat>
#include "bnn_device.cuh"
#include "w1a8_gemv.cuh"
#include "w1a8_mma.cuh"

namespace bnn {

enum InputKind : int { kInputI8 = 1, kInputF32 = 2 };

constexpr int kPrepThreads = 256;


struct PrepArgs {
    const unsigned char* in;  // first logical row (buffer base + view offset)
    size_t in_stride;         // bytes between rows
    int kind;                 // kInputI8 / kInputF32
    uint32_t k, m;
    uint32_t* act;            // [M][G][32] sliced words (dp4a path), or
    unsigned char* a_sw;      // non-null: pre-tiled rows for w1a8_mma_kernel instead
    uint32_t row0;            // row index of this launch's first row within a_sw
    int32_t* totals;          // [M][G]
    float* row_scale;         // [M]
    int* status;
};

// One CTA per logical input row. Shared memory: K floats + K int8.
static __global__ void __launch_bounds__(kPrepThreads) w1a8_prep_kernel(PrepArgs a) {
    extern __shared__ __align__(16) unsigned char prep_smem[];
    float* xs = reinterpret_cast<float*>(prep_smem);
    int8_t* qs = reinterpret_cast<int8_t*>(prep_smem + (size_t)a.k * sizeof(float));
    __shared__ int s_bad;
    __shared__ float s_red[kPrepThreads / 32];

    const uint32_t m = blockIdx.x;
    const uint32_t tid = threadIdx.x;
    const unsigned char* row = a.in + (size_t)m * a.in_stride;
    if (tid == 0)
        s_bad = 0;
    __syncthreads();

    int bad = 0;
    float scale = 0.0f;
    if (a.kind == kInputF32) {
        float amax = 0.0f;
        for (uint32_t k = tid; k < a.k; k += kPrepThreads) {
            float x = load_f32_any(row + (size_t)k * 4u);
            xs[k] = x;
            bad |= !isfinite(x);
            amax = fmaxf(amax, fabsf(x));  // max is order independent
        }
        for (int o = 16; o > 0; o >>= 1)
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if ((tid & 31) == 0)
            s_red[tid >> 5] = amax;
        if (bad)
            s_bad = 1;
        __syncthreads();
        if (s_bad) {
            if (tid == 0)
                atomicOr(a.status, kStatusBadInput);
            return;
        }
        amax = s_red[0];
        for (int w = 1; w < kPrepThreads / 32; ++w)
            amax = fmaxf(amax, s_red[w]);
        scale = row_scale_from_absmax(amax);
        const RowQuantizer quant(scale);
        for (uint32_t k = tid; k < a.k; k += kPrepThreads)
            qs[k] = quant(xs[k]);
    } else {
        for (uint32_t k = tid; k < a.k; k += kPrepThreads) {
            int8_t v = (int8_t)row[k];
            qs[k] = v;
            bad |= (v == INT8_MIN);
        }
        if (bad)
            s_bad = 1;
        __syncthreads();
        if (s_bad) {
            if (tid == 0)
                atomicOr(a.status, kStatusBadInput);
            return;
        }
    }
    __syncthreads();

    const uint32_t groups = a.k / kGroup;
    if (a.a_sw) {
        // tensor-core operand: 16-byte chunks into the 128B-swizzled row tiles
        for (uint32_t c = tid; c < groups * 8u; c += kPrepThreads) {
            const uint32_t g = c / 8u, j = c % 8u;
            *reinterpret_cast<uint4*>(a.a_sw + mma_a_offset(a.row0 + m, g, groups, j)) =
                *reinterpret_cast<const uint4*>(qs + g * kGroup + j * 16u);
        }
        if (tid == 0)
            a.row_scale[m] = scale;
        return;
    }
    uint32_t* act = a.act + (size_t)m * groups * kWordsPerGroup;
    for (uint32_t w = tid; w < groups * kWordsPerGroup; w += kPrepThreads) {
        uint32_t g = w / kWordsPerGroup, tj = w % kWordsPerGroup;
        act[w] = pack_slice(qs + g * kGroup, tj >> 3, tj & 7u);
    }
    // Per-group activation totals (soft :226-234), one warp per group.
    const uint32_t lane = tid & 31, warp = tid >> 5;
    for (uint32_t g = warp; g < groups; g += kPrepThreads / 32) {
        const int8_t* qg = qs + g * kGroup + lane * 4u;
        int t = (int)qg[0] + (int)qg[1] + (int)qg[2] + (int)qg[3];
        for (int o = 16; o > 0; o >>= 1)
            t += __shfl_xor_sync(0xffffffffu, t, o);
        if (lane == 0)
            a.totals[(size_t)m * groups + g] = t;
    }
    if (tid == 0)
        a.row_scale[m] = scale;
}

inline size_t prep_smem_bytes(uint32_t k) { return (size_t)k * 5u; }

}  // namespace bnn
