// w1a8_kernels.cuh - the W1A8 hot path of BNN_Execute.
//
//   w1a8_prep_kernel      validate one logical input row, quantise it
//                         (F32 ops) and re-slice it for the contraction
//                         (QuantizeRow/Validate*, soft-bnn-accelerator.c:175-211, 278-308)
//   w1a8_contract_kernel  per (row, group): exact integer dot of +-1 weights
//                         with int8 activations, then the ordered FP32
//                         scale-accumulate (ComputeRow, soft :219-276)
//
// Device weight layout (written by BNN_MatrixCreate): blocks of 8 output
// rows; block b, group g, row r holds the 16 bytes of row 8b+r, group g:
//     wbits[((b * G + g) * 8 + r)]   (uint4)
// so a warp whose lanes are (r = lane % 8, g = 4q + lane / 8) reads 512
// contiguous bytes. Scales stay in the public [N][G] binary16 layout.
//
// Sliced activation layout (written by the prep kernel): for row m, group g,
// 32 words; word (t, j) = t * 8 + j packs q[g*128 + 32t + 8i + j], i = 0..3.
// Masking weight word t with (0x01010101 << j) leaves, in byte i, bit
// (8i + j) of that word scaled by 2^j; dp4a with word (t, j) therefore sums
// 2^j * q over the four weights whose bit is set. Eight such partial sums
// (one per j, kept apart) give pos = sum_j acc_j >> j exactly, and the group
// dot is D = 2 * pos - total (soft :251-258).
#pragma once

#include <cstdint>
#include <cfloat>
#include "bnn_device.cuh"

namespace bnn {

enum InputKind : int { kInputI8 = 1, kInputF32 = 2 };

constexpr int kPrepThreads = 256;
constexpr int kContractThreads = 128;
constexpr int kRowsPerCta = 8;  // activation rows per contraction CTA

// Status bits written by the prep kernel.
constexpr int kStatusBadInput = 1;

struct PrepArgs {
    const unsigned char* in;  // first logical row (buffer base + view offset)
    size_t in_stride;         // bytes between rows
    int kind;                 // kInputI8 / kInputF32
    uint32_t k, m;
    uint32_t* act;            // [M][G][32]
    int32_t* totals;          // [M][G]
    float* row_scale;         // [M]
    int* status;
};

// One CTA per logical input row. Shared memory: K floats + K int8.
__global__ void __launch_bounds__(kPrepThreads) w1a8_prep_kernel(PrepArgs a) {
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
        for (uint32_t k = tid; k < a.k; k += kPrepThreads)
            qs[k] = quantize_one(xs[k], scale);
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

struct ContractArgs {
    const uint4* wbits;       // repacked weight blocks
    const uint16_t* scales;   // [N][G] binary16
    const uint32_t* act;      // [M][G][32]
    const int32_t* totals;    // [M][G]
    const float* row_scale;   // [M] (F32 ops) or nullptr (I8 ops return Z)
    const int* status;        // non-zero: a prep CTA rejected its row
    uint32_t n, groups, m;
    unsigned char* out;       // first logical output row (buffer base + view offset)
    size_t out_stride;
};

// Integer part for one (row, group) unit: returns D for activation row mm.
__device__ __forceinline__ int group_dot(const uint32_t (&mk)[32], const uint32_t* act_s,
                                         int total) {
    int acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
        acc[j] = 0;
    const uint4* a4 = reinterpret_cast<const uint4*>(act_s);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        uint4 lo = a4[t * 2], hi = a4[t * 2 + 1];
        acc[0] = dp4a_us(mk[t * 8 + 0], lo.x, acc[0]);
        acc[1] = dp4a_us(mk[t * 8 + 1], lo.y, acc[1]);
        acc[2] = dp4a_us(mk[t * 8 + 2], lo.z, acc[2]);
        acc[3] = dp4a_us(mk[t * 8 + 3], lo.w, acc[3]);
        acc[4] = dp4a_us(mk[t * 8 + 4], hi.x, acc[4]);
        acc[5] = dp4a_us(mk[t * 8 + 5], hi.y, acc[5]);
        acc[6] = dp4a_us(mk[t * 8 + 6], hi.z, acc[6]);
        acc[7] = dp4a_us(mk[t * 8 + 7], hi.w, acc[7]);
    }
    int pos = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j)
        pos += acc[j] >> j;  // acc[j] is an exact multiple of 2^j
    return 2 * pos - total;
}

// MODE 0: DOT_GROUPS (int16 [M][N][G]); MODE 1: scaled FP32 [M][N].
// Grid: x = 8-row weight blocks, y = chunks of kRowsPerCta activation rows.
template <int MODE>
__global__ void __launch_bounds__(kContractThreads) w1a8_contract_kernel(ContractArgs a) {
    if (*a.status != 0)
        return;  // a rejected input leaves the output untouched
    extern __shared__ __align__(16) unsigned char c_smem[];
    const uint32_t G = a.groups;
    uint32_t* act_s = reinterpret_cast<uint32_t*>(c_smem);                    // [8][G][36]
    int32_t* tot_s = reinterpret_cast<int32_t*>(act_s + kRowsPerCta * G * kActStride);  // [8][G]
    int32_t* d_s = tot_s + kRowsPerCta * G;                                   // [8][8][G]

    const uint32_t blk = blockIdx.x;
    const uint32_t m0 = blockIdx.y * kRowsPerCta;
    const uint32_t mrows = min((uint32_t)kRowsPerCta, a.m - m0);
    const uint32_t tid = threadIdx.x;

    // Stage this CTA's activation rows (sliced words) and group totals.
    for (uint32_t i = tid; i < mrows * G * (kWordsPerGroup / 4); i += kContractThreads) {
        uint32_t mm = i / (G * 8), rest = i % (G * 8), g = rest / 8, c = rest % 8;
        const uint4* src = reinterpret_cast<const uint4*>(a.act + ((size_t)(m0 + mm) * G + g) * kWordsPerGroup);
        reinterpret_cast<uint4*>(act_s + (mm * G + g) * kActStride)[c] = src[c];
    }
    for (uint32_t i = tid; i < mrows * G; i += kContractThreads)
        tot_s[i] = a.totals[(size_t)m0 * G + i];
    __syncthreads();

    const uint32_t lane = tid & 31, warp = tid >> 5;
    const uint32_t r = lane & 7;
    const uint32_t n = blk * kRowBlock + r;
    for (uint32_t q = warp; q * 4 < G; q += kContractThreads / 32) {
        const uint32_t g = q * 4 + (lane >> 3);
        if (g >= G)
            continue;
        const uint4 w = a.wbits[((size_t)blk * G + g) * kRowBlock + r];
        uint32_t mk[32];
        const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int t = 0; t < 4; ++t)
#pragma unroll
            for (int j = 0; j < 8; ++j)
                mk[t * 8 + j] = words[t] & (0x01010101u << j);
        for (uint32_t mm = 0; mm < mrows; ++mm) {
            int d = group_dot(mk, act_s + (mm * G + g) * kActStride, tot_s[mm * G + g]);
            if (MODE == 0) {
                if (n < a.n)
                    store_i16_any(a.out + (size_t)(m0 + mm) * a.out_stride +
                                      ((size_t)n * G + g) * 2u,
                                  (int16_t)d);
            } else {
                d_s[(mm * kRowBlock + r) * G + g] = d;
            }
        }
    }
    if (MODE == 0)
        return;
    __syncthreads();
    // Ordered FP32 scale-accumulate, one thread per (activation row, output
    // row): acc = fl(acc + fl(F32(scale_g) * D_g)) for g ascending, then
    // Y = fl(acc * s) for F32 ops (soft :260-274).
    if (tid < mrows * kRowBlock) {
        const uint32_t mm = tid / kRowBlock, rr = tid % kRowBlock;
        const uint32_t nn = blk * kRowBlock + rr;
        if (nn < a.n) {
            const uint16_t* sc = a.scales + (size_t)nn * G;
            const int32_t* dd = d_s + (mm * kRowBlock + rr) * G;
            float acc = 0.0f;
            for (uint32_t g = 0; g < G; ++g)
                acc = __fadd_rn(acc, __fmul_rn(h2f(sc[g]), (float)dd[g]));
            if (a.row_scale)
                acc = __fmul_rn(acc, a.row_scale[m0 + mm]);
            store_f32_any(a.out + (size_t)(m0 + mm) * a.out_stride + (size_t)nn * 4u, acc);
        }
    }
}

// Repack the public [N][K/8] bit layout into 8-row blocks (see header).
// One thread per 16-byte (row, group) chunk; rows past N are zero.
__global__ void w1a8_repack_kernel(const uint8_t* __restrict__ bits, uint32_t n, uint32_t groups,
                                   uint4* __restrict__ out) {
    const size_t nblocks = (n + kRowBlock - 1) / kRowBlock;
    const size_t total = nblocks * groups * kRowBlock;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i % kRowBlock, g = (i / kRowBlock) % groups, b = i / (kRowBlock * groups);
        const size_t row = b * kRowBlock + r;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (row < n) {
            const uint8_t* src = bits + row * (groups * 16u) + g * 16u;
            uint32_t w[4];
#pragma unroll
            for (int t = 0; t < 4; ++t)
                w[t] = (uint32_t)src[4 * t] | ((uint32_t)src[4 * t + 1] << 8) |
                       ((uint32_t)src[4 * t + 2] << 16) | ((uint32_t)src[4 * t + 3] << 24);
            v = make_uint4(w[0], w[1], w[2], w[3]);
        }
        out[i] = v;
    }
}

inline size_t contract_smem_bytes(uint32_t groups, int mode) {
    size_t b = (size_t)kRowsPerCta * groups * kActStride * 4u + (size_t)kRowsPerCta * groups * 4u;
    if (mode == 1)
        b += (size_t)kRowsPerCta * kRowBlock * groups * 4u;
    return b;
}

inline size_t prep_smem_bytes(uint32_t k) { return (size_t)k * 5u; }

}  // namespace bnn
