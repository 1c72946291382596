// w1a8_gemv.cuh - the W1A8 contraction (ComputeRow, soft-bnn-accelerator.c:219-276).
//
// Packed weight layout (written once by w1a8_pack_kernel): blocks of 8 output
// rows; block b is G*144 bytes:
//     [G][8][16 B]  sign bits of row 8b+r, group g, public bit order
//     [8][G]        binary16 scales of row 8b+r, group g
// A tile of B = 1, 2, 4 or 8 consecutive blocks is one contiguous range that the
// producer warp streams into shared memory with a single 1D bulk copy, bits
// and scales together. Allocations are padded to kBlockPad blocks.
//
// Activations are int8 "sliced" words: per row and group 32 words, word
// (t, j) = t*8 + j packs q[g*128 + 32t + 8i + j], i = 0..3. Masking weight
// word t with (0x01010101 << j) keeps, in byte i, the weight bit that meets
// exactly that activation, scaled by 2^j; dp4a sums 2^j * q over those four
// weights, the eight slices are kept apart, and
//     pos = sum_j acc_j >> j,   D = 2 * pos - total    (soft :251-258).
// The FP32 epilogue then runs acc = fl(acc + fl(F32(scale_g) * D_g)) in
// increasing g, one lane per (activation row, output row) (soft :260-274).
//
// Prologues (where the int8 activations come from):
//   kProSliced   pre-sliced words/totals/row scales in global memory (BNN_Execute)
//   kProQuant    FP32 rows, quantised in the CTA (QuantizeRow, soft :175-211)
//   kProRmsNorm  FP32 rows, RMSNorm (qwen3.c:361-372) then quantised
//   kProI8       int8 rows as given, validated (no -128) and sliced in the CTA
// Epilogues (what is written):
//   kEpiDotGroups  int16 D into a BNN view          (DOT_GROUPS)
//   kEpiView       FP32 Z or Z*s into a BNN view    (GEMV/GEMM[_F32])
//   kEpiResidual   x[n] = fl(x[n] + Y)              (qwen3.c:482-483, 498-499)
//   kEpiSwiGLU     h = fl(fl(g / fl(1 + exp(-g))) * u) over gate/up block pairs
//                  (qwen3.c:491-495); the matrix stores gate and up rows in
//                  alternating 8-row blocks
//
// Pipeline: persistent CTAs of 8 compute warps + 1 producer warp. The
// producer starts streaming weights at once (they never depend on earlier
// kernels), before the compute warps wait for the preceding kernel
// (programmatic dependent launch) and build the activations (the RMSNorm sum
// and every elementwise pass on all 8). 8/B warps share
// one block, each taking a subset of its groups (the integer D's meet in
// shared memory, so the FP32 order is unchanged); small matrices use B = 1 so
// that every SM gets blocks. All waits are bounded.
#pragma once

#include <cstdint>
#include "bnn_device.cuh"
#include "bnn_sync.cuh"
#include "exact_sum.cuh"

namespace bnn {

constexpr int kRowsPerCta = 8;      // activation rows per CTA (grid y covers more)
constexpr int kStatusBadInput = 1;  // an input row had NaN/Inf (F32) or -128 (I8)
constexpr int kStatusNonFinite = 4; // a normalisation divisor was not finite
constexpr uint32_t kBlockPad = 4;
constexpr uint32_t kComputeWarps = 8;
constexpr uint32_t kSumWarps = kSumThreads / 32;  // the RMSNorm sum runs on compute warps 0..kSumWarps-1
static_assert(kComputeWarps >= kSumWarps, "the RMSNorm sum needs four compute warps");
// Prologues that build the activations in the CTA hold up to this many inputs
// (in registers: kMaxPrologueK / 512 float4 per compute thread).
constexpr uint32_t kMaxPrologueK = 8192;

// Test hook (bnn_b200_test_wait_limit): when set, the producer warps of this
// translation unit's contraction kernels issue no copies and arrive on no
// barrier, so every consumer wait for a weight tile runs out.
static __device__ int g_test_starve_producer = 0;

enum Prologue : int { kProSliced = 0, kProQuant = 1, kProRmsNorm = 2, kProI8 = 3 };
enum Epilogue : int { kEpiDotGroups = 0, kEpiView = 1, kEpiResidual = 2, kEpiSwiGLU = 3 };

__host__ __device__ inline size_t block_bytes(uint32_t groups) { return (size_t)groups * 144u; }

// Public [N][K/8] bits + [N][G] scales -> packed blocks (rows past N zero).
static __global__ void w1a8_pack_kernel(const uint8_t* __restrict__ bits, const uint16_t* __restrict__ scales,
                                        uint32_t n, uint32_t groups, size_t nblocks,
                                        unsigned char* __restrict__ out) {
    const size_t bb = block_bytes(groups);
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t first = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    const size_t chunks = nblocks * groups * kRowBlock;
    for (size_t i = first; i < chunks; i += stride) {
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
        *reinterpret_cast<uint4*>(out + b * bb + (g * kRowBlock + r) * 16u) = v;
    }
    const size_t nscales = nblocks * kRowBlock * groups;
    for (size_t i = first; i < nscales; i += stride) {
        const size_t g = i % groups, r = (i / groups) % kRowBlock, b = i / (kRowBlock * groups);
        const size_t row = b * kRowBlock + r;
        const uint16_t sc = row < n ? scales[row * groups + g] : (uint16_t)0;
        *reinterpret_cast<uint16_t*>(out + b * bb + (size_t)groups * 128u + (r * groups + g) * 2u) = sc;
    }
}

struct GemvArgs {
    const unsigned char* wblocks;  // packed blocks (see header)
    uint32_t n, groups, m;         // packed output rows, K/128, activation rows
    uint32_t tiles, stages;        // tiles of B blocks; shared-memory ring depth
    uint32_t blocks_per_tile;      // B = 1, 2, 4 or 8
    // kProSliced
    const uint32_t* act;           // [M][G][32]
    const int32_t* totals;         // [M][G]
    const float* row_scale;        // [M]; nullptr: the I8 ops return Z unscaled
    // kProQuant / kProRmsNorm
    const float* x;                // FP32 rows
    size_t x_stride;               // floats (kProI8: bytes) between rows
    const int8_t* xq;              // kProI8: int8 rows, 4-byte aligned
    const float* gain;             // kProRmsNorm gains [K]
    float eps;
    int exact;                     // 1: the reference's serial sum for RMSNorm
    // output
    unsigned char* out;            // first logical output row
    size_t out_stride;             // bytes between output rows
    int* status;
    int* status_next;              // when set: cleared for the next job of the stream (once, after the wait)
    // kProQuant / kProI8: 1 when no kernel that may still be running writes x (the
    // host tracks the outputs of the jobs in flight): the prologue then
    // loads and quantises x before the grid-dependency wait, under the
    // previous kernel's tail; status words are touched only after the wait
    int early_input;
    // kEpiView: when set, best[m] collects max over the row's outputs of
    // (order-preserving bits of the value) << 32 | ~(index_base + index),
    // i.e. the greedy pick (first index of the maximum); non-finite outputs
    // set the status
    unsigned long long* best;
    uint32_t index_base;           // global index of output row 0 (a column shard's first row)
    // kEpiResidual: out = fl(res + Y) with res rows at res (res_stride bytes
    // apart); nullptr: in place, out = fl(out + Y)
    const unsigned char* res;
    size_t res_stride;
};

// 64-bit argmax key of output `n` with value y (-0 counts as +0; larger
// values, then smaller indices, give larger keys).
__device__ __forceinline__ unsigned long long argmax_key(float y, uint32_t n) {
    const uint32_t u = y == 0.0f ? 0u : __float_as_uint(y);
    const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)ord << 32) | (0xffffffffu - n);
}

struct GemvSmem {
    size_t bars, rs, act, tot, xbuf, seg, dsm, epi, amort, stage, total;
};

// One activation row, one block per compute warp (bpt == kComputeWarps), a
// View or residual epilogue and at most 32 groups: each warp gathers the
// integer D and the scales of four of its blocks and then runs their 32
// ordered FP32 chains at once, one per lane (instead of eight chains on
// eight lanes after every block).
constexpr uint32_t kAmortBlocks = 4;
__host__ __device__ inline bool gemv_amortised(uint32_t groups, uint32_t mrows, uint32_t bpt, int epi) {
    return mrows == 1 && bpt == kComputeWarps && (epi == 1 /* kEpiView */ || epi == 2 /* kEpiResidual */) &&
           (groups == 8 || groups == 16 || groups == 32);
}

// One activation row, one block per compute warp and G = 8/16/32: the lane
// layout of the amortised epilogue (each lane keeps one group's sliced
// activations in registers); DOT_GROUPS stores its integers directly.
__host__ __device__ inline bool gemv_one_row_lanes(uint32_t groups, uint32_t mrows, uint32_t bpt, int epi) {
    return gemv_amortised(groups, mrows, bpt, epi) ||
           (epi == 0 /* kEpiDotGroups */ && mrows == 1 && bpt == kComputeWarps &&
            (groups == 8 || groups == 16 || groups == 32));
}

__host__ __device__ inline GemvSmem gemv_smem_plan(uint32_t groups, uint32_t mrows, uint32_t bpt,
                                                   uint32_t stages, int pro, int epi) {
    GemvSmem p;
    p.bars = 0;     // full[stages], empty[stages] (stages <= 8)
    p.rs = 128;     // row scales + status flags
    p.act = 448;  // after the row scales, flags and 64 reduction slots
    p.tot = p.act + (size_t)mrows * groups * kActStride * 4u;
    p.xbuf = (p.tot + (size_t)mrows * groups * 4u + 15) & ~(size_t)15;  // float4 stores
    p.seg = p.xbuf + (pro == kProQuant || pro == kProRmsNorm ? (size_t)groups * kGroup * 4u : 0);  // FP32 row
    p.dsm = p.seg + (pro == kProRmsNorm ? kSumSmemBytes : 0);
    p.epi = p.dsm + (epi != kEpiDotGroups ? (size_t)bpt * mrows * kRowBlock * groups * 2u : 0);
    p.epi = (p.epi + 15) & ~(size_t)15;
    p.amort = p.epi + (epi == kEpiSwiGLU ? (size_t)bpt * mrows * kRowBlock * 4u : 0);
    // per warp: D [4 blocks][8 rows][G] int16 then scales [4][8][G] binary16
    p.stage = p.amort + (gemv_amortised(groups, mrows, bpt, epi)
                             ? (size_t)kComputeWarps * kAmortBlocks * kRowBlock * groups * 4u : 0);
    p.stage = (p.stage + 127) & ~(size_t)127;
    p.total = p.stage + (size_t)stages * bpt * block_bytes(groups);
    return p;
}

// Integer part of one (row, group) unit for one activation row.
__device__ __forceinline__ int group_dot(const uint32_t (&mk)[32], const uint32_t* act_s, int total) {
    int acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
        acc[j] = 0;
    const uint4* a4 = reinterpret_cast<const uint4*>(act_s);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const uint4 lo = a4[t * 2], hi = a4[t * 2 + 1];
        acc[0] = dp4a_us(mk[t * 8 + 0], lo.x, acc[0]);
        acc[1] = dp4a_us(mk[t * 8 + 1], lo.y, acc[1]);
        acc[2] = dp4a_us(mk[t * 8 + 2], lo.z, acc[2]);
        acc[3] = dp4a_us(mk[t * 8 + 3], lo.w, acc[3]);
        acc[4] = dp4a_us(mk[t * 8 + 4], hi.x, acc[4]);
        acc[5] = dp4a_us(mk[t * 8 + 5], hi.y, acc[5]);
        acc[6] = dp4a_us(mk[t * 8 + 6], hi.z, acc[6]);
        acc[7] = dp4a_us(mk[t * 8 + 7], hi.w, acc[7]);
    }
    // 128 * pos = sum_j acc_j * 2^(7-j): acc_j is an exact multiple of 2^j.
    int pos128 = acc[7];
#pragma unroll
    for (int j = 6; j >= 0; --j)
        pos128 += acc[j] << (7 - j);
    return (pos128 >> 6) - total;
}

// group_dot with the group's 32 sliced activation words already in registers.
__device__ __forceinline__ int group_dot_regs(uint4 w, const uint4 (&av)[8], int total) {
    int acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
        acc[j] = 0;
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const uint4 lo = av[t * 2], hi = av[t * 2 + 1];
        const uint32_t wd = words[t];
        acc[0] = dp4a_us(wd & 0x01010101u, lo.x, acc[0]);
        acc[1] = dp4a_us(wd & 0x02020202u, lo.y, acc[1]);
        acc[2] = dp4a_us(wd & 0x04040404u, lo.z, acc[2]);
        acc[3] = dp4a_us(wd & 0x08080808u, lo.w, acc[3]);
        acc[4] = dp4a_us(wd & 0x10101010u, hi.x, acc[4]);
        acc[5] = dp4a_us(wd & 0x20202020u, hi.y, acc[5]);
        acc[6] = dp4a_us(wd & 0x40404040u, hi.z, acc[6]);
        acc[7] = dp4a_us(wd & 0x80808080u, hi.w, acc[7]);
    }
    int pos128 = acc[7];
#pragma unroll
    for (int j = 6; j >= 0; --j)
        pos128 += acc[j] << (7 - j);
    return (pos128 >> 6) - total;
}

// group_dot for one activation row, the masks built word by word from the
// weight words (fewer live registers; the same integers).
__device__ __forceinline__ int group_dot_w(uint4 w, const uint32_t* act_s, int total) {
    int acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
        acc[j] = 0;
    const uint4* a4 = reinterpret_cast<const uint4*>(act_s);
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const uint4 lo = a4[t * 2], hi = a4[t * 2 + 1];
        const uint32_t wd = words[t];
        acc[0] = dp4a_us(wd & 0x01010101u, lo.x, acc[0]);
        acc[1] = dp4a_us(wd & 0x02020202u, lo.y, acc[1]);
        acc[2] = dp4a_us(wd & 0x04040404u, lo.z, acc[2]);
        acc[3] = dp4a_us(wd & 0x08080808u, lo.w, acc[3]);
        acc[4] = dp4a_us(wd & 0x10101010u, hi.x, acc[4]);
        acc[5] = dp4a_us(wd & 0x20202020u, hi.y, acc[5]);
        acc[6] = dp4a_us(wd & 0x40404040u, hi.z, acc[6]);
        acc[7] = dp4a_us(wd & 0x80808080u, hi.w, acc[7]);
    }
    int pos128 = acc[7];
#pragma unroll
    for (int j = 6; j >= 0; --j)
        pos128 += acc[j] << (7 - j);
    return (pos128 >> 6) - total;
}

// GC: the group count when fixed at compile time (0: a.groups). The one-row
// amortised contraction at G = 16 (K = 2048, every Qwen3-1.7B linear but
// down and the shape of lm_head) runs ~10 % fewer instructions with every
// index and loop bound constant.
template <int PRO, int EPI, int GC = 0>
__global__ void __launch_bounds__((kComputeWarps + 1) * 32, 3) w1a8_gemv_kernel(GemvArgs a) {
    griddep_launch_dependents();
    extern __shared__ __align__(128) unsigned char sm[];
    const uint32_t G = GC != 0 ? (uint32_t)GC : a.groups;
    const uint32_t consumers = kComputeWarps;
    const uint32_t cthreads = consumers * 32;
    const uint32_t bpt = a.blocks_per_tile, wpb = kComputeWarps / bpt;
    const uint32_t m0 = blockIdx.y * kRowsPerCta;
    const uint32_t mrows = min((uint32_t)kRowsPerCta, a.m - m0);
    const GemvSmem plan = gemv_smem_plan(G, mrows, bpt, a.stages, PRO, EPI);
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + plan.bars);
    uint64_t* empty = full + a.stages;
    float* rs_s = reinterpret_cast<float*>(sm + plan.rs);          // [8] row scales
    int* flags = reinterpret_cast<int*>(sm + plan.rs + 32);        // [0] abort
    float* red = reinterpret_cast<float*>(sm + plan.rs + 64);      // reduction slots (64)
    uint32_t* act_s = reinterpret_cast<uint32_t*>(sm + plan.act);
    int32_t* tot_s = reinterpret_cast<int32_t*>(sm + plan.tot);
    float* xbuf = reinterpret_cast<float*>(sm + plan.xbuf);
    unsigned char* sum_mem = sm + plan.seg;  // exact RMS sum scratch
    int16_t* dsm = reinterpret_cast<int16_t*>(sm + plan.dsm);
    float* epi_s = reinterpret_cast<float*>(sm + plan.epi);
    unsigned char* stage0 = sm + plan.stage;
    const uint32_t bb = (uint32_t)block_bytes(G);
    const uint32_t tile_bytes = bpt * bb;
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    if (tid == 0) {
        for (uint32_t s = 0; s < a.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], consumers);
        }
        fence_barrier_init();
        flags[0] = 0;
    }
    __syncthreads();

    if (warp == consumers) {  // producer warp: weights never depend on earlier kernels
        if (lane == 0 && !*reinterpret_cast<volatile int*>(&g_test_starve_producer)) {
            uint32_t i = 0;
            for (uint32_t tile = blockIdx.x; tile < a.tiles; tile += gridDim.x, ++i) {
                const uint32_t s = i % a.stages;
                if (i >= a.stages && !mbar_wait(&empty[s], ((i / a.stages) - 1) & 1)) {
                    atomicOr(a.status, kStatusTimeout);
                    break;
                }
                mbar_arrive_expect_tx(&full[s], tile_bytes);
                bulk_g2s(stage0 + (size_t)s * tile_bytes, a.wblocks + (size_t)tile * tile_bytes, tile_bytes,
                         &full[s]);
            }
            // No bulk copy may still be in flight when the CTA exits.
            for (uint32_t j = i > a.stages ? i - a.stages : 0; j < i; ++j)
                if (!mbar_wait(&full[j % a.stages], (j / a.stages) & 1))
                    atomicOr(a.status, kStatusTimeout);
        }
        return;
    }

    // ---- consumers: wait for the producers of our activations, then build them
    const bool early = (PRO == kProQuant || PRO == kProI8) && a.early_input != 0;
    auto after_wait = [&]() {
        if (tid == 0) {
            if (*a.status != 0 && flags[0] != 2)
                flags[0] = 1;  // an earlier kernel failed: skip the work, keep the protocol
            if (a.status_next != nullptr && blockIdx.x == 0 && blockIdx.y == 0)
                *a.status_next = 0;
        }
    };
    if (!early) {
        griddep_wait();
        after_wait();
    }
    if (PRO == kProSliced) {
        for (uint32_t i = tid; i < mrows * G * (kWordsPerGroup / 4); i += cthreads) {
            const uint32_t mm = i / (G * 8), rest = i % (G * 8), g = rest / 8, c = rest % 8;
            const uint4* src =
                reinterpret_cast<const uint4*>(a.act + ((size_t)(m0 + mm) * G + g) * kWordsPerGroup);
            reinterpret_cast<uint4*>(act_s + (mm * G + g) * kActStride)[c] = src[c];
        }
        for (uint32_t i = tid; i < mrows * G; i += cthreads)
            tot_s[i] = a.totals[(size_t)m0 * G + i];
        if (tid < mrows)
            rs_s[tid] = a.row_scale ? a.row_scale[m0 + tid] : 1.0f;
        named_barrier(1, cthreads);
    } else if constexpr (PRO == kProI8) {
        // int8 rows as given (ValidateI8Input, soft :279-292: no -128). One
        // warp slices one group per pass: lane L holds the group's bytes
        // 4L .. 4L+3, the same 4x4 byte transpose as the FP32 prologue leaves
        // lane L with its slice word; totals with one dp4a and a reduction.
        const uint32_t slot = (lane >> 3) * 8u + (lane & 1u) * 4u + ((lane >> 1) & 3u);
        int bad = 0;
        for (uint32_t mm = 0; mm < mrows; ++mm) {
            const uint32_t* xr = reinterpret_cast<const uint32_t*>(a.xq + (size_t)(m0 + mm) * a.x_stride);
#pragma unroll 1
            for (uint32_t g = warp; g < G; g += consumers) {
                uint32_t w = xr[g * 32u + lane];
                bad |= __vcmpeq4(w, 0x80808080u) != 0u;
                const int total = __reduce_add_sync(0xffffffffu, __dp4a((int)w, 0x01010101, 0));
                uint32_t o = __shfl_xor_sync(0xffffffffu, w, 4);
                w = (lane & 4u) ? __byte_perm(w, o, 0x3276) : __byte_perm(w, o, 0x5410);
                o = __shfl_xor_sync(0xffffffffu, w, 2);
                w = (lane & 2u) ? __byte_perm(w, o, 0x3715) : __byte_perm(w, o, 0x6240);
                act_s[(mm * G + g) * kActStride + slot] = w;
                if (lane == 0)
                    tot_s[mm * G + g] = total;
            }
        }
        if (bad)
            flags[0] = 2;
        if (tid < mrows)
            rs_s[tid] = 1.0f;
        named_barrier(1, cthreads);
        if (early) {
            griddep_wait();
            after_wait();
        }
        if (tid == 0 && flags[0] == 2)
            atomicOr(a.status, kStatusBadInput);
        named_barrier(1, cthreads);
    } else {
        // The row is staged in shared memory once; every later pass is a
        // rolled loop over it (compact code: the kernels of a decode step take
        // turns on every SM, so their instruction footprint matters).
        const uint32_t K = G * kGroup;
        float4* xb4 = reinterpret_cast<float4*>(xbuf);
        for (uint32_t mm = 0; mm < mrows; ++mm) {
            const float4* xr = reinterpret_cast<const float4*>(a.x + (size_t)(m0 + mm) * a.x_stride);
            int bad = 0;
            float amax = 0.0f;
#pragma unroll 4
            for (uint32_t i = tid; i < K / 4; i += cthreads) {
                const float4 v = xr[i];
                bad |= !isfinite(v.x) | !isfinite(v.y) | !isfinite(v.z) | !isfinite(v.w);
                amax = fmaxf(fmaxf(amax, fmaxf(fabsf(v.x), fabsf(v.y))), fmaxf(fabsf(v.z), fabsf(v.w)));
                xb4[i] = v;
            }
            // A linear rejects non-finite input (ValidateF32Input, soft :294-308);
            // before RMSNorm it shows up as a non-finite divisor instead.
            if (bad && PRO == kProQuant)
                flags[0] = 2;
            named_barrier(1, cthreads);
            if (PRO == kProRmsNorm) {
                // The reference's RMSNorm sum fl(...fl(fl(x0*x0) + x1*x1)...) in
                // index order (qwen3.c:361-372): exact mode reproduces it bit for
                // bit with the compute warps (exact_sum.cuh); fast mode sums
                // in a fixed tree order.
                // Both run on warps 0..kSumWarps-1 (named barrier 2); the fast tree.s
                // order is that of kSumThreads threads.
                if (warp < kSumWarps) {
                    float sum;
                    if (a.exact) {
                        sum = exact_sumsq(xbuf, (int)K, sum_mem, 2);
                    } else {
                        float t = 0.0f;
                        for (uint32_t i = tid; i < K; i += kSumThreads)
                            t = __fadd_rn(t, __fmul_rn(xbuf[i], xbuf[i]));
                        for (int o = 16; o > 0; o >>= 1)
                            t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, o));
                        if (lane == 0)
                            red[16 + warp] = t;
                        named_barrier(2, kSumThreads);
                        sum = 0.0f;
                        for (uint32_t w = 0; w < kSumWarps; ++w)
                            sum = __fadd_rn(sum, red[16 + w]);
                    }
                    if (tid == 0)
                        red[48] = sum;
                }
                named_barrier(1, cthreads);
                const float sum = red[48];
                const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)K), a.eps));
                amax = 0.0f;
                if (!isfinite(rms) || rms == 0.0f) {
                    if (tid == 0) {
                        flags[0] = 1;
                        atomicOr(a.status, kStatusNonFinite);
                    }
                } else {
                    const float4* gr = reinterpret_cast<const float4*>(a.gain);
#pragma unroll 2
                    for (uint32_t i = tid; i < K / 4; i += cthreads) {
                        float4 v = xb4[i];
                        const float4 gn = gr[i];
                        v.x = __fmul_rn(__fdiv_rn(v.x, rms), gn.x);
                        v.y = __fmul_rn(__fdiv_rn(v.y, rms), gn.y);
                        v.z = __fmul_rn(__fdiv_rn(v.z, rms), gn.z);
                        v.w = __fmul_rn(__fdiv_rn(v.w, rms), gn.w);
                        amax = fmaxf(fmaxf(amax, fmaxf(fabsf(v.x), fabsf(v.y))), fmaxf(fabsf(v.z), fabsf(v.w)));
                        xb4[i] = v;
                    }
                }
            }
            for (int o = 16; o > 0; o >>= 1)
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            if (lane == 0)
                red[32 + warp] = amax;
            named_barrier(1, cthreads);
            amax = red[32];
            for (uint32_t w = 1; w < consumers; ++w)
                amax = fmaxf(amax, red[32 + w]);
            const float s = row_scale_from_absmax(amax);
            const RowQuantizer quant(s);
            // One warp quantises one group per pass (32 lanes x 4 values).
            // Lane L = 8t + 2i + h holds q[32t + 8i + 4h + b], b = 0..3; a
            // 4x4 byte transpose across the lanes that share (t, h) leaves lane
            // L with slice word (t, j = 4h + i): the bytes q[32t + 8i' + j].
            const uint32_t slot = (lane >> 3) * 8u + (lane & 1u) * 4u + ((lane >> 1) & 3u);
            auto quant_group = [&](uint32_t g) {
                const float4 v = xb4[g * 32u + lane];
                const int8_t q0 = quant(v.x), q1 = quant(v.y), q2 = quant(v.z), q3 = quant(v.w);
                uint32_t w = (uint32_t)(uint8_t)q0 | ((uint32_t)(uint8_t)q1 << 8) | ((uint32_t)(uint8_t)q2 << 16) |
                             ((uint32_t)(uint8_t)q3 << 24);
                const int total = __reduce_add_sync(0xffffffffu, (int)q0 + (int)q1 + (int)q2 + (int)q3);
                uint32_t o = __shfl_xor_sync(0xffffffffu, w, 4);
                w = (lane & 4u) ? __byte_perm(w, o, 0x3276) : __byte_perm(w, o, 0x5410);
                o = __shfl_xor_sync(0xffffffffu, w, 2);
                w = (lane & 2u) ? __byte_perm(w, o, 0x3715) : __byte_perm(w, o, 0x6240);
                act_s[(mm * G + g) * kActStride + slot] = w;
                if (lane == 0)
                    tot_s[mm * G + g] = total;
            };
            if constexpr (GC != 0 && GC % kComputeWarps == 0) {
                // every warp owns GC / 8 groups: unrolled, their chains interleave
#pragma unroll
                for (uint32_t j = 0; j < (uint32_t)GC / kComputeWarps; ++j)
                    quant_group(warp + j * consumers);
            } else {
#pragma unroll 1
                for (uint32_t g = warp; g < G; g += consumers)
                    quant_group(g);
            }
            if (tid == 0)
                rs_s[mm] = s;
            named_barrier(1, cthreads);  // xbuf and red are reused by the next row
        }
        if (early) {
            griddep_wait();  // the row loop's last barrier made every flag visible to thread 0
            after_wait();
        }
        if (tid == 0 && flags[0] == 2)
            atomicOr(a.status, kStatusBadInput);
        named_barrier(1, cthreads);
    }
    const bool abort = flags[0] != 0;

    // ---- contraction over this CTA's tiles
    unsigned long long best0 = 0ull, best1 = 0ull;  // kEpiView argmax: outputs p = lane, lane + 32
    const uint32_t r = lane & 7;
    const uint32_t my_block = warp / wpb, part = warp % wpb;
    int16_t* blk_d = dsm + (size_t)my_block * mrows * kRowBlock * G;
    // With one warp per block the warps never share a tile's D or epilogue
    // slots (SwiGLU pairs excepted: a 64-thread barrier per gate/up pair), so
    // they run through the tiles without waiting for each other.
    const bool solo = wpb == 1;
    auto tile_sync = [&]() {
        if (!solo)
            named_barrier(1, cthreads);
        else if (EPI == kEpiSwiGLU) {
            // constant barrier ids 3..6 (one per pair of an 8-block tile)
            switch (my_block >> 1) {
                case 0: named_barrier(3, 64); break;
                case 1: named_barrier(4, 64); break;
                case 2: named_barrier(5, 64); break;
                default: named_barrier(6, 64); break;
            }
        }
        else
            __syncwarp();
    };
    if (EPI == kEpiDotGroups && gemv_one_row_lanes(G, mrows, bpt, EPI)) {
        // ---- one row, DOT_GROUPS: lane L works on group L / (32 / G), rows
        // (L % (32 / G)) * (G / 4) .. + G / 4 - 1 of every block, its group's
        // activations in registers; each int16 D goes straight to the output
        const uint32_t lpg = 32u / G, rpl = G / 4u;
        const uint32_t ga = lane / lpg, ra = (lane % lpg) * rpl;
        uint4 av[8];
#pragma unroll
        for (int c = 0; c < 8; ++c)
            av[c] = reinterpret_cast<const uint4*>(act_s + ga * kActStride)[c];
        const int tot_a = tot_s[ga];
        unsigned char* orow = a.out + (size_t)m0 * a.out_stride;
        uint32_t s = 0, phase = 0;
        for (uint32_t tile = blockIdx.x; tile < a.tiles; tile += gridDim.x) {
            const bool ready = mbar_wait(&full[s], phase);
            if (!ready && lane == 0)
                atomicOr(a.status, kStatusTimeout);
            if (ready && !abort) {
                const uint4* wt = reinterpret_cast<const uint4*>(stage0 + (size_t)s * tile_bytes +
                                                                 (size_t)my_block * bb) + ga * kRowBlock + ra;
                const uint32_t n0 = (tile * bpt + my_block) * kRowBlock + ra;
#pragma unroll 2
                for (uint32_t i2 = 0; i2 < rpl; ++i2) {
                    const int d = group_dot_regs(wt[i2], av, tot_a);
                    if (n0 + i2 < a.n)
                        store_i16_any(orow + ((size_t)(n0 + i2) * G + ga) * 2u, (int16_t)d);
                }
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&empty[s]);  // this warp no longer reads the stage
            if (++s == a.stages) {
                s = 0;
                phase ^= 1u;
            }
        }
        return;
    }
    if (EPI == kEpiView || EPI == kEpiResidual) {
        if (gemv_amortised(G, mrows, bpt, EPI)) {
            // ---- amortised epilogue (see gemv_amortised)
            int16_t* am_d = reinterpret_cast<int16_t*>(sm + plan.amort) + (size_t)warp * kAmortBlocks * kRowBlock * G * 2;
            uint16_t* am_s = reinterpret_cast<uint16_t*>(am_d + kAmortBlocks * kRowBlock * G);
            uint32_t pend = 0;       // blocks gathered
            uint32_t pend_live = 0;  // slot k computed (bit k)
            uint32_t pend_tile = 0;  // tile of slot 0; slot k holds tile pend_tile + k * gridDim.x
            // lane L works on group g = L / (32 / G), rows (L % (32 / G)) * (G / 4) .. + G / 4 - 1
            // of every block: its group's activations stay in registers for every tile
            const uint32_t lpg = 32u / G, rpl = G / 4u;
            const uint32_t ga = lane / lpg, ra = (lane % lpg) * rpl;
            uint4 av[8];
#pragma unroll
            for (int c = 0; c < 8; ++c)
                av[c] = reinterpret_cast<const uint4*>(act_s + ga * kActStride)[c];
            const int tot_a = tot_s[ga];
            uint32_t s = 0, phase = 0;  // ring stage and its parity (no division per tile)
            for (uint32_t tile = blockIdx.x; tile < a.tiles; tile += gridDim.x) {
                const bool ready = mbar_wait(&full[s], phase);
                if (!ready && lane == 0)
                    atomicOr(a.status, kStatusTimeout);
                const bool work = ready && !abort;
                const unsigned char* wblk = stage0 + (size_t)s * tile_bytes + (size_t)my_block * bb;
                if (work) {
                    const uint4* wt = reinterpret_cast<const uint4*>(wblk) + ga * kRowBlock + ra;
                    int16_t* dcol = am_d + (size_t)(pend * kRowBlock + ra) * G + ga;
#pragma unroll 2
                    for (uint32_t i2 = 0; i2 < rpl; ++i2)
                        dcol[(size_t)i2 * G] = (int16_t)group_dot_regs(wt[i2], av, tot_a);
                    // the block's scales (8 rows x G binary16) follow it out of the stage
                    const uint4* sc4 = reinterpret_cast<const uint4*>(wblk + (size_t)G * 128u);
                    uint4* dst4 = reinterpret_cast<uint4*>(am_s + (size_t)pend * kRowBlock * G);
                    for (uint32_t c = lane; c < kRowBlock * G / 8; c += 32)
                        dst4[c] = sc4[c];
                }
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(&empty[s]);  // this warp no longer reads the stage
                if (++s == a.stages) {
                    s = 0;
                    phase ^= 1u;
                }
                if (pend == 0)
                    pend_tile = tile;
                pend_live |= (work ? 1u : 0u) << pend;
                ++pend;
                if (pend == kAmortBlocks || tile + gridDim.x >= a.tiles) {
                    // lane L: block slot L / 8, row L % 8
                    const uint32_t k = lane >> 3, rr = lane & 7;
                    const uint32_t bk = (pend_tile + k * gridDim.x) * bpt + my_block;
                    const uint32_t n = bk * kRowBlock + rr;
                    if (k < pend && ((pend_live >> k) & 1u) && n < a.n) {
                        float acc = 0.0f;
                        const uint16_t* sc = am_s + ((size_t)k * kRowBlock + rr) * G;
                        const int16_t* dd = am_d + ((size_t)k * kRowBlock + rr) * G;
                        for (uint32_t g0 = 0; g0 < G; g0 += 8) {
                            const uint4 sv = *reinterpret_cast<const uint4*>(sc + g0);
                            const uint4 dv = *reinterpret_cast<const uint4*>(dd + g0);
                            const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
                            const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w};
                            float pr[8];
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                const int d0 = (int)(int16_t)(dw[j] & 0xffffu), d1 = (int)(int16_t)(dw[j] >> 16);
                                const float f0 = __fsub_rn(__int_as_float(0x4b400000 + d0), 12582912.0f);
                                const float f1 = __fsub_rn(__int_as_float(0x4b400000 + d1), 12582912.0f);
                                pr[2 * j] = __fmul_rn(h2f((uint16_t)(sw[j] & 0xffffu)), f0);
                                pr[2 * j + 1] = __fmul_rn(h2f((uint16_t)(sw[j] >> 16)), f1);
                            }
#pragma unroll
                            for (int j = 0; j < 8; ++j)
                                acc = __fadd_rn(acc, pr[j]);
                        }
                        if ((PRO != kProSliced && PRO != kProI8) || a.row_scale)
                            acc = __fmul_rn(acc, rs_s[0]);
                        if (EPI == kEpiView) {
                            store_f32_any(a.out + (size_t)m0 * a.out_stride + (size_t)n * 4u, acc);
                            if (a.best) {
                                if (!isfinite(acc))
                                    atomicOr(a.status, kStatusNonFinite);
                                const unsigned long long key = argmax_key(acc, a.index_base + n);
                                best0 = key > best0 ? key : best0;
                            }
                        } else {
                            float* dst = reinterpret_cast<float*>(a.out + (size_t)m0 * a.out_stride) + n;
                            const float base =
                                a.res ? reinterpret_cast<const float*>(a.res + (size_t)m0 * a.res_stride)[n] : *dst;
                            *dst = __fadd_rn(base, acc);
                        }
                    }
                    __syncwarp();  // the slots are reused
                    pend = 0;
                    pend_live = 0;
                }
            }
            if (EPI == kEpiView && a.best != nullptr) {
                for (int o = 16; o > 0; o >>= 1) {
                    const unsigned long long ob = __shfl_xor_sync(0xffffffffu, best0, o);
                    best0 = ob > best0 ? ob : best0;
                }
                if (lane == 0 && best0 != 0ull)
                    atomicMax(&a.best[m0], best0);
            }
            return;
        }
    }
    uint32_t i = 0;
    for (uint32_t tile = blockIdx.x; tile < a.tiles; tile += gridDim.x, ++i) {
        const uint32_t s = i % a.stages;
        const bool ready = mbar_wait(&full[s], (i / a.stages) & 1);
        if (!ready && lane == 0)
            atomicOr(a.status, kStatusTimeout);
        const bool work = ready && !abort;
        const uint32_t blk = tile * bpt + my_block;
        const unsigned char* wblk = stage0 + (size_t)s * tile_bytes + (size_t)my_block * bb;
        const uint4* wt = reinterpret_cast<const uint4*>(wblk);
        if (work) {
            for (uint32_t q = part; q * 4 < G; q += wpb) {
                const uint32_t g = q * 4 + (lane >> 3);
                if (g >= G)
                    continue;
                const uint4 w = wt[g * kRowBlock + r];
                uint32_t mk[32];
                const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int t = 0; t < 4; ++t)
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        mk[t * 8 + j] = words[t] & (0x01010101u << j);
                const uint32_t n = blk * kRowBlock + r;
                for (uint32_t mm = 0; mm < mrows; ++mm) {
                    const int d = group_dot(mk, act_s + (mm * G + g) * kActStride, tot_s[mm * G + g]);
                    if (EPI == kEpiDotGroups) {
                        if (n < a.n)
                            store_i16_any(a.out + (size_t)(m0 + mm) * a.out_stride + ((size_t)n * G + g) * 2u,
                                          (int16_t)d);
                    } else {
                        blk_d[(mm * kRowBlock + r) * G + g] = (int16_t)d;
                    }
                }
            }
        }
        if (EPI != kEpiDotGroups) {
            tile_sync();  // every group's D of the block is in shared memory
            // Ordered FP32 scale-accumulate, by the first warp of each block;
            // the scales come from the same stage.
            const uint16_t* sc_blk = reinterpret_cast<const uint16_t*>(wblk + (size_t)G * 128u);
            if (part == 0) {
                for (uint32_t p = lane; p < mrows * kRowBlock; p += 32) {
                    const uint32_t mm = p / kRowBlock, rr = p % kRowBlock;
                    const uint32_t n = blk * kRowBlock + rr;
                    float acc = 0.0f;
                    if (work && n < a.n) {
                        const uint16_t* sc = sc_blk + rr * G;
                        const int16_t* dd = blk_d + (mm * kRowBlock + rr) * G;
                        if ((G & 7u) == 0) {
                            // eight groups per pair of 16-byte loads; D (|D| <= 16256)
                            // to float exactly through the 1.5 * 2^23 bias
                            for (uint32_t g0 = 0; g0 < G; g0 += 8) {
                                const uint4 sv = *reinterpret_cast<const uint4*>(sc + g0);
                                const uint4 dv = *reinterpret_cast<const uint4*>(dd + g0);
                                const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
                                const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w};
                                float p[8];
#pragma unroll
                                for (int j = 0; j < 4; ++j) {
                                    const int d0 = (int)(int16_t)(dw[j] & 0xffffu), d1 = (int)(int16_t)(dw[j] >> 16);
                                    const float f0 = __fsub_rn(__int_as_float(0x4b400000 + d0), 12582912.0f);
                                    const float f1 = __fsub_rn(__int_as_float(0x4b400000 + d1), 12582912.0f);
                                    p[2 * j] = __fmul_rn(h2f((uint16_t)(sw[j] & 0xffffu)), f0);
                                    p[2 * j + 1] = __fmul_rn(h2f((uint16_t)(sw[j] >> 16)), f1);
                                }
#pragma unroll
                                for (int j = 0; j < 8; ++j)
                                    acc = __fadd_rn(acc, p[j]);
                            }
                        } else {
#pragma unroll 8
                            for (uint32_t g = 0; g < G; ++g)
                                acc = __fadd_rn(acc, __fmul_rn(h2f(sc[g]), (float)dd[g]));
                        }
                        if ((PRO != kProSliced && PRO != kProI8) || a.row_scale)
                            acc = __fmul_rn(acc, rs_s[mm]);
                        if (EPI == kEpiView) {
                            store_f32_any(a.out + (size_t)(m0 + mm) * a.out_stride + (size_t)n * 4u, acc);
                            if (a.best) {
                                if (!isfinite(acc))
                                    atomicOr(a.status, kStatusNonFinite);
                                const unsigned long long key = argmax_key(acc, a.index_base + n);
                                if (p < 32)
                                    best0 = key > best0 ? key : best0;
                                else
                                    best1 = key > best1 ? key : best1;
                            }
                        } else if (EPI == kEpiResidual) {
                            float* dst = reinterpret_cast<float*>(a.out + (size_t)(m0 + mm) * a.out_stride) + n;
                            const float base =
                                a.res ? reinterpret_cast<const float*>(a.res + (size_t)(m0 + mm) * a.res_stride)[n]
                                      : *dst;
                            *dst = __fadd_rn(base, acc);
                        }
                    }
                    if (EPI == kEpiSwiGLU)
                        epi_s[(my_block * mrows + mm) * kRowBlock + rr] = acc;
                }
            }
            if (EPI == kEpiSwiGLU) {
                // Blocks 2k (gate rows) and 2k+1 (up rows) hold the same 8 rows.
                tile_sync();
                if (part == 0 && (my_block & 1) == 0 && work) {
                    for (uint32_t p = lane; p < mrows * kRowBlock; p += 32) {
                        const uint32_t mm = p / kRowBlock, rr = p % kRowBlock;
                        if (blk * kRowBlock + rr >= a.n)
                            continue;
                        const float g = epi_s[(my_block * mrows + mm) * kRowBlock + rr];
                        const float u = epi_s[((my_block + 1) * mrows + mm) * kRowBlock + rr];
                        const float silu = __fdiv_rn(g, __fadd_rn(1.0f, expf_cr(-g)));
                        reinterpret_cast<float*>(a.out + (size_t)(m0 + mm) * a.out_stride)[(blk / 2) * kRowBlock + rr] =
                            __fmul_rn(silu, u);
                    }
                }
            }
            tile_sync();  // shared D/epilogue buffers and the stage are free again
        }
        __syncwarp();
        if (lane == 0)
            mbar_arrive(&empty[s]);  // this warp no longer reads the stage
    }
    if (EPI == kEpiView && a.best != nullptr && part == 0) {
        // lanes 8k..8k+7 hold outputs of one activation row: reduce, one atomic
#pragma unroll
        for (uint32_t k = 0; k < 2; ++k) {
            unsigned long long b = k == 0 ? best0 : best1;
#pragma unroll
            for (int o = 4; o > 0; o >>= 1) {
                const unsigned long long ob = __shfl_xor_sync(0xffffffffu, b, o);
                b = ob > b ? ob : b;
            }
            const uint32_t p = lane + 32u * k;
            if ((lane & 7) == 0 && p < mrows * kRowBlock && b != 0ull)
                atomicMax(&a.best[m0 + p / kRowBlock], b);
        }
    }
}

// Launch shape for one matrix, row count and variant.
struct GemvLaunch {
    uint32_t blocks_per_tile, stages, tiles, grid_x;
    size_t smem;
    int pro, epi;
    int gc;  // compile-time group count of the chosen kernel (0: general)
};

using GemvFn = void (*)(GemvArgs);

// One-row amortised variants compiled for G = 16.
constexpr uint32_t kGemvFixedGroups = 16;
inline GemvFn gemv_fn_fixed(int pro, int epi) {
    if (pro == kProSliced && epi == kEpiView) return w1a8_gemv_kernel<kProSliced, kEpiView, 16>;
    if (pro == kProSliced && epi == kEpiResidual) return w1a8_gemv_kernel<kProSliced, kEpiResidual, 16>;
    if (pro == kProQuant && epi == kEpiView) return w1a8_gemv_kernel<kProQuant, kEpiView, 16>;
    if (pro == kProRmsNorm && epi == kEpiView) return w1a8_gemv_kernel<kProRmsNorm, kEpiView, 16>;
    if (pro == kProI8 && epi == kEpiView) return w1a8_gemv_kernel<kProI8, kEpiView, 16>;
    if (pro == kProI8 && epi == kEpiDotGroups) return w1a8_gemv_kernel<kProI8, kEpiDotGroups, 16>;
    return nullptr;
}

inline GemvFn gemv_fn(int pro, int epi, int gc = 0) {
    if (gc == (int)kGemvFixedGroups)
        return gemv_fn_fixed(pro, epi);
    if (pro == kProSliced && epi == kEpiDotGroups) return w1a8_gemv_kernel<kProSliced, kEpiDotGroups>;
    if (pro == kProSliced && epi == kEpiView) return w1a8_gemv_kernel<kProSliced, kEpiView>;
    if (pro == kProSliced && epi == kEpiResidual) return w1a8_gemv_kernel<kProSliced, kEpiResidual>;
    if (pro == kProSliced && epi == kEpiSwiGLU) return w1a8_gemv_kernel<kProSliced, kEpiSwiGLU>;
    if (pro == kProQuant && epi == kEpiView) return w1a8_gemv_kernel<kProQuant, kEpiView>;
    if (pro == kProQuant && epi == kEpiResidual) return w1a8_gemv_kernel<kProQuant, kEpiResidual>;
    if (pro == kProRmsNorm && epi == kEpiView) return w1a8_gemv_kernel<kProRmsNorm, kEpiView>;
    if (pro == kProRmsNorm && epi == kEpiSwiGLU) return w1a8_gemv_kernel<kProRmsNorm, kEpiSwiGLU>;
    if (pro == kProI8 && epi == kEpiDotGroups) return w1a8_gemv_kernel<kProI8, kEpiDotGroups>;
    if (pro == kProI8 && epi == kEpiView) return w1a8_gemv_kernel<kProI8, kEpiView>;
    return nullptr;
}

constexpr size_t kGemvSmemBudget = 200u * 1024u;

// Blocks per tile so even small matrices spread over every SM (B = 1 gives
// one block per CTA, its groups split over the 4 compute warps); ring depth
// that fits the shared-memory budget; persistent grid from the occupancy of
// that configuration. SwiGLU needs gate/up block pairs in a tile.
inline GemvLaunch plan_gemv(int sm_count, uint32_t n, uint32_t groups, uint32_t m, int pro, int epi) {
    const uint32_t nblocks = (n + kRowBlock - 1) / kRowBlock;
    const uint32_t mrows = m < (uint32_t)kRowsPerCta ? m : (uint32_t)kRowsPerCta;
    const uint32_t min_bpt = epi == kEpiSwiGLU ? 2u : 1u;
    GemvLaunch c;
    c.pro = pro;
    c.epi = epi;
    // one block per compute warp when there are blocks to spare (no split groups,
    // no hand-off between warps inside a block)
    c.blocks_per_tile = nblocks >= 16u * sm_count ? kComputeWarps
                        : nblocks >= 8u * sm_count ? 4u
                        : (nblocks >= 2u * sm_count ? 2u : 1u);
    if (c.blocks_per_tile < min_bpt)
        c.blocks_per_tile = min_bpt;
    c.stages = 4;
    for (;;) {
        c.smem = gemv_smem_plan(groups, mrows, c.blocks_per_tile, c.stages, pro, epi).total;
        if (c.smem <= kGemvSmemBudget)
            break;
        if (c.stages > 2)
            --c.stages;
        else if (c.blocks_per_tile > min_bpt)
            c.blocks_per_tile /= 2;
        else
            break;
    }
    const GemvFn fn = gemv_fn(pro, epi);
    // The attribute is per function, shared by every matrix's launches.
    cudaFuncSetAttribute((const void*)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemvSmemBudget);
    const uint32_t mchunks = (m + kRowsPerCta - 1) / kRowsPerCta;
    uint32_t slots = 1;
    // Every CTA repeats the prologue, so each should get one tile: widen the
    // tiles (up to one block per compute warp) until they fit in one wave; a
    // CTA with a single tile needs only two ring stages.
    auto occupancy = [&](size_t smem) {
        int occ = 1;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, (const void*)fn, (int)(kComputeWarps + 1) * 32,
                                                          smem) != cudaSuccess ||
            occ < 1)
            occ = 1;
        const uint32_t sl = (uint32_t)sm_count * (uint32_t)occ;
        return sl > mchunks ? sl / mchunks : 1u;
    };
    for (uint32_t bpt = c.blocks_per_tile;; bpt *= 2) {
        const uint32_t tiles = (nblocks + bpt - 1) / bpt;
        const size_t smem2 = gemv_smem_plan(groups, mrows, bpt, 2, pro, epi).total;
        if (smem2 > kGemvSmemBudget)
            break;
        const uint32_t sl = occupancy(smem2);
        if (tiles <= sl) {
            c.blocks_per_tile = bpt;
            c.stages = 2;
            c.smem = smem2;
            break;
        }
        if (bpt >= kComputeWarps)
            break;
    }
    c.tiles = (nblocks + c.blocks_per_tile - 1) / c.blocks_per_tile;
    slots = occupancy(c.smem);
    if (c.tiles > slots) {
        // CTAs loop over several tiles (large matrices): the shallowest ring
        // that gives the most CTAs per SM (more warps hide the dot latency;
        // the bytes in flight per SM stay the same)
        for (uint32_t st = 2; st < c.stages; ++st) {
            const size_t sm2 = gemv_smem_plan(groups, mrows, c.blocks_per_tile, st, pro, epi).total;
            const uint32_t sl = occupancy(sm2);
            if (sl > slots) {
                c.stages = st;
                c.smem = sm2;
                slots = sl;
                break;
            }
        }
    }
    c.grid_x = c.tiles < slots ? c.tiles : slots;
    c.gc = 0;
    if (groups == kGemvFixedGroups && gemv_one_row_lanes(groups, mrows, c.blocks_per_tile, epi)) {
        const GemvFn fixed = gemv_fn_fixed(pro, epi);
        if (fixed != nullptr &&
            cudaFuncSetAttribute((const void*)fixed, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kGemvSmemBudget) == cudaSuccess)
            c.gc = (int)kGemvFixedGroups;
        cudaGetLastError();
    }
    return c;
}

// Launches on `s`; with pdl the launch may overlap the previous kernel of the
// stream (the kernel waits for it before touching activations).
inline cudaError_t launch_gemv(const GemvLaunch& c, uint32_t m, const GemvArgs& a, cudaStream_t s, bool pdl) {
    const GemvFn fn = gemv_fn(c.pro, c.epi, c.gc);
    if (!fn)
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c.grid_x, (m + kRowsPerCta - 1) / kRowsPerCta);
    cfg.blockDim = dim3((kComputeWarps + 1) * 32);
    cfg.dynamicSmemBytes = c.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, fn, a);
}

}  // namespace bnn
