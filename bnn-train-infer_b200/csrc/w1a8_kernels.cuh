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
#include "bnn_sync.cuh"

namespace bnn {

enum InputKind : int { kInputI8 = 1, kInputF32 = 2 };

constexpr int kPrepThreads = 256;
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
    const uint4* wbits;       // repacked weight blocks, padded to whole tiles
    const uint16_t* scales;   // [N][G] binary16
    const uint32_t* act;      // [M][G][32]
    const int32_t* totals;    // [M][G]
    const float* row_scale;   // [M] (F32 ops) or nullptr (I8 ops return Z)
    int* status;              // non-zero on entry: a prep CTA rejected its row
    uint32_t n, groups, m;
    unsigned char* out;       // first logical output row (buffer base + view offset)
    size_t out_stride;
    const float* residual;    // MODE 1: if set, Y = fl(residual + Y) (same layout as out)
    uint32_t tiles;           // tiles of `consumers` 8-row blocks
    uint32_t stages;          // depth of the shared-memory weight ring
};

// Integer part for one (row, group) unit: returns D for one activation row.
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
    // 128 * pos = sum_j acc_j * 2^(7-j): acc_j is an exact multiple of 2^j.
    int pos128 = acc[7];
#pragma unroll
    for (int j = 6; j >= 0; --j)
        pos128 += acc[j] << (7 - j);
    return (pos128 >> 6) - total;  // D = 2 * pos - total
}

// Shared-memory plan of the contraction kernel (see w1a8_contract_kernel).
struct ContractSmem {
    size_t bars, act, tot, dsm, stage, total;
};

__host__ __device__ inline ContractSmem contract_smem_plan(uint32_t groups, uint32_t mrows,
                                                          uint32_t consumers, uint32_t stages,
                                                          int mode) {
    ContractSmem p;
    p.bars = 0;
    p.act = 128;
    p.tot = p.act + (size_t)mrows * groups * kActStride * 4u;
    p.dsm = p.tot + (size_t)mrows * groups * 4u;
    size_t dsm_bytes = mode == 1 ? (size_t)consumers * mrows * kRowBlock * groups * 2u : 0;
    p.stage = (p.dsm + dsm_bytes + 127) & ~(size_t)127;
    p.total = p.stage + (size_t)stages * consumers * groups * kRowBlock * 16u;
    return p;
}

// Persistent W1A8 contraction.
//
// Grid: x = persistent CTAs striding over weight tiles, y = chunks of
// kRowsPerCta activation rows. Block: `consumers` compute warps + 1 producer
// warp. A tile is `consumers` consecutive 8-row weight blocks (contiguous in
// the repacked layout); the producer streams tiles into a `stages`-deep
// shared-memory ring with 1D bulk copies (TMA), and consumer warp w computes
// block w of each tile:
//   lanes (r = lane % 8, g = 4q + lane / 8) take one 16-byte (row, group)
//   unit per step; activation words are broadcast reads from shared memory;
//   the group dots D go to a per-warp shared array, and lanes then run the
//   ordered FP32 scale-accumulate of one (activation row, output row) each.
// MODE 0 writes DOT_GROUPS (int16 [M][N][G]) directly; MODE 1 writes FP32.
template <int MODE>
__global__ void w1a8_contract_kernel(ContractArgs a) {
    if (*a.status != 0)
        return;  // a rejected input leaves the output untouched
    extern __shared__ __align__(128) unsigned char c_smem[];
    const uint32_t G = a.groups;
    const uint32_t nwarps = blockDim.x / 32, consumers = nwarps - 1;
    const uint32_t m0 = blockIdx.y * kRowsPerCta;
    const uint32_t mrows = min((uint32_t)kRowsPerCta, a.m - m0);
    const ContractSmem plan = contract_smem_plan(G, mrows, consumers, a.stages, MODE);
    uint64_t* full = reinterpret_cast<uint64_t*>(c_smem + plan.bars);
    uint64_t* empty = full + a.stages;
    uint32_t* act_s = reinterpret_cast<uint32_t*>(c_smem + plan.act);
    int32_t* tot_s = reinterpret_cast<int32_t*>(c_smem + plan.tot);
    int16_t* dsm = reinterpret_cast<int16_t*>(c_smem + plan.dsm);
    unsigned char* stage0 = c_smem + plan.stage;
    const uint32_t tile_bytes = consumers * G * kRowBlock * 16u;
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    if (tid == 0) {
        for (uint32_t s = 0; s < a.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], consumers);
        }
        fence_barrier_init();
    }
    for (uint32_t i = tid; i < mrows * G * (kWordsPerGroup / 4); i += blockDim.x) {
        uint32_t mm = i / (G * 8), rest = i % (G * 8), g = rest / 8, c = rest % 8;
        const uint4* src = reinterpret_cast<const uint4*>(a.act + ((size_t)(m0 + mm) * G + g) * kWordsPerGroup);
        reinterpret_cast<uint4*>(act_s + (mm * G + g) * kActStride)[c] = src[c];
    }
    for (uint32_t i = tid; i < mrows * G; i += blockDim.x)
        tot_s[i] = a.totals[(size_t)m0 * G + i];
    __syncthreads();  // the only CTA-wide barrier

    if (warp == consumers) {  // producer warp
        if (lane == 0) {
            uint32_t i = 0;
            bool ok = true;
            for (uint32_t tile = blockIdx.x; tile < a.tiles && ok; tile += gridDim.x, ++i) {
                const uint32_t s = i % a.stages;
                if (i >= a.stages && !mbar_wait(&empty[s], ((i / a.stages) - 1) & 1)) {
                    atomicOr(a.status, kStatusTimeout);
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&full[s], tile_bytes);
                bulk_g2s(stage0 + (size_t)s * tile_bytes,
                         reinterpret_cast<const unsigned char*>(a.wbits) + (size_t)tile * tile_bytes,
                         tile_bytes, &full[s]);
            }
            // No bulk copy may still be in flight when the CTA exits.
            for (uint32_t j = i > a.stages ? i - a.stages : 0; j < i; ++j)
                if (!mbar_wait(&full[j % a.stages], (j / a.stages) & 1))
                    atomicOr(a.status, kStatusTimeout);
        }
        return;
    }

    const uint32_t r = lane & 7;
    int16_t* my_d = dsm + (size_t)warp * mrows * kRowBlock * G;
    uint32_t i = 0;
    for (uint32_t tile = blockIdx.x; tile < a.tiles; tile += gridDim.x, ++i) {
        const uint32_t s = i % a.stages;
        const bool ready = mbar_wait(&full[s], (i / a.stages) & 1);
        if (!ready && lane == 0)
            atomicOr(a.status, kStatusTimeout);
        const uint32_t blk = tile * consumers + warp;  // global 8-row block
        const uint4* wt = reinterpret_cast<const uint4*>(stage0 + (size_t)s * tile_bytes) +
                          (size_t)warp * G * kRowBlock;
        if (ready) {
            for (uint32_t q = 0; q * 4 < G; ++q) {
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
                    if (MODE == 0) {
                        if (n < a.n)
                            store_i16_any(a.out + (size_t)(m0 + mm) * a.out_stride +
                                              ((size_t)n * G + g) * 2u,
                                          (int16_t)d);
                    } else {
                        my_d[(mm * kRowBlock + r) * G + g] = (int16_t)d;
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0)
            mbar_arrive(&empty[s]);  // weights of this stage are no longer read
        if (MODE == 1 && ready) {
            // Ordered FP32 scale-accumulate (soft :260-274): one lane per
            // (activation row, output row), groups in increasing order.
            for (uint32_t p = lane; p < mrows * kRowBlock; p += 32) {
                const uint32_t mm = p / kRowBlock, rr = p % kRowBlock;
                const uint32_t n = blk * kRowBlock + rr;
                if (n >= a.n)
                    continue;
                const uint16_t* sc = a.scales + (size_t)n * G;
                const int16_t* dd = my_d + (mm * kRowBlock + rr) * G;
                float acc = 0.0f;
#pragma unroll 8
                for (uint32_t g = 0; g < G; ++g)
                    acc = __fadd_rn(acc, __fmul_rn(h2f(__ldg(sc + g)), (float)dd[g]));
                if (a.row_scale)
                    acc = __fmul_rn(acc, a.row_scale[m0 + mm]);
                unsigned char* dst = a.out + (size_t)(m0 + mm) * a.out_stride + (size_t)n * 4u;
                if (a.residual)
                    acc = __fadd_rn(*reinterpret_cast<const float*>(
                                        reinterpret_cast<const unsigned char*>(a.residual) +
                                        (dst - a.out)),
                                    acc);
                store_f32_any(dst, acc);
            }
        }
        __syncwarp();
    }
}

// Repack the public [N][K/8] bit layout into 8-row blocks (see header).
// One thread per 16-byte (row, group) chunk; rows past N (up to `nblocks`
// whole blocks, the allocation's padding) are zero.
static __global__ void w1a8_repack_kernel(const uint8_t* __restrict__ bits, uint32_t n, uint32_t groups,
                                   size_t nblocks, uint4* __restrict__ out) {
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

// Weight blocks are allocated in multiples of this many 8-row blocks so a
// tile of 1, 2 or 4 consumer blocks never reads past the allocation.
constexpr uint32_t kBlockPad = 4;

inline size_t prep_smem_bytes(uint32_t k) { return (size_t)k * 5u; }

// Launch shape of the contraction kernel for one matrix and row count.
struct ContractLaunch {
    uint32_t consumers, stages, tiles, grid_x;
    size_t smem;
    int mode;
};

// Picks consumer warps (8-row blocks per tile) so small matrices still
// spread over every SM, a ring depth that fits shared memory, and a
// persistent grid sized from the occupancy of that configuration.
inline ContractLaunch plan_contract(int sm_count, uint32_t n, uint32_t groups, uint32_t m, int mode) {
    constexpr size_t kSmemBudget = 200u * 1024u;
    const uint32_t nblocks = (n + kRowBlock - 1) / kRowBlock;
    const uint32_t mrows = m < (uint32_t)kRowsPerCta ? m : (uint32_t)kRowsPerCta;
    ContractLaunch c;
    c.mode = mode;
    c.consumers = nblocks >= 8u * sm_count ? 4u : (nblocks >= 2u * sm_count ? 2u : 1u);
    c.stages = 4;
    for (;;) {
        c.smem = contract_smem_plan(groups, mrows, c.consumers, c.stages, mode).total;
        if (c.smem <= kSmemBudget)
            break;
        if (c.stages > 2)
            --c.stages;
        else if (c.consumers > 1)
            c.consumers /= 2;
        else
            break;
    }
    c.tiles = (nblocks + c.consumers - 1) / c.consumers;
    int occ = 1;
    const void* fn = mode == 0 ? (const void*)w1a8_contract_kernel<0> : (const void*)w1a8_contract_kernel<1>;
    // The attribute is per function, shared by every matrix's launches: set it
    // to the whole budget rather than this plan's need.
    cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBudget);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, (int)(c.consumers + 1) * 32, c.smem) != cudaSuccess ||
        occ < 1)
        occ = 1;
    const uint32_t mchunks = (m + kRowsPerCta - 1) / kRowsPerCta;
    uint32_t slots = (uint32_t)sm_count * (uint32_t)occ;
    slots = slots > mchunks ? slots / mchunks : 1u;
    c.grid_x = c.tiles < slots ? c.tiles : slots;
    return c;
}

inline cudaError_t launch_contract(const ContractLaunch& c, uint32_t mchunks, int mode,
                                   const ContractArgs& a, cudaStream_t s) {
    dim3 grid(c.grid_x, mchunks), block((c.consumers + 1) * 32);
    if (mode == 0)
        w1a8_contract_kernel<0><<<grid, block, c.smem, s>>>(a);
    else
        w1a8_contract_kernel<1><<<grid, block, c.smem, s>>>(a);
    return cudaGetLastError();
}

}  // namespace bnn
