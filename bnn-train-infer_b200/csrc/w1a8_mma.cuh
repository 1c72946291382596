// w1a8_mma.cuh - the W1A8 contraction for many activation rows on the
// 5th-generation tensor cores (ComputeRow, soft-bnn-accelerator.c:219-276).
//
// With weights w in {-1, +1} and int8 activations q, the reference's group
// dot D = 2 * pos - total (soft :251-258) is exactly sum_k w_k * q_k, an int8
// x int8 product with an int32 sum. So a tile of 128 activation rows x NT
// (128, or 64 when 128-wide tiles would leave SMs idle) output rows runs as tcgen05.mma kind::i8 (A = q, B = +-1, both K-major,
// 128-byte swizzle), four K=32 instructions per 128-wide group, each group
// into its own TMEM accumulator (NT columns). Groups are processed in chunks
// of kMmaChunk, double-buffered in TMEM (2 x 2 x NT columns), so the
// MMAs of one chunk overlap the epilogue of the previous one. The epilogue
// reads D per group with tcgen05.ld and does the reference's FP32 work in
// its order: acc = fl(acc + fl(F32(scale_g) * D_g)) for increasing g, then
// Y = fl(acc * s) (F32 ops) or Z = acc (I8 ops); DOT_GROUPS stores (int16)D.
// D (|D| <= 16256) becomes a float exactly through the 1.5 * 2^23 bias, and
// the multiply and the add run two columns at a time (f32x2, round to
// nearest, per element exactly the scalar operations).
//
// Operands in shared memory:
//   A  the prep kernel writes the quantised rows pre-tiled: block (m_tile, g)
//      is the 16 KB 128B-swizzled K-major image of 128 rows x 128 bytes, so
//      one 1D bulk copy per group fills a ring stage;
//   B  the epilogue warps fetch each chunk's weight bits and scales (the
//      w1a8_gemv.cuh 8-row block layout) from global memory one chunk ahead,
//      expand the bits to +-1 bytes in the swizzled layout and convert the
//      scales to FP32 once per tile.
//
// Warp roles (320 threads): warp 0 streams the A copies, warp 1 owns the
// TMEM allocation and one of its lanes issues the MMAs, warps 2-9 expand B
// and run the epilogue (warp w reads TMEM lanes 32 * (w % 4) .. + 31, i.e.
// tile rows, and half (w - 2) / 4 of the tile's columns). Every wait is
// bounded; a timeout sets the status word, and the TMEM is released only
// after a final commit shows every issued MMA completed.
#pragma once

#include <cstdint>
#include "bnn_device.cuh"
#include "bnn_sync.cuh"
#include "w1a8_gemv.cuh"

namespace bnn {

constexpr uint32_t kMmaM = 128;                      // activation rows per tile (TMEM lanes)
constexpr uint32_t kMmaN = 128;                      // output rows per tile, wide form (16 weight blocks)
constexpr uint32_t kMmaNarrow = 64;                  // narrow form, for matrices that give few wide tiles
constexpr uint32_t kMmaChunk = 2;                    // groups per TMEM buffer
constexpr uint32_t kMmaStages = 4;                   // A ring depth
constexpr uint32_t kMmaATile = kMmaM * kGroup;       // 16 KB: one group of 128 rows
constexpr uint32_t kMmaEpiWarps = 8;                 // two per TMEM lane quadrant
constexpr uint32_t kMmaThreads = 64 + kMmaEpiWarps * 32;
constexpr uint32_t kMmaEpiThreads = kMmaEpiWarps * 32;
constexpr uint32_t kMmaMinRows = 64;                 // BNN_Execute's tensor-core threshold
static_assert(kMmaChunk * kMmaN == kMmaEpiThreads, "at most one B row-group per epilogue thread and chunk");

// Instruction descriptor: D s32, A and B signed 8-bit, both K-major, N, M.
__host__ __device__ constexpr uint32_t mma_idesc(uint32_t n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((kMmaM >> 4) << 24);
}

// Byte offset of activation (row, group g, 16-byte chunk c) in the pre-tiled A.
__host__ __device__ inline size_t mma_a_offset(uint32_t row, uint32_t g, uint32_t groups, uint32_t c) {
    const uint32_t mt = row / kMmaM, r = row % kMmaM;
    return ((size_t)mt * groups + g) * kMmaATile + (r / 8u) * 1024u + (r % 8u) * 128u + ((c ^ (r % 8u)) * 16u);
}

inline size_t mma_a_bytes(uint32_t rows, uint32_t groups) {
    return (size_t)((rows + kMmaM - 1) / kMmaM) * groups * kMmaATile;
}

struct MmaArgs {
    const unsigned char* wblocks;  // packed 8-row blocks, padded to 4 blocks
    uint32_t n, groups, m;         // output rows, K/128, activation rows of this launch
    const unsigned char* a_sw;     // pre-tiled int8 activations of this launch
    const float* row_scale;        // [M], or nullptr: the I8 ops return Z unscaled
    unsigned char* out;            // first logical output row
    size_t out_stride;             // bytes between output rows
    int epi;                       // kEpiView, kEpiDotGroups; engine prefill: kEpiResidual
                                   // (out = fl(out + Y), 4-byte aligned F32 rows) or kEpiSwiGLU
                                   // (gate/up interleaved by 8-row blocks, out = h rows)
    int* status;
};

struct MmaSmem {
    size_t a, b, sf, bars, total;
};

__host__ __device__ inline MmaSmem mma_smem_plan(uint32_t nt) {
    MmaSmem p;
    p.a = 0;
    p.b = p.a + (size_t)kMmaStages * kMmaATile;
    p.sf = p.b + (size_t)2 * kMmaChunk * nt * kGroup;       // FP32 scales [2][kMmaChunk][nt]
    p.bars = p.sf + (size_t)2 * kMmaChunk * nt * 4u;
    p.total = p.bars + 256 + 1024;  // barriers and words, plus slack to 1024-align the base
    return p;
}

// ---- tcgen05 primitives (inline PTX)
__device__ __forceinline__ uint64_t mma_smem_desc(uint32_t saddr) {
    // K-major, 128-byte swizzle: 8-row groups 1024 B apart (SBO), LBO 16 B
    // (unused for this layout), descriptor version 1, layout type 2
    const uint32_t lo = ((saddr >> 4) & 0x3fffu) | (1u << 16);
    const uint32_t hi = (1024u >> 4) | (1u << 14) | (2u << 29);
    return ((uint64_t)hi << 32) | lo;
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t accumulate, uint32_t idesc) {
    const uint32_t mask = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(mask));
}

// Arrives on `bar` once every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive TMEM columns of this warp's 32 lanes; complete after tmem_wait().
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* v) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Two-wide FP32 arithmetic, round to nearest even per element (sm_100).
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    return (uint64_t)__float_as_uint(lo) | ((uint64_t)__float_as_uint(hi) << 32);
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// Four weight bits (LSB first) as four bytes: +1 for a set bit, -1 otherwise.
__device__ __forceinline__ uint32_t expand_signs4(uint32_t v) {
    const uint32_t b = (v * 0x00204081u) & 0x01010101u;  // byte i = bit i
    return (b * 0xfeu) ^ 0xffffffffu;
}

// Grid (ceil(N / NT), ceil(M / 128)); kMmaThreads threads; mma_smem_plan(NT).total
// bytes of dynamic shared memory.
template <uint32_t NT>
static __global__ void __launch_bounds__(kMmaThreads, 1) w1a8_mma_kernel(MmaArgs a) {
    constexpr uint32_t kMmaBTile = NT * kGroup;             // one group of NT rows as +-1 bytes
    constexpr uint32_t kMmaCols = NT / (kMmaEpiWarps / 4);  // columns per epilogue thread
    constexpr uint32_t kMmaTmemCols = 2 * kMmaChunk * NT;   // 512 or 256
    constexpr uint32_t kFetchThreads = kMmaChunk * NT;      // one B row-group each per chunk
    constexpr uint32_t kIdesc = mma_idesc(NT);
    extern __shared__ __align__(1024) unsigned char mma_smem_raw[];
    // the swizzle pattern follows shared-memory address bits: 1024-align the base
    const uint32_t raw = smem_addr(mma_smem_raw);
    unsigned char* sm = mma_smem_raw + (((raw + 1023u) & ~1023u) - raw);
    const uint32_t G = a.groups;
    const MmaSmem plan = mma_smem_plan(NT);
    unsigned char* a_ring = sm + plan.a;
    unsigned char* b_buf = sm + plan.b;
    float* sf = reinterpret_cast<float*>(sm + plan.sf);  // [2][kMmaChunk][NT]
    uint64_t* afull = reinterpret_cast<uint64_t*>(sm + plan.bars);
    uint64_t* aempty = afull + kMmaStages;
    uint64_t* bready = aempty + kMmaStages;
    uint64_t* dready = bready + 2;
    uint64_t* tfree = dready + 2;
    uint64_t* mdone = tfree + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + 1);

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t nt = blockIdx.x, mt = blockIdx.y;
    const uint32_t nchunks = (G + kMmaChunk - 1) / kMmaChunk;
    const uint32_t nblocks = (a.n + kRowBlock - 1) / kRowBlock;  // weight blocks that exist

    if (*a.status != 0)
        return;  // an input row was rejected: no output is written

    if (tid == 0) {
        for (uint32_t s = 0; s < kMmaStages; ++s) {
            mbar_init(&afull[s], 1);
            mbar_init(&aempty[s], 1);
        }
        for (uint32_t b = 0; b < 2; ++b) {
            mbar_init(&bready[b], kMmaEpiThreads);
            mbar_init(&dready[b], 1);
            mbar_init(&tfree[b], kMmaEpiThreads);
        }
        mbar_init(mdone, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(kMmaTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---- producer: one A block per group
        if (lane == 0) {
            uint32_t g = 0;
            for (; g < G; ++g) {
                const uint32_t s = g % kMmaStages;
                if (g >= kMmaStages && !mbar_wait(&aempty[s], ((g / kMmaStages) - 1) & 1)) {
                    atomicOr(a.status, kStatusTimeout);
                    break;
                }
                mbar_arrive_expect_tx(&afull[s], kMmaATile);
                bulk_g2s(a_ring + (size_t)s * kMmaATile, a.a_sw + ((size_t)mt * G + g) * kMmaATile, kMmaATile,
                         &afull[s]);
            }
            // no copy may still be in flight when the CTA exits
            for (uint32_t j = g > kMmaStages ? g - kMmaStages : 0; j < g; ++j)
                if (!mbar_wait(&afull[j % kMmaStages], (j / kMmaStages) & 1))
                    atomicOr(a.status, kStatusTimeout);
        }
    } else if (warp == 1) {
        // ---- MMA issuer
        if (lane == 0) {
            for (uint32_t c = 0; c < nchunks; ++c) {
                const uint32_t b = c & 1;
                bool ok = mbar_wait(&bready[b], (c >> 1) & 1);
                if (ok && c >= 2)
                    ok = mbar_wait(&tfree[b], ((c >> 1) - 1) & 1);
                if (!ok) {
                    atomicOr(a.status, kStatusTimeout);
                    break;
                }
                tc_fence_after();
                const uint32_t g0 = c * kMmaChunk, gn = min(kMmaChunk, G - g0);
                for (uint32_t gi = 0; gi < gn; ++gi) {
                    const uint32_t g = g0 + gi, s = g % kMmaStages;
                    if (!mbar_wait(&afull[s], (g / kMmaStages) & 1)) {
                        atomicOr(a.status, kStatusTimeout);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_base = smem_addr(a_ring + (size_t)s * kMmaATile);
                    const uint32_t b_base = smem_addr(b_buf + (size_t)(b * kMmaChunk + gi) * kMmaBTile);
                    const uint32_t d = tmem + (b * kMmaChunk + gi) * NT;
#pragma unroll
                    for (uint32_t k = 0; k < kGroup / 32; ++k)
                        mma_i8(d, mma_smem_desc(a_base + 32u * k), mma_smem_desc(b_base + 32u * k), k, kIdesc);
                    mma_commit(&aempty[s]);  // the A stage is free once these MMAs have read it
                }
                if (!ok)
                    break;
                mma_commit(&dready[b]);
            }
            mma_commit(mdone);  // completes when every MMA issued above has completed
        }
        __syncwarp();
    } else {
        // ---- warps 2..9: fetch + expand B chunks, then the ordered FP32 epilogue
        const uint32_t et = tid - 64;                    // 0..255
        const uint32_t quad = warp & 3;                  // TMEM lane quadrant this warp may read
        const uint32_t half = (warp - 2) >> 2;           // which half of the tile's columns
        const uint32_t row = quad * 32 + lane;           // tile row = TMEM lane
        const uint32_t m = mt * kMmaM + row;
        const uint32_t col0 = half * kMmaCols;           // first tile column of this thread
        const bool dot_groups = a.epi == kEpiDotGroups;
        const bool live = m < a.m;
        // B fetch of one chunk: thread et owns (group gi = et / 128, tile row n = et % 128):
        // 16 bytes of sign bits, and the scale of that row and group
        const bool fetcher = et < kFetchThreads;        // the others only arrive on bready
        const uint32_t fgi = fetcher ? et / NT : 0, fn = et % NT;
        const uint32_t fblk = nt * (NT / kRowBlock) + fn / kRowBlock, fr = fn % kRowBlock;
        const unsigned char* fbase = a.wblocks + (size_t)fblk * G * 144u;
        uint4 fbits = make_uint4(0u, 0u, 0u, 0u);
        uint16_t fscale = 0;
        auto fetch = [&](uint32_t c) {
            const uint32_t g = c * kMmaChunk + fgi;
            fbits = make_uint4(0u, 0u, 0u, 0u);
            fscale = 0;
            if (fetcher && fblk < nblocks && g < G) {
                fbits = *reinterpret_cast<const uint4*>(fbase + (size_t)g * 128u + fr * 16u);
                fscale = *reinterpret_cast<const uint16_t*>(fbase + (size_t)G * 128u + ((size_t)fr * G + g) * 2u);
            }
        };
        auto expand = [&](uint32_t c) {
            const uint32_t b = c & 1;
            if (!fetcher) {
                mbar_arrive(&bready[b]);
                return;
            }
            unsigned char* dst =
                b_buf + (size_t)(b * kMmaChunk + fgi) * kMmaBTile + (fn / 8u) * 1024u + (fn % 8u) * 128u;
            const uint32_t w[4] = {fbits.x, fbits.y, fbits.z, fbits.w};
#pragma unroll
            for (uint32_t j = 0; j < 8; ++j) {  // 16-byte chunk j of the row: bits 16j .. 16j + 15
                const uint32_t bits = (w[j >> 1] >> ((j & 1u) * 16u)) & 0xffffu;
                uint4 o;
                o.x = expand_signs4(bits & 0xfu);
                o.y = expand_signs4((bits >> 4) & 0xfu);
                o.z = expand_signs4((bits >> 8) & 0xfu);
                o.w = expand_signs4(bits >> 12);
                *reinterpret_cast<uint4*>(dst + ((j ^ (fn % 8u)) * 16u)) = o;
            }
            sf[(b * kMmaChunk + fgi) * NT + fn] = h2f(fscale);
            fence_proxy_async();  // the MMAs read these bytes through the async proxy
            mbar_arrive(&bready[b]);
        };
        fetch(0);
        expand(0);
        if (nchunks > 1) {
            fetch(1);
            expand(1);
        }
        uint64_t acc[kMmaCols / 2];
#pragma unroll
        for (uint32_t j = 0; j < kMmaCols / 2; ++j)
            acc[j] = 0ull;
        bool ok = true;
        const uint64_t bias2 = f2_pack(-12582912.0f, -12582912.0f);  // -1.5 * 2^23
        for (uint32_t c = 0; c < nchunks; ++c) {
            const uint32_t b = c & 1, g0 = c * kMmaChunk, gn = min(kMmaChunk, G - g0);
            if (c + 2 < nchunks)
                fetch(c + 2);  // global loads in flight during this chunk's epilogue
            if (ok && !mbar_wait(&dready[b], (c >> 1) & 1)) {
                atomicOr(a.status, kStatusTimeout);
                ok = false;
            }
            tc_fence_after();
            for (uint32_t gi = 0; gi < gn && ok; ++gi) {
                uint32_t d[kMmaCols];
                const uint32_t taddr = tmem + ((quad * 32u) << 16) + (b * kMmaChunk + gi) * NT + col0;
#pragma unroll
                for (uint32_t q = 0; q < kMmaCols / 32; ++q)
                    tmem_ld32(taddr + 32u * q, d + 32 * q);
                tmem_wait();
                const uint32_t g = g0 + gi;
                if (dot_groups) {
                    if (live)
#pragma unroll
                        for (uint32_t j = 0; j < kMmaCols; ++j) {
                            const uint32_t on = nt * NT + col0 + j;
                            if (on < a.n)
                                store_i16_any(a.out + (size_t)m * a.out_stride + ((size_t)on * G + g) * 2u,
                                              (int16_t)(int32_t)d[j]);
                        }
                } else {
                    const float4* sc4 = reinterpret_cast<const float4*>(sf + (b * kMmaChunk + gi) * NT + col0);
#pragma unroll
                    for (uint32_t q = 0; q < kMmaCols / 4; ++q) {
                        const float4 sc = sc4[q];
                        // D + 1.5 * 2^23 as float bits, minus the bias: D exactly
                        const uint64_t d01 = f2_add(f2_pack(__int_as_float((int)d[4 * q] + 0x4b400000),
                                                            __int_as_float((int)d[4 * q + 1] + 0x4b400000)),
                                                    bias2);
                        const uint64_t d23 = f2_add(f2_pack(__int_as_float((int)d[4 * q + 2] + 0x4b400000),
                                                            __int_as_float((int)d[4 * q + 3] + 0x4b400000)),
                                                    bias2);
                        acc[2 * q] = f2_add(acc[2 * q], f2_mul(f2_pack(sc.x, sc.y), d01));
                        acc[2 * q + 1] = f2_add(acc[2 * q + 1], f2_mul(f2_pack(sc.z, sc.w), d23));
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&tfree[b]);
            if (c + 2 < nchunks) {
                // every epilogue thread is done with sf[b] before it is rewritten
                asm volatile("bar.sync 1, %0;" ::"r"(kMmaEpiThreads) : "memory");
                expand(c + 2);  // buffer b is free: the MMAs of chunk c have completed
            }
        }
        if (ok && live && !dot_groups) {
            const float s = a.row_scale ? a.row_scale[m] : 1.0f;
            const uint64_t s2 = f2_pack(s, s);
            float y[kMmaCols];
#pragma unroll
            for (uint32_t j = 0; j < kMmaCols / 2; ++j) {
                const uint64_t v = a.row_scale ? f2_mul(acc[j], s2) : acc[j];
                y[2 * j] = f2_lo(v);
                y[2 * j + 1] = f2_hi(v);
            }
            unsigned char* orow = a.out + (size_t)m * a.out_stride;
            const uint32_t n0 = nt * NT + col0;
            if (a.epi == kEpiSwiGLU) {
                // weight blocks 2k (gate rows) and 2k + 1 (up rows) hold the same
                // 8 FFN rows: h[k * 8 + r] (w1a8_gemv.cuh)
#pragma unroll
                for (uint32_t p = 0; p < kMmaCols / 16; ++p)
#pragma unroll
                    for (uint32_t r = 0; r < kRowBlock; ++r) {
                        if (n0 + 16u * p + r >= a.n)
                            continue;
                        const float gv = y[16 * p + r], uv = y[16 * p + 8 + r];
                        const float silu = __fdiv_rn(gv, __fadd_rn(1.0f, expf_cr(-gv)));
                        reinterpret_cast<float*>(orow)[(n0 / 16u + p) * kRowBlock + r] = __fmul_rn(silu, uv);
                    }
            } else if (a.epi == kEpiResidual) {
                float* dst = reinterpret_cast<float*>(orow) + n0;
#pragma unroll
                for (uint32_t j = 0; j < kMmaCols; ++j)
                    if (n0 + j < a.n)
                        dst[j] = __fadd_rn(dst[j], y[j]);  // x = fl(x + Y)
            } else if (n0 + kMmaCols <= a.n && ((reinterpret_cast<uintptr_t>(orow) + n0 * 4u) & 15u) == 0) {
                float4* dst = reinterpret_cast<float4*>(orow + (size_t)n0 * 4u);
#pragma unroll
                for (uint32_t q = 0; q < kMmaCols / 4; ++q)
                    dst[q] = make_float4(y[4 * q], y[4 * q + 1], y[4 * q + 2], y[4 * q + 3]);
            } else {
#pragma unroll
                for (uint32_t j = 0; j < kMmaCols; ++j)
                    if (n0 + j < a.n)
                        store_f32_any(orow + (size_t)(n0 + j) * 4u, y[j]);
            }
        }
    }

    // ---- teardown: TMEM reads are done; free TMEM after every MMA completed
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        if (!mbar_wait(mdone, 0) && lane == 0)
            atomicOr(a.status, kStatusTimeout);
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kMmaTmemCols));
    }
}

// Launches the contraction of `a.m` rows (a.m <= 65535 * kMmaM) on `s`:
// 128-wide tiles, or 64-wide when the wide grid would leave SMs idle on a
// device of `sms` streaming multiprocessors.
inline cudaError_t launch_mma(const MmaArgs& a, int sms, cudaStream_t s) {
    const uint32_t mtiles = (a.m + kMmaM - 1) / kMmaM;
    const bool narrow = (size_t)((a.n + kMmaN - 1) / kMmaN) * mtiles < (size_t)sms;
    const uint32_t nt = narrow ? kMmaNarrow : kMmaN;
    const MmaSmem p = mma_smem_plan(nt);
    const void* fn = narrow ? (const void*)w1a8_mma_kernel<kMmaNarrow> : (const void*)w1a8_mma_kernel<kMmaN>;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.total);
    if (e != cudaSuccess)
        return e;
    const dim3 grid((a.n + nt - 1) / nt, mtiles);
    if (narrow)
        w1a8_mma_kernel<kMmaNarrow><<<grid, kMmaThreads, p.total, s>>>(a);
    else
        w1a8_mma_kernel<kMmaN><<<grid, kMmaThreads, p.total, s>>>(a);
    return cudaGetLastError();
}

}  // namespace bnn
