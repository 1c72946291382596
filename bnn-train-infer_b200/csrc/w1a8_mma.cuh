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
// D (|D| <= 16256) becomes a float exactly through the 1.5 * 2^23 bias the
// accumulators start from, and the multiply and the add run two columns at a
// time (f32x2, round to nearest, per element exactly the scalar operations).
//
// Operands in shared memory:
//   A  the prep kernel writes the quantised rows pre-tiled: block (m_tile, g)
//      is the 16 KB 128B-swizzled K-major image of 128 rows x 128 bytes, so
//      one 1D bulk copy per group fills a ring stage;
//      (one copy of a chunk's kMmaChunk blocks; a single thread issues
//      every copy, so copies are few and large);
//   W  each expansion thread's own 16-byte rows of weight bits, fetched with
//      cp.async from the w1a8_gemv.cuh 8-row block layout kMmaXDepth chunks
//      ahead (private slots: no cross-thread hand-off);
//   B  the +-1 bytes expanded from W (a 16-entry table turns 4 bits into 4
//      bytes) in the swizzled layout, a ring of kMmaBBufs chunks;
//   the FP32 group scales of the whole tile, converted once.
//
// Warp roles (704 threads): warp 0 streams A with bulk copies, warp 1
// owns the TMEM allocation and one of its lanes issues the MMAs, warps 2-5
// fetch and expand W into B, warps 6-21 run the epilogue (warp w reads TMEM lanes
// 32 * (w % 4) .. + 31, i.e. tile rows, and quarter (w - 6) / 4 of the
// tile's columns). No warp on the MMA's critical path waits on a global
// load. Every accumulator starts at the bits of 1.5 * 2^23 (the epilogue
// rewrites them after each read), so a finished accumulator holds the float
// Db = 1.5 * 2^23 + D, and one packed FMA per two outputs,
// s * Db - s * 1.5 * 2^23, gives fl(scale * D) directly (the second product
// is exact and kept beside the scales). Every wait is bounded; a timeout sets the status word, and the
// TMEM is released only after a final commit shows every issued MMA
// completed.
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
constexpr uint32_t kMmaAStages = 3;                  // A ring depth (chunks of kMmaChunk groups)
constexpr uint32_t kMmaXDepth = 3;                   // chunks of weight bits in flight per expansion thread
constexpr uint32_t kMmaBBufs = 2;                    // expanded B ring depth (chunks)
constexpr uint32_t kMmaATile = kMmaM * kGroup;       // 16 KB: one group of 128 rows
constexpr uint32_t kMmaXWarps = 4;                   // B expansion
constexpr uint32_t kMmaEpiWarps = 16;                // four per TMEM lane quadrant
constexpr uint32_t kMmaXThreads = kMmaXWarps * 32;
constexpr uint32_t kMmaEpiThreads = kMmaEpiWarps * 32;
constexpr uint32_t kMmaEpiWarp0 = 2 + kMmaXWarps;    // first epilogue warp
constexpr uint32_t kMmaThreads = (kMmaEpiWarp0 + kMmaEpiWarps) * 32;
constexpr uint32_t kMmaMinRows = 64;                 // BNN_Execute's tensor-core threshold
// Every accumulator starts at 1.5 * 2^23 (as int32 bits): after the MMAs the
// word holds the float bits of 1.5 * 2^23 + D exactly (|D| <= 16256).
constexpr uint32_t kMmaBias = 0x4b400000u;
// Epilogue warp w reads TMEM lane quadrant w % 4: any four consecutive
// epilogue warps cover the four quadrants once (one column quarter).

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
    size_t a, b, w, sf, sb, bars, total;
};

// Shared memory of a tile of nt output rows over `groups` groups.
__host__ __device__ inline MmaSmem mma_smem_plan(uint32_t nt, uint32_t groups) {
    MmaSmem p;
    p.a = 0;                                                          // [kMmaAStages][kMmaChunk][16 KB]
    p.b = p.a + (size_t)kMmaAStages * kMmaChunk * kMmaATile;         // [kMmaBBufs][kMmaChunk][nt x 128 B]
    p.w = p.b + (size_t)kMmaBBufs * kMmaChunk * nt * kGroup;         // [kMmaXDepth][rows per thread][threads][16 B]
    p.sf = p.w + (size_t)kMmaXDepth * kMmaChunk * nt * 16u;          // FP32 scales s [groups][nt]
    p.sb = p.sf + (size_t)groups * nt * 4u;                           // -s * 1.5 * 2^23 [groups][nt]
    p.bars = p.sb + (size_t)groups * nt * 4u;
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

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* v) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// The same word x into 32 (16) consecutive TMEM columns of this warp's 32
// lanes; complete after tmem_wait_st().
__device__ __forceinline__ void tmem_fill32(uint32_t taddr, uint32_t x) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
        "%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr),
        "r"(x)
        : "memory");
}
__device__ __forceinline__ void tmem_fill16(uint32_t taddr, uint32_t x) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
        "%1};" ::"r"(taddr),
        "r"(x)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

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
// a * b + c, rounded once per element
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

// Four weight bits (LSB first) as four bytes: +1 for a set bit, -1 otherwise.
__device__ __forceinline__ uint32_t expand_signs4(uint32_t v) {
    const uint32_t b = (v * 0x00204081u) & 0x01010101u;  // byte i = bit i
    return (b * 0xfeu) ^ 0xffffffffu;
}

// h = fl(silu(g) * u) of the SwiGLU epilogue (qwen3.c:487-495), out of line:
// the correctly rounded exp needs registers the contraction loop does not have.
static __device__ __noinline__ float swiglu_one(float gv, float uv) {
    const float silu = __fdiv_rn(gv, __fadd_rn(1.0f, expf_cr(-gv)));
    return __fmul_rn(silu, uv);
}

// 16 bytes global -> shared, asynchronous (this thread's own copy; complete
// after cp_async_wait<n> leaves at most n newer commit groups pending).
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Grid (ceil(N / NT), ceil(M / 128)); kMmaThreads threads; mma_smem_plan(NT).total
// bytes of dynamic shared memory.
template <uint32_t NT>
static __global__ void __launch_bounds__(kMmaThreads, 1) w1a8_mma_kernel(MmaArgs a) {
    constexpr uint32_t kMmaBTile = NT * kGroup;             // one group of NT rows as +-1 bytes
    constexpr uint32_t kMmaCols = NT / (kMmaEpiWarps / 4);  // columns per epilogue thread (32 or 16)
    constexpr uint32_t kMmaTmemCols = 2 * kMmaChunk * NT;   // 512 or 256
    constexpr uint32_t kBlk = NT / kRowBlock;               // weight blocks per tile
    constexpr uint32_t kXRows = kMmaChunk * NT / kMmaXThreads;  // 16-byte weight rows per expansion thread
    constexpr uint32_t kAStage = kMmaChunk * kMmaATile;     // A bytes of one chunk
    constexpr uint32_t kIdesc = mma_idesc(NT);
    static_assert(kMmaCols == 32 || kMmaCols == 16, "TMEM access width");
    static_assert((kMmaChunk * NT) % kMmaXThreads == 0, "row-groups per expansion thread");
    extern __shared__ __align__(1024) unsigned char mma_smem_raw[];
    __shared__ uint32_t sign_lut[16];  // 4 weight bits -> 4 bytes of +-1
    // the swizzle pattern follows shared-memory address bits: 1024-align the base
    const uint32_t raw = smem_addr(mma_smem_raw);
    unsigned char* sm = mma_smem_raw + (((raw + 1023u) & ~1023u) - raw);
    const uint32_t G = a.groups;
    const MmaSmem plan = mma_smem_plan(NT, G);
    unsigned char* a_ring = sm + plan.a;
    unsigned char* b_ring = sm + plan.b;
    unsigned char* w_slots = sm + plan.w;
    float* sf = reinterpret_cast<float*>(sm + plan.sf);  // [G][NT] scales s
    float* sb = reinterpret_cast<float*>(sm + plan.sb);  // [G][NT] -s * 1.5 * 2^23, exact
    uint64_t* afull = reinterpret_cast<uint64_t*>(sm + plan.bars);
    uint64_t* aempty = afull + kMmaAStages;
    uint64_t* bready = aempty + kMmaAStages;
    uint64_t* bfree = bready + kMmaBBufs;
    uint64_t* dready = bfree + kMmaBBufs;
    uint64_t* tfree = dready + 2;
    uint64_t* sready = tfree + 2;
    uint64_t* mdone = sready + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + 1);

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t nt = blockIdx.x, mt = blockIdx.y;
    const uint32_t nchunks = (G + kMmaChunk - 1) / kMmaChunk;
    const uint32_t nblocks = (a.n + kRowBlock - 1) / kRowBlock;  // weight blocks that exist
    __shared__ int skip_cta;
    // With programmatic dependent launch the set-up below (barriers, TMEM,
    // the first weight bits) overlaps the previous kernel; nothing that an
    // earlier kernel writes is read before the grid-dependency wait.
    griddep_launch_dependents();

    // ---- warps 2..5: weight bits kMmaXDepth chunks ahead (each thread its
    // own kXRows 16-byte rows): where they come from and where they go
    const uint32_t xt = tid - 64;  // 0 .. kMmaXThreads - 1 on those warps
    auto row_src = [&](uint32_t c, uint32_t k, uint32_t* gi, uint32_t* n) -> const unsigned char* {
        const uint32_t rg = xt + k * kMmaXThreads;
        *gi = rg / NT;
        *n = rg % NT;
        const uint32_t g = c * kMmaChunk + *gi, blk = nt * kBlk + *n / kRowBlock;
        if (g >= G || blk >= nblocks)
            return nullptr;
        return a.wblocks + (size_t)blk * G * 144u + (size_t)g * 128u + (*n % kRowBlock) * 16u;
    };
    auto slot = [&](uint32_t c, uint32_t k) {
        return w_slots + (((size_t)(c % kMmaXDepth) * kXRows + k) * kMmaXThreads + xt) * 16u;
    };
    auto fetch = [&](uint32_t c) {  // one commit group per chunk, empty past the end
        if (c < nchunks)
#pragma unroll
            for (uint32_t k = 0; k < kXRows; ++k) {
                uint32_t gi, n;
                const unsigned char* src = row_src(c, k, &gi, &n);
                if (src)
                    cp_async16(slot(c, k), src);
            }
        cp_async_commit();
    };
    const bool expander = warp >= 2 && warp < kMmaEpiWarp0;

    if (tid == 0) {
        for (uint32_t s = 0; s < kMmaAStages; ++s) {
            mbar_init(&afull[s], 1);
            mbar_init(&aempty[s], 1);
        }
        for (uint32_t s = 0; s < kMmaBBufs; ++s) {
            mbar_init(&bready[s], kMmaXThreads);
            mbar_init(&bfree[s], 1);
        }
        for (uint32_t b = 0; b < 2; ++b) {
            mbar_init(&dready[b], 1);
            mbar_init(&tfree[b], kMmaEpiThreads);
        }
        mbar_init(sready, kMmaXThreads);
        mbar_init(mdone, 1);
        fence_barrier_init();
    }
    if (tid < 16)
        sign_lut[tid] = expand_signs4(tid);
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(kMmaTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // weights never depend on earlier kernels
    if (expander)
#pragma unroll
        for (uint32_t c = 0; c < kMmaXDepth; ++c)
            fetch(c);
    griddep_wait();
    if (tid == 0)
        skip_cta = *a.status != 0;  // an input row was rejected: no output is written
    __syncthreads();
    if (skip_cta) {
        if (expander)
            cp_async_wait<0>();  // no copy in flight when the CTA exits
        tc_fence_before();
        __syncthreads();
        if (warp == 1) {  // no MMA was issued
            tc_fence_after();
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kMmaTmemCols));
        }
        return;
    }

    if (warp == 0) {
        // ---- producer: one bulk copy of A per chunk (its groups are adjacent)
        if (lane == 0) {
            uint32_t c = 0;
            for (; c < nchunks; ++c) {
                const uint32_t st = c % kMmaAStages, gn = min(kMmaChunk, G - c * kMmaChunk);
                if (c >= kMmaAStages && !mbar_wait(&aempty[st], ((c / kMmaAStages) - 1) & 1)) {
                    atomicOr(a.status, kStatusTimeout);
                    break;
                }
                mbar_arrive_expect_tx(&afull[st], gn * kMmaATile);
                bulk_g2s(a_ring + (size_t)st * kAStage, a.a_sw + ((size_t)mt * G + c * kMmaChunk) * kMmaATile,
                         gn * kMmaATile, &afull[st]);
            }
            // no copy may still be in flight when the CTA exits
            for (uint32_t j = c > kMmaAStages ? c - kMmaAStages : 0; j < c; ++j)
                if (!mbar_wait(&afull[j % kMmaAStages], (j / kMmaAStages) & 1))
                    atomicOr(a.status, kStatusTimeout);
        }
    } else if (warp == 1) {
        // ---- MMA issuer: every MMA accumulates (onto the bias the epilogue wrote)
        if (lane == 0) {
            for (uint32_t c = 0; c < nchunks; ++c) {
                const uint32_t b = c & 1, bb = c % kMmaBBufs;
                bool ok = mbar_wait(&bready[bb], (c / kMmaBBufs) & 1) && mbar_wait(&tfree[b], (c >> 1) & 1);
                if (!ok) {
                    atomicOr(a.status, kStatusTimeout);
                    break;
                }
                const uint32_t st = c % kMmaAStages, gn = min(kMmaChunk, G - c * kMmaChunk);
                if (!mbar_wait(&afull[st], (c / kMmaAStages) & 1)) {
                    atomicOr(a.status, kStatusTimeout);
                    break;
                }
                tc_fence_after();
                // K step outer, group inner: consecutive MMAs feed different
                // accumulators, so they need not wait for one another
                const uint32_t a_base = smem_addr(a_ring + (size_t)st * kAStage);
                const uint32_t b_base = smem_addr(b_ring + (size_t)bb * kMmaChunk * kMmaBTile);
#pragma unroll
                for (uint32_t k = 0; k < kGroup / 32; ++k)
                    for (uint32_t gi = 0; gi < gn; ++gi)
                        mma_i8(tmem + (b * kMmaChunk + gi) * NT, mma_smem_desc(a_base + gi * kMmaATile + 32u * k),
                               mma_smem_desc(b_base + gi * kMmaBTile + 32u * k), 1u, kIdesc);
                mma_commit(&aempty[st]);  // the A stage is free once these MMAs have read it
                mma_commit(&dready[b]);
                mma_commit(&bfree[bb]);
            }
            mma_commit(mdone);  // completes when every MMA issued above has completed
        }
        __syncwarp();
    } else if (expander) {
        // ---- warps 2..5: B chunk by chunk from the fetched weight bits (the
        // first kMmaXDepth chunks are in flight already); after the first
        // chunk, the tile's FP32 scales (the epilogue's first read comes after
        // that chunk's MMAs)
        bool scaled = false;
        auto convert_scales = [&]() {
            scaled = true;
            for (uint32_t i = xt; i < G * NT; i += kMmaXThreads) {
                const uint32_t g = i / NT, n = i % NT, blk = nt * kBlk + n / kRowBlock;
                const float v = blk < nblocks ? h2f(*reinterpret_cast<const uint16_t*>(
                                                    a.wblocks + (size_t)blk * G * 144u + (size_t)G * 128u +
                                                    ((size_t)(n % kRowBlock) * G + g) * 2u))
                                              : 0.0f;
                sf[i] = v;
                // exact: 11 significant bits times 2 (the matrix scales are finite)
                sb[i] = __fmul_rn(v, -12582912.0f);
            }
            mbar_arrive(sready);
        };
        bool ok = true;
        for (uint32_t c = 0; c < nchunks && ok; ++c) {
            if (c == 1)
                convert_scales();
            const uint32_t bb = c % kMmaBBufs;
            cp_async_wait<kMmaXDepth - 1>();  // this thread's rows of chunk c are in place
            if (c >= kMmaBBufs && !mbar_wait(&bfree[bb], ((c / kMmaBBufs) - 1) & 1)) {
                atomicOr(a.status, kStatusTimeout);
                ok = false;
                break;
            }
#pragma unroll
            for (uint32_t k = 0; k < kXRows; ++k) {
                uint32_t gi, n;
                if (!row_src(c, k, &gi, &n))
                    continue;
                const uint4 bits4 = *reinterpret_cast<const uint4*>(slot(c, k));
                const uint32_t w[4] = {bits4.x, bits4.y, bits4.z, bits4.w};
                unsigned char* dst =
                    b_ring + (size_t)(bb * kMmaChunk + gi) * kMmaBTile + (n / 8u) * 1024u + (n % 8u) * 128u;
#pragma unroll
                for (uint32_t j = 0; j < 8; ++j) {  // 16-byte chunk j of the row: bits 16j .. 16j + 15
                    const uint32_t bits = (w[j >> 1] >> ((j & 1u) * 16u)) & 0xffffu;
                    uint4 o;
                    o.x = sign_lut[bits & 0xfu];
                    o.y = sign_lut[(bits >> 4) & 0xfu];
                    o.z = sign_lut[(bits >> 8) & 0xfu];
                    o.w = sign_lut[bits >> 12];
                    *reinterpret_cast<uint4*>(dst + ((j ^ (n % 8u)) * 16u)) = o;
                }
            }
            fence_proxy_async();  // the MMAs read these bytes through the async proxy
            mbar_arrive(&bready[bb]);
            fetch(c + kMmaXDepth);  // into the slots just read
        }
        cp_async_wait<0>();  // no copy in flight when the CTA exits
        if (!scaled)
            convert_scales();  // a one-chunk tile, or a wait that gave up first: still release the epilogue
    } else {
        // ---- warps 6..21: the ordered FP32 epilogue
        const uint32_t quad = warp & 3;                          // TMEM lane quadrant this warp may read
        const uint32_t quarter = (warp - kMmaEpiWarp0) >> 2;     // which quarter of the tile's columns
        const uint32_t row = quad * 32 + lane;                   // tile row = TMEM lane
        const uint32_t m = mt * kMmaM + row;
        const uint32_t col0 = quarter * kMmaCols;                // first tile column of this thread
        const bool dot_groups = a.epi == kEpiDotGroups;
        const bool live = m < a.m;
        const uint32_t tbase = tmem + ((quad * 32u) << 16) + col0;  // this thread's lane and columns
        auto fill = [&](uint32_t slot) {  // slot = buffer * kMmaChunk + group of the chunk
            if constexpr (kMmaCols == 32)
                tmem_fill32(tbase + slot * NT, kMmaBias);
            else
                tmem_fill16(tbase + slot * NT, kMmaBias);
        };
        // both TMEM buffers start at the bias: phase 0 of tfree releases them
        for (uint32_t slot = 0; slot < 2 * kMmaChunk; ++slot)
            fill(slot);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&tfree[0]);
        mbar_arrive(&tfree[1]);
        uint64_t acc[kMmaCols / 2];
#pragma unroll
        for (uint32_t j = 0; j < kMmaCols / 2; ++j)
            acc[j] = 0ull;
        bool ok = mbar_wait(sready, 0);
        if (!ok)
            atomicOr(a.status, kStatusTimeout);
        for (uint32_t c = 0; c < nchunks && ok; ++c) {
            const uint32_t b = c & 1, g0 = c * kMmaChunk, gn = min(kMmaChunk, G - g0);
            if (!mbar_wait(&dready[b], (c >> 1) & 1)) {
                atomicOr(a.status, kStatusTimeout);
                ok = false;
                break;
            }
            tc_fence_after();
            // 16 TMEM columns per wait (an 80-register budget at 22 warps)
            for (uint32_t gi = 0; gi < gn; ++gi) {
                const uint32_t slot = b * kMmaChunk + gi, g = g0 + gi;
#pragma unroll
                for (uint32_t h = 0; h < kMmaCols / 16; ++h) {
                    uint32_t d[16];
                    tmem_ld16(tbase + slot * NT + 16u * h, d);
                    tmem_wait();
                    if (dot_groups) {
                        if (live)
#pragma unroll
                            for (uint32_t j = 0; j < 16; ++j) {
                                const uint32_t on = nt * NT + col0 + 16u * h + j;
                                if (on < a.n)
                                    store_i16_any(a.out + (size_t)m * a.out_stride + ((size_t)on * G + g) * 2u,
                                                  (int16_t)(int32_t)(d[j] - kMmaBias));
                            }
                    } else {
                        const float4* sc4 = reinterpret_cast<const float4*>(sf + (size_t)g * NT + col0 + 16u * h);
                        const float4* sb4 = reinterpret_cast<const float4*>(sb + (size_t)g * NT + col0 + 16u * h);
#pragma unroll
                        for (uint32_t q = 0; q < 4; ++q) {
                            const float4 sc = sc4[q], bs = sb4[q];
                            // The words are Db = the float bits of 1.5 * 2^23 + D, and
                            // fma(s, Db, -s * 1.5 * 2^23) = RN(s * Db - s * 1.5 * 2^23) =
                            // RN(s * D) = fl(scale * D): the subtrahend is exact (s has 11
                            // significant bits) and the FMA rounds once.
                            const uint64_t p01 = f2_fma(f2_pack(sc.x, sc.y),
                                                        f2_pack(__uint_as_float(d[4 * q]), __uint_as_float(d[4 * q + 1])),
                                                        f2_pack(bs.x, bs.y));
                            const uint64_t p23 = f2_fma(
                                f2_pack(sc.z, sc.w), f2_pack(__uint_as_float(d[4 * q + 2]), __uint_as_float(d[4 * q + 3])),
                                f2_pack(bs.z, bs.w));
                            const uint32_t k = 8u * h + 2u * q;
                            acc[k] = f2_add(acc[k], p01);
                            acc[k + 1] = f2_add(acc[k + 1], p23);
                        }
                    }
                }
                fill(slot);  // the bias again, for chunk c + 2
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&tfree[b]);
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
                        reinterpret_cast<float*>(orow)[(n0 / 16u + p) * kRowBlock + r] =
                            swiglu_one(y[16 * p + r], y[16 * p + 8 + r]);
                    }
            } else if (a.epi == kEpiResidual) {
                // x = fl(x + Y): every load of x issued before the first store
                float* dst = reinterpret_cast<float*>(orow) + n0;
                float xv[kMmaCols];
                if (n0 + kMmaCols <= a.n && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
#pragma unroll
                    for (uint32_t q = 0; q < kMmaCols / 4; ++q) {
                        const float4 v = reinterpret_cast<const float4*>(dst)[q];
                        xv[4 * q] = v.x;
                        xv[4 * q + 1] = v.y;
                        xv[4 * q + 2] = v.z;
                        xv[4 * q + 3] = v.w;
                    }
#pragma unroll
                    for (uint32_t q = 0; q < kMmaCols / 4; ++q)
                        reinterpret_cast<float4*>(dst)[q] =
                            make_float4(__fadd_rn(xv[4 * q], y[4 * q]), __fadd_rn(xv[4 * q + 1], y[4 * q + 1]),
                                        __fadd_rn(xv[4 * q + 2], y[4 * q + 2]), __fadd_rn(xv[4 * q + 3], y[4 * q + 3]));
                } else {
#pragma unroll
                    for (uint32_t j = 0; j < kMmaCols; ++j)
                        xv[j] = n0 + j < a.n ? dst[j] : 0.0f;
#pragma unroll
                    for (uint32_t j = 0; j < kMmaCols; ++j)
                        if (n0 + j < a.n)
                            dst[j] = __fadd_rn(xv[j], y[j]);
                }
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

constexpr size_t kMmaSmemMax = 227u * 1024u;  // dynamic shared memory per CTA

// Whether a matrix of `groups` groups fits the tensor-core kernel's shared
// memory (the scales of a whole tile stay on chip): up to 183 groups.
inline bool mma_fits(uint32_t groups) { return mma_smem_plan(kMmaNarrow, groups).total <= kMmaSmemMax; }

// Launches the contraction of `a.m` rows (a.m <= 65535 * kMmaM, mma_fits)
// on `s`: 128-wide tiles, or 64-wide when the wide grid would leave SMs idle
// on a device of `sms` streaming multiprocessors or its scales do not fit.
// With pdl the launch may overlap the previous kernel of the stream (the
// kernel waits for it before it reads anything but the weights).
inline cudaError_t launch_mma(const MmaArgs& a, int sms, cudaStream_t s, bool pdl = false) {
    const uint32_t mtiles = (a.m + kMmaM - 1) / kMmaM;
    const bool narrow = (size_t)((a.n + kMmaN - 1) / kMmaN) * mtiles < (size_t)sms ||
                        mma_smem_plan(kMmaN, a.groups).total > kMmaSmemMax;
    const uint32_t nt = narrow ? kMmaNarrow : kMmaN;
    const MmaSmem p = mma_smem_plan(nt, a.groups);
    const void* fn = narrow ? (const void*)w1a8_mma_kernel<kMmaNarrow> : (const void*)w1a8_mma_kernel<kMmaN>;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.total);
    if (e != cudaSuccess)
        return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.n + nt - 1) / nt, mtiles);
    cfg.blockDim = dim3(kMmaThreads);
    cfg.dynamicSmemBytes = p.total;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return narrow ? cudaLaunchKernelEx(&cfg, w1a8_mma_kernel<kMmaNarrow>, a)
                  : cudaLaunchKernelEx(&cfg, w1a8_mma_kernel<kMmaN>, a);
}

}  // namespace bnn
