// exact_sum.cuh - the reference's serial FP32 sum of squares, computed in parallel.
//
// qwen3_rmsnorm (bnn-sw-v2/qwen3/qwen3.c:361-372) accumulates
//     s_0 = 0,  s_{i+1} = fl(s_i + fl(x_i * x_i)),  i = 0..n-1
// in index order. Run literally that is a chain of n dependent adds; this
// file produces the identical float with the 256 threads of eight warps.
//
// Every term a_i = fl(x_i * x_i) is >= 0, so s is non-decreasing. While s_i
// and s_{i+1} lie in one binade [2^e, 2^(e+1)), with grid spacing
// u = 2^(e-23), the rounded add is s_i + u * RN(a_i / u), where RN is round
// to nearest and a tie (a_i / u exactly half-way) is broken by the parity of
// s_i. So a run of steps inside one binade with no tie adds the exact integer
// D = sum RN(a_i / u), independent of where the run starts.
//
// Which binade each s_i is in is guessed from an approximate FP32 prefix p_i
// of the squares (per-thread sums and a block scan). A step counts as
// "inside binade e" only with a relative margin of 2^-12 on both sides; steps
// that cross a binade, start below 2^-100 or hit a tie are "singles".
//
// Each thread classifies a contiguous chunk and records only where an op
// starts: every single, and the first element of each run (a change of
// binade). Records carry the running total of the increments RN(a_i / u)
// before them, so a run's D is the difference of two neighbouring records;
// a run that continues the previous thread's last run is dropped, which
// merges the two. One warp then walks the ops 32 at a time: all lanes run
// the same chain of adds (one add per op) and each keeps the value before
// and after its op; each lane checks its op, and the chain restarts after
// the first op that fails, which is replayed step by step. A single always
// passes; a run passes when s starts inside binade e and the sum stays below
// 2^(e+1). So the result never depends on the margin argument, only the
// speed does.
#pragma once

#include <cstdint>
#include <cmath>
#include <cstring>

namespace bnn {

constexpr int kSumThreads = 256;       // eight warps
constexpr int kSumWarpsN = kSumThreads / 32;
constexpr int kSumSlots = 8;           // records per thread before its chunk goes serial
constexpr int kSumBatch = 8;           // elements loaded ahead per step
constexpr int kRunEMin = -100;         // runs only in binades where u and 2^(23-e) are normal
constexpr int kRunEMax = 125;
constexpr uint32_t kLoMant = 1u << 11;                  // p >= 2^e * (1 + 2^-12)
constexpr uint32_t kHiMant = (1u << 23) - (1u << 12);   // p <= 2^(e+1) * (1 - 2^-12)
constexpr int kTagSingle = 0;          // record tags: a single, a run (e + 128), a serial chunk
constexpr int kTagChunk = 255;

// One op record: key = first element | tag << 16; cum = increments before it.
struct SumRec {
    int key;
    int cum;
};

__host__ __device__ inline int rec_first(int key) { return key & 0xffff; }
__host__ __device__ inline int rec_tag(int key) { return (key >> 16) & 0xff; }

// Shared memory of one sum: per-thread record slots (stride padded against
// bank conflicts), the compacted op list (+ sentinel), last tags, scratch.
constexpr int kSumSlotStride = kSumSlots + 1;
constexpr int kSumListMax = kSumThreads * kSumSlots;
constexpr size_t kSumSlotsOffset = 0;
constexpr size_t kSumListOffset = kSumSlotsOffset + (size_t)kSumThreads * kSumSlotStride * sizeof(SumRec);
constexpr size_t kSumTagsOffset = kSumListOffset + (size_t)(kSumListMax + 2) * sizeof(SumRec);
constexpr size_t kSumMiscOffset = kSumTagsOffset + kSumThreads * sizeof(int);
constexpr size_t kSumSmemBytes = kSumMiscOffset + 64 * sizeof(float);

__host__ __device__ inline uint32_t fbits(float v) {
#ifdef __CUDA_ARCH__
    return __float_as_uint(v);
#else
    uint32_t b;
    memcpy(&b, &v, sizeof b);
    return b;
#endif
}

__host__ __device__ inline float fvalue(uint32_t b) {
#ifdef __CUDA_ARCH__
    return __uint_as_float(b);
#else
    float v;
    memcpy(&v, &b, sizeof v);
    return v;
#endif
}

__host__ __device__ inline float pow2f(int e) {
    // 2^e for -126 <= e <= 127, exactly
    return fvalue((uint32_t)(e + 127) << 23);
}

#ifdef __CUDA_ARCH__
__device__ __forceinline__ float sq_rn(float x) { return __fmul_rn(x, x); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
#else
inline float sq_rn(float x) {
    volatile float r = x * x;
    return r;
}
inline float add_rn(float a, float b) {
    volatile float r = a + b;
    return r;
}
inline float mul_rn(float a, float b) {
    volatile float r = a * b;
    return r;
}
#endif

// Elements per thread: odd, so that the threads' i-th elements fall in
// different shared-memory banks.
__host__ __device__ inline int sum_chunk_len(int n) { return ((n + kSumThreads - 1) / kSumThreads) | 1; }

// Serial sum of squares over [first, last) starting from s.
__host__ __device__ inline float sum_serial(const float* xs, float s, int first, int last) {
    for (int i = first; i < last; ++i)
        s = add_rn(s, sq_rn(xs[i]));
    return s;
}

// Approximate sum of squares of xs[first, last) (any order will do).
__host__ __device__ inline float sum_approx(const float* xs, int first, int last) {
    float q[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int i = first; i < last; i += kSumBatch) {
#pragma unroll
        for (int j = 0; j < kSumBatch; ++j) {
            const float v = sq_rn(xs[i + j < last ? i + j : first]);
            q[j & 3] = add_rn(q[j & 3], i + j < last ? v : 0.0f);
        }
    }
    return add_rn(add_rn(q[0], q[1]), add_rn(q[2], q[3]));
}

// Classifies [first, last), whose approximate prefix before `first` is p0.
// Records each op start into out[0..kSumSlots) (cum relative to `first`;
// out[kSumSlots] is scratch); returns the count, or -1 when more are needed.
// Sets *inc_total to the sum of the run increments and *last_tag to the tag
// of the last element (-1 if the range is empty).
// Written stage by stage over a batch of kSumBatch elements: only the prefix
// adds, the start tests and the counts are chained, every other stage is
// kSumBatch independent operations that issue back to back.
__host__ __device__ inline int sum_classify(const float* xs, int first, int last, float p0, SumRec* out,
                                            int* inc_total, int* last_tag) {
    constexpr float kMagic = 8388608.0f;  // 2^23: t = fl(2^23 + v) holds RNE(v) for 0 <= v < 2^23
    int count = 0, cum = 0, prev = -1;
    float p = p0;
    for (int base = first; base < last; base += kSumBatch) {
        float a[kSumBatch], pb[kSumBatch], pe[kSumBatch];
#pragma unroll
        for (int j = 0; j < kSumBatch; ++j)
            a[j] = base + j < last ? sq_rn(xs[base + j < last ? base + j : first]) : 0.0f;
#pragma unroll
        for (int j = 0; j < kSumBatch; ++j) {
            pb[j] = p;
            p = add_rn(p, a[j]);  // past the end a = +0 leaves p as is
            pe[j] = p;
        }
        uint32_t eb[kSumBatch];
#pragma unroll
        for (int j = 0; j < kSumBatch; ++j)
            eb[j] = fbits(pb[j]) >> 23;  // p >= 0: the biased exponent
        bool in[kSumBatch];
#pragma unroll
        for (int j = 0; j < kSumBatch; ++j) {
            // inside binade e = eb - 127 with the margin: p >= 2^e (1 + 2^-12)
            // and pn <= 2^(e+1) (1 - 2^-12); false for NaN and infinity too
            in[j] = eb[j] - (uint32_t)(kRunEMin + 127) <= (uint32_t)(kRunEMax - kRunEMin) &&
                    pb[j] >= fvalue((eb[j] << 23) | kLoMant) && pe[j] <= fvalue((eb[j] << 23) | kHiMant);
        }
        float v[kSumBatch];
#pragma unroll
        for (int j = 0; j < kSumBatch; ++j)  // a / u = a * 2^(23 - e), exact; 2^(23-e) has biased exponent 277 - eb
            v[j] = mul_rn(a[j], fvalue((in[j] ? 277u - eb[j] : 127u) << 23));
        float t[kSumBatch];
#pragma unroll
        for (int j = 0; j < kSumBatch; ++j)
            t[j] = add_rn(v[j], kMagic);
        bool lin[kSumBatch];
#pragma unroll
        for (int j = 0; j < kSumBatch; ++j)
            lin[j] = in[j] && v[j] < kMagic && fabsf(add_rn(v[j], -add_rn(t[j], -kMagic))) != 0.5f;  // not a tie
        int inc[kSumBatch], tag[kSumBatch];
#pragma unroll
        for (int j = 0; j < kSumBatch; ++j) {
            inc[j] = lin[j] ? (int)(fbits(t[j]) - 0x4b000000u) : 0;
            tag[j] = lin[j] ? (int)eb[j] + 1 : kTagSingle;  // e + 128
        }
#pragma unroll
        for (int j = 0; j < kSumBatch; ++j) {
            const int i = base + j;
            const bool valid = i < last;
            const bool start = valid && (!lin[j] || tag[j] != prev);
            // unconditional store: uncounted records go to the scratch slot
            out[start && count < kSumSlots ? count : kSumSlots] = SumRec{i | (tag[j] << 16), cum};
            count += start;
            cum += valid ? inc[j] : 0;
            prev = valid ? tag[j] : prev;
        }
    }
    *inc_total = cum;
    *last_tag = prev;
    return count <= kSumSlots ? count : -1;
}

// The op that list[k] starts, applied to s on the host (the reference of
// what the warp walk does): returns the new s.
__host__ __device__ inline float sum_apply(const float* xs, float s, SumRec rec, SumRec next) {
    const int tag = rec_tag(rec.key), first = rec_first(rec.key), last = rec_first(next.key);
    if (tag == kTagSingle)
        return add_rn(s, sq_rn(xs[first]));
    if (tag != kTagChunk) {
        const int e = tag - 128, d = next.cum - rec.cum;
        if (d >= 0 && d < (1 << 24) && s >= pow2f(e) && s < pow2f(e + 1)) {
            const float t = add_rn(s, mul_rn((float)d, pow2f(e - 23)));
            if (t < pow2f(e + 1))
                return t;
        }
    }
    return sum_serial(xs, s, first, last);
}

// ---- the wide form: 512 threads (16 warps), 4 consecutive elements per
// thread, rows of up to 2048 elements per pass (longer rows in passes of
// 2048 from the exact sum so far). One approximate block scan, one
// classification pass per element (sum_classify's rules), one block scan of
// (op count, increment sum) and one list write, then the same walk. A run
// never continues across a warp boundary (the first element of every warp
// starts an op), so no thread needs its neighbour warp's tags: that costs at
// most 15 extra ops, each checked like any other.
constexpr int kWideThreads = 512;
constexpr int kWideWarps = kWideThreads / 32;
constexpr int kWidePer = 4;
constexpr int kWideChunk = kWideThreads * kWidePer;
constexpr size_t kWideAddOffset = 256;    // [64] addends of a walk round
constexpr size_t kWideListOffset = 512;

// An op of the wide form: first element | tag << 16, increments before it
// (mod 2^32), and for a single its addend (the square).
struct WideRec {
    int key;
    int cum;
    float add;
    int pad;
};
constexpr size_t kWideSmemBytes = kWideListOffset + (size_t)(kWideChunk + 2) * sizeof(WideRec);

// One element's op tag (kTagSingle, or e + 128 for a run in binade e) and its
// increment RN(a / 2^(e-23)), given the approximate sum pb before it; the
// same tests as sum_classify.
__host__ __device__ inline void sum_classify_one(float a, float pb, int* tag, uint32_t* inc) {
    constexpr float kMagic = 8388608.0f;
    const float pe = add_rn(pb, a);
    const uint32_t eb = fbits(pb) >> 23;
    const bool in = eb - (uint32_t)(kRunEMin + 127) <= (uint32_t)(kRunEMax - kRunEMin) &&
                    pb >= fvalue((eb << 23) | kLoMant) && pe <= fvalue((eb << 23) | kHiMant);
    const float v = mul_rn(a, fvalue((in ? 277u - eb : 127u) << 23));
    const float t = add_rn(v, kMagic);
    const bool lin = in && v < kMagic && fabsf(add_rn(v, -add_rn(t, -kMagic))) != 0.5f;
    *inc = lin ? fbits(t) - 0x4b000000u : 0u;
    *tag = lin ? (int)eb + 1 : kTagSingle;
}

#ifdef __CUDACC__
__device__ __forceinline__ void sum_bar(int id) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(kSumThreads) : "memory");
}

// Called by the 256 threads of warps 0..7 of a CTA; returns the serial sum of
// squares of xs[0..n), 1 <= n <= 65535 (shared memory), to all of them.
// Uses named barrier `bar` (256 threads) and kSumSmemBytes of 16-byte
// aligned shared memory at `mem`.
static __device__ __forceinline__ float exact_sumsq(const float* xs, int n, unsigned char* mem, int bar) {
    SumRec* slots = reinterpret_cast<SumRec*>(mem + kSumSlotsOffset);
    SumRec* list = reinterpret_cast<SumRec*>(mem + kSumListOffset);
    int* tags = reinterpret_cast<int*>(mem + kSumTagsOffset);
    float* misc = reinterpret_cast<float*>(mem + kSumMiscOffset);
    float* wsum = misc;                              // [8] warp sums of the partials
    int* wcnt = reinterpret_cast<int*>(misc + 8);    // [8] warp record counts
    int* winc = reinterpret_cast<int*>(misc + 16);   // [8] warp increment totals
    float* abuf = misc + 24;                         // [32] addends of a walk round
    float* result = misc + 56;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int len = sum_chunk_len(n);
    const int first = min(t * len, n), last = min(first + len, n);

    // approximate prefix before `first`: block scan of the chunk sums
    const float part = sum_approx(xs, first, last);
    float incl = part;
    for (int o = 1; o < 32; o <<= 1) {
        const float v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o)
            incl = add_rn(incl, v);
    }
    float excl = __shfl_up_sync(0xffffffffu, incl, 1);
    if (lane == 0)
        excl = 0.0f;
    if (lane == 31)
        wsum[warp] = incl;
    sum_bar(bar);
    for (int w = 0; w < warp; ++w)
        excl = add_rn(excl, wsum[w]);

    SumRec* mine = slots + t * kSumSlotStride;
    int inc_total, last_tag;
    int cnt = sum_classify(xs, first, last, excl, mine, &inc_total, &last_tag);
    if (cnt < 0) {
        mine[0] = SumRec{first | (kTagChunk << 16), 0};
        cnt = 1;
        last_tag = kTagChunk;
    }
    tags[t] = last_tag;
    int iincl = inc_total;
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, iincl, o);
        if (lane >= o)
            iincl += v;
    }
    if (lane == 31)
        winc[warp] = iincl;
    sum_bar(bar);

    // A first record that continues the previous thread's last run is
    // dropped: the two runs become one op.
    const int tag0 = cnt > 0 ? rec_tag(mine[0].key) : -1;
    const bool drop = tag0 != -1 && tag0 != kTagSingle && tag0 != kTagChunk && t > 0 && tags[t - 1] == tag0;
    const int keep = cnt - (drop ? 1 : 0);
    int cincl = keep;
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, cincl, o);
        if (lane >= o)
            cincl += v;
    }
    if (lane == 31)
        wcnt[warp] = cincl;
    sum_bar(bar);
    int coff = cincl - keep, ioff = iincl - inc_total;
    for (int w = 0; w < warp; ++w) {
        coff += wcnt[w];
        ioff += winc[w];
    }
    int total = 0, inc_all = 0;
#pragma unroll
    for (int w = 0; w < kSumWarpsN; ++w) {
        total += wcnt[w];
        inc_all += winc[w];
    }
    for (int k = drop ? 1 : 0; k < cnt; ++k) {
        SumRec r = mine[k];
        r.cum += ioff;
        list[coff + k - (drop ? 1 : 0)] = r;
    }
    if (t == 0)  // sentinel: where the last op ends, and the final total
        list[total] = list[total + 1] = SumRec{n, inc_all};
    sum_bar(bar);

    if (warp == 0) {
        float s = 0.0f;
        int k = 0;
        while (k < total) {
            const int idx = k + lane;
            const bool valid = idx < total;
            const int ci = valid ? idx : total;  // the sentinel (and the slot after it) past the end
            const SumRec rec = list[ci], nx = list[ci + 1];
            const int tag = rec_tag(rec.key);
            const float a = sq_rn(xs[min(rec_first(rec.key), n - 1)]);
            // a run is exact when s starts inside binade e and the sum stays
            // below 2^(e+1): 0 <= d < 2^24 with u = 2^(e-23) normal makes
            // d * u a float, and s and d * u are multiples of u
            const int d = nx.cum - rec.cum;
            const bool single = tag == kTagSingle;
            const bool run = valid && !single && tag != kTagChunk && d >= 0 && d < (1 << 24);
            const int e = run ? tag - 128 : 0;
            const float addend = !valid ? 0.0f : single ? a : run ? mul_rn((float)d, pow2f(e - 23)) : 0.0f;
            bool ok = !valid || single || run;  // a chunk (or a bad d) fails
            abuf[lane] = addend;
            __syncwarp();
            float ad[32];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 v = reinterpret_cast<const float4*>(abuf)[q];
                ad[4 * q] = v.x;
                ad[4 * q + 1] = v.y;
                ad[4 * q + 2] = v.z;
                ad[4 * q + 3] = v.w;
            }
            float cur = s, before = s, after = s;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const float next = add_rn(cur, ad[j]);
                before = lane == j ? cur : before;
                after = lane == j ? next : after;
                cur = next;
            }
            if (run)
                ok = before >= pow2f(e) && before < pow2f(e + 1) && after < pow2f(e + 1);
            const unsigned bad = __ballot_sync(0xffffffffu, !ok);
            if (bad == 0) {
                s = cur;
                k += 32;
                continue;
            }
            // replay the first failing op step by step, restart after it
            const int f = __ffs(bad) - 1;
            s = __shfl_sync(0xffffffffu, before, f);
            s = sum_serial(xs, s, rec_first(list[k + f].key), rec_first(list[k + f + 1].key));
            k += f + 1;
        }
        if (lane == 0)
            *result = s;
    }
    sum_bar(bar);
    return *result;
}

__device__ __forceinline__ void wide_bar(int id) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(kWideThreads) : "memory");
}

// Called by the 512 threads of warps 0..15; returns the serial sum of squares
// of xs[0..n) (shared memory, n >= 1) to all of them. Uses named barrier
// `bar` and kWideSmemBytes of 16-byte aligned shared memory at `mem`.
static __device__ __forceinline__ float exact_sumsq_wide(const float* xs, int n, unsigned char* mem, int bar) {
    float* wt = reinterpret_cast<float*>(mem);             // [16] warp totals of the approximate sums
    int* wc = reinterpret_cast<int*>(mem + 64);            // [16] warp op counts
    uint32_t* wk = reinterpret_cast<uint32_t*>(mem + 128); // [16] warp increment sums (mod 2^32)
    float* result = reinterpret_cast<float*>(mem + 192);
    float* abuf = reinterpret_cast<float*>(mem + kWideAddOffset);
    WideRec* list = reinterpret_cast<WideRec*>(mem + kWideListOffset);
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    float s0 = 0.0f;  // the exact sum before this pass
    for (int base = 0; base < n; base += kWideChunk) {
        const int m = min(kWideChunk, n - base);
        const float* xc = xs + base;
        const int j0 = t * kWidePer;
        float a[kWidePer], loc[kWidePer];
        if (j0 + kWidePer <= m && ((reinterpret_cast<uintptr_t>(xc) & 15u) == 0)) {
            const float4 v = reinterpret_cast<const float4*>(xc)[t];
            a[0] = sq_rn(v.x);
            a[1] = sq_rn(v.y);
            a[2] = sq_rn(v.z);
            a[3] = sq_rn(v.w);
        } else {
#pragma unroll
            for (int q = 0; q < kWidePer; ++q)
                a[q] = j0 + q < m ? sq_rn(xc[j0 + q]) : 0.0f;
        }
        loc[0] = a[0];
#pragma unroll
        for (int q = 1; q < kWidePer; ++q)
            loc[q] = add_rn(loc[q - 1], a[q]);
        // approximate prefix before this thread's first element
        float incl = loc[kWidePer - 1];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o)
                incl = add_rn(incl, v);
        }
        float excl = __shfl_up_sync(0xffffffffu, incl, 1);
        if (lane == 0)
            excl = 0.0f;
        if (lane == 31)
            wt[warp] = incl;
        wide_bar(bar);
        // the earlier warps' totals, summed by a shuffle tree (any order
        // will do for the approximate prefix; this one is wide_warp_prefix)
        float wp = lane < warp ? wt[lane] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            wp = add_rn(wp, __shfl_xor_sync(0xffffffffu, wp, o));
        float pb = add_rn(add_rn(s0, wp), excl);
        // classify, mark op starts, count
        int tag[kWidePer];
        uint32_t inc[kWidePer];
#pragma unroll
        for (int q = 0; q < kWidePer; ++q) {
            sum_classify_one(a[q], pb, &tag[q], &inc[q]);
            pb = add_rn(pb, a[q]);
        }
        int prev = __shfl_up_sync(0xffffffffu, tag[kWidePer - 1], 1);
        if (lane == 0)
            prev = -1;
        bool start[kWidePer];
        int cnt = 0;
        uint32_t ksum = 0;
#pragma unroll
        for (int q = 0; q < kWidePer; ++q) {
            const bool valid = j0 + q < m;
            start[q] = valid && (tag[q] == kTagSingle || tag[q] != (q ? tag[q - 1] : prev));
            cnt += start[q];
            ksum += valid ? inc[q] : 0u;
        }
        int ci = cnt;
        uint32_t ki = ksum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int vc = __shfl_up_sync(0xffffffffu, ci, o);
            const uint32_t vk = __shfl_up_sync(0xffffffffu, ki, o);
            if (lane >= o) {
                ci += vc;
                ki += vk;
            }
        }
        if (lane == 31) {
            wc[warp] = ci;
            wk[warp] = ki;
        }
        wide_bar(bar);
        const int cw = lane < kWideWarps ? wc[lane] : 0;
        const uint32_t kw = lane < kWideWarps ? wk[lane] : 0u;
        int coff = ci - cnt + __reduce_add_sync(0xffffffffu, lane < warp ? cw : 0);
        uint32_t kc = ki - ksum + __reduce_add_sync(0xffffffffu, lane < warp ? kw : 0u);
        const int total = __reduce_add_sync(0xffffffffu, cw);
        const uint32_t kall = __reduce_add_sync(0xffffffffu, kw);
#pragma unroll
        for (int q = 0; q < kWidePer; ++q) {
            if (start[q])
                list[coff++] = WideRec{(j0 + q) | (tag[q] << 16), (int)kc, a[q], 0};
            kc += j0 + q < m ? inc[q] : 0u;
        }
        if (t == 0)  // sentinel: where the last op ends, and the final increment sum
            list[total] = list[total + 1] = WideRec{m, (int)kall, 0.0f, 0};
        wide_bar(bar);
        if (warp == 0) {
            // 64 ops a round: lane j prepares ops k + j and k + 32 + j
            float s = s0;
            int k = 0;
            while (k < total) {
                float ad[2];
                bool run[2], okp[2];
                int e[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int idx = k + 32 * h + lane;
                    const bool valid = idx < total;
                    const WideRec rec = list[valid ? idx : total], nx = list[(valid ? idx : total) + 1];
                    const int tg = rec_tag(rec.key);
                    const uint32_t d = (uint32_t)nx.cum - (uint32_t)rec.cum;
                    const bool single = tg == kTagSingle;
                    run[h] = valid && !single && d < (1u << 24);
                    e[h] = run[h] ? tg - 128 : 0;
                    ad[h] = !valid ? 0.0f : single ? rec.add : run[h] ? mul_rn((float)d, pow2f(e[h] - 23)) : 0.0f;
                    okp[h] = !valid || single || run[h];
                }
                abuf[lane] = ad[0];
                abuf[32 + lane] = ad[1];
                __syncwarp();
                // all lanes run the same chain of adds; lane j keeps the values
                // before and after ops k + j and k + 32 + j
                float av[64];
#pragma unroll
                for (int q = 0; q < 16; ++q) {
                    const float4 v = reinterpret_cast<const float4*>(abuf)[q];
                    av[4 * q] = v.x;
                    av[4 * q + 1] = v.y;
                    av[4 * q + 2] = v.z;
                    av[4 * q + 3] = v.w;
                }
                float cur = s, b0 = s, a0 = s, b1 = s, a1 = s;
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) {
                    const float next = add_rn(cur, av[jj]);
                    b0 = lane == jj ? cur : b0;
                    a0 = lane == jj ? next : a0;
                    cur = next;
                }
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) {
                    const float next = add_rn(cur, av[32 + jj]);
                    b1 = lane == jj ? cur : b1;
                    a1 = lane == jj ? next : a1;
                    cur = next;
                }
                bool ok0 = okp[0], ok1 = okp[1];
                if (run[0])
                    ok0 = b0 >= pow2f(e[0]) && b0 < pow2f(e[0] + 1) && a0 < pow2f(e[0] + 1);
                if (run[1])
                    ok1 = b1 >= pow2f(e[1]) && b1 < pow2f(e[1] + 1) && a1 < pow2f(e[1] + 1);
                const unsigned bad0 = __ballot_sync(0xffffffffu, !ok0);
                const unsigned bad1 = __ballot_sync(0xffffffffu, !ok1);  // (also orders abuf's reuse)
                if ((bad0 | bad1) == 0) {
                    s = cur;
                    k += 64;
                    continue;
                }
                // replay the first failing op step by step, restart after it
                const int f = bad0 ? __ffs(bad0) - 1 : 32 + __ffs(bad1) - 1;
                const float bf0 = __shfl_sync(0xffffffffu, b0, f & 31), bf1 = __shfl_sync(0xffffffffu, b1, f & 31);
                s = f < 32 ? bf0 : bf1;
                s = sum_serial(xc, s, rec_first(list[k + f].key), rec_first(list[k + f + 1].key));
                k += f + 1;
            }
            if (lane == 0)
                *result = s;
        }
        wide_bar(bar);
        s0 = *result;  // (the next pass rewrites result and the list only after two more barriers)
    }
    return s0;
}
#endif

}  // namespace bnn
