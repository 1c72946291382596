// exact_sum.cuh - the reference's serial FP32 sum of squares, computed in parallel.
//
// qwen3_rmsnorm (bnn-sw-v2/qwen3/qwen3.c:361-372) accumulates
//     s_0 = 0,  s_{i+1} = fl(s_i + fl(x_i * x_i)),  i = 0..n-1
// in index order. Run literally that is a chain of n dependent adds; this
// file produces the identical float with the four compute warps of a CTA.
//
// Every term a_i = fl(x_i * x_i) is >= 0, so s is non-decreasing. While s_i
// and s_{i+1} lie in one binade [2^e, 2^(e+1)), with grid spacing
// u = 2^(e-23), the rounded add is s_i + u * RN(a_i / u), where RN is round
// to nearest and a tie (a_i / u exactly half-way) is broken by the parity of
// s_i. So a run of steps inside one binade with no tie adds the exact integer
// D = sum RN(a_i / u), independent of where the run starts, and runs of the
// same binade that follow one another add their D's.
//
// Which binade each s_i is in is guessed from an approximate FP32 prefix p_i
// of the squares. A step counts as "inside binade e" only with a relative
// margin of 2^-12 on both sides; steps that cross a binade, start below
// 2^-100, or hit a tie are done serially ("singles").
//
// Work split: one warp sums the head [0, H) serially (the sum crosses most
// binades early, where a_i is large relative to s_i); 96 lanes classify
// contiguous chunks of [H, n) into runs and singles with one uniform,
// predicated loop; the entries are compacted and consecutive runs of one
// binade merged into an op list; one warp then walks the ops in order from
// the head's value. A merged run is applied in one exact add only after
// checking that s starts inside binade e and ends below 2^(e+1); otherwise
// its elements are replayed serially. So the result never depends on the
// margin argument, only the speed does.
#pragma once

#include <cstdint>
#include <cmath>
#include <cstring>

namespace bnn {

constexpr int kSegMax = 8;           // entries per lane before the lane goes fully serial
constexpr int kSegSlot = kSegMax + 1;  // per-lane slot stride (one scratch entry)
constexpr int kSegSingle = -1000;    // op: one serial step; d holds the bits of a_first
constexpr int kSegChunk = -1001;     // op: serial steps over [first, last)
constexpr int kRunEMin = -100;       // runs only in binades where u and 2^(23-e) are normal
constexpr int kRunEMax = 125;
constexpr uint32_t kLoMant = 1u << 11;                  // p >= 2^e * (1 + 2^-12)
constexpr uint32_t kHiMant = (1u << 23) - (1u << 12);   // p <= 2^(e+1) * (1 - 2^-12)
constexpr int kSumLanes = 96;        // classifying lanes: warps 0..2
constexpr int kSumHeadWarp = 3;      // warp that sums the head serially

struct SumSeg {
    int e;      // binade exponent of a run, or kSegSingle / kSegChunk
    int first;  // first element index
    int last;   // one past the last element index
    int d;      // run: sum of RN(a_i / u); single: bits of a_first
};

// Shared memory of one sum: per-lane slots (reused for the ops), the
// compacted list, and a few words of cross-warp state.
constexpr int kSumSlotEntries = kSumLanes * kSegSlot;
constexpr int kSumListEntries = kSumLanes * kSegMax;
constexpr size_t kSumSmemBytes = (size_t)(kSumSlotEntries + kSumListEntries) * sizeof(SumSeg) + 64;

__host__ __device__ inline uint32_t fbits(float v) {
    uint32_t b;
    memcpy(&b, &v, sizeof b);
    return b;
}

__host__ __device__ inline float fvalue(uint32_t b) {
    float v;
    memcpy(&v, &b, sizeof v);
    return v;
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

// Head length H and chunk length of the classifying lanes for n terms.
__host__ __device__ inline int sum_head_len(int n) {
    const int h = 32 + n / 32;
    return n - h < kSumLanes * 4 ? n : h;  // short rows: all serial
}

__host__ __device__ inline int sum_chunk_len(int n, int h) {
    // odd, so that the lanes' i-th elements fall in different banks
    return ((n - h + kSumLanes - 1) / kSumLanes) | 1;
}

// Serial sum of squares over [first, last) starting from s.
__host__ __device__ inline float sum_serial(const float* xs, float s, int first, int last) {
    for (int i = first; i < last; ++i)
        s = add_rn(s, sq_rn(xs[i]));
    return s;
}

// Classifies [first, last), whose approximate prefix before `first` is p0,
// into out[0..kSegMax): runs and singles in element order. Returns their
// count, or -1 when more are needed (the chunk is then replayed serially).
// One uniform loop with predicated updates, so the lanes never diverge.
__host__ __device__ inline int sum_classify(const float* xs, int first, int last, float p0, SumSeg* out) {
    int count = 0;
    int run_e = kSegSingle, run_d = 0, run_first = first;
    float p = p0;
    for (int i = first; i < last; ++i) {
        const float a = sq_rn(xs[i]);
        const float pn = add_rn(p, a);
        const uint32_t eb = fbits(p) >> 23;  // p >= 0: the biased exponent
        const int e = (int)eb - 127;
        // inside binade e with the margin: p >= 2^e (1 + 2^-12) and
        // pn <= 2^(e+1) (1 - 2^-12); false for NaN and infinity too
        const bool in = e >= kRunEMin && e <= kRunEMax && p >= fvalue((eb << 23) | kLoMant) &&
                        pn <= fvalue((eb << 23) | kHiMant);
        const int ec = in ? e : 0;
        const float v = mul_rn(a, fvalue((uint32_t)(150 - ec) << 23));  // a / u, exact
        const float r = rintf(v);
        const bool lin = in && fabsf(v - r) != 0.5f;
        const int inc = lin ? (int)r : 0;
        const bool cont = lin && e == run_e;
        if (!cont && run_e != kSegSingle) {  // the current run ends before i
            if (count < kSegMax)
                out[count] = SumSeg{run_e, run_first, i, run_d};
            ++count;
        }
        if (!lin) {
            if (count < kSegMax)
                out[count] = SumSeg{kSegSingle, i, i + 1, (int)fbits(a)};
            ++count;
        }
        run_d = cont ? run_d + inc : inc;
        run_first = cont ? run_first : i;
        run_e = lin ? e : kSegSingle;
        p = pn;
    }
    if (run_e != kSegSingle) {
        if (count < kSegMax)
            out[count] = SumSeg{run_e, run_first, last, run_d};
        ++count;
    }
    return count <= kSegMax ? count : -1;
}

// Merges consecutive runs of one binade in the compacted list into ops;
// returns the op count. (The device does the same with one warp.)
inline int sum_merge_host(const SumSeg* list, int count, SumSeg* ops) {
    int g = -1;
    for (int k = 0; k < count; ++k) {
        const SumSeg it = list[k];
        if (it.e >= kRunEMin && k > 0 && list[k - 1].e == it.e) {
            ops[g].d += it.d;
            ops[g].last = it.last;
        } else {
            ops[++g] = it;
        }
    }
    return g + 1;
}

// Applies the ops in order to s.
__host__ __device__ inline float sum_walk(const float* xs, float s, const SumSeg* ops, int count) {
#pragma unroll 4
    for (int k = 0; k < count; ++k) {
        const SumSeg g = ops[k];
        if (g.e >= kRunEMin) {
            // exact when s starts inside binade e and the sum stays below
            // 2^(e+1): 0 <= d < 2^24 with u = 2^(e-23) normal makes d * u a
            // float, and s and d * u are multiples of u
            const float lo = pow2f(g.e), hi = pow2f(g.e + 1);
            const bool dok = g.d >= 0 && g.d < (1 << 24);
            const float t = add_rn(s, mul_rn((float)(dok ? g.d : 0), pow2f(g.e - 23)));
            if (dok && s >= lo && s < hi && t < hi)
                s = t;
            else
                s = sum_serial(xs, s, g.first, g.last);
        } else if (g.e == kSegSingle) {
            s = add_rn(s, fvalue((uint32_t)g.d));
        } else {
            s = sum_serial(xs, s, g.first, g.last);
        }
    }
    return s;
}

#ifdef __CUDACC__
__device__ __forceinline__ void sum_bar(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Serial sum of squares of xs[0..h), loads and squares batched ahead of the
// dependent adds.
__device__ __forceinline__ float sum_head(const float* xs, int h) {
    float s = 0.0f;
    int i = 0;
    for (; i + 8 <= h; i += 8) {
        float a[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            a[j] = sq_rn(xs[i + j]);
#pragma unroll
        for (int j = 0; j < 8; ++j)
            s = add_rn(s, a[j]);
    }
    for (; i < h; ++i)
        s = add_rn(s, sq_rn(xs[i]));
    return s;
}

// Called by the 128 threads of warps 0..3 of a CTA; returns the serial sum of
// squares of xs[0..n), n >= 1 (shared memory), to all of them. Uses named
// barriers `bar` (128 threads) and `bar + 1` (warps 0..2) and kSumSmemBytes
// of 16-byte aligned shared memory at `mem`.
static __device__ __noinline__ float exact_sumsq(const float* xs, int n, unsigned char* mem, int bar) {
    SumSeg* slots = reinterpret_cast<SumSeg*>(mem);  // per-lane slots, then the ops
    SumSeg* list = slots + kSumSlotEntries;
    float* xf = reinterpret_cast<float*>(list + kSumListEntries);  // [0..2] chunk sums, [3..5] head parts
    int* xi = reinterpret_cast<int*>(xf + 6);                       // [0..2] entry counts
    float* head_value = xf + 12;
    float* result = xf + 13;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = sum_head_len(n);
    if (warp == kSumHeadWarp) {
        if (lane == 0)
            *head_value = sum_head(xs, h);
        sum_bar(bar, 128);  // head value ready
        sum_bar(bar, 128);  // result ready
        return *result;
    }
    int nops = 0;
    if (h < n) {
        const int c = sum_chunk_len(n, h);
        const int first = min(h + tid * c, n), last = min(first + c, n);
        float part0 = 0.0f, part1 = 0.0f, hp = 0.0f;
        int i = first;
        for (; i + 1 < last; i += 2) {
            part0 = add_rn(part0, sq_rn(xs[i]));
            part1 = add_rn(part1, sq_rn(xs[i + 1]));
        }
        if (i < last)
            part0 = add_rn(part0, sq_rn(xs[i]));
        for (int j = tid; j < h; j += kSumLanes)
            hp = add_rn(hp, sq_rn(xs[j]));
        float incl = add_rn(part0, part1);
        for (int o = 1; o < 32; o <<= 1) {
            const float t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o)
                incl = add_rn(incl, t);
            hp = add_rn(hp, __shfl_xor_sync(0xffffffffu, hp, o));
        }
        if (lane == 31) {
            xf[warp] = incl;
            xf[3 + warp] = hp;
        }
        sum_bar(bar + 1, kSumLanes);
        float base = add_rn(add_rn(xf[3], xf[4]), xf[5]);
        if (warp > 0)
            base = add_rn(base, xf[0]);
        if (warp > 1)
            base = add_rn(base, xf[1]);
        float excl = __shfl_up_sync(0xffffffffu, incl, 1);
        if (lane == 0)
            excl = 0.0f;
        SumSeg* mine = slots + tid * kSegSlot;
        int cnt = sum_classify(xs, first, last, add_rn(base, excl), mine);
        if (cnt < 0) {
            mine[0] = SumSeg{kSegChunk, first, last, 0};
            cnt = 1;
        }
        // compact the entries into the list: exclusive scan of the counts
        int off = cnt;
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, off, o);
            if (lane >= o)
                off += t;
        }
        if (lane == 31)
            xi[warp] = off;
        sum_bar(bar + 1, kSumLanes);
        const int total = xi[0] + xi[1] + xi[2];
        off += (warp > 0 ? xi[0] : 0) + (warp > 1 ? xi[1] : 0) - cnt;
        for (int k = 0; k < cnt; ++k)
            list[off + k] = mine[k];
        sum_bar(bar + 1, kSumLanes);  // list complete, slots free
        if (warp == 0) {
            // merge consecutive runs of one binade into ops (over the slots)
            for (int r = 0; r < total; r += 32) {
                const int k = r + lane;
                const bool valid = k < total;
                SumSeg it{kSegSingle, 0, 0, 0};
                bool head = false;
                if (valid) {
                    it = list[k];
                    head = !(it.e >= kRunEMin && k > 0 && list[k - 1].e == it.e);
                }
                const unsigned hb = __ballot_sync(0xffffffffu, head);
                const int gid = nops + __popc(hb & ((2u << lane) - 1u)) - 1;
                if (head)
                    slots[gid] = it;
                __syncwarp();
                if (valid && !head) {
                    atomicAdd(&slots[gid].d, it.d);
                    atomicMax(&slots[gid].last, it.last);
                }
                __syncwarp();
                nops += __popc(hb);
            }
        }
    }
    sum_bar(bar, 128);  // head value ready
    if (warp == 0) {
        const float s = sum_walk(xs, *head_value, slots, nops);
        if (lane == 0)
            *result = s;
    }
    sum_bar(bar, 128);  // result ready
    return *result;
}
#endif

}  // namespace bnn
