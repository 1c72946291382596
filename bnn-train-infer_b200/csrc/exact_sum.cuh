// exact_sum.cuh - the reference's serial FP32 sum of squares, computed in parallel.
//
// qwen3_rmsnorm (bnn-sw-v2/qwen3/qwen3.c:361-372) accumulates
//     s_0 = 0,  s_{i+1} = fl(s_i + fl(x_i * x_i)),  i = 0..n-1
// in index order. Run literally that is a chain of n dependent adds; this
// file produces the identical float with one warp.
//
// Every term a_i = fl(x_i * x_i) is >= 0, so s is non-decreasing. While s_i
// and s_{i+1} lie in one binade [2^e, 2^(e+1)), with grid spacing
// u = 2^(e-23), the rounded add is s_i + u * RN(a_i / u), where RN is round
// to nearest and a tie (a_i / u exactly half-way) is broken by the parity of
// s_i. So a run of steps inside one binade with no tie adds the exact integer
// D = sum RN(a_i / u), independent of where the run starts.
//
// The binade of each s_i is found from a double-precision prefix p_i of the
// exact real sums. The rounded s_i differs from that real sum by at most
// i * 2^-24 relative (each rounding costs at most half an ulp of a value that
// is <= s_i), so a step is taken as "in binade e" only with a margin
// 2^-9 >= 8192 * 2^-24 on both sides. Steps that cross a binade, start from
// 0 or from below 2^-100, or hit a tie are done serially.
//
// Lanes classify contiguous chunks into runs and single steps; lane 0 then
// walks the entries in order, adding each run's D * u in one exact float add.
// The walk re-checks every run (start inside binade e, end below 2^(e+1))
// and replays it serially if the check fails, so the result never depends on
// the margin argument: only the speed does.
#pragma once

#include <cstdint>
#include <cmath>
#include <cstring>

namespace bnn {

constexpr int kSegMax = 16;          // entries per lane before the lane goes fully serial
constexpr int kSegSingle = -100000; // kind marker of a single serial step

struct SumSeg {
    int e;          // binade exponent of a run, or kSegSingle
    int first;      // first element index
    int last;       // one past the last element index
    int pad;
    long long d;    // run: sum of RN(a_i / u)
};

__host__ __device__ inline double pow2d(int e) {
    // 2^e for -1022 <= e <= 1023, exactly
    unsigned long long bits = (unsigned long long)(e + 1023) << 52;
    double r;
    memcpy(&r, &bits, sizeof r);
    return r;
}

__host__ __device__ inline float pow2f(int e) {
    // 2^e for -126 <= e <= 127, exactly
    uint32_t bits = (uint32_t)(e + 127) << 23;
    float r;
    memcpy(&r, &bits, sizeof r);
    return r;
}

__host__ __device__ inline int ilog2d(double p) {
    // floor(log2(p)) for a normal positive double
    unsigned long long bits;
    memcpy(&bits, &p, sizeof bits);
    return (int)((bits >> 52) & 0x7ff) - 1023;
}

#ifdef __CUDA_ARCH__
__device__ __forceinline__ float sq_rn(float x) { return __fmul_rn(x, x); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
#else
inline float sq_rn(float x) {
    volatile float r = x * x;
    return r;
}
inline float add_rn(float a, float b) {
    volatile float r = a + b;
    return r;
}
#endif

// Classifies elements [first, last) whose exact real prefix before `first`
// is p0. Writes at most kSegMax entries; returns their count, or -1 if the
// chunk needs more (then it is replayed serially).
__host__ __device__ inline int sum_classify(const float* xs, int first, int last, double p0, SumSeg* out) {
    const double margin = 1.0 / 512.0;
    // Fast path: the whole chunk stays inside one binade.
    if (p0 > 0.0 && first < last) {
        const int e = ilog2d(p0);
        if (e >= -100 && e <= 126 && p0 >= pow2d(e) * (1.0 + margin)) {
            const double scale = pow2d(23 - e), limit = pow2d(e + 1) * (1.0 - margin);
            double p = p0;
            long long d = 0;
            bool ok = true;
            for (int i = first; i < last && ok; ++i) {
                const float a = sq_rn(xs[i]);
                p += (double)a;
                const double v = (double)a * scale;
                const double fl = floor(v);
                const double fr = v - fl;
                ok = p <= limit && fr != 0.5;
                d += (long long)fl + (fr > 0.5 ? 1 : 0);
            }
            if (ok) {
                out[0] = SumSeg{e, first, last, 0, d};
                return 1;
            }
        }
    }
    int count = 0;
    int run_e = kSegSingle;
    long long run_d = 0;
    int run_first = first;
    double p = p0;
    for (int i = first; i < last; ++i) {
        const float a = sq_rn(xs[i]);
        const double pn = p + (double)a;
        bool lin = false;
        int e = 0;
        long long inc = 0;
        if (p > 0.0) {
            e = ilog2d(p);
            if (e >= -100 && e <= 126 && p >= pow2d(e) * (1.0 + margin) && pn <= pow2d(e + 1) * (1.0 - margin)) {
                const double v = (double)a * pow2d(23 - e);  // exact: a < 2^(e+1)
                const double fl = floor(v);
                const double fr = v - fl;
                if (fr != 0.5) {
                    lin = true;
                    inc = (long long)fl + (fr > 0.5 ? 1 : 0);
                }
            }
        }
        if (lin && e == run_e) {
            run_d += inc;
        } else {
            if (run_e != kSegSingle) {
                if (count == kSegMax)
                    return -1;
                out[count++] = SumSeg{run_e, run_first, i, 0, run_d};
                run_e = kSegSingle;
            }
            if (lin) {
                run_e = e;
                run_d = inc;
                run_first = i;
            } else {
                if (count == kSegMax)
                    return -1;
                out[count++] = SumSeg{kSegSingle, i, i + 1, 0, 0};
            }
        }
        p = pn;
    }
    if (run_e != kSegSingle) {
        if (count == kSegMax)
            return -1;
        out[count++] = SumSeg{run_e, run_first, last, 0, run_d};
    }
    return count;
}

// Applies one lane's entries (or, for count < 0, its whole chunk) to s.
__host__ __device__ inline float sum_walk(const float* xs, float s, const SumSeg* seg, int count, int first,
                                          int last) {
    if (count < 0) {
        for (int i = first; i < last; ++i)
            s = add_rn(s, sq_rn(xs[i]));
        return s;
    }
    for (int k = 0; k < count; ++k) {
        const SumSeg g = seg[k];
        if (g.e != kSegSingle) {
            const float lo = pow2f(g.e), hi = pow2f(g.e + 1);
            if (s >= lo && s < hi && g.d < (1ll << 24)) {
                // exact: d < 2^24, u a power of two, and the sum is a
                // multiple of u below 2^(e+1) (checked next)
                const float t = add_rn(s, (float)g.d * pow2f(g.e - 23));
                if (t < hi) {
                    s = t;
                    continue;
                }
            }
        }
        for (int i = g.first; i < g.last; ++i)
            s = add_rn(s, sq_rn(xs[i]));
    }
    return s;
}

// Warp-cooperative: all 32 lanes of one warp call it; returns the serial sum
// of squares of xs[0..n) (shared or global memory) to every lane. seg needs
// 32 * kSegMax entries and cnt 32 ints of shared memory.
static __device__ __noinline__ float exact_sumsq_warp(const float* xs, int n, SumSeg* seg, int* cnt) {
    const int lane = threadIdx.x & 31;
    const int chunk = (n + 31) / 32;
    const int first = min(lane * chunk, n), last = min(first + chunk, n);
    double part = 0.0;
    bool finite = true;
    for (int i = first; i < last; ++i) {
        const float a = sq_rn(xs[i]);
        finite &= isfinite(a);
        part += (double)a;
    }
    double incl = part;
    for (int o = 1; o < 32; o <<= 1) {
        const double t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o)
            incl += t;
    }
    finite = __all_sync(0xffffffffu, finite);
    cnt[lane] = finite ? sum_classify(xs, first, last, incl - part, seg + lane * kSegMax) : -1;
    __syncwarp();
    float s = 0.0f;
    if (lane == 0) {
        for (int l = 0; l < 32; ++l) {
            const int f = min(l * chunk, n), e = min(f + chunk, n);
            s = sum_walk(xs, s, seg + l * kSegMax, cnt[l], f, e);
        }
    }
    return __shfl_sync(0xffffffffu, s, 0);
}

}  // namespace bnn
