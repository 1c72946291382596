// Host emulation of exact_sumsq (bnn-train-infer_b200/csrc/exact_sum.cuh): the
// 256-thread parallel form of the reference's serial FP32 sum of squares
// (qwen3.c:361-372), replayed step by step with the header's own host-callable
// pieces (sum_approx, sum_classify, sum_serial) and the same order of every
// float operation as the device code (warp scans, block scan, walk of 32 ops
// with per-lane checks and replay of the first failing op). Each vector's
// result is compared bit for bit with the plain serial loop.
//
// Usage: exact_sum_host <vectors per family> <seed> [plant]; prints one
// line per family (with how many ops took the run path, the single path, or
// were replayed) and "mismatches N" at the end (exit status 1 when N > 0).
// "plant" plants a mistake in this emulation (every run adds one unit more
// than its increments), which the comparison with the serial loop must
// catch.
#define __host__
#define __device__
#define __forceinline__ inline
#include "exact_sum.cuh"

#include <algorithm>
#include <string>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <vector>

using namespace bnn;

namespace {

bool g_plant = false;
long g_runs = 0, g_singles = 0, g_replays = 0;

float exact_sumsq_host(const float* xs, int n) {
    const int T = kSumThreads, W = kSumWarpsN;
    const int len = sum_chunk_len(n);
    std::vector<float> part(T), incl(T), excl(T), wsum(W);
    for (int t = 0; t < T; ++t) {
        const int first = std::min(t * len, n), last = std::min(first + len, n);
        part[t] = sum_approx(xs, first, last);
    }
    // warp inclusive scans (Hillis-Steele: lane l adds lane l - o of the previous round)
    incl = part;
    for (int w = 0; w < W; ++w)
        for (int o = 1; o < 32; o <<= 1) {
            float prev[32];
            for (int l = 0; l < 32; ++l)
                prev[l] = incl[w * 32 + l];
            for (int l = o; l < 32; ++l)
                incl[w * 32 + l] = add_rn(prev[l], prev[l - o]);
        }
    for (int w = 0; w < W; ++w)
        wsum[w] = incl[w * 32 + 31];
    for (int t = 0; t < T; ++t) {
        const int w = t / 32, l = t % 32;
        float e = l == 0 ? 0.0f : incl[t - 1];
        for (int v = 0; v < w; ++v)
            e = add_rn(e, wsum[v]);
        excl[t] = e;
    }
    // classification
    std::vector<SumRec> slots((size_t)T * kSumSlotStride);
    std::vector<int> cnt(T), inc_total(T), last_tag(T);
    for (int t = 0; t < T; ++t) {
        const int first = std::min(t * len, n), last = std::min(first + len, n);
        SumRec* mine = &slots[(size_t)t * kSumSlotStride];
        int c = sum_classify(xs, first, last, excl[t], mine, &inc_total[t], &last_tag[t]);
        if (c < 0) {
            mine[0] = SumRec{first | (kTagChunk << 16), 0};
            c = 1;
            last_tag[t] = kTagChunk;
        }
        cnt[t] = c;
    }
    // increments before each thread, kept records, compaction (integer sums: order-free)
    std::vector<int> keep(T), coff(T), ioff(T);
    std::vector<bool> drop(T);
    int total = 0, inc_all = 0;
    for (int t = 0; t < T; ++t) {
        const SumRec* mine = &slots[(size_t)t * kSumSlotStride];
        const int tag0 = cnt[t] > 0 ? rec_tag(mine[0].key) : -1;
        drop[t] = tag0 != -1 && tag0 != kTagSingle && tag0 != kTagChunk && t > 0 && last_tag[t - 1] == tag0;
        keep[t] = cnt[t] - (drop[t] ? 1 : 0);
        coff[t] = total;
        ioff[t] = inc_all;
        total += keep[t];
        inc_all += inc_total[t];
    }
    std::vector<SumRec> list((size_t)kSumListMax + 2);
    for (int t = 0; t < T; ++t) {
        const SumRec* mine = &slots[(size_t)t * kSumSlotStride];
        for (int k = drop[t] ? 1 : 0; k < cnt[t]; ++k) {
            SumRec r = mine[k];
            r.cum += ioff[t];
            list[coff[t] + k - (drop[t] ? 1 : 0)] = r;
        }
    }
    list[total] = list[total + 1] = SumRec{n, inc_all};
    // the walk of warp 0
    float s = 0.0f;
    int k = 0;
    while (k < total) {
        float ad[32], before[32], after[32];
        bool ok[32], run[32];
        int e[32];
        for (int lane = 0; lane < 32; ++lane) {
            const int idx = k + lane;
            const bool valid = idx < total;
            const int ci = valid ? idx : total;
            const SumRec rec = list[ci], nx = list[ci + 1];
            const int tag = rec_tag(rec.key);
            const float a = sq_rn(xs[std::min(rec_first(rec.key), n - 1)]);
            const int d = nx.cum - rec.cum;
            const bool single = tag == kTagSingle;
            run[lane] = valid && !single && tag != kTagChunk && d >= 0 && d < (1 << 24);
            e[lane] = run[lane] ? tag - 128 : 0;
            const int dd = d + (g_plant ? 1 : 0);
            ad[lane] = !valid ? 0.0f : single ? a : run[lane] ? mul_rn((float)dd, pow2f(e[lane] - 23)) : 0.0f;
            ok[lane] = !valid || single || run[lane];
        }
        float cur = s;
        for (int j = 0; j < 32; ++j) {
            const float next = add_rn(cur, ad[j]);
            before[j] = cur;
            after[j] = next;
            cur = next;
        }
        int f = -1;
        for (int lane = 0; lane < 32; ++lane) {
            if (run[lane])
                ok[lane] = before[lane] >= pow2f(e[lane]) && before[lane] < pow2f(e[lane] + 1) &&
                           after[lane] < pow2f(e[lane] + 1);
            if (!ok[lane] && f < 0)
                f = lane;
        }
        for (int lane = 0; lane < (f < 0 ? 32 : f); ++lane)
            if (k + lane < total) {
                g_runs += run[lane];
                g_singles += !run[lane];
            }
        if (f < 0) {
            s = cur;
            k += 32;
            continue;
        }
        ++g_replays;
        s = before[f];
        s = sum_serial(xs, s, rec_first(list[k + f].key), rec_first(list[k + f + 1].key));
        k += f + 1;
    }
    return s;
}

// The same walk over a compacted op list, starting from s (the wide form's
// walk is the 256-thread walk over its own list).
float walk_host(const float* xs, int n, const std::vector<SumRec>& list, int total, float s) {
    int k = 0;
    while (k < total) {
        float ad[32], before[32], after[32];
        bool ok[32], run[32];
        int e[32];
        for (int lane = 0; lane < 32; ++lane) {
            const int idx = k + lane;
            const bool valid = idx < total;
            const int ci = valid ? idx : total;
            const SumRec rec = list[ci], nx = list[ci + 1];
            const int tag = rec_tag(rec.key);
            const float a = sq_rn(xs[std::min(rec_first(rec.key), n - 1)]);
            const uint32_t d = (uint32_t)nx.cum - (uint32_t)rec.cum;
            const bool single = tag == kTagSingle;
            run[lane] = valid && !single && d < (1u << 24);
            e[lane] = run[lane] ? tag - 128 : 0;
            const uint32_t dd = d + (g_plant ? 1u : 0u);
            ad[lane] = !valid ? 0.0f : single ? a : run[lane] ? mul_rn((float)dd, pow2f(e[lane] - 23)) : 0.0f;
            ok[lane] = !valid || single || run[lane];
        }
        float cur = s;
        for (int j = 0; j < 32; ++j) {
            const float next = add_rn(cur, ad[j]);
            before[j] = cur;
            after[j] = next;
            cur = next;
        }
        int f = -1;
        for (int lane = 0; lane < 32; ++lane) {
            if (run[lane])
                ok[lane] = before[lane] >= pow2f(e[lane]) && before[lane] < pow2f(e[lane] + 1) &&
                           after[lane] < pow2f(e[lane] + 1);
            if (!ok[lane] && f < 0)
                f = lane;
        }
        for (int lane = 0; lane < (f < 0 ? 32 : f); ++lane)
            if (k + lane < total) {
                g_runs += run[lane];
                g_singles += !run[lane];
            }
        if (f < 0) {
            s = cur;
            k += 32;
            continue;
        }
        ++g_replays;
        s = before[f];
        s = sum_serial(xs, s, rec_first(list[k + f].key), rec_first(list[k + f + 1].key));
        k += f + 1;
    }
    return s;
}

// Host emulation of exact_sumsq_wide (512 threads, 4 elements each, passes
// of 2048), with the device code's order of float operations.
float exact_sumsq_wide_host(const float* xs, int n) {
    const int T = kWideThreads, W = kWideWarps, P = kWidePer;
    float s0 = 0.0f;
    for (int base = 0; base < n; base += kWideChunk) {
        const int m = std::min(kWideChunk, n - base);
        const float* xc = xs + base;
        std::vector<float> a((size_t)T * P), incl(T), wt(W);
        for (int t = 0; t < T; ++t) {
            float loc = 0.0f;
            for (int q = 0; q < P; ++q) {
                const int j = t * P + q;
                a[(size_t)t * P + q] = j < m ? sq_rn(xc[j]) : 0.0f;
                loc = q == 0 ? a[(size_t)t * P] : add_rn(loc, a[(size_t)t * P + q]);
            }
            incl[t] = loc;
        }
        for (int w = 0; w < W; ++w)
            for (int o = 1; o < 32; o <<= 1) {
                float prev[32];
                for (int l = 0; l < 32; ++l)
                    prev[l] = incl[w * 32 + l];
                for (int l = o; l < 32; ++l)
                    incl[w * 32 + l] = add_rn(prev[l], prev[l - o]);
            }
        for (int w = 0; w < W; ++w)
            wt[w] = incl[w * 32 + 31];
        std::vector<int> tag((size_t)T * P), cnt(T);
        std::vector<uint32_t> inc((size_t)T * P), ksum(T);
        std::vector<char> start((size_t)T * P);
        // the earlier warps' totals by the device's xor-shuffle tree
        std::vector<float> wpre(W);
        for (int w = 0; w < W; ++w) {
            float v[32];
            for (int l = 0; l < 32; ++l)
                v[l] = l < w ? wt[l] : 0.0f;
            for (int o = 16; o > 0; o >>= 1) {
                float nv[32];
                for (int l = 0; l < 32; ++l)
                    nv[l] = add_rn(v[l], v[l ^ o]);
                std::copy(nv, nv + 32, v);
            }
            wpre[w] = v[0];
        }
        for (int t = 0; t < T; ++t) {
            const int w = t / 32, l = t % 32;
            float pb = add_rn(add_rn(s0, wpre[w]), l == 0 ? 0.0f : incl[t - 1]);
            for (int q = 0; q < P; ++q) {
                sum_classify_one(a[(size_t)t * P + q], pb, &tag[(size_t)t * P + q], &inc[(size_t)t * P + q]);
                pb = add_rn(pb, a[(size_t)t * P + q]);
            }
        }
        for (int t = 0; t < T; ++t) {
            const int prev = t % 32 == 0 ? -1 : tag[(size_t)t * P + P - 1 - P];
            cnt[t] = 0;
            ksum[t] = 0;
            for (int q = 0; q < P; ++q) {
                const int j = t * P + q;
                const bool valid = j < m;
                const int pt = q ? tag[(size_t)j - 1] : prev;
                start[j] = valid && (tag[j] == kTagSingle || tag[j] != pt);
                cnt[t] += start[j];
                ksum[t] += valid ? inc[j] : 0u;
            }
        }
        std::vector<SumRec> list((size_t)kWideChunk + 2);
        int total = 0;
        uint32_t kc = 0;
        for (int t = 0; t < T; ++t)
            for (int q = 0; q < P; ++q) {
                const int j = t * P + q;
                if (start[j])
                    list[total++] = SumRec{j | (tag[j] << 16), (int)kc};
                kc += j < m ? inc[j] : 0u;
            }
        list[total] = list[total + 1] = SumRec{m, (int)kc};
        s0 = walk_host(xc, m, list, total, s0);
    }
    return s0;
}

uint32_t bits_of(float v) { return fbits(v); }

}  // namespace

int main(int argc, char** argv) {
    const int per = argc > 1 ? atoi(argv[1]) : 200;
    const unsigned seed = argc > 2 ? (unsigned)atoi(argv[2]) : 1u;
    bool wide = false;
    for (int i = 3; i < argc; ++i) {
        g_plant |= std::string(argv[i]) == "plant";
        wide |= std::string(argv[i]) == "wide";
    }
    std::mt19937 rng(seed);
    std::normal_distribution<float> normal(0.0f, 1.0f);
    std::uniform_real_distribution<float> uni(0.0f, 1.0f);
    const int lens[] = {1, 2, 3, 31, 255, 256, 257, 511, 1024, 2048, 4099, 6144, 8192};
    auto pick_len = [&]() {
        return (rng() & 1) ? lens[rng() % (sizeof lens / sizeof lens[0])] : 1 + (int)(rng() % 8192);
    };
    const char* names[] = {"normal", "outliers", "wide-range", "half-ulp ties", "tiny/huge/zero", "long"};
    long mismatches = 0, checked = 0;
    for (int fam = 0; fam < 6; ++fam) {
        long fam_bad = 0;
        g_runs = g_singles = g_replays = 0;
        for (int v = 0; v < per; ++v) {
            const int n = fam == 5 ? 16384 + (int)(rng() % 49151) : pick_len();
            std::vector<float> x(n);
            for (int i = 0; i < n; ++i) {
                float r = normal(rng);
                switch (fam) {
                    case 0: x[i] = r; break;
                    case 1: x[i] = uni(rng) < 0.01f ? r * 20.0f : r; break;
                    case 2: x[i] = std::ldexp(1.0f + uni(rng), -60 + (int)(rng() % 110)) * (r < 0 ? -1.0f : 1.0f); break;
                    case 3: {
                        // x^2 = half a unit of the running sum's last place: 1, then
                        // 2^-12 (2^-24 = u/2 at s in [1, 2)), with a few other binades
                        const int shift = (int)(rng() % 4) * 2;
                        x[i] = i == 0 ? std::ldexp(1.0f, shift) : std::ldexp(uni(rng) < 0.9f ? 1.0f : 1.5f, -12 + shift / 2);
                        break;
                    }
                    case 4: {
                        const float u = uni(rng);
                        x[i] = u < 0.2f ? 0.0f : u < 0.4f ? r * 1e-25f : u < 0.5f ? r * 1e18f : u < 0.6f ? r * 1e-20f : r;
                        break;
                    }
                    default: x[i] = r * (uni(rng) < 0.001f ? 1e3f : 1.0f); break;
                }
            }
            const float want = sum_serial(x.data(), 0.0f, 0, n);
            const float got = wide ? exact_sumsq_wide_host(x.data(), n) : exact_sumsq_host(x.data(), n);
            ++checked;
            if (bits_of(want) != bits_of(got)) {
                ++fam_bad;
                if (fam_bad <= 3)
                    printf("  %s n=%d: serial %a, parallel %a\n", names[fam], n, want, got);
            }
        }
        printf("%-15s %d vectors, %ld mismatches; ops: %ld runs, %ld singles, %ld replays\n", names[fam], per,
               fam_bad, g_runs, g_singles, g_replays);
        mismatches += fam_bad;
    }
    printf("checked %ld mismatches %ld\n", checked, mismatches);
    return mismatches ? 1 : 0;
}
