// engine_kernels.cuh - the device-resident glue of the Qwen3 / bnn-mlp step.
//
// Each kernel restates one piece of the reference's host glue with the same
// FP32 operation order (bnn-sw-v2/qwen3/qwen3.c, bnn-mlp/bnn-mlp.c), using
// explicit round-to-nearest intrinsics so nothing is fused or reassociated:
//   embed_kernel            qwen3_embed               qwen3.c:374-385
//   attention_kernel        per-head q/k RMSNorm, RoPE, KV append and
//                           causal softmax attention  qwen3.c:418-478
//   mlp_post_kernel         post_scale/bias + ReLU    bnn-mlp.c:189-193
// RMSNorm before a linear, the row quantisation, SwiGLU and the greedy pick
// (bnn-infer-v2.c:48-54, engine.c:262-267: first index of the maximum, any
// non-finite logit an error) run inside the W1A8 linears (w1a8_gemv.cuh
// prologues/epilogues). In exact mode every long
// sum is accumulated serially in index order, as the reference does; fast
// mode uses a fixed-order tree instead.
#pragma once

#include <cstdint>
#include "bnn_device.cuh"
#include "bnn_sync.cuh"

namespace bnn {
namespace eng {

constexpr int kStatusNonFinite = 4;  // RMSNorm divisor, softmax or logits not finite

// Block-wide reductions (blockDim.x a multiple of 32, <= 1024).
__device__ __forceinline__ float block_max(float v, float* red) {
    for (int o = 16; o > 0; o >>= 1)
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0)
        red[w] = v;
    __syncthreads();
    v = red[0];
    for (int i = 1; i < nw; ++i)
        v = fmaxf(v, red[i]);
    return v;
}

// Sum of `vals[0..n)` (shared memory). exact: serial in index order by
// thread 0 (the reference's loop); otherwise a fixed-order tree. The result
// is returned to every thread.
static __device__ float block_sum_ordered(const float* vals, uint32_t n, bool exact, float* red) {
    __syncthreads();
    if (exact) {
        if (threadIdx.x == 0) {
            float s = 0.0f;
            for (uint32_t i = 0; i < n; ++i)
                s = __fadd_rn(s, vals[i]);
            red[0] = s;
        }
        __syncthreads();
        return red[0];
    }
    float s = 0.0f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x)
        s = __fadd_rn(s, vals[i]);
    for (int o = 16; o > 0; o >>= 1)
        s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if ((threadIdx.x & 31) == 0)
        red[32 + w] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int i = 0; i < nw; ++i)
            t = __fadd_rn(t, red[32 + i]);
        red[0] = t;
    }
    __syncthreads();
    return red[0];
}

// qwen3_embed: x[c] = bit ? scale : -scale, read from lm_head's packed
// blocks (token_embd and lm_head are the same tied matrix). best (one entry
// per row, or null) is the greedy pick the step's lm_head will fill.
__global__ void embed_kernel(const int32_t* tokens, const unsigned char* wblocks, uint32_t c, float* x,
                             unsigned long long* best) {
    const uint32_t row = blockIdx.x;
    if (best && threadIdx.x == 0)
        best[row] = 0ull;  // the step's greedy pick starts empty
    const uint32_t tok = (uint32_t)tokens[row];
    const uint32_t groups = c / kGroup;
    const uint32_t r = tok % kRowBlock;
    const unsigned char* blk = wblocks + (size_t)(tok / kRowBlock) * groups * 144u;
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(blk + (size_t)groups * 128u) + (size_t)r * groups;
    for (uint32_t k = threadIdx.x; k < c; k += blockDim.x) {
        const uint32_t g = k / kGroup, b = k % kGroup;
        const uint32_t word = reinterpret_cast<const uint32_t*>(blk + (g * kRowBlock + r) * 16u)[b >> 5];
        const float scale = h2f(sc[g]);
        x[(size_t)row * c + k] = ((word >> (b & 31)) & 1u) ? scale : -scale;
    }
}

// ---- attention: q/k RMSNorm, RoPE, KV append and causal softmax attention
// in one kernel per (KV head, row). The KV cache of a layer is laid out
// [rows][kv_heads][n_ctx][head_dim], so the positions of one head are
// contiguous: K and V are streamed through shared memory as tiles of
// kAttnTile positions with 1D bulk copies (K rows padded against bank
// conflicts), in a two-stage ring; the first K tiles are requested before
// the kernel waits for the q|k|v projection, since the cache rows it reads
// were written by earlier steps. The current position's k and v are used
// straight from shared memory. While the whole history fits in shared memory
// (n <= resident_max), K and V are instead copied whole at the start and
// every phase spreads over all threads: no tiles, no per-tile waits.
constexpr uint32_t kAttnThreads = 512;
constexpr uint32_t kAttnTile = 128;
constexpr uint32_t kAttnStages = 2;

struct AttnArgs {
    const float* qkv;       // [rows][C + 2KV]: q | k | v projections
    const float* q_norm;    // [HD]
    const float* k_norm;    // [HD]
    const float* rope_cos;  // [n_ctx][HD/2]
    const float* rope_sin;
    const uint32_t* pos;    // [rows]
    float* kcache;          // this layer: [rows][kv_heads][n_ctx][kcache_row(HD)]
    float* vcache;          // this layer: [rows][kv_heads][n_ctx][HD]
    float* scores;          // [rows][heads][attn_sc_stride(n_ctx)] when they do not fit in shared memory, else null
    float* y;               // output rows: this block's heads at y + row * y_stride + head * HD
    uint32_t y_stride;      // floats between output rows
    uint32_t c, kv, hd, heads, kv_heads, n_ctx;
    float eps;
    float scale;            // 1 / sqrtf(head_dim), computed on the host as qwen3.c:404
    int exact;
    int* status;
    uint32_t resident_max;  // positions n up to which K and V are held whole in shared memory (0: never)
};

// Floats per K-cache position: the head vector and 4 floats of padding, so a
// run of positions copied into shared memory with one bulk copy already has
// the bank-spread row stride the score loops read (padding never read).
__host__ __device__ constexpr uint32_t kcache_row(uint32_t hd) { return hd + 4u; }

// Scores of one query head occupy a row of this many floats (a multiple of
// 4, so the V pass can read four probabilities at once).
__host__ __device__ inline uint32_t attn_sc_stride(uint32_t n_ctx) { return (n_ctx + 3u) & ~3u; }

struct AttnSmem {
    size_t bars, red, q, kn, vn, gq, gk, rc, rs, sc, ring, stage_bytes, total;
};

// Positions held whole (K rows padded, V dense) in `bytes` of shared memory past the ring start.
__host__ __device__ inline uint32_t attn_resident_rows(uint32_t hd, size_t bytes) {
    return (uint32_t)(bytes / ((size_t)(2u * hd + 4u) * 4u));
}

__host__ __device__ inline AttnSmem attn_smem_plan(uint32_t hd, uint32_t kv_mul, uint32_t n_ctx, bool sc_smem) {
    AttnSmem p;
    p.bars = 0;                                // full[kAttnStages]
    p.red = 64;                                // 64 floats
    p.q = p.red + 64 * 4;                      // [kv_mul][hd]
    p.kn = p.q + (size_t)kv_mul * hd * 4;      // [hd]
    p.vn = p.kn + (size_t)hd * 4;              // [hd]
    p.gq = p.vn + (size_t)hd * 4;              // q_norm gain [hd]
    p.gk = p.gq + (size_t)hd * 4;              // k_norm gain [hd]
    p.rc = p.gk + (size_t)hd * 4;              // cos row of this position [hd/2]
    p.rs = p.rc + (size_t)hd * 2;              // sin row [hd/2]
    p.sc = p.rs + (size_t)hd * 2;              // [kv_mul][attn_sc_stride(n_ctx)] when in shared memory
    p.ring = (p.sc + (sc_smem ? (size_t)kv_mul * attn_sc_stride(n_ctx) * 4 : 0) + 127) & ~(size_t)127;
    p.stage_bytes = (size_t)kAttnTile * (hd + 4) * 4;  // K rows padded by 4 floats; V tiles dense
    p.total = p.ring + kAttnStages * p.stage_bytes;
    return p;
}

// qwen3_rmsnorm of one head vector (HD floats in shared memory, by one warp)
// followed by qwen3_rope (qwen3.c:418-438), in place; gain, cos and sin rows
// in shared memory. Returns false when the divisor is not finite or zero.
template <int HD>
__device__ inline bool attn_norm_rope(float* v, const float* gain, const float* cs, const float* sn, float eps,
                                      bool exact) {
    constexpr int kPer = HD / 32;
    const uint32_t lane = threadIdx.x & 31;
    float x[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k)
        x[k] = v[lane + 32 * k];
    float sum = 0.0f;
    if (exact) {
        // the reference's serial sum, index order (loads batched ahead)
        if (lane == 0) {
#pragma unroll
            for (int i = 0; i < HD; i += 16) {
                float a[16];
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    a[j] = __fmul_rn(v[i + j], v[i + j]);
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    sum = __fadd_rn(sum, a[j]);
            }
        }
        sum = __shfl_sync(0xffffffffu, sum, 0);
    } else {
#pragma unroll
        for (int k = 0; k < kPer; ++k)
            sum = __fadd_rn(sum, __fmul_rn(x[k], x[k]));
        for (int o = 16; o > 0; o >>= 1)
            sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
    }
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)HD), eps));
    if (!isfinite(rms) || rms == 0.0f)
        return false;
    const float rr = __frcp_rn(rms);
#pragma unroll
    for (int k = 0; k < kPer; ++k)
        v[lane + 32 * k] = __fmul_rn(div_cr(x[k], rms, rr), gain[lane + 32 * k]);
    __syncwarp();
    constexpr int kHalf = HD / 2;
    float out[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const int i = lane + 32 * k;
        if (i < kHalf)
            out[k] = __fsub_rn(__fmul_rn(v[i], cs[i]), __fmul_rn(v[i + kHalf], sn[i]));
        else
            out[k] = __fadd_rn(__fmul_rn(v[i - kHalf], sn[i - kHalf]), __fmul_rn(v[i], cs[i - kHalf]));
    }
    __syncwarp();
#pragma unroll
    for (int k = 0; k < kPer; ++k)
        v[lane + 32 * k] = out[k];
    __syncwarp();
    return true;
}

// One block of kAttnThreads per (KV head g, row); it serves the kv_mul query
// heads g * kv_mul .. that share the KV head (qwen3.c:440-478):
//   scores[t] = fl(dot(q, k_t)) * scale, the dot accumulated serially over
//   the head dimension; softmax with expf(s - max), a serial sum over t and a
//   division; y_i = sum_t p_t * v_t,i, serial in t.
// Fast mode replaces the serial sums of the norms and the softmax by trees.
// SCS: the scores live in shared memory (a.scores null); a compile-time
// choice, so every score access is a shared-memory access (a pointer that
// may be either costs a serial softmax sum more than twice the cycles).
template <int HD, int KVM, bool SCS>
__global__ void __launch_bounds__(kAttnThreads, 1) attention_kernel(AttnArgs a) {
    griddep_launch_dependents();
    extern __shared__ __align__(128) unsigned char e_smem[];
    const uint32_t g = blockIdx.x, row = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr uint32_t kv_mul = KVM;  // query heads per KV head (a.heads / a.kv_heads)
    constexpr bool sc_smem = SCS;
    const AttnSmem plan = attn_smem_plan(HD, kv_mul, a.n_ctx, sc_smem);
    uint64_t* full = reinterpret_cast<uint64_t*>(e_smem + plan.bars);
    float* red = reinterpret_cast<float*>(e_smem + plan.red);
    float* q_s = reinterpret_cast<float*>(e_smem + plan.q);
    float* kn_s = reinterpret_cast<float*>(e_smem + plan.kn);
    float* vn_s = reinterpret_cast<float*>(e_smem + plan.vn);
    float* gq_s = reinterpret_cast<float*>(e_smem + plan.gq);
    float* gk_s = reinterpret_cast<float*>(e_smem + plan.gk);
    float* rc_s = reinterpret_cast<float*>(e_smem + plan.rc);
    float* rs_s = reinterpret_cast<float*>(e_smem + plan.rs);
    const uint32_t sc_stride = attn_sc_stride(a.n_ctx);  // per-head rows of scores, float4-aligned
    float* sc = sc_smem ? reinterpret_cast<float*>(e_smem + plan.sc)
                        : a.scores + ((size_t)row * a.heads + (size_t)g * kv_mul) * sc_stride;
    unsigned char* ring = e_smem + plan.ring;
    int* flag = reinterpret_cast<int*>(red + 62);  // [0] abort: earlier failure, non-finite, timeout

    const uint32_t pos = a.pos[row], n = pos + 1;
    const uint32_t ntiles = (n + kAttnTile - 1) / kAttnTile, nloads = 2 * ntiles;
    constexpr uint32_t kstride = kcache_row(HD);  // K rows in the cache and in shared memory
    const size_t head_base = ((size_t)row * a.kv_heads + g) * a.n_ctx * HD;
    const size_t khead_base = ((size_t)row * a.kv_heads + g) * a.n_ctx * kstride;
    const float* kc = a.kcache + khead_base;
    const float* vc = a.vcache + head_base;
    const bool resident = n <= a.resident_max;
    float* kres = reinterpret_cast<float*>(ring);                // [resident_max][kstride]
    float* vres = kres + (size_t)a.resident_max * kstride;       // [resident_max][HD]

    if (tid == 0) {
        for (uint32_t s = 0; s < kAttnStages; ++s)
            mbar_init(&full[s], 1);
        fence_barrier_init();
        *flag = 0;
    }
    __syncthreads();
    // Load L (< ntiles: K tile L, rows padded; else V tile L - ntiles, dense)
    // into stage L % kAttnStages; issued by warp 0.
    auto issue = [&](uint32_t L) {
        const uint32_t s = L % kAttnStages;
        const bool is_k = L < ntiles;
        const uint32_t t0 = (is_k ? L : L - ntiles) * kAttnTile;
        const uint32_t rows_in = min(kAttnTile, n - t0);
        unsigned char* dst = ring + (size_t)s * plan.stage_bytes;
        if (lane == 0) {
            // K tile: padded rows, V tile: dense rows; one bulk copy each
            const uint32_t bytes = rows_in * (is_k ? kstride : (uint32_t)HD) * 4u;
            mbar_arrive_expect_tx(&full[s], bytes);
            bulk_g2s(dst, is_k ? kc + (size_t)t0 * kstride : vc + (size_t)t0 * HD, bytes, &full[s]);
        }
        __syncwarp();
    };
    if (warp == 0) {
        if (resident) {
            // every earlier position of the head at once: K rows padded, V dense
            if (lane == 0) {
                mbar_arrive_expect_tx(&full[0], pos * (kstride + HD) * 4u);
                if (pos > 0) {
                    bulk_g2s(kres, kc, pos * kstride * 4u, &full[0]);
                    bulk_g2s(vres, vc, pos * HD * 4u, &full[0]);
                }
            }
            __syncwarp();
        } else {
            for (uint32_t L = 0; L < kAttnStages && L < nloads; ++L)
                issue(L);
        }
    }
    // weights and rope rows do not depend on earlier kernels either
    for (uint32_t i = tid; i < HD; i += kAttnThreads) {
        gq_s[i] = a.q_norm[i];
        gk_s[i] = a.k_norm[i];
    }
    for (uint32_t i = tid; i < HD / 2; i += kAttnThreads) {
        rc_s[i] = a.rope_cos[(size_t)pos * (HD / 2) + i];
        rs_s[i] = a.rope_sin[(size_t)pos * (HD / 2) + i];
    }

    // ---- wait for the q|k|v projection; norm + rope of the q heads and the k head
    griddep_wait();
    const size_t width = a.c + 2u * a.kv;
    const float* qkv_row = a.qkv + (size_t)row * width;
    for (uint32_t i = tid; i < kv_mul * HD; i += kAttnThreads)
        q_s[i] = qkv_row[(size_t)g * kv_mul * HD + i];
    for (uint32_t i = tid; i < HD; i += kAttnThreads) {
        kn_s[i] = qkv_row[a.c + (size_t)g * HD + i];
        vn_s[i] = qkv_row[a.c + a.kv + (size_t)g * HD + i];
    }
    if (tid == 0 && *a.status != 0)
        *flag = 1;  // an earlier kernel failed: skip the work, keep the copy protocol
    __syncthreads();
    if (warp <= kv_mul) {
        float* v = warp < kv_mul ? q_s + (size_t)warp * HD : kn_s;
        if (!attn_norm_rope<HD>(v, warp < kv_mul ? gq_s : gk_s, rc_s, rs_s, a.eps, a.exact != 0) && lane == 0) {
            *flag = 1;
            atomicOr(a.status, kStatusNonFinite);
        }
    }
    __syncthreads();
    // append this position's k and v to the cache (read back by later steps)
    for (uint32_t i = tid; i < HD; i += kAttnThreads) {
        a.kcache[khead_base + (size_t)pos * kstride + i] = kn_s[i];
        a.vcache[head_base + (size_t)pos * HD + i] = vn_s[i];
    }
    int bad = 0;
    if (resident) {
        for (uint32_t i = tid; i < HD; i += kAttnThreads) {
            kres[(size_t)pos * kstride + i] = kn_s[i];
            vres[(size_t)pos * HD + i] = vn_s[i];
        }
        if (!mbar_wait(&full[0], 0) && lane == 0) {
            *flag = 1;
            atomicOr(a.status, kStatusTimeout);
        }
        __syncthreads();
        if (*flag == 0) {
            // scores: every (query head, position) pair over all threads
            for (uint32_t i = tid; i < kv_mul * n; i += kAttnThreads) {
                const uint32_t h = i / n, t = i % n;
                const float4* k4 = reinterpret_cast<const float4*>(kres + (size_t)t * kstride);
                const float4* q4 = reinterpret_cast<const float4*>(q_s + (size_t)h * HD);
                float dot = 0.0f;
#pragma unroll
                for (uint32_t j = 0; j < HD / 4; ++j) {
                    const float4 kk = k4[j], qq = q4[j];
                    dot = __fadd_rn(dot, __fmul_rn(qq.x, kk.x));
                    dot = __fadd_rn(dot, __fmul_rn(qq.y, kk.y));
                    dot = __fadd_rn(dot, __fmul_rn(qq.z, kk.z));
                    dot = __fadd_rn(dot, __fmul_rn(qq.w, kk.w));
                }
                const float score = __fmul_rn(dot, a.scale);
                bad |= !isfinite(score);
                sc[(size_t)h * sc_stride + t] = score;
            }
        }
    }

    // ---- scores (tiled)
    uint32_t L = 0;
    for (uint32_t tile = 0; tile < (resident ? 0u : ntiles); ++tile, ++L) {
        const uint32_t s = L % kAttnStages, t0 = tile * kAttnTile, rows_in = min(kAttnTile, n - t0);
        if (!mbar_wait(&full[s], (L / kAttnStages) & 1) && lane == 0) {
            *flag = 1;
            atomicOr(a.status, kStatusTimeout);
        }
        float* kt = reinterpret_cast<float*>(ring + (size_t)s * plan.stage_bytes);
        if (pos >= t0 && pos < t0 + rows_in)
            for (uint32_t i = tid; i < HD; i += kAttnThreads)
                kt[(size_t)(pos - t0) * kstride + i] = kn_s[i];
        __syncthreads();
        if (*flag == 0) {
            for (uint32_t pr = tid; pr < kv_mul * kAttnTile; pr += kAttnThreads) {
                const uint32_t h = pr / kAttnTile, tt = pr % kAttnTile;
                if (tt >= rows_in)
                    continue;
                const float4* k4 = reinterpret_cast<const float4*>(kt + (size_t)tt * kstride);
                const float4* q4 = reinterpret_cast<const float4*>(q_s + (size_t)h * HD);
                float dot = 0.0f;
#pragma unroll
                for (uint32_t i = 0; i < HD / 4; ++i) {
                    const float4 kk = k4[i], qq = q4[i];
                    dot = __fadd_rn(dot, __fmul_rn(qq.x, kk.x));
                    dot = __fadd_rn(dot, __fmul_rn(qq.y, kk.y));
                    dot = __fadd_rn(dot, __fmul_rn(qq.z, kk.z));
                    dot = __fadd_rn(dot, __fmul_rn(qq.w, kk.w));
                }
                const float score = __fmul_rn(dot, a.scale);
                bad |= !isfinite(score);
                sc[(size_t)h * sc_stride + t0 + tt] = score;
            }
        }
        fence_proxy_async();  // this thread's accesses to stage s come before the next bulk copy into it
        __syncthreads();      // stage s is free again
        if (warp == 0 && L + kAttnStages < nloads)
            issue(L + kAttnStages);
    }
    if (__syncthreads_or(bad) && tid == 0) {
        *flag = 1;
        atomicOr(a.status, kStatusNonFinite);  // "attention score is not finite"
    }
    __syncthreads();

    // ---- softmax per query head: max, expf(s - max), serial sum, division
    const bool live = *flag == 0;
    if (live) {
        if (warp < kv_mul) {
            float mx = -INFINITY;
            for (uint32_t t = lane; t < n; t += 32)
                mx = fmaxf(mx, sc[(size_t)warp * sc_stride + t]);
            for (int o = 16; o > 0; o >>= 1)
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            if (lane == 0)
                red[warp] = mx;
        }
        __syncthreads();
        for (uint32_t i = tid; i < kv_mul * n; i += kAttnThreads) {
            const uint32_t h = i / n, t = i % n;
            float* e = &sc[(size_t)h * sc_stride + t];
            *e = expf_cr(__fsub_rn(*e, red[h]));
        }
        __syncthreads();
        if (warp < kv_mul) {
            const float* e = sc + (size_t)warp * sc_stride;
            float sum = 0.0f;
            if (a.exact) {
                if (lane == 0) {
                    // serial in index order; terms load two float4s ahead of
                    // their adds (rows are float4-aligned)
                    const float4* e4 = reinterpret_cast<const float4*>(e);
                    const uint32_t n4 = n / 4;
                    const float4 zero = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    float4 cur = n4 > 0 ? e4[0] : zero, nxt = n4 > 1 ? e4[1] : zero;
                    for (uint32_t b = 0; b < n4; ++b) {
                        const float4 ahead = b + 2 < n4 ? e4[b + 2] : nxt;
                        sum = __fadd_rn(sum, cur.x);
                        sum = __fadd_rn(sum, cur.y);
                        sum = __fadd_rn(sum, cur.z);
                        sum = __fadd_rn(sum, cur.w);
                        cur = nxt;
                        nxt = ahead;
                    }
                    for (uint32_t t = n4 * 4; t < n; ++t)
                        sum = __fadd_rn(sum, e[t]);
                }
            } else {
                for (uint32_t t = lane; t < n; t += 32)
                    sum = __fadd_rn(sum, e[t]);
                for (int o = 16; o > 0; o >>= 1)
                    sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
            }
            if (lane == 0) {
                red[16 + warp] = sum;
                if (!(sum > 0.0f) || !isfinite(sum)) {  // "attention softmax failed"
                    *flag = 1;
                    atomicOr(a.status, kStatusNonFinite);
                }
            }
        }
        __syncthreads();
        if (*flag == 0)
            for (uint32_t i = tid; i < kv_mul * n; i += kAttnThreads) {
                const uint32_t h = i / n, t = i % n;
                float* e = &sc[(size_t)h * sc_stride + t];
                *e = __fdiv_rn(*e, red[16 + h]);
            }
    }
    __syncthreads();

    // ---- y = sum_t p_t * v_t, one serial chain per (query head, dim): thread
    // d < HD runs the chains of dim d for every query head of the block, so
    // each v element is read once; p comes four positions at a time.
    const bool live2 = *flag == 0;
    float acc[KVM];
#pragma unroll
    for (uint32_t h = 0; h < KVM; ++h)
        acc[h] = 0.0f;
    if (resident) {
        // y: one serial chain per (query head, dim) over all threads
        if (live2)
            for (uint32_t i = tid; i < kv_mul * HD; i += kAttnThreads) {
                const uint32_t h = i / HD, d = i % HD;
                const float* ph = sc + (size_t)h * sc_stride;
                float v = 0.0f;
                uint32_t t = 0;
                for (; t + 8 <= n; t += 8) {
                    // products of eight positions first (independent), then
                    // the serial chain of adds
                    const float4 p0 = *reinterpret_cast<const float4*>(ph + t);
                    const float4 p1 = *reinterpret_cast<const float4*>(ph + t + 4);
                    float w[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        w[j] = vres[(size_t)(t + j) * HD + d];
                    const float pr[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        w[j] = __fmul_rn(pr[j], w[j]);
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        v = __fadd_rn(v, w[j]);
                }
                for (; t < n; ++t)
                    v = __fadd_rn(v, __fmul_rn(ph[t], vres[(size_t)t * HD + d]));
                if (*flag == 0)
                    a.y[(size_t)row * a.y_stride + ((size_t)g * kv_mul + h) * HD + d] = v;
            }
        return;
    }
    for (uint32_t tile = 0; tile < ntiles; ++tile, ++L) {
        const uint32_t s = L % kAttnStages, t0 = tile * kAttnTile, rows_in = min(kAttnTile, n - t0);
        if (!mbar_wait(&full[s], (L / kAttnStages) & 1) && lane == 0) {
            *flag = 1;
            atomicOr(a.status, kStatusTimeout);
        }
        float* vt = reinterpret_cast<float*>(ring + (size_t)s * plan.stage_bytes);
        if (pos >= t0 && pos < t0 + rows_in)
            for (uint32_t i = tid; i < HD; i += kAttnThreads)
                vt[(size_t)(pos - t0) * HD + i] = vn_s[i];
        __syncthreads();
        if (live2 && tid < HD) {
            const uint32_t d = tid;
            uint32_t tt = 0;
            for (; tt + 4 <= rows_in; tt += 4) {
                const float v0 = vt[(size_t)tt * HD + d], v1 = vt[(size_t)(tt + 1) * HD + d];
                const float v2 = vt[(size_t)(tt + 2) * HD + d], v3 = vt[(size_t)(tt + 3) * HD + d];
#pragma unroll
                for (uint32_t h = 0; h < KVM; ++h) {
                    const float4 p = *reinterpret_cast<const float4*>(sc + (size_t)h * sc_stride + t0 + tt);
                    float v = acc[h];
                    v = __fadd_rn(v, __fmul_rn(p.x, v0));
                    v = __fadd_rn(v, __fmul_rn(p.y, v1));
                    v = __fadd_rn(v, __fmul_rn(p.z, v2));
                    v = __fadd_rn(v, __fmul_rn(p.w, v3));
                    acc[h] = v;
                }
            }
            for (; tt < rows_in; ++tt) {
                const float v0 = vt[(size_t)tt * HD + d];
#pragma unroll
                for (uint32_t h = 0; h < KVM; ++h)
                    acc[h] = __fadd_rn(acc[h], __fmul_rn(sc[(size_t)h * sc_stride + t0 + tt], v0));
            }
        }
        fence_proxy_async();
        __syncthreads();
        if (warp == 0 && L + kAttnStages < nloads)
            issue(L + kAttnStages);
    }
    if (live2 && *flag == 0 && tid < HD) {
#pragma unroll
        for (uint32_t h = 0; h < KVM; ++h)
            a.y[(size_t)row * a.y_stride + ((size_t)g * kv_mul + h) * HD + tid] = acc[h];
    }
}

// GGUF Q1_0 rows straight into the contraction's packed blocks (loader).
// A Q1_0 block is 18 bytes per 128 weights: the binary16 scale
// (little-endian) then 16 sign bytes in the public bit order
// (linear.c:26-62). Source row o of the slice goes to matrix row
// dst_row0 + o, or with half >= 0 to the interleaved gate/up position
// (o / 8) * 16 + half * 8 + o % 8. A non-finite scale sets *bad.
__global__ void q1_0_pack_kernel(const uint8_t* raw, uint32_t rows, uint32_t groups, uint32_t dst_row0, int half,
                                 unsigned char* wblocks, int* bad) {
    const size_t total = (size_t)rows * groups;
    const size_t bb = (size_t)groups * 144u;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const uint32_t o = (uint32_t)(i / groups), g = (uint32_t)(i % groups);
        const uint8_t* src = raw + i * 18u;
        const uint32_t row = half < 0 ? dst_row0 + o : (o / 8u) * 16u + (uint32_t)half * 8u + o % 8u;
        const uint32_t blk = row / kRowBlock, r = row % kRowBlock;
        const uint16_t sc = (uint16_t)(src[0] | (src[1] << 8));
        if ((sc & 0x7c00u) == 0x7c00u)
            atomicOr(bad, 1);
        uint32_t w[4];
#pragma unroll
        for (int t = 0; t < 4; ++t)
            w[t] = (uint32_t)src[2 + 4 * t] | ((uint32_t)src[3 + 4 * t] << 8) | ((uint32_t)src[4 + 4 * t] << 16) |
                   ((uint32_t)src[5 + 4 * t] << 24);
        unsigned char* b = wblocks + (size_t)blk * bb;
        *reinterpret_cast<uint4*>(b + ((size_t)g * kRowBlock + r) * 16u) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint16_t*>(b + (size_t)groups * 128u + ((size_t)r * groups + g) * 2u) = sc;
    }
}

// End of a decode step: advance every row's position; the greedy pick (the
// lm_head epilogue's packed key: index = ~low word) becomes the next input
// and is appended to the generation history.
// With column-sharded lm_head (world > 1) best holds every rank's key,
// [world][rows], and the pick is their maximum.
__global__ void step_end_kernel(uint32_t rows, uint32_t* pos, int32_t* tok_in, int32_t* tok_next,
                                const unsigned long long* best, uint32_t world, int32_t* hist,
                                uint32_t* hist_count, uint32_t hist_cap, int has_logits) {
    const uint32_t r = threadIdx.x;
    if (r < rows) {
        pos[r] += 1;
        if (has_logits) {
            unsigned long long b = best[r];
            for (uint32_t p = 1; p < world; ++p)
                b = best[(size_t)p * rows + r] > b ? best[(size_t)p * rows + r] : b;
            tok_next[r] = b ? (int32_t)(0xffffffffu - (uint32_t)(b & 0xffffffffull)) : 0;
            tok_in[r] = tok_next[r];
            const uint32_t h = *hist_count;
            if (h < hist_cap)
                hist[(size_t)h * rows + r] = tok_next[r];
        }
    }
    __syncthreads();
    if (r == 0 && has_logits)
        *hist_count += 1;
}

// Rank-major all-gather result [world][rows][slice] -> row-major
// [rows][width] (column p * slice + j comes from rank p), width <= world * slice.
__global__ void gather_rows_kernel(const float* st, float* dst, uint32_t world, uint32_t rows, uint32_t slice,
                                   uint32_t width, uint32_t dst_stride) {
    const size_t total = (size_t)rows * width;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const uint32_t r = (uint32_t)(i / width), col = (uint32_t)(i % width);
        const uint32_t p = col / slice, j = col % slice;
        dst[(size_t)r * dst_stride + col] = st[((size_t)p * rows + r) * slice + j];
    }
}

// bnn-mlp post-op: y = fl(fl(post_scale * y) + post_bias), ReLU if y < 0.
__global__ void mlp_post_kernel(float* y, const float* ps, const float* pb, uint32_t n, uint32_t rows,
                                int relu) {
    const size_t total = (size_t)rows * n;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const uint32_t o = (uint32_t)(i % n);
        float v = __fadd_rn(__fmul_rn(ps[o], y[i]), pb[o]);
        if (relu && v < 0.0f)
            v = 0.0f;
        y[i] = v;
    }
}

// Non-finite check of an FP32 array (BNNE_Classify's logit check). After an
// earlier kernel failed (a rejected layer input, whose layer was skipped) the
// array is stale and the first error stands, as the reference stops at it.
__global__ void finite_check_kernel(const float* v, size_t n, int* status, int bit) {
    if (*status != 0)
        return;
    int bad = 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        bad |= !isfinite(v[i]);
    if (__syncthreads_or(bad) && threadIdx.x == 0)
        atomicOr(status, bit);
}

}  // namespace eng
}  // namespace bnn
