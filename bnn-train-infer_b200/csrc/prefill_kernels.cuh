// prefill_kernels.cuh - batched prefill: every prompt position of every row
// is one activation row of a GEMM on the tensor cores (w1a8_mma.cuh).
//
// The reference prefills one token at a time (BNNE_Decode, engine.c:241-273:
// qwen3_step per token, each linear a GEMV_F32 of one row). Every output of a
// linear depends only on its own input row (per-row quantisation, exact group
// dots, per-output FP32 order), and the attention of position p reads only
// positions <= p. So the prompt runs layer by layer over all positions at
// once with the same per-element arithmetic as the decode step:
//
//   rows_prep_kernel   RMSNorm (optional, qwen3.c:361-372) + QuantizeRow
//                      (soft-bnn-accelerator.c:175-211) of one row, written
//                      pre-tiled for the tensor cores; the sums and the
//                      element order are those of the decode prologue
//                      (w1a8_gemv.cuh kProRmsNorm / kProQuant)
//   kv_append_kernel   k-norm + RoPE of every position's k heads and the
//                      K/V cache append (qwen3.c:418-438), before attention
//   prefill_attention_kernel  per tile of positions: q-norm + RoPE and
//                      causal attention over the cache, each K/V tile read
//                      once for the whole tile (decode-kernel arithmetic)
//
// The linears' epilogues (View, residual add, SwiGLU) run inside the
// tensor-core kernel. Greedy logits come from the decode step's lm_head on
// the last position of each row.
#pragma once

#include <cstdint>
#include "bnn_device.cuh"
#include "exact_sum.cuh"
#include "w1a8_mma.cuh"
#include "engine_kernels.cuh"

namespace bnn {
namespace eng {

constexpr uint32_t kRowsPrepThreads = kWideThreads;  // the wide exact sum's threads

struct RowsPrepArgs {
    const float* x;      // [m][k] F32 rows, x_stride floats apart
    size_t x_stride;
    const float* gain;   // RMSNorm gains [k], or null: quantise the row as it is
    float eps;
    int exact;           // RMSNorm sum: serial (reference order) or the decode prologue's tree
    uint32_t k, m;
    unsigned char* a_sw; // pre-tiled int8 rows (mma_a_offset), or null:
    uint32_t* act;       //   sliced words [m][k/128][32] and
    int32_t* totals;     //   group totals [m][k/128] for the dp4a contraction (kProSliced)
    float* row_scale;    // [m]
    int* status;
    int early_next;      // 1: let the next kernel of the stream launch at once (PDL)
};

inline size_t rows_prep_smem(uint32_t k, bool exact) {
    return (size_t)k * 5u + (exact ? kWideSmemBytes : 0);  // row, its int8 codes, the sum's scratch
}

// One CTA of kRowsPrepThreads per row. A non-finite input without RMSNorm is
// rejected (kStatusBadInput, ValidateF32Input); with RMSNorm it shows up as a
// non-finite divisor (kStatusNonFinite), as in the decode step.
__global__ void __launch_bounds__(kRowsPrepThreads) rows_prep_kernel(RowsPrepArgs a) {
    extern __shared__ __align__(16) unsigned char rp_smem[];
    __shared__ float red[32];  // [1..8] fast-mode warp sums, [16..31] warp maxima
    __shared__ int s_flag;
    float* xb = reinterpret_cast<float*>(rp_smem);
    float4* xb4 = reinterpret_cast<float4*>(rp_smem);
    int8_t* qs = reinterpret_cast<int8_t*>(rp_smem + (size_t)a.k * 4u);  // sliced mode
    unsigned char* sum_mem = rp_smem + (size_t)a.k * 5u;
    const uint32_t row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t K = a.k, G = K / kGroup;
    constexpr uint32_t nt = kRowsPrepThreads, nw = kRowsPrepThreads / 32;
    // everything below reads what earlier kernels wrote (a no-op unless
    // launched with programmatic dependent launch)
    if (a.early_next)
        griddep_launch_dependents();
    griddep_wait();

    if (tid == 0)
        s_flag = *a.status != 0;  // an earlier kernel failed: nothing more is written
    const float4* xr = reinterpret_cast<const float4*>(a.x + (size_t)row * a.x_stride);
    int bad = 0;
    float amax = 0.0f;
    for (uint32_t i = tid; i < K / 4; i += nt) {
        const float4 v = xr[i];
        bad |= !isfinite(v.x) | !isfinite(v.y) | !isfinite(v.z) | !isfinite(v.w);
        amax = fmaxf(fmaxf(amax, fmaxf(fabsf(v.x), fabsf(v.y))), fmaxf(fabsf(v.z), fabsf(v.w)));
        xb4[i] = v;
    }
    if (__syncthreads_or(bad) && !a.gain) {
        if (tid == 0 && !s_flag)
            atomicOr(a.status, kStatusBadInput);
        return;
    }
    if (s_flag)
        return;
    if (a.gain) {
        float sum;
        if (a.exact) {
            sum = exact_sumsq_wide(xb, (int)K, sum_mem, 1);
        } else {
            // the decode prologue's tree: kSumThreads lane-strided sums
            if (tid < kSumThreads) {
                float t = 0.0f;
                for (uint32_t i = tid; i < K; i += kSumThreads)
                    t = __fadd_rn(t, __fmul_rn(xb[i], xb[i]));
                for (int o = 16; o > 0; o >>= 1)
                    t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, o));
                if (lane == 0)
                    red[1 + warp] = t;
            }
            __syncthreads();
            sum = 0.0f;
            for (uint32_t w = 0; w < (uint32_t)kSumWarpsN; ++w)
                sum = __fadd_rn(sum, red[1 + w]);
        }
        const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)K), a.eps));
        if (!isfinite(rms) || rms == 0.0f) {
            if (tid == 0)
                atomicOr(a.status, kStatusNonFinite);
            return;  // uniform: every thread computed the same rms
        }
        amax = 0.0f;
        const float rr = __frcp_rn(rms);  // div_cr: x / rms correctly rounded, as __fdiv_rn
        const float4* gr = reinterpret_cast<const float4*>(a.gain);
        for (uint32_t i = tid; i < K / 4; i += nt) {
            float4 v = xb4[i];
            const float4 gn = gr[i];
            v.x = __fmul_rn(div_cr(v.x, rms, rr), gn.x);
            v.y = __fmul_rn(div_cr(v.y, rms, rr), gn.y);
            v.z = __fmul_rn(div_cr(v.z, rms, rr), gn.z);
            v.w = __fmul_rn(div_cr(v.w, rms, rr), gn.w);
            amax = fmaxf(fmaxf(amax, fmaxf(fabsf(v.x), fabsf(v.y))), fmaxf(fabsf(v.z), fabsf(v.w)));
            xb4[i] = v;
        }
    }
    for (int o = 16; o > 0; o >>= 1)
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0)
        red[16 + warp] = amax;
    __syncthreads();
    amax = red[16];
    for (uint32_t w = 1; w < nw; ++w)
        amax = fmaxf(amax, red[16 + w]);
    const float s = row_scale_from_absmax(amax);
    const RowQuantizer quant(s);
    if (!a.a_sw) {
        // QuantizeRow into shared memory, then the contraction's sliced words
        // and per-group totals (w1a8_prep_kernel's layout)
        for (uint32_t k = tid; k < K; k += nt)
            qs[k] = quant(xb[k]);
        __syncthreads();
        uint32_t* act = a.act + (size_t)row * G * kWordsPerGroup;
        for (uint32_t w = tid; w < G * kWordsPerGroup; w += nt) {
            const uint32_t g = w / kWordsPerGroup, tj = w % kWordsPerGroup;
            act[w] = pack_slice(qs + g * kGroup, tj >> 3, tj & 7u);
        }
        for (uint32_t g = warp; g < G; g += nw) {
            const int8_t* qg = qs + g * kGroup + lane * 4u;
            int t = (int)qg[0] + (int)qg[1] + (int)qg[2] + (int)qg[3];
            for (int o = 16; o > 0; o >>= 1)
                t += __shfl_xor_sync(0xffffffffu, t, o);
            if (lane == 0)
                a.totals[(size_t)row * G + g] = t;
        }
        if (tid == 0)
            a.row_scale[row] = s;
        return;
    }
    // 16 quantised values (one swizzled 16-byte chunk) per thread and pass
    for (uint32_t c = tid; c < G * 8u; c += nt) {
        const float4* src = xb4 + (size_t)c * 4u;
        uint32_t w[4];
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
            const float4 v = src[j];
            w[j] = (uint32_t)(uint8_t)quant(v.x) | ((uint32_t)(uint8_t)quant(v.y) << 8) |
                   ((uint32_t)(uint8_t)quant(v.z) << 16) | ((uint32_t)(uint8_t)quant(v.w) << 24);
        }
        *reinterpret_cast<uint4*>(a.a_sw + mma_a_offset(row, c / 8u, G, c % 8u)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    if (tid == 0)
        a.row_scale[row] = s;
}

struct KvAppendArgs {
    const float* qkv;       // [rows][c + 2kv]: q | k | v projections
    const float* k_norm;    // [HD]
    const float* rope_cos;  // [n_ctx][HD/2]
    const float* rope_sin;
    const uint32_t* pos;    // [rows]
    const uint32_t* slot;   // [rows] KV cache row
    float* kcache;          // this layer: [cache rows][kv_heads][n_ctx][kcache_row(HD)]
    float* vcache;
    uint32_t c, kv, kv_heads, n_ctx;
    float eps;
    int exact;
    int* status;
};

inline size_t kv_append_smem(uint32_t hd, uint32_t kv_heads) { return (size_t)(2u + kv_heads) * hd * 4u; }

// One CTA per row, one warp per KV head: the decode step's k-norm + RoPE
// (attn_norm_rope, the same function) and the append of k and v.
template <int HD>
__global__ void kv_append_kernel(KvAppendArgs a) {
    extern __shared__ __align__(16) float kv_smem[];
    float* gk = kv_smem;            // [HD]
    float* rc = gk + HD;            // [HD/2]
    float* rs = rc + HD / 2;        // [HD/2]
    float* kb = rs + HD / 2;        // [kv_heads][HD]
    const uint32_t row = blockIdx.x, tid = threadIdx.x, g = tid >> 5, lane = tid & 31;
    griddep_launch_dependents();
    griddep_wait();
    if (*a.status != 0)
        return;
    const uint32_t pos = a.pos[row];
    const float* qkv_row = a.qkv + (size_t)row * (a.c + 2u * a.kv);
    for (uint32_t i = tid; i < HD; i += blockDim.x)
        gk[i] = a.k_norm[i];
    for (uint32_t i = tid; i < HD / 2; i += blockDim.x) {
        rc[i] = a.rope_cos[(size_t)pos * (HD / 2) + i];
        rs[i] = a.rope_sin[(size_t)pos * (HD / 2) + i];
    }
    for (uint32_t i = tid; i < a.kv; i += blockDim.x)
        kb[i] = qkv_row[a.c + i];
    __syncthreads();
    if (g >= a.kv_heads)
        return;
    float* v = kb + (size_t)g * HD;
    if (!attn_norm_rope<HD>(v, gk, rc, rs, a.eps, a.exact != 0) && lane == 0)
        atomicOr(a.status, kStatusNonFinite);
    __syncwarp();
    const size_t cell = ((size_t)a.slot[row] * a.kv_heads + g) * a.n_ctx + pos;
    for (uint32_t i = lane; i < HD; i += 32) {
        a.kcache[cell * kcache_row(HD) + i] = v[i];
        a.vcache[cell * HD + i] = qkv_row[a.c + a.kv + (size_t)g * HD + i];
    }
}

// ---- causal attention over a tile of prompt positions
//
// One CTA per (KV head g, kPfQT consecutive positions of one row): the
// kv_mul query heads of g at each position, every K and V tile of the cache
// read once for all of them. Per query head the arithmetic is the decode
// kernel's (attention_kernel): q-norm + RoPE (attn_norm_rope), each score a
// serial FP32 dot over the head dimension times the scale, the maximum,
// expf_cr(s - max), the sum in the same order (serial in exact mode, the
// same lane-strided tree in fast mode), the division, and y accumulated
// serially over the positions 0 .. pos. So outputs are bit-identical to one
// decode step per position.
constexpr uint32_t kPfQT = 16;        // query positions per CTA
constexpr uint32_t kPfKT = 64;        // K/V positions per shared-memory tile
constexpr uint32_t kPfThreads = 512;  // (query pair, key) and (query, 4 dims) per thread
constexpr uint32_t kPfSmemBudget = 200u * 1024u;
static_assert(kPfThreads == kPfQT / 2 * kPfKT && kPfThreads == kPfQT * 32, "thread maps of the score and V phases");

struct PfAttnArgs {
    const float* qkv;       // [rows][c + 2kv]
    const float* q_norm;    // [HD]
    const float* rope_cos;  // [n_ctx][HD/2]
    const float* rope_sin;
    const uint32_t* pos;    // [rows]: consecutive positions within a row of the chunk
    const uint32_t* slot;   // [rows] KV cache row
    const float* kcache;    // this layer: [cache rows][kv_heads][n_ctx][kcache_row(HD)]
    const float* vcache;
    float* scores;          // [rows][heads][sc_stride] when they do not fit in shared memory, else null
    float* y;               // [rows][y_stride]: head h at h * HD
    uint32_t y_stride;
    uint32_t c, kv, heads, kv_heads, n_ctx;
    uint32_t len;           // positions of each row in this chunk (rows = R * len)
    uint32_t sc_stride;     // floats per score row (a multiple of 4)
    float eps, scale;
    int exact;
    int* status;
};

struct PfSmem {
    size_t q, kv, gq, rc, rs, red, sc, total;
};

__host__ __device__ inline PfSmem pf_smem_plan(uint32_t hd, uint32_t kv_mul, uint32_t sc_stride, bool sc_smem) {
    PfSmem p;
    p.q = 0;                                                    // [kPfQT * kv_mul][hd]
    p.kv = p.q + (size_t)kPfQT * kv_mul * hd * 4u;              // [2][kPfKT][hd + 4] (double-buffered)
    p.gq = p.kv + (size_t)2 * kPfKT * (hd + 4u) * 4u;           // [hd]
    p.rc = p.gq + (size_t)hd * 4u;                              // [kPfQT][hd / 2]
    p.rs = p.rc + (size_t)kPfQT * (hd / 2u) * 4u;
    p.red = p.rs + (size_t)kPfQT * (hd / 2u) * 4u;              // 64 floats
    p.sc = p.red + 64u * 4u;                                    // [kPfQT * kv_mul][sc_stride]
    p.total = p.sc + (sc_smem ? (size_t)kPfQT * kv_mul * sc_stride * 4u : 0u);
    return p;
}

// SCS: a tile's scores live in shared memory (a.scores null), fixed at compile
// time so that score accesses are shared-memory accesses.
template <int HD, int KVM, bool SCS>
__global__ void __launch_bounds__(kPfThreads, 1) prefill_attention_kernel(PfAttnArgs a) {
    extern __shared__ __align__(16) unsigned char pf_smem[];
    constexpr uint32_t kStride = HD + 4;  // padded K/V rows
    const uint32_t g = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t tiles = (a.len + kPfQT - 1) / kPfQT;
    // the last positions (most keys) first: the longest CTAs start in the first wave
    const uint32_t r = blockIdx.y / tiles, i0 = (tiles - 1 - blockIdx.y % tiles) * kPfQT;
    const uint32_t nq = min(kPfQT, a.len - i0);
    const uint32_t p0 = r * a.len + i0;  // activation row of the first query
    constexpr bool sc_smem = SCS;
    const PfSmem plan = pf_smem_plan(HD, KVM, a.sc_stride, sc_smem);
    float* q_s = reinterpret_cast<float*>(pf_smem + plan.q);
    float* kv_s = reinterpret_cast<float*>(pf_smem + plan.kv);
    float* gq_s = reinterpret_cast<float*>(pf_smem + plan.gq);
    float* rc_s = reinterpret_cast<float*>(pf_smem + plan.rc);
    float* rs_s = reinterpret_cast<float*>(pf_smem + plan.rs);
    float* red = reinterpret_cast<float*>(pf_smem + plan.red);
    int* flag = reinterpret_cast<int*>(red + 63);
    // score row of (query qi, head h): the decode layout [row][head][stride] when global
    auto sc_row = [&](uint32_t qi, uint32_t h) -> float* {
        return sc_smem ? reinterpret_cast<float*>(pf_smem + plan.sc) + (size_t)(qi * KVM + h) * a.sc_stride
                       : a.scores + ((size_t)(p0 + qi) * a.heads + g * KVM + h) * a.sc_stride;
    };
    griddep_launch_dependents();
    griddep_wait();
    if (*a.status != 0)
        return;
    const uint32_t pos0 = a.pos[p0];
    const uint32_t n_max = a.pos[p0 + nq - 1] + 1;  // keys of the last query
    const size_t head_cells = ((size_t)a.slot[p0] * a.kv_heads + g) * a.n_ctx;
    const float* kc = a.kcache + head_cells * kcache_row(HD);  // padded K rows
    const float* vc = a.vcache + head_cells * HD;
    const size_t width = a.c + 2u * a.kv;

    if (tid == 0)
        *flag = 0;
    for (uint32_t i = tid; i < HD; i += kPfThreads)
        gq_s[i] = a.q_norm[i];
    for (uint32_t i = tid; i < kPfQT * (HD / 2); i += kPfThreads) {
        const uint32_t qi = i / (HD / 2), j = i % (HD / 2);
        const uint32_t ps = qi < nq ? pos0 + qi : pos0;
        rc_s[i] = a.rope_cos[(size_t)ps * (HD / 2) + j];
        rs_s[i] = a.rope_sin[(size_t)ps * (HD / 2) + j];
    }
    for (uint32_t i = tid; i < kPfQT * KVM * HD; i += kPfThreads) {
        const uint32_t v = i / HD, d = i % HD, qi = v / KVM, h = v % KVM;
        q_s[i] = qi < nq ? a.qkv[(size_t)(p0 + qi) * width + (size_t)(g * KVM + h) * HD + d] : 0.0f;
    }
    __syncthreads();
    for (uint32_t v = warp; v < nq * KVM; v += kPfThreads / 32) {
        const uint32_t qi = v / KVM;
        if (!attn_norm_rope<HD>(q_s + (size_t)v * HD, gq_s, rc_s + qi * (HD / 2), rs_s + qi * (HD / 2), a.eps,
                                a.exact != 0) &&
            lane == 0) {
            *flag = 1;
            atomicOr(a.status, kStatusNonFinite);
        }
    }
    __syncthreads();
    if (*flag)
        return;

    // K/V tiles are double-buffered: this thread's share of tile t + 1 is
    // loaded into registers while tile t is in use, then stored to the
    // other buffer
    constexpr uint32_t kPer = (kPfKT * (HD / 4) + kPfThreads - 1) / kPfThreads;  // float4 per thread and tile
    float4 pre[kPer];
    auto tile_load = [&](const float* src, uint32_t src_row, uint32_t t0) {
        const uint32_t rows_in = min(kPfKT, n_max - t0);
#pragma unroll
        for (uint32_t j = 0; j < kPer; ++j) {
            const uint32_t i = tid + j * kPfThreads;
            if (i < rows_in * (HD / 4))
                pre[j] = reinterpret_cast<const float4*>(src + (size_t)(t0 + i / (HD / 4)) * src_row)[i % (HD / 4)];
        }
    };
    auto tile_store = [&](float* dst, uint32_t t0) {
        const uint32_t rows_in = min(kPfKT, n_max - t0);
#pragma unroll
        for (uint32_t j = 0; j < kPer; ++j) {
            const uint32_t i = tid + j * kPfThreads;
            if (i < rows_in * (HD / 4))
                reinterpret_cast<float4*>(dst + (size_t)(i / (HD / 4)) * kStride)[i % (HD / 4)] = pre[j];
        }
    };
    auto kvb = [&](uint32_t b) { return kv_s + (b ? (size_t)kPfKT * kStride : (size_t)0); };

    // ---- scores: thread (queries 2sp and 2sp + 1, key kp of the tile), all
    // KVM heads: each K row read from shared memory serves both queries
    const uint32_t sp = tid / kPfKT, kp = tid % kPfKT;
    const uint32_t sq0 = 2 * sp, sq1 = sq0 + 1;
    const uint32_t n0 = pos0 + sq0 + 1, n1 = n0 + 1;  // keys of each query
    int bad = 0;
    tile_load(kc, kcache_row(HD), 0);
    tile_store(kvb(0), 0);
    __syncthreads();
    for (uint32_t t0 = 0, buf = 0; t0 < n_max; t0 += kPfKT, buf ^= 1) {
        const bool more = t0 + kPfKT < n_max;
        if (more)
            tile_load(kc, kcache_row(HD), t0 + kPfKT);
        const uint32_t ta = t0 + kp;
        const bool v0 = sq0 < nq && ta < n0, v1 = sq1 < nq && ta < n1;
        if (v0 || v1) {
            const float4* ka = reinterpret_cast<const float4*>(kvb(buf) + (size_t)kp * kStride);
            float d0[KVM], d1[KVM];
#pragma unroll
            for (int h = 0; h < KVM; ++h)
                d0[h] = d1[h] = 0.0f;
#pragma unroll 4
            for (uint32_t i = 0; i < HD / 4; ++i) {
                const float4 x = ka[i];
#pragma unroll
                for (int h = 0; h < KVM; ++h) {
                    const float4 q0 = reinterpret_cast<const float4*>(q_s + (size_t)(sq0 * KVM + h) * HD)[i];
                    const float4 q1 = reinterpret_cast<const float4*>(q_s + (size_t)(sq1 * KVM + h) * HD)[i];
                    d0[h] = __fadd_rn(d0[h], __fmul_rn(q0.x, x.x));
                    d1[h] = __fadd_rn(d1[h], __fmul_rn(q1.x, x.x));
                    d0[h] = __fadd_rn(d0[h], __fmul_rn(q0.y, x.y));
                    d1[h] = __fadd_rn(d1[h], __fmul_rn(q1.y, x.y));
                    d0[h] = __fadd_rn(d0[h], __fmul_rn(q0.z, x.z));
                    d1[h] = __fadd_rn(d1[h], __fmul_rn(q1.z, x.z));
                    d0[h] = __fadd_rn(d0[h], __fmul_rn(q0.w, x.w));
                    d1[h] = __fadd_rn(d1[h], __fmul_rn(q1.w, x.w));
                }
            }
#pragma unroll
            for (int h = 0; h < KVM; ++h) {
                if (v0) {
                    const float sa = __fmul_rn(d0[h], a.scale);
                    bad |= !isfinite(sa);
                    sc_row(sq0, h)[ta] = sa;
                }
                if (v1) {
                    const float sa = __fmul_rn(d1[h], a.scale);
                    bad |= !isfinite(sa);
                    sc_row(sq1, h)[ta] = sa;
                }
            }
        }
        if (more)
            tile_store(kvb(buf ^ 1), t0 + kPfKT);
        __syncthreads();  // the next tile is in place; this one is free again
    }
    if (__syncthreads_or(bad)) {
        if (tid == 0)
            atomicOr(a.status, kStatusNonFinite);  // "attention score is not finite"
        return;
    }

    // ---- softmax per (query, head) row, one warp per row
    for (uint32_t v = warp; v < nq * KVM; v += kPfThreads / 32) {
        const uint32_t qi = v / KVM, h = v % KVM, n = pos0 + qi + 1;
        float* e = sc_row(qi, h);
        float mx = -INFINITY;
        for (uint32_t t = lane; t < n; t += 32)
            mx = fmaxf(mx, e[t]);
        for (int o = 16; o > 0; o >>= 1)
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        for (uint32_t t = lane; t < n; t += 32)
            e[t] = expf_cr(__fsub_rn(e[t], mx));
        __syncwarp();
        float sum = 0.0f;
        if (a.exact) {
            if (lane == 0) {
                uint32_t t = 0;
                for (; t + 8 <= n; t += 8) {
                    float w[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        w[j] = e[t + j];
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        sum = __fadd_rn(sum, w[j]);
                }
                for (; t < n; ++t)
                    sum = __fadd_rn(sum, e[t]);
            }
            sum = __shfl_sync(0xffffffffu, sum, 0);
        } else {
            for (uint32_t t = lane; t < n; t += 32)
                sum = __fadd_rn(sum, e[t]);
            for (int o = 16; o > 0; o >>= 1)
                sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
        }
        if (!(sum > 0.0f) || !isfinite(sum)) {  // "attention softmax failed"
            if (lane == 0) {
                *flag = 1;
                atomicOr(a.status, kStatusNonFinite);
            }
            continue;
        }
        for (uint32_t t = lane; t < n; t += 32)
            e[t] = __fdiv_rn(e[t], sum);
    }
    __syncthreads();
    if (*flag)
        return;

    // ---- y: thread (query vq, dims DV vd .. DV vd + DV - 1), all KVM heads; serial over t
    constexpr int DV = HD / 32;
    const uint32_t vq = tid / 32, vd = (tid % 32) * DV;
    const uint32_t vn = vq < nq ? pos0 + vq + 1 : 0;
    float acc[KVM][DV];
#pragma unroll
    for (int h = 0; h < KVM; ++h)
#pragma unroll
        for (int j = 0; j < DV; ++j)
            acc[h][j] = 0.0f;
    tile_load(vc, HD, 0);
    tile_store(kvb(0), 0);
    __syncthreads();
    for (uint32_t t0 = 0, buf = 0; t0 < n_max; t0 += kPfKT, buf ^= 1) {
        const uint32_t rows_in = min(kPfKT, n_max - t0);
        const bool more = t0 + kPfKT < n_max;
        if (more)
            tile_load(vc, HD, t0 + kPfKT);
        const float* vt = kvb(buf);
        const uint32_t tend = vn > t0 ? min(rows_in, vn - t0) : 0;
        for (uint32_t tt = 0; tt < tend; ++tt) {
            float v[DV];
#pragma unroll
            for (int j = 0; j < DV; ++j)
                v[j] = vt[(size_t)tt * kStride + vd + j];
#pragma unroll
            for (int h = 0; h < KVM; ++h) {
                const float p = sc_row(vq, h)[t0 + tt];
#pragma unroll
                for (int j = 0; j < DV; ++j)
                    acc[h][j] = __fadd_rn(acc[h][j], __fmul_rn(p, v[j]));
            }
        }
        if (more)
            tile_store(kvb(buf ^ 1), t0 + kPfKT);
        __syncthreads();
    }
    if (vq < nq) {
        float* yr = a.y + (size_t)(p0 + vq) * a.y_stride;
#pragma unroll
        for (int h = 0; h < KVM; ++h)
#pragma unroll
            for (int j = 0; j < DV; ++j)
                yr[(size_t)(g * KVM + h) * HD + vd + j] = acc[h][j];
    }
}

}  // namespace eng
}  // namespace bnn
