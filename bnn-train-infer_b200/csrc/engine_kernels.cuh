// engine_kernels.cuh - the device-resident glue of the Qwen3 / bnn-mlp step.
//
// Each kernel restates one piece of the reference's host glue with the same
// FP32 operation order (bnn-sw-v2/qwen3/qwen3.c, bnn-mlp/bnn-mlp.c), using
// explicit round-to-nearest intrinsics so nothing is fused or reassociated:
//   embed_kernel            qwen3_embed               qwen3.c:374-385
//   qk_norm_rope_kernel     per-head q/k RMSNorm, RoPE, KV append  qwen3.c:418-438
//   attention_kernel        causal softmax attention  qwen3.c:440-478
//   argmax_kernel           greedy pick + finite check  bnn-infer-v2.c:48-54, engine.c:262-267
//   mlp_post_kernel         post_scale/bias + ReLU    bnn-mlp.c:189-193
// RMSNorm before a linear, the row quantisation and SwiGLU run inside the
// W1A8 linears (w1a8_gemv.cuh prologues/epilogues). In exact mode every long
// sum is accumulated serially in index order, as the reference does; fast
// mode uses a fixed-order tree instead.
#pragma once

#include <cstdint>
#include "bnn_device.cuh"

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
// blocks (token_embd and lm_head are the same tied matrix).
__global__ void embed_kernel(const int32_t* tokens, const unsigned char* wblocks, uint32_t c, float* x) {
    const uint32_t row = blockIdx.x;
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

struct QkArgs {
    float* qkv;            // [rows][C + 2KV]: q | k | v
    const float* q_norm;   // [HD]
    const float* k_norm;   // [HD]
    const float* rope_cos; // [n_ctx][HD/2]
    const float* rope_sin;
    const uint32_t* pos;   // [rows]
    float* kcache;         // this layer: [rows][n_ctx][KV]
    float* vcache;
    uint32_t c, kv, hd, heads, kv_heads, n_ctx;
    float eps;
    int exact;
    int* status;
};

// One block per (head, row), blockDim.x == head_dim. Q heads are normalised
// and rotated in place; K heads are normalised, rotated and appended to the
// K cache at this row's position, together with the matching V head.
__global__ void qk_norm_rope_kernel(QkArgs a) {
    extern __shared__ __align__(16) unsigned char e_smem[];
    float* v = reinterpret_cast<float*>(e_smem);
    float* sq = v + a.hd;
    __shared__ float red[64];
    const uint32_t hh = blockIdx.x, row = blockIdx.y, i = threadIdx.x;
    const bool is_q = hh < a.heads;
    const uint32_t kvh = is_q ? 0 : hh - a.heads;
    const size_t width = a.c + 2u * a.kv;
    float* vec = a.qkv + (size_t)row * width + (is_q ? hh * a.hd : a.c + kvh * a.hd);
    const float x = vec[i];
    v[i] = x;
    sq[i] = __fmul_rn(x, x);
    const float sum = block_sum_ordered(sq, a.hd, a.exact != 0, red);
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)a.hd), a.eps));
    if (!isfinite(rms) || rms == 0.0f) {
        if (i == 0)
            atomicOr(a.status, kStatusNonFinite);
        return;
    }
    const float* gain = is_q ? a.q_norm : a.k_norm;
    v[i] = __fmul_rn(__fdiv_rn(x, rms), gain[i]);
    __syncthreads();
    const uint32_t half = a.hd / 2, p = a.pos[row];
    float out;
    if (i < half) {
        const float c = a.rope_cos[(size_t)p * half + i], s = a.rope_sin[(size_t)p * half + i];
        out = __fsub_rn(__fmul_rn(v[i], c), __fmul_rn(v[i + half], s));
    } else {
        const uint32_t j = i - half;
        const float c = a.rope_cos[(size_t)p * half + j], s = a.rope_sin[(size_t)p * half + j];
        out = __fadd_rn(__fmul_rn(v[j], s), __fmul_rn(v[i], c));
    }
    if (is_q) {
        vec[i] = out;
    } else {
        const size_t slot = ((size_t)row * a.n_ctx + p) * a.kv + kvh * a.hd + i;
        a.kcache[slot] = out;
        a.vcache[slot] = a.qkv[(size_t)row * width + a.c + a.kv + kvh * a.hd + i];
    }
}

struct AttnArgs {
    const float* qkv;     // q part: [rows][C + 2KV]
    const float* kcache;  // this layer: [rows][n_ctx][KV]
    const float* vcache;
    const uint32_t* pos;
    float* y;             // [rows][C]
    uint32_t c, kv, hd, heads, kv_heads, n_ctx;
    float scale;          // 1 / sqrtf(head_dim), computed on the host as qwen3.c:404
    int exact;
    int* status;
};

// One block per (q head, row). scores[t] = fl(dot(q, k_t)) * scale, dots
// accumulated serially over the head dimension; softmax with expf(s - max),
// a sequential sum over t and a division; then y_i = sum_t p_t * v_t,i,
// sequential in t, one thread per i.
__global__ void attention_kernel(AttnArgs a) {
    extern __shared__ __align__(16) unsigned char e_smem[];
    float* q = reinterpret_cast<float*>(e_smem);
    float* sc = q + a.hd;
    __shared__ float red[64];
    const uint32_t h = blockIdx.x, row = blockIdx.y;
    const uint32_t kvh = h / (a.heads / a.kv_heads);
    const uint32_t n = a.pos[row] + 1;  // positions 0..pos inclusive
    const size_t width = a.c + 2u * a.kv;
    for (uint32_t i = threadIdx.x; i < a.hd; i += blockDim.x)
        q[i] = a.qkv[(size_t)row * width + h * a.hd + i];
    __syncthreads();
    const float* kbase = a.kcache + (size_t)row * a.n_ctx * a.kv + kvh * a.hd;
    const float* vbase = a.vcache + (size_t)row * a.n_ctx * a.kv + kvh * a.hd;
    int bad = 0;
    float mx = -INFINITY;
    for (uint32_t t = threadIdx.x; t < n; t += blockDim.x) {
        const float4* k4 = reinterpret_cast<const float4*>(kbase + (size_t)t * a.kv);
        float dot = 0.0f;
        for (uint32_t i = 0; i < a.hd / 4; ++i) {
            const float4 kk = k4[i];
            dot = __fadd_rn(dot, __fmul_rn(q[4 * i], kk.x));
            dot = __fadd_rn(dot, __fmul_rn(q[4 * i + 1], kk.y));
            dot = __fadd_rn(dot, __fmul_rn(q[4 * i + 2], kk.z));
            dot = __fadd_rn(dot, __fmul_rn(q[4 * i + 3], kk.w));
        }
        const float s = __fmul_rn(dot, a.scale);
        bad |= !isfinite(s);
        sc[t] = s;
        mx = fmaxf(mx, s);
    }
    mx = block_max(mx, red);
    if (__syncthreads_or(bad)) {
        if (threadIdx.x == 0)
            atomicOr(a.status, kStatusNonFinite);
        return;
    }
    for (uint32_t t = threadIdx.x; t < n; t += blockDim.x)
        sc[t] = expf_cr(__fsub_rn(sc[t], mx));
    const float sum = block_sum_ordered(sc, n, a.exact != 0, red);
    if (!(sum > 0.0f) || !isfinite(sum)) {
        if (threadIdx.x == 0)
            atomicOr(a.status, kStatusNonFinite);
        return;
    }
    for (uint32_t t = threadIdx.x; t < n; t += blockDim.x)
        sc[t] = __fdiv_rn(sc[t], sum);
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < a.hd; i += blockDim.x) {
        float acc = 0.0f;
        for (uint32_t t = 0; t < n; ++t)
            acc = __fadd_rn(acc, __fmul_rn(sc[t], vbase[(size_t)t * a.kv + i]));
        a.y[(size_t)row * a.c + h * a.hd + i] = acc;
    }
}

// Greedy pick per row: the first index holding the maximum (strict > scan in
// index order); any non-finite logit flags the step (BNNE_Decode's check).
__global__ void argmax_kernel(const float* logits, uint32_t v, int32_t* out, int* status) {
    __shared__ float bv[32];
    __shared__ uint32_t bi[32];
    __shared__ int bad_any;
    const uint32_t row = blockIdx.x;
    const float* l = logits + (size_t)row * v;
    if (threadIdx.x == 0)
        bad_any = 0;
    __syncthreads();
    float best = -INFINITY;
    uint32_t idx = 0xffffffffu;
    int bad = 0;
    for (uint32_t i = threadIdx.x; i < v; i += blockDim.x) {
        const float x = l[i];
        bad |= !isfinite(x);
        if (x > best || (x == best && i < idx)) {
            best = x;
            idx = i;
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ob > best || (ob == best && oi < idx)) {
            best = ob;
            idx = oi;
        }
    }
    if (bad)
        bad_any = 1;
    const uint32_t w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        bv[w] = best;
        bi[w] = idx;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (uint32_t k = 1; k < (blockDim.x >> 5); ++k)
            if (bv[k] > best || (bv[k] == best && bi[k] < idx)) {
                best = bv[k];
                idx = bi[k];
            }
        out[row] = (int32_t)(idx == 0xffffffffu ? 0 : idx);
        if (bad_any)
            atomicOr(status, kStatusNonFinite);
    }
}

// End of a decode step: advance every row's position; the greedy pick
// becomes the next input and is appended to the generation history.
__global__ void step_end_kernel(uint32_t rows, uint32_t* pos, int32_t* tok_in, const int32_t* tok_next,
                                int32_t* hist, uint32_t* hist_count, uint32_t hist_cap, int has_logits) {
    const uint32_t r = threadIdx.x;
    if (r < rows) {
        pos[r] += 1;
        if (has_logits) {
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

// Non-finite check of an FP32 array (BNNE_Classify's input/logit checks).
__global__ void finite_check_kernel(const float* v, size_t n, int* status, int bit) {
    int bad = 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        bad |= !isfinite(v[i]);
    if (__syncthreads_or(bad) && threadIdx.x == 0)
        atomicOr(status, bit);
}

}  // namespace eng
}  // namespace bnn
