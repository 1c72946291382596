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
//   attention_kernel   (engine_kernels.cuh) with append = 0: per position,
//                      q-norm + RoPE and causal attention over the cache
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

constexpr uint32_t kRowsPrepThreads = kSumThreads;  // the decode prologue's four compute warps

struct RowsPrepArgs {
    const float* x;      // [m][k] F32 rows, x_stride floats apart
    size_t x_stride;
    const float* gain;   // RMSNorm gains [k], or null: quantise the row as it is
    float eps;
    int exact;           // RMSNorm sum: serial (reference order) or the decode prologue's tree
    uint32_t k, m;
    unsigned char* a_sw; // pre-tiled int8 rows (mma_a_offset)
    float* row_scale;    // [m]
    int* status;
};

inline size_t rows_prep_smem(uint32_t k, bool exact) {
    return (size_t)k * 4u + (exact ? kSumSmemBytes : 0);
}

// One CTA of kRowsPrepThreads per row. A non-finite input without RMSNorm is
// rejected (kStatusBadInput, ValidateF32Input); with RMSNorm it shows up as a
// non-finite divisor (kStatusNonFinite), as in the decode step.
__global__ void __launch_bounds__(kRowsPrepThreads) rows_prep_kernel(RowsPrepArgs a) {
    extern __shared__ __align__(16) unsigned char rp_smem[];
    __shared__ float red[16];
    __shared__ int s_flag;
    float* xb = reinterpret_cast<float*>(rp_smem);
    float4* xb4 = reinterpret_cast<float4*>(rp_smem);
    unsigned char* sum_mem = rp_smem + (size_t)a.k * 4u;
    const uint32_t row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t K = a.k, G = K / kGroup;
    constexpr uint32_t nt = kRowsPrepThreads, nw = kRowsPrepThreads / 32;

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
            sum = exact_sumsq(xb, (int)K, sum_mem, 1);
        } else {
            float t = 0.0f;
            for (uint32_t i = tid; i < K; i += nt)
                t = __fadd_rn(t, __fmul_rn(xb[i], xb[i]));
            for (int o = 16; o > 0; o >>= 1)
                t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, o));
            if (lane == 0)
                red[1 + warp] = t;
            __syncthreads();
            sum = 0.0f;
            for (uint32_t w = 0; w < nw; ++w)
                sum = __fadd_rn(sum, red[1 + w]);
        }
        const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)K), a.eps));
        if (!isfinite(rms) || rms == 0.0f) {
            if (tid == 0)
                atomicOr(a.status, kStatusNonFinite);
            return;  // uniform: every thread computed the same rms
        }
        amax = 0.0f;
        const float4* gr = reinterpret_cast<const float4*>(a.gain);
        for (uint32_t i = tid; i < K / 4; i += nt) {
            float4 v = xb4[i];
            const float4 gn = gr[i];
            v.x = __fmul_rn(__fdiv_rn(v.x, rms), gn.x);
            v.y = __fmul_rn(__fdiv_rn(v.y, rms), gn.y);
            v.z = __fmul_rn(__fdiv_rn(v.z, rms), gn.z);
            v.w = __fmul_rn(__fdiv_rn(v.w, rms), gn.w);
            amax = fmaxf(fmaxf(amax, fmaxf(fabsf(v.x), fabsf(v.y))), fmaxf(fabsf(v.z), fabsf(v.w)));
            xb4[i] = v;
        }
    }
    for (int o = 16; o > 0; o >>= 1)
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0)
        red[8 + warp] = amax;
    __syncthreads();
    amax = red[8];
    for (uint32_t w = 1; w < nw; ++w)
        amax = fmaxf(amax, red[8 + w]);
    const float s = row_scale_from_absmax(amax);
    const RowQuantizer quant(s);
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
    float* kcache;          // this layer: [cache rows][kv_heads][n_ctx][HD]
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
    const size_t base = (((size_t)a.slot[row] * a.kv_heads + g) * a.n_ctx + pos) * HD;
    for (uint32_t i = lane; i < HD; i += 32) {
        a.kcache[base + i] = v[i];
        a.vcache[base + i] = qkv_row[a.c + a.kv + (size_t)g * HD + i];
    }
}

}  // namespace eng
}  // namespace bnn
