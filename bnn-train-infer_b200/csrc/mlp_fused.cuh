// mlp_fused.cuh - the whole bnn-mlp classifier in one launch, one sample per CTA.
//
// bnn_mlp_classify (bnn-sw-v2/bnn-mlp/bnn-mlp.c:176-197) runs every sample
// through every layer: the linear as one GEMV_F32 job (QuantizeRow of the
// row, soft-bnn-accelerator.c:175-211; the binary group dots :219-258; the
// ordered FP32 scale-accumulate :260-274 times the row scale), then
// fl(fl(post_scale * y) + post_bias) and ReLU (bnn-mlp.c:188-193). The
// classifier's weights are ~0.1 MB, so a batch is latency-bound: here one
// CTA keeps its sample's rows in shared memory from the input to the logits
// and streams each layer's packed weights (w1a8_gemv.cuh layout) into shared
// memory with one bulk copy, the next layer's copy in flight while this one
// computes, with the arithmetic of the contraction kernels (the same sliced
// activations, the same integers, the same FP32 order), so the logits are
// bit-identical to the per-layer launches.
#pragma once

#include <cstdint>
#include "bnn_device.cuh"
#include "bnn_sync.cuh"
#include "w1a8_gemv.cuh"

namespace bnn {
namespace eng {

struct MlpLayerDev {
    const unsigned char* wblocks;  // packed 8-row blocks
    const float* post_scale;       // [out]
    const float* post_bias;        // [out]
    uint32_t in, out;
    int relu;
};

struct MlpFusedArgs {
    const MlpLayerDev* layers;  // device array
    uint32_t n_layers;
    uint32_t max_in;            // widest layer input (floats per shared row)
    uint32_t max_wbytes;        // largest layer's packed weights (bytes, a multiple of 16)
    const float* x;             // [samples][layers[0].in]
    float* logits;              // [samples][last layer's out]
    int* status;
};

constexpr uint32_t kMlpThreads = 512;
constexpr uint32_t kMlpWarps = kMlpThreads / 32;
constexpr uint32_t kMlpFusedMaxSamples = 256;  // larger batches: per-layer launches on the tensor cores
// The call's input itself held NaN/Inf (BNNE_Classify's input check, mapped
// to BNND_EINVAL): the input is checked here instead of on the host.
constexpr int kStatusInputNotFinite = 16;

// Packed weight bytes of a layer: its 8-row blocks.
__host__ __device__ inline uint32_t mlp_layer_wbytes(uint32_t in, uint32_t out) {
    return (out + kRowBlock - 1) / kRowBlock * (uint32_t)block_bytes(in / kGroup);
}

// Two weight buffers + two rows (input, output) + the sliced activations and
// group totals + each warp's [8 rows][G] integer dots + reduction slots + two
// mbarriers.
inline size_t mlp_fused_smem(uint32_t max_in, uint32_t max_wbytes) {
    const size_t g = max_in / kGroup;
    return (size_t)2 * max_wbytes + (size_t)2 * max_in * 4u + g * kActStride * 4u + g * 4u +
           (size_t)kMlpWarps * kRowBlock * g * 4u + kMlpWarps * 4u + 16u;
}

// QuantizeRow of one group held as 32 lanes x float4 (lane L: values
// 4L .. 4L+3) into the contraction's sliced words and the group total (the
// layout of w1a8_gemv_kernel's F32 prologue).
__device__ __forceinline__ void mlp_slice_group(float4 v, const RowQuantizer& quant, uint32_t lane, uint32_t* act_g,
                                                int32_t* tot_g) {
    const int8_t q0 = quant(v.x), q1 = quant(v.y), q2 = quant(v.z), q3 = quant(v.w);
    uint32_t w = (uint32_t)(uint8_t)q0 | ((uint32_t)(uint8_t)q1 << 8) | ((uint32_t)(uint8_t)q2 << 16) |
                 ((uint32_t)(uint8_t)q3 << 24);
    const int total = __reduce_add_sync(0xffffffffu, (int)q0 + (int)q1 + (int)q2 + (int)q3);
    uint32_t o = __shfl_xor_sync(0xffffffffu, w, 4);
    w = (lane & 4u) ? __byte_perm(w, o, 0x3276) : __byte_perm(w, o, 0x5410);
    o = __shfl_xor_sync(0xffffffffu, w, 2);
    w = (lane & 2u) ? __byte_perm(w, o, 0x3715) : __byte_perm(w, o, 0x6240);
    act_g[(lane >> 3) * 8u + (lane & 1u) * 4u + ((lane >> 1) & 3u)] = w;
    if (lane == 0)
        *tot_g = total;
}

// A non-finite input row sets kStatusInputNotFinite; a non-finite hidden
// row (after a post-scale overflow) is rejected as the accelerator rejects a
// linear's input (kStatusBadInput); either stops the sample. Non-finite
// logits set kStatusNonFinite.
__global__ void __launch_bounds__(kMlpThreads) mlp_fused_kernel(MlpFusedArgs a) {
    extern __shared__ __align__(16) unsigned char mf_smem[];
    const uint32_t gmax = a.max_in / kGroup;
    unsigned char* wbuf = mf_smem;                                                     // [2][max_wbytes]
    float* rows = reinterpret_cast<float*>(mf_smem + 2 * (size_t)a.max_wbytes);        // [2][max_in]
    uint32_t* act_s = reinterpret_cast<uint32_t*>(rows + 2 * a.max_in);                // [gmax][kActStride]
    int32_t* tot_s = reinterpret_cast<int32_t*>(act_s + gmax * kActStride);
    int32_t* dots = tot_s + gmax;                                                      // [warps][8][gmax]
    float* red = reinterpret_cast<float*>(dots + kMlpWarps * kRowBlock * gmax);
    uint64_t* wfull = reinterpret_cast<uint64_t*>(
        (reinterpret_cast<uintptr_t>(red + kMlpWarps) + 7u) & ~uintptr_t(7));           // [2]
    const uint32_t sample = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    // layer l's weights go to buffer l & 1 (thread 0 issues; its use waits)
    auto fetch = [&](uint32_t l) {
        const MlpLayerDev& L = a.layers[l];
        const uint32_t bytes = mlp_layer_wbytes(L.in, L.out);
        mbar_arrive_expect_tx(&wfull[l & 1u], bytes);
        bulk_g2s(wbuf + (size_t)(l & 1u) * a.max_wbytes, L.wblocks, bytes, &wfull[l & 1u]);
    };
    if (tid == 0) {
        mbar_init(&wfull[0], 1);
        mbar_init(&wfull[1], 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0)
        for (uint32_t l = 0; l < a.n_layers && l < 2; ++l)
            fetch(l);
    uint32_t issued = a.n_layers < 2 ? a.n_layers : 2;  // copies issued (thread 0's view)
    // no bulk copy may be in flight when the CTA exits
    auto drain = [&](uint32_t waited) {
        if (tid == 0)
            for (uint32_t l = waited; l < issued; ++l)
                mbar_wait(&wfull[l & 1u], (l >> 1) & 1u);
    };

    const uint32_t k0 = a.layers[0].in;
    const float4* xg = reinterpret_cast<const float4*>(a.x + (size_t)sample * k0);
    for (uint32_t i = tid; i < k0 / 4; i += kMlpThreads)
        reinterpret_cast<float4*>(rows)[i] = xg[i];
    __syncthreads();

    int bad_out = 0;
    for (uint32_t l = 0; l < a.n_layers; ++l) {
        const MlpLayerDev L = a.layers[l];
        const float4* xin = reinterpret_cast<const float4*>(rows + (l & 1u) * a.max_in);
        float* yout = rows + ((l & 1u) ^ 1u) * a.max_in;
        const uint32_t K = L.in, G = K / kGroup, N = L.out;
        const bool last = l + 1 == a.n_layers;

        // ValidateF32Input (soft :294-308) and the row's absmax
        int bad = 0;
        float amax = 0.0f;
        for (uint32_t i = tid; i < K / 4; i += kMlpThreads) {
            const float4 v = xin[i];
            bad |= !isfinite(v.x) | !isfinite(v.y) | !isfinite(v.z) | !isfinite(v.w);
            amax = fmaxf(fmaxf(amax, fmaxf(fabsf(v.x), fabsf(v.y))), fmaxf(fabsf(v.z), fabsf(v.w)));
        }
        for (int o = 16; o > 0; o >>= 1)
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if (lane == 0)
            red[warp] = amax;
        if (__syncthreads_or(bad)) {
            if (tid == 0)
                atomicOr(a.status, l == 0 ? kStatusInputNotFinite : kStatusBadInput);
            drain(l);
            return;
        }
        amax = red[0];
        for (uint32_t w = 1; w < kMlpWarps; ++w)
            amax = fmaxf(amax, red[w]);
        const float s = row_scale_from_absmax(amax);
        const RowQuantizer quant(s);
        for (uint32_t g = warp; g < G; g += kMlpWarps)
            mlp_slice_group(xin[g * 32u + lane], quant, lane, act_s + g * kActStride, tot_s + g);
        __syncthreads();

        // this layer's weights in shared memory
        if (!mbar_wait(&wfull[l & 1u], (l >> 1) & 1u)) {
            if (tid == 0)
                atomicOr(a.status, kStatusTimeout);
            drain(l + 1);
            return;  // every thread gave up on the same barrier
        }
        const unsigned char* wl = wbuf + (size_t)(l & 1u) * a.max_wbytes;

        // warp w: output blocks w, w + 16, ...; its lanes take the block's
        // (group, row) units, then lanes 0..7 run the rows' ordered epilogues
        int32_t* dw = dots + warp * kRowBlock * gmax;
        const uint32_t nblocks = (N + kRowBlock - 1) / kRowBlock;
        const size_t bb = block_bytes(G);
        for (uint32_t b = warp; b < nblocks; b += kMlpWarps) {
            const unsigned char* wb = wl + (size_t)b * bb;
            for (uint32_t u = lane; u < G * kRowBlock; u += 32) {
                const uint32_t g = u / kRowBlock, r = u % kRowBlock;
                const uint4 w = *reinterpret_cast<const uint4*>(wb + (size_t)(g * kRowBlock + r) * 16u);
                dw[r * G + g] = group_dot_w(w, act_s + g * kActStride, tot_s[g]);
            }
            __syncwarp();
            const uint32_t n = b * kRowBlock + lane;
            if (lane < kRowBlock && n < N) {
                const uint16_t* sc = reinterpret_cast<const uint16_t*>(wb + (size_t)G * 128u) + lane * G;
                float acc = 0.0f;
                for (uint32_t g = 0; g < G; ++g)
                    acc = __fadd_rn(acc, __fmul_rn(h2f(sc[g]), (float)dw[lane * G + g]));
                acc = __fmul_rn(acc, s);
                float v = __fadd_rn(__fmul_rn(L.post_scale[n], acc), L.post_bias[n]);
                if (L.relu && v < 0.0f)
                    v = 0.0f;
                if (last) {
                    a.logits[(size_t)sample * N + n] = v;
                    bad_out |= !isfinite(v);
                } else {
                    yout[n] = v;
                }
            }
            __syncwarp();  // dw is reused by the next block
        }
        __syncthreads();  // yout complete; act_s, tot_s and this layer's weight buffer free
        if (tid == 0 && l + 2 < a.n_layers) {
            fetch(l + 2);
            issued = l + 3;
        }
    }
    if (__syncthreads_or(bad_out) && tid == 0)
        atomicOr(a.status, kStatusNonFinite);
}

}  // namespace eng
}  // namespace bnn
