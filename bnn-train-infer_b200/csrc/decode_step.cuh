// decode_step.cuh - one whole Qwen3 decode step (qwen3_step, qwen3.c:396-512)
// as a single persistent kernel, for one context row on one GPU.
//
// The step kernel runs one CTA per SM (a cooperative launch, so every CTA is
// resident) in two roles:
//   * attention CTAs 0 .. heads-1, one per query head: q/k RMSNorm, RoPE,
//     K/V append and causal softmax attention (qwen3.c:418-478); each keeps
//     its KV head's whole K/V history in shared memory, bulk-copied while the
//     contraction CTAs work on the previous layer;
//   * contraction CTAs (the rest): each owns fixed row ranges of every linear
//     (step_schedule.h) and one producer warp that streams those weight rows
//     (and the RMSNorm gains) through a shared-memory ring from the first
//     instruction on - weights never depend on activations, so the ring runs
//     up to ~3 layers ahead and every contraction finds its rows on chip.
// Phases of a layer, each a dataflow hand-off: the producing CTAs write their
// rows as 8-byte (value, generation) pairs and the consumers poll the rows
// themselves until every pair carries the phase's generation (no flag, no
// fence: one L2 round trip once the last row lands):
//   A  x ready      -> RMSNorm + quantise (every CTA, the full row) -> q|k|v rows
//   B  q|k|v ready  -> attention (attention CTAs) -> y
//   C  y ready      -> quantise y -> o rows, x += o   (rows the CTA owns)
//   D  x ready      -> RMSNorm + quantise -> gate|up pairs -> SwiGLU h
//   E  h ready      -> quantise h -> down rows, x += d
// then RMSNorm + lm_head + the greedy pick; the last CTA to finish advances
// the position, feeds the pick back and clears the counters for the next
// step. Every FP32 operation and its order are those of the per-kernel path
// (w1a8_gemv.cuh, engine_kernels.cuh, exact_sum.cuh): the results are
// bit-identical to it and to the reference. Every wait is bounded; a wait
// that gives up sets the status word, and once the status is set every CTA
// skips its work but keeps arriving on every counter, so the kernel always
// ends promptly.
#pragma once

#include <cstdint>
#include "bnn_device.cuh"
#include "bnn_sync.cuh"
#include "engine_kernels.cuh"
#include "exact_sum.cuh"
#include "step_schedule.h"
#include "w1a8_gemv.cuh"

namespace bnn {
namespace step {

constexpr uint32_t kWarps = 16;                     // compute warps of a CTA
constexpr uint32_t kCThreads = kWarps * 32;         // 512
constexpr uint32_t kThreads = kCThreads + 32;       // + the producer warp
constexpr uint32_t kBarCompute = 1;                 // named barrier of the compute warps
constexpr uint32_t kBarSum = 2;                     // the exact RMS sum (all compute warps)
constexpr uint32_t kHD = 128;                       // head_dim of the step kernel
constexpr size_t kSmemBudget = 226u * 1024u;  // dynamic; the static exit flag takes the rest of 227 KB

// Hand-offs of one layer. The generation a writer stamps on its pairs is
// epoch * 256 + layer * 5 + phase (at most 51 layers), never the all-ones
// pattern the buffers are cleared to.
enum : uint32_t { kPhQkv = 0, kPhY = 1, kPhXo = 2, kPhH = 3, kPhXd = 4, kPhPerLayer = 5 };
constexpr uint32_t kMaxStepLayers = 51;

__device__ __forceinline__ uint32_t hand_gen(uint32_t epoch, uint32_t l, uint32_t ph) {
    return epoch * 256u + l * kPhPerLayer + ph;
}

// One value of a hand-off row, with its generation (8-byte stores are single-copy atomic).
__device__ __forceinline__ void put_tagged(unsigned long long* dst, float v, uint32_t gen) {
    __stcg(dst, ((unsigned long long)gen << 32) | __float_as_uint(v));
}

struct LayerPtrs {
    const float* q_norm;   // [HD]
    const float* k_norm;   // [HD]
    float* kcache;         // this layer, KV head 0: [kv_heads][n_ctx][HD + 4]
    float* vcache;         // [kv_heads][n_ctx][HD]
};

struct StepArgs {
    const LayerPtrs* layers;
    uint32_t n_layers;
    uint32_t C, F, V, qkv_rows, heads, kv_heads, n_ctx;
    uint32_t n_attn, n_gemv;        // CTAs 0..n_attn-1 attention, the rest contraction
    const Copy* sched;              // [n_gemv][sched_stride]
    const uint32_t* sched_len;      // [n_gemv]
    uint32_t sched_stride;
    uint32_t ring_bytes;            // ring capacity of a contraction CTA
    uint32_t dsm_bytes;             // its integer-D buffer (one copy's blocks)
    uint32_t kv_resident;           // positions an attention CTA holds in shared memory
    const unsigned char* lm_head;   // packed blocks (also the tied embedding)
    int32_t* tok_in;
    uint32_t* pos;
    int32_t* tok_next;
    int32_t* hist;
    uint32_t* hist_count;
    uint32_t hist_cap;
    float* logits;
    unsigned long long* best;
    const float* rope_cos;          // [n_ctx][HD/2]
    const float* rope_sin;
    // hand-off rows as (value, generation) pairs: a reader polls the data
    // itself, each 8-byte pair valid once it carries the phase's generation
    unsigned long long *xt, *qkvt, *yt, *ht;
    uint32_t* epoch;                // step generation (advanced by the step's last CTA)
    uint32_t* sync;                 // [1]: the exit ticket, zero at step start
    int* status;
    float eps, scale;
    unsigned long long* trace;      // null, or [gridDim.x][n_layers + 1][kTraceSlots] %globaltimer stamps
    uint32_t poll_ns;               // pause between two polls of a hand-off row (doubling up to 8x while nothing arrives)
};

constexpr uint32_t kTraceSlots = 16;

__device__ __forceinline__ unsigned long long* trace_slot(const StepArgs& a, uint32_t l, uint32_t k) {
    return a.trace ? a.trace + ((size_t)blockIdx.x * (a.n_layers + 1) + l) * kTraceSlots + k : nullptr;
}

// Phase timestamp `k` of layer record `l` of this CTA (thread 0), when tracing.
__device__ __forceinline__ void stamp(const StepArgs& a, uint32_t l, uint32_t k) {
    if (a.trace != nullptr && threadIdx.x == 0)
        a.trace[((size_t)blockIdx.x * (a.n_layers + 1) + l) * kTraceSlots + k] = globaltimer_ns();
}

// ---- shared memory plans (one dynamic size; the two roles lay it out apart)
constexpr uint32_t kOwnRowsMax = 64;  // residual rows a contraction CTA owns (8 blocks)

constexpr uint32_t kSchedMax = 1024;  // copies per step a contraction CTA may stream

struct GemvPlan {
    size_t bars, red, xown, offs, xs, sum, act, tot, dsm, ring, total;
};

__host__ __device__ inline GemvPlan gemv_plan(uint32_t C, uint32_t F, uint32_t dsm_bytes) {
    GemvPlan p;
    const uint32_t kmax = C > F ? C : F;
    p.bars = 0;                                                   // full[kSlots], empty[kSlots]
    p.red = 2 * kSlots * 8;                                       // 64 floats + flags
    p.xown = p.red + 64 * 4 + 64;                                 // the CTA's residual rows [kOwnRowsMax]
    p.offs = p.xown + kOwnRowsMax * 4;                            // ring offsets of the copies [kSchedMax]
    p.xs = (p.offs + kSchedMax * 4 + 15) & ~(size_t)15;           // FP32 row [kmax]
    p.sum = (p.xs + (size_t)kmax * 4 + 15) & ~(size_t)15;         // exact RMS sum scratch
    p.act = (p.sum + kWideSmemBytes + 15) & ~(size_t)15;          // sliced words [G][kActStride]
    p.tot = p.act + (size_t)(kmax / kGroup) * kActStride * 4;     // group totals [G]
    p.dsm = (p.tot + (size_t)(kmax / kGroup) * 4 + 15) & ~(size_t)15;  // int16 D of one copy
    p.ring = (p.dsm + dsm_bytes + 127) & ~(size_t)127;
    p.total = kSmemBudget;
    return p;
}

struct AttnPlan {
    size_t bar, red, q, k, v, gq, gk, rc, rs, sc, kres, vres, total;
};

__host__ __device__ inline AttnPlan attn_plan(uint32_t resident) {
    AttnPlan p;
    p.bar = 0;
    p.red = 64;                                   // 64 floats + flags
    p.q = p.red + 64 * 4 + 64;
    p.k = p.q + kHD * 4;
    p.v = p.k + kHD * 4;
    p.gq = p.v + kHD * 4;
    p.gk = p.gq + kHD * 4;
    p.rc = p.gk + kHD * 4;
    p.rs = p.rc + kHD * 2;
    p.sc = p.rs + kHD * 2;                                          // scores [resident + 1], float4 rows
    p.kres = (p.sc + (size_t)((resident + 4) & ~3u) * 4 + 127) & ~(size_t)127;  // [resident][HD + 4]
    p.vres = p.kres + (size_t)resident * (kHD + 4) * 4;               // [resident][HD]
    p.total = p.vres + (size_t)resident * kHD * 4;
    return p;
}

// Largest K/V history an attention CTA can hold.
__host__ inline uint32_t attn_resident_max() {
    uint32_t r = 0;
    while (attn_plan(r + 1).total <= kSmemBudget)
        ++r;
    return r;
}

// ---- cross-CTA counters
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ int status_now(const int* status) {
    return *reinterpret_cast<const volatile int*>(status);
}

// By the compute warps: loads the K values of hand-off row `src` into xs
// once every pair carries `gen` (bounded; gives up at once when the status
// word is set). Each thread keeps all of its 16-byte loads in flight and
// reissues only the pairs not yet written. Returns, to all threads, whether
// the CTA should do its work; *amax_out and *bad_out (any non-finite value)
// cover the whole row.
__device__ __noinline__ bool poll_row(const unsigned long long* src, uint32_t K, uint32_t gen, float* xs, int* status,
                                      int* flag, float* red, float* amax_out, int* bad_out, uint32_t poll_ns) {
    constexpr uint32_t kMine = 16;  // 16-byte chunks per thread at most (K <= 16384)
    const uint32_t tid = threadIdx.x, chunks = K / 2;
    const ulonglong2* s2 = reinterpret_cast<const ulonglong2*>(src);
    if (tid == 0)
        *flag = 1;
    named_barrier(kBarCompute, kCThreads);
    uint32_t pending = 0;
    float amax = 0.0f;
    int bad = 0;
    auto take = [&](uint32_t i, ulonglong2 v) {
        const uint32_t c = tid + i * kCThreads;
        const bool ok0 = (uint32_t)(v.x >> 32) == gen, ok1 = (uint32_t)(v.y >> 32) == gen;
        if (ok0 && ok1) {
            const float f0 = __uint_as_float((uint32_t)v.x), f1 = __uint_as_float((uint32_t)v.y);
            bad |= !isfinite(f0) | !isfinite(f1);
            amax = fmaxf(amax, fmaxf(fabsf(f0), fabsf(f1)));
            reinterpret_cast<float2*>(xs)[c] = make_float2(f0, f1);
        } else {
            pending |= 1u << i;
        }
    };
#pragma unroll
    for (uint32_t i = 0; i < kMine; ++i)
        if (tid + i * kCThreads < chunks)
            take(i, __ldcg(s2 + tid + i * kCThreads));
    if (pending) {
        const uint64_t t0 = globaltimer_ns();
        const uint64_t limit = *reinterpret_cast<volatile unsigned long long*>(&g_wait_ns_limit);
        uint32_t pause = poll_ns;
        for (uint32_t round = 0; pending; ++round) {
            __nanosleep(pause);
            const uint32_t was = pending;
            pending = 0;
#pragma unroll
            for (uint32_t i = 0; i < kMine; ++i)
                if (was & (1u << i))
                    take(i, __ldcg(s2 + tid + i * kCThreads));
            pause = pending == was ? min(2u * pause, 8u * poll_ns) : poll_ns;
            if (pending && (round & 15u) == 15u &&
                (status_now(status) != 0 || globaltimer_ns() - t0 > limit)) {
                if (status_now(status) == 0)
                    atomicOr(status, kStatusTimeout);
                *flag = 0;
                break;
            }
        }
    }
    for (int o = 16; o > 0; o >>= 1)
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    bad = __reduce_or_sync(0xffffffffu, bad);
    if ((tid & 31) == 0) {
        red[32 + (tid >> 5)] = amax;
        if (bad)
            red[49] = 1.0f;
    }
    named_barrier(kBarCompute, kCThreads);
    float m = red[32];
    for (uint32_t w = 1; w < kWarps; ++w)
        m = fmaxf(m, red[32 + w]);
    *amax_out = m;
    *bad_out = red[49] != 0.0f;
    const bool live = *reinterpret_cast<volatile int*>(flag) != 0;
    named_barrier(kBarCompute, kCThreads);  // red and flag are reused next
    if (tid == 0)
        red[49] = 0.0f;
    return live;
}

// ---- the contraction pieces (the larger ones kept out of line: a contraction
// CTA runs phases A, C, D and E every layer, and one shared copy of each
// piece stays in the instruction cache where inlined copies evict each other)
// Integer D of every (block, row, group) of a copy of nb blocks at w into
// dsm [b][row][g]: one warp per (block, group quad), as w1a8_gemv_kernel.
__device__ __noinline__ void copy_dots(const unsigned char* w, uint32_t nb, uint32_t G, const uint32_t* act_s,
                                          const int32_t* tot_s, int16_t* dsm) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, r = lane & 7;
    const uint32_t quads = (G + 3) / 4, items = nb * quads;
    for (uint32_t it = warp; it < items; it += kWarps) {
        const uint32_t b = it / quads, g = (it % quads) * 4 + (lane >> 3);
        if (g >= G)
            continue;
        const uint4 wv = reinterpret_cast<const uint4*>(w + (size_t)b * G * 144u)[g * kRowBlock + r];
        dsm[(b * kRowBlock + r) * G + g] = (int16_t)group_dot_w(wv, act_s + g * kActStride, tot_s[g]);
    }
}

// acc = fl(acc + fl(F32(scale_g) * D_g)) in increasing g (soft :260-274),
// eight groups per pair of 16-byte loads when G % 8 == 0.
__device__ __forceinline__ float ordered_acc(const uint16_t* sc, const int16_t* dd, uint32_t G) {
    float acc = 0.0f;
    if ((G & 7u) == 0) {
        for (uint32_t g0 = 0; g0 < G; g0 += 8) {
            const uint4 sv = *reinterpret_cast<const uint4*>(sc + g0);
            const uint4 dv = *reinterpret_cast<const uint4*>(dd + g0);
            const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
            const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w};
            float p[8];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int d0 = (int)(int16_t)(dw[j] & 0xffffu), d1 = (int)(int16_t)(dw[j] >> 16);
                const float f0 = __fsub_rn(__int_as_float(0x4b400000 + d0), 12582912.0f);
                const float f1 = __fsub_rn(__int_as_float(0x4b400000 + d1), 12582912.0f);
                p[2 * j] = __fmul_rn(h2f((uint16_t)(sw[j] & 0xffffu)), f0);
                p[2 * j + 1] = __fmul_rn(h2f((uint16_t)(sw[j] >> 16)), f1);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j)
                acc = __fadd_rn(acc, p[j]);
        }
    } else {
        for (uint32_t g = 0; g < G; ++g)
            acc = __fadd_rn(acc, __fmul_rn(h2f(sc[g]), (float)dd[g]));
    }
    return acc;
}

// Block-wide maximum over the compute warps (red[32..47] scratch).
__device__ __forceinline__ float compute_max(float v, float* red) {
    for (int o = 16; o > 0; o >>= 1)
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0)
        red[32 + (threadIdx.x >> 5)] = v;
    named_barrier(kBarCompute, kCThreads);
    v = red[32];
    for (uint32_t w = 1; w < kWarps; ++w)
        v = fmaxf(v, red[32 + w]);
    named_barrier(kBarCompute, kCThreads);  // red is reused next
    return v;
}

// QuantizeRow of the K floats in xs (absmax given) into the sliced words and
// group totals (the layout and lane transposes of w1a8_gemv_kernel).
__device__ __noinline__ float quantize_slice(const float* xs, uint32_t K, float amax, uint32_t* act_s,
                                                int32_t* tot_s) {
    const float s = row_scale_from_absmax(amax);
    const RowQuantizer quant(s);
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t slot = (lane >> 3) * 8u + (lane & 1u) * 4u + ((lane >> 1) & 3u);
    const float4* xb4 = reinterpret_cast<const float4*>(xs);
    const uint32_t G = K / kGroup;
#pragma unroll 1
    for (uint32_t g = warp; g < G; g += kWarps) {
        const float4 v = xb4[g * 32u + lane];
        const int8_t q0 = quant(v.x), q1 = quant(v.y), q2 = quant(v.z), q3 = quant(v.w);
        uint32_t w = (uint32_t)(uint8_t)q0 | ((uint32_t)(uint8_t)q1 << 8) | ((uint32_t)(uint8_t)q2 << 16) |
                     ((uint32_t)(uint8_t)q3 << 24);
        const int total = __reduce_add_sync(0xffffffffu, (int)q0 + (int)q1 + (int)q2 + (int)q3);
        uint32_t o = __shfl_xor_sync(0xffffffffu, w, 4);
        w = (lane & 4u) ? __byte_perm(w, o, 0x3276) : __byte_perm(w, o, 0x5410);
        o = __shfl_xor_sync(0xffffffffu, w, 2);
        w = (lane & 2u) ? __byte_perm(w, o, 0x3715) : __byte_perm(w, o, 0x6240);
        act_s[g * kActStride + slot] = w;
        if (lane == 0)
            tot_s[g] = total;
    }
    named_barrier(kBarCompute, kCThreads);
    return s;
}

// RMSNorm (qwen3.c:361-372, the reference's serial sum) of the K floats in
// xs with `gain`, in place, then QuantizeRow. Returns false (status set)
// when the divisor is not finite or zero.
__device__ __noinline__ bool rms_quantize(float* xs, const float* gain, uint32_t K, float eps,
                                             unsigned char* sum_mem, float* red, uint32_t* act_s, int32_t* tot_s,
                                             float* s_out, int* status, unsigned long long* trace_at = nullptr) {
    named_barrier(kBarCompute, kCThreads);  // xs complete
    const float sum = exact_sumsq_wide(xs, (int)K, sum_mem, kBarSum);
    if (threadIdx.x == 0)
        red[48] = sum;
    named_barrier(kBarCompute, kCThreads);
    if (trace_at != nullptr && threadIdx.x == 0)
        *trace_at = globaltimer_ns();
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(red[48], (float)K), eps));
    if (!isfinite(rms) || rms == 0.0f) {
        if (threadIdx.x == 0)
            atomicOr(status, kStatusNonFinite);
        return false;
    }
    const float rr = __frcp_rn(rms);
    float amax = 0.0f;
    float4* xb4 = reinterpret_cast<float4*>(xs);
    const float4* gr = reinterpret_cast<const float4*>(gain);
    for (uint32_t i = threadIdx.x; i < K / 4; i += kCThreads) {
        float4 v = xb4[i];
        const float4 gn = gr[i];
        v.x = __fmul_rn(div_cr(v.x, rms, rr), gn.x);
        v.y = __fmul_rn(div_cr(v.y, rms, rr), gn.y);
        v.z = __fmul_rn(div_cr(v.z, rms, rr), gn.z);
        v.w = __fmul_rn(div_cr(v.w, rms, rr), gn.w);
        amax = fmaxf(fmaxf(amax, fmaxf(fabsf(v.x), fabsf(v.y))), fmaxf(fabsf(v.z), fabsf(v.w)));
        xb4[i] = v;
    }
    amax = compute_max(amax, red);
    *s_out = quantize_slice(xs, K, amax, act_s, tot_s);
    return true;
}

// Waits for copy i of the ring (bounded); false when it will not come (the
// copy warp stopped before it) or the wait ran out.
__device__ __forceinline__ bool take_copy(uint64_t* full, uint32_t i, const volatile int* stopped_at) {
    uint64_t* bar = &full[i % kSlots];
    const uint32_t parity = (i / kSlots) & 1u;
    if (mbar_try_wait(bar, parity))
        return true;
    const uint64_t t0 = globaltimer_ns();
    const uint64_t limit = *reinterpret_cast<volatile unsigned long long*>(&g_wait_ns_limit);
    for (uint32_t k = 0; k < kWaitPollLimit; ++k) {
        if (mbar_try_wait_suspend(bar, parity))
            return true;
        if ((uint32_t)*stopped_at <= i || globaltimer_ns() - t0 > limit)
            return false;
    }
    return false;
}

// The step's last CTA: advance the position, feed the greedy pick back,
// record it, and clear the counters and the pick for the next step
// (step_end_kernel's work, engine_kernels.cuh).
__device__ __forceinline__ void finish_step(const StepArgs& a, uint32_t pos) {
    __threadfence();
    if (threadIdx.x == 0) {
        const unsigned long long b = *reinterpret_cast<volatile unsigned long long*>(a.best);
        const int32_t tok = b ? (int32_t)(0xffffffffu - (uint32_t)(b & 0xffffffffull)) : 0;
        a.pos[0] = pos + 1;
        a.tok_next[0] = tok;
        a.tok_in[0] = tok;
        const uint32_t hc = *a.hist_count;
        if (hc < a.hist_cap)
            a.hist[hc] = tok;
        *a.hist_count = hc + 1;
        *a.best = 0ull;
        // the next step stamps new generations; the exit ticket starts again
        *a.epoch = (*a.epoch + 1u) & 0xffffffu;
        a.sync[0] = 0u;
    }
}

// By the compute warps after the CTA's last phase: true in the CTA that
// arrives last (every other CTA has passed all of its waits).
__device__ __forceinline__ bool exit_ticket(uint32_t* done, int* flag) {
    named_barrier(kBarCompute, kCThreads);
    if (threadIdx.x == 0) {
        __threadfence();
        *flag = atomicAdd(done, 1u) == gridDim.x - 1;
    }
    named_barrier(kBarCompute, kCThreads);
    return *reinterpret_cast<volatile int*>(flag) != 0;
}

// ---- attention CTA: query head blockIdx.x (qwen3.c:418-478), every layer
__device__ __forceinline__ void attention_role(const StepArgs& a, unsigned char* sm, uint32_t pos) {
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const AttnPlan p = attn_plan(a.kv_resident);
    uint64_t* kvbar = reinterpret_cast<uint64_t*>(sm + p.bar);
    float* red = reinterpret_cast<float*>(sm + p.red);
    int* flag = reinterpret_cast<int*>(sm + p.red + 64 * 4);
    float *q_s = reinterpret_cast<float*>(sm + p.q), *k_s = reinterpret_cast<float*>(sm + p.k);
    float *v_s = reinterpret_cast<float*>(sm + p.v), *gq_s = reinterpret_cast<float*>(sm + p.gq);
    float *gk_s = reinterpret_cast<float*>(sm + p.gk), *rc_s = reinterpret_cast<float*>(sm + p.rc);
    float *rs_s = reinterpret_cast<float*>(sm + p.rs), *sc = reinterpret_cast<float*>(sm + p.sc);
    float *kres = reinterpret_cast<float*>(sm + p.kres), *vres = reinterpret_cast<float*>(sm + p.vres);
    constexpr uint32_t HD = kHD, kstride = eng::kcache_row(kHD);
    const uint32_t L = a.n_layers, hq = blockIdx.x, kv_mul = a.heads / a.kv_heads, g = hq / kv_mul, n = pos + 1;
    const uint32_t epoch = *a.epoch;
    const size_t khead = (size_t)g * a.n_ctx * kstride, vhead = (size_t)g * a.n_ctx * HD;
    if (tid == 0) {
        mbar_init(kvbar, 1);
        fence_barrier_init();
        // the greedy pick starts empty (an earlier per-kernel step may have
        // left a key); every atomicMax on it comes after this CTA's first
        // arrival, so this store is ordered before them
        if (hq == 0)
            *a.best = 0ull;
    }
    named_barrier(kBarCompute, kCThreads);
    // the K/V history of layer l (positions 0 .. pos-1), one bulk copy each;
    // it does not depend on this step, so it is in flight while the
    // contraction CTAs finish the layers before
    auto prefetch = [&](uint32_t l) {
        if (tid == 0 && pos > 0) {
            const LayerPtrs& Lp = a.layers[l];
            mbar_arrive_expect_tx(kvbar, pos * (kstride + HD) * 4u);
            bulk_g2s(kres, Lp.kcache + khead, pos * kstride * 4u, kvbar);
            bulk_g2s(vres, Lp.vcache + vhead, pos * HD * 4u, kvbar);
        }
    };
    prefetch(0);
    for (uint32_t i = tid; i < HD / 2; i += kCThreads) {
        rc_s[i] = a.rope_cos[(size_t)pos * (HD / 2) + i];
        rs_s[i] = a.rope_sin[(size_t)pos * (HD / 2) + i];
    }
    for (uint32_t l = 0; l < L; ++l) {
        const LayerPtrs& Lp = a.layers[l];
        for (uint32_t i = tid; i < HD; i += kCThreads) {
            gq_s[i] = Lp.q_norm[i];
            gk_s[i] = Lp.k_norm[i];
        }
        // q (this head), k and v (its KV head) as they are written: threads
        // 0..63, 64..127, 128..191 each poll one 16-byte chunk (two pairs)
        if (tid == 0)
            *flag = 0;
        named_barrier(kBarCompute, kCThreads);
        if (tid < 3 * HD / 2) {
            const uint32_t part = tid / (HD / 2), c = tid % (HD / 2);
            const size_t base = part == 0 ? (size_t)hq * HD
                                          : a.C + (size_t)(part - 1) * a.kv_heads * HD + (size_t)g * HD;
            const ulonglong2* src = reinterpret_cast<const ulonglong2*>(a.qkvt + base) + c;
            float* dst = part == 0 ? q_s : part == 1 ? k_s : v_s;
            const uint32_t want = hand_gen(epoch, l, kPhQkv);
            ulonglong2 v = __ldcg(src);
            const uint64_t t0 = globaltimer_ns();
            const uint64_t limit = *reinterpret_cast<volatile unsigned long long*>(&g_wait_ns_limit);
            uint32_t pause = a.poll_ns;
            for (uint32_t round = 0; (uint32_t)(v.x >> 32) != want || (uint32_t)(v.y >> 32) != want; ++round) {
                if ((round & 15u) == 15u && (status_now(a.status) != 0 || globaltimer_ns() - t0 > limit)) {
                    if (status_now(a.status) == 0)
                        atomicOr(a.status, kStatusTimeout);
                    *flag = 1;
                    break;
                }
                __nanosleep(pause);
                pause = min(2u * pause, 8u * a.poll_ns);
                v = __ldcg(src);
            }
            dst[2 * c] = __uint_as_float((uint32_t)v.x);
            dst[2 * c + 1] = __uint_as_float((uint32_t)v.y);
        }
        named_barrier(kBarCompute, kCThreads);
        bool live = *reinterpret_cast<volatile int*>(flag) == 0;
        stamp(a, l, 0);
        named_barrier(kBarCompute, kCThreads);
        if (live && warp < 2) {
            if (!eng::attn_norm_rope<HD>(warp == 0 ? q_s : k_s, warp == 0 ? gq_s : gk_s, rc_s, rs_s, a.eps, true) &&
                lane == 0) {
                *flag = 1;
                atomicOr(a.status, kStatusNonFinite);
            }
        }
        named_barrier(kBarCompute, kCThreads);
        live = live && *reinterpret_cast<volatile int*>(flag) == 0;
        stamp(a, l, 1);
        // append this position's k and v (the first query head of the KV head writes)
        if (live && hq % kv_mul == 0 && tid < HD) {
            Lp.kcache[khead + (size_t)pos * kstride + tid] = k_s[tid];
            Lp.vcache[vhead + (size_t)pos * HD + tid] = v_s[tid];
        }
        if (pos > 0 && !mbar_wait(kvbar, l & 1u)) {
            if (lane == 0)
                atomicOr(a.status, kStatusTimeout);
            live = false;
        }
        stamp(a, l, 2);
        // scores: one position per thread, each dot serial over the head
        // dimension; their maximum is reduced on the way (per warp here, across
        // the warps after the barrier)
        int bad = 0;
        float mx = -INFINITY;
        if (live) {
            for (uint32_t t = tid; t < n; t += kCThreads) {
                const float4* k4 = reinterpret_cast<const float4*>(t < pos ? kres + (size_t)t * kstride : k_s);
                const float4* q4 = reinterpret_cast<const float4*>(q_s);
                float dot = 0.0f;
#pragma unroll
                for (uint32_t jj = 0; jj < HD / 4; ++jj) {
                    const float4 kk = k4[jj], qq = q4[jj];
                    dot = __fadd_rn(dot, __fmul_rn(qq.x, kk.x));
                    dot = __fadd_rn(dot, __fmul_rn(qq.y, kk.y));
                    dot = __fadd_rn(dot, __fmul_rn(qq.z, kk.z));
                    dot = __fadd_rn(dot, __fmul_rn(qq.w, kk.w));
                }
                const float score = __fmul_rn(dot, a.scale);
                bad |= !isfinite(score);
                sc[t] = score;
                mx = fmaxf(mx, score);
            }
        }
        bad = __reduce_or_sync(0xffffffffu, bad);
        for (int o = 16; o > 0; o >>= 1)
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0)
            red[32 + warp] = mx;  // read after the barrier; rewritten only in the next layer
        if (bad && lane == 0) {
            *flag = 1;
            atomicOr(a.status, kStatusNonFinite);  // "attention score is not finite"
        }
        named_barrier(kBarCompute, kCThreads);
        live = live && *reinterpret_cast<volatile int*>(flag) == 0;
        stamp(a, l, 3);
        // softmax: max (the scores are finite here), expf(s - max), serial sum, division
        mx = red[32];
        for (uint32_t w = 1; w < kWarps; ++w)
            mx = fmaxf(mx, red[32 + w]);
        if (live)
            for (uint32_t t = tid; t < n; t += kCThreads)
                sc[t] = expf_cr(__fsub_rn(sc[t], mx));
        named_barrier(kBarCompute, kCThreads);
        if (live && tid == 0) {
            // serial in index order; terms load two float4s ahead of their adds
            const float4* e4 = reinterpret_cast<const float4*>(sc);
            const uint32_t n4 = n / 4;
            float sum = 0.0f;
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
                sum = __fadd_rn(sum, sc[t]);
            red[16] = sum;
            if (!(sum > 0.0f) || !isfinite(sum)) {  // "attention softmax failed"
                *flag = 1;
                atomicOr(a.status, kStatusNonFinite);
            }
        }
        named_barrier(kBarCompute, kCThreads);
        live = live && *reinterpret_cast<volatile int*>(flag) == 0;
        if (live) {
            const float sum = red[16], rs = __frcp_rn(sum);
            for (uint32_t t = tid; t < n; t += kCThreads)
                sc[t] = div_cr(sc[t], sum, rs);
        }
        named_barrier(kBarCompute, kCThreads);
        stamp(a, l, 4);
        // y_d = sum_t p_t * v_t,d: one serial chain per dimension
        if (live && tid < HD) {
            const uint32_t d = tid;
            float v = 0.0f;
            uint32_t t = 0;
            for (; t + 8 <= pos; t += 8) {
                const float4 p0 = *reinterpret_cast<const float4*>(sc + t);
                const float4 p1 = *reinterpret_cast<const float4*>(sc + t + 4);
                float w[8];
#pragma unroll
                for (int jj = 0; jj < 8; ++jj)
                    w[jj] = vres[(size_t)(t + jj) * HD + d];
                const float pr[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
                for (int jj = 0; jj < 8; ++jj)
                    w[jj] = __fmul_rn(pr[jj], w[jj]);
#pragma unroll
                for (int jj = 0; jj < 8; ++jj)
                    v = __fadd_rn(v, w[jj]);
            }
            for (; t < pos; ++t)
                v = __fadd_rn(v, __fmul_rn(sc[t], vres[(size_t)t * HD + d]));
            v = __fadd_rn(v, __fmul_rn(sc[pos], v_s[d]));
            put_tagged(a.yt + (size_t)hq * HD + d, v, hand_gen(epoch, l, kPhY));
        }
        // the history buffers are free again: the next layer's copies start
        fence_proxy_async();
        named_barrier(kBarCompute, kCThreads);
        if (l + 1 < L)
            prefetch(l + 1);
        stamp(a, l, 5);
    }
}

// ---- contraction CTA j = blockIdx.x - n_attn
__device__ __forceinline__ void contraction_role(const StepArgs& a, unsigned char* sm, uint32_t pos) {
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t j = blockIdx.x - a.n_attn, L = a.n_layers;
    const uint32_t C = a.C, F = a.F, GC = C / kGroup, GF = F / kGroup;
    const GemvPlan p = gemv_plan(C, F, a.dsm_bytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + p.bars);
    uint64_t* empty = full + kSlots;
    float* red = reinterpret_cast<float*>(sm + p.red);
    int* flag = reinterpret_cast<int*>(sm + p.red + 64 * 4);
    volatile int* stopped_at = reinterpret_cast<volatile int*>(sm + p.red + 64 * 4 + 4);
    float* xs = reinterpret_cast<float*>(sm + p.xs);
    float* xown = reinterpret_cast<float*>(sm + p.xown);  // x rows [8 o0, 8 o1), kept here between phases
    unsigned char* sum_mem = sm + p.sum;
    uint32_t* act_s = reinterpret_cast<uint32_t*>(sm + p.act);
    int32_t* tot_s = reinterpret_cast<int32_t*>(sm + p.tot);
    int16_t* dsm = reinterpret_cast<int16_t*>(sm + p.dsm);
    unsigned char* ring = sm + p.ring;
    const Copy* sched = a.sched + (size_t)j * a.sched_stride;
    const uint32_t nsched = a.sched_len[j];

    uint32_t* offs = reinterpret_cast<uint32_t*>(sm + p.offs);
    if (tid == 0) {
        for (uint32_t s = 0; s < kSlots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_barrier_init();
        *stopped_at = 0x7fffffff;
    }
    // the ring offset of every copy, read once (the consumers need it on the
    // critical path; a global load there costs an L2 round trip)
    for (uint32_t i = tid; i < nsched; i += kThreads)
        offs[i] = sched[i].ring_off;
    __syncthreads();
    if (warp == kWarps) {
        // copy warp: the whole step's weight rows and gains, in consumption order
        if (lane == 0) {
            uint32_t released = 0;
            for (uint32_t i = 0; i < nsched; ++i) {
                const Copy c = sched[i];
                bool ok = true;
                while (released < c.need) {
                    if (!mbar_wait(&empty[released % kSlots], (released / kSlots) & 1u)) {
                        ok = false;
                        break;
                    }
                    ++released;
                }
                if (!ok) {
                    atomicOr(a.status, kStatusTimeout);
                    *stopped_at = (int)i;  // copies from i on never come
                    break;
                }
                mbar_arrive_expect_tx(&full[i % kSlots], c.bytes);
                bulk_g2s(ring + c.ring_off, reinterpret_cast<const void*>(c.src), c.bytes, &full[i % kSlots]);
            }
        }
        return;
    }

    uint32_t ci = 0;  // next copy to consume
    auto take = [&]() -> const unsigned char* {
        if (!take_copy(full, ci, stopped_at) && lane == 0)
            atomicOr(a.status, kStatusTimeout);
        return ring + offs[ci];
    };
    auto release = [&]() {
        named_barrier(kBarCompute, kCThreads);
        if (tid == 0)
            mbar_arrive(&empty[ci % kSlots]);
        ++ci;
    };
    const uint32_t epoch = *a.epoch;
    auto gen = [&](uint32_t l, uint32_t ph) { return hand_gen(epoch, l, ph); };
    // QuantizeRow of a hand-off row of K floats that other CTAs wrote (y or h)
    auto quant_prologue = [&](const unsigned long long* src, uint32_t K, uint32_t g, float* s) -> bool {
        float amax;
        int bad;
        const bool live = poll_row(src, K, g, xs, a.status, flag, red, &amax, &bad, a.poll_ns);
        // a linear rejects non-finite input (ValidateF32Input, soft :294-308)
        if (live && bad && tid == 0)
            atomicOr(a.status, kStatusBadInput);
        const bool ok = live && !bad;
        if (ok)
            *s = quantize_slice(xs, K, amax, act_s, tot_s);
        return ok;
    };
    // the ordered FP32 epilogue of output (block b, row r) of a copy at w
    auto acc_of = [&](const unsigned char* w, uint32_t G, uint32_t b, uint32_t r) {
        const uint16_t* sc = reinterpret_cast<const uint16_t*>(w + (size_t)b * G * 144u + (size_t)G * 128u) + r * G;
        return ordered_acc(sc, dsm + (size_t)(b * kRowBlock + r) * G, G);
    };

    const uint32_t nb_qkv = a.qkv_rows / kRowBlock, nb_c = C / kRowBlock, np_gu = F / kRowBlock;
    const uint32_t nb_v = (a.V + kRowBlock - 1) / kRowBlock;
    uint32_t q0, q1, o0, o1, p0, p1, v0, v1;
    split(j, a.n_gemv, nb_qkv, &q0, &q1);
    split(j, a.n_gemv, nb_c, &o0, &o1);
    split(j, a.n_gemv, np_gu, &p0, &p1);
    split(j, a.n_gemv, nb_v, &v0, &v1);
    float s = 1.0f;

    // qwen3_embed (qwen3.c:374-385): the token's row of the tied lm_head
    // blocks; the full row stays in xs for layer 0's RMSNorm, the rows this
    // CTA owns stay in xown for the residual adds
    if (tid == 0)
        red[49] = 0.0f;
    if (q1 > q0 || o1 > o0) {
        const uint32_t tok = (uint32_t)a.tok_in[0];
        const unsigned char* blk = a.lm_head + (size_t)(tok / kRowBlock) * GC * 144u;
        const uint32_t r = tok % kRowBlock;
        const uint16_t* scl = reinterpret_cast<const uint16_t*>(blk + (size_t)GC * 128u) + (size_t)r * GC;
        for (uint32_t k = tid; k < C; k += kCThreads) {
            const uint32_t g = k / kGroup, bit = k % kGroup;
            const uint32_t word = reinterpret_cast<const uint32_t*>(blk + (g * kRowBlock + r) * 16u)[bit >> 5];
            const float scale = h2f(scl[g]);
            xs[k] = ((word >> (bit & 31)) & 1u) ? scale : -scale;
        }
        named_barrier(kBarCompute, kCThreads);
        for (uint32_t k = o0 * kRowBlock + tid; k < o1 * kRowBlock; k += kCThreads)
            xown[k - o0 * kRowBlock] = xs[k];
    }
    if (tid == 0)
        *flag = status_now(a.status) == 0;
    named_barrier(kBarCompute, kCThreads);
    const bool live0 = *reinterpret_cast<volatile int*>(flag) != 0;

    for (uint32_t l = 0; l < L; ++l) {
        // ---- A: attn_norm + q|k|v rows
        stamp(a, l, 0);
        if (q1 > q0) {
            bool live = live0;
            if (l > 0) {
                float amax;
                int bad;
                live = poll_row(a.xt, C, gen(l - 1, kPhXd), xs, a.status, flag, red, &amax, &bad, a.poll_ns);
            }
            stamp(a, l, 1);
            const float* gain = reinterpret_cast<const float*>(take());
            live = live && rms_quantize(xs, gain, C, a.eps, sum_mem, red, act_s, tot_s, &s, a.status,
                                        trace_slot(a, l, 13));
            release();
            stamp(a, l, 2);
            const unsigned char* w = take();
            const uint32_t nb = q1 - q0;
            if (live) {
                copy_dots(w, nb, GC, act_s, tot_s, dsm);
                named_barrier(kBarCompute, kCThreads);
                const uint32_t g = gen(l, kPhQkv);
                for (uint32_t q = tid; q < nb * kRowBlock; q += kCThreads) {
                    const uint32_t n = q0 * kRowBlock + q;
                    if (n < a.qkv_rows)
                        put_tagged(a.qkvt + n, __fmul_rn(acc_of(w, GC, q / kRowBlock, q % kRowBlock), s), g);
                }
            }
            release();
        }
        stamp(a, l, 3);
        // ---- C: o rows, x += o
        if (o1 > o0) {
            bool live = quant_prologue(a.yt, C, gen(l, kPhY), &s);
            stamp(a, l, 4);
            stamp(a, l, 5);
            const unsigned char* w = take();
            const uint32_t nb = o1 - o0;
            if (live) {
                copy_dots(w, nb, GC, act_s, tot_s, dsm);
                named_barrier(kBarCompute, kCThreads);
                const uint32_t g = gen(l, kPhXo);
                for (uint32_t q = tid; q < nb * kRowBlock; q += kCThreads) {
                    const float y = __fmul_rn(acc_of(w, GC, q / kRowBlock, q % kRowBlock), s);
                    const float xn = __fadd_rn(xown[q], y);
                    xown[q] = xn;
                    put_tagged(a.xt + o0 * kRowBlock + q, xn, g);
                }
            }
            release();
        }
        stamp(a, l, 6);
        // ---- D: ffn_norm + gate|up pairs + SwiGLU
        if (p1 > p0) {
            float amax;
            int bad;
            bool live = poll_row(a.xt, C, gen(l, kPhXo), xs, a.status, flag, red, &amax, &bad, a.poll_ns);
            stamp(a, l, 7);
            const float* gain = reinterpret_cast<const float*>(take());
            live = live && rms_quantize(xs, gain, C, a.eps, sum_mem, red, act_s, tot_s, &s, a.status,
                                        trace_slot(a, l, 14));
            release();
            stamp(a, l, 8);
            const unsigned char* w = take();
            const uint32_t np = p1 - p0;
            if (live) {
                copy_dots(w, 2 * np, GC, act_s, tot_s, dsm);
                named_barrier(kBarCompute, kCThreads);
                // one ordered chain per thread (gate and up rows apart), then SwiGLU
                float* gu_s = xs;  // the normalised row is no longer needed
                for (uint32_t q = tid; q < 2 * np * kRowBlock; q += kCThreads)
                    gu_s[q] = __fmul_rn(acc_of(w, GC, q / kRowBlock, q % kRowBlock), s);
                named_barrier(kBarCompute, kCThreads);
                const uint32_t g = gen(l, kPhH);
                for (uint32_t q = tid; q < np * kRowBlock; q += kCThreads) {
                    const uint32_t k = q / kRowBlock, r = q % kRowBlock;
                    const float gt = gu_s[(2 * k) * kRowBlock + r], up = gu_s[(2 * k + 1) * kRowBlock + r];
                    const float silu = __fdiv_rn(gt, __fadd_rn(1.0f, expf_cr(-gt)));
                    put_tagged(a.ht + (size_t)(p0 + k) * kRowBlock + r, __fmul_rn(silu, up), g);
                }
            }
            release();
        }
        stamp(a, l, 9);
        // ---- E: down rows, x += d
        if (o1 > o0) {
            bool live = quant_prologue(a.ht, F, gen(l, kPhH), &s);
            stamp(a, l, 10);
            stamp(a, l, 11);
            const unsigned char* w = take();
            const uint32_t nb = o1 - o0;
            if (live) {
                copy_dots(w, nb, GF, act_s, tot_s, dsm);
                named_barrier(kBarCompute, kCThreads);
                const uint32_t g = gen(l, kPhXd);
                for (uint32_t q = tid; q < nb * kRowBlock; q += kCThreads) {
                    const float d = __fmul_rn(acc_of(w, GF, q / kRowBlock, q % kRowBlock), s);
                    const float xn = __fadd_rn(xown[q], d);
                    xown[q] = xn;
                    put_tagged(a.xt + o0 * kRowBlock + q, xn, g);
                }
            }
            release();
        }
        stamp(a, l, 12);
    }

    // ---- out_norm + lm_head + greedy pick (bnn-infer-v2.c:48-54: first maximum)
    if (v1 > v0) {
        float amax;
        int bad;
        bool live = poll_row(a.xt, C, gen(L - 1, kPhXd), xs, a.status, flag, red, &amax, &bad, a.poll_ns);
        stamp(a, L, 0);
        const float* gain = reinterpret_cast<const float*>(take());
        live = live && rms_quantize(xs, gain, C, a.eps, sum_mem, red, act_s, tot_s, &s, a.status);
        release();
        stamp(a, L, 1);
        unsigned long long best = 0ull;
        int nonfinite = 0;
        for (uint32_t b0 = v0; b0 < v1; b0 += kLmChunkBlocks) {
            const uint32_t nb = min(kLmChunkBlocks, v1 - b0);
            const unsigned char* w = take();
            if (live) {
                copy_dots(w, nb, GC, act_s, tot_s, dsm);
                named_barrier(kBarCompute, kCThreads);
                for (uint32_t q = tid; q < nb * kRowBlock; q += kCThreads) {
                    const uint32_t n = b0 * kRowBlock + q;
                    if (n >= a.V)
                        continue;
                    const float y = __fmul_rn(acc_of(w, GC, q / kRowBlock, q % kRowBlock), s);
                    a.logits[n] = y;
                    nonfinite |= !isfinite(y);
                    const unsigned long long key = argmax_key(y, n);
                    best = key > best ? key : best;
                }
            }
            release();
        }
        stamp(a, L, 2);
        if (nonfinite)
            atomicOr(a.status, kStatusNonFinite);
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long ob = __shfl_xor_sync(0xffffffffu, best, o);
            best = ob > best ? ob : best;
        }
        if (lane == 0 && best != 0ull)
            atomicMax(a.best, best);
    }
}

static_assert(kCThreads == (uint32_t)kWideThreads, "the exact RMS sum runs on every compute thread");

__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(StepArgs a) {
    extern __shared__ __align__(128) unsigned char sm[];
    const uint32_t pos = *a.pos;
    stamp(a, a.n_layers, 15);
    if (blockIdx.x < a.n_attn) {
        if (threadIdx.x >= kCThreads)
            return;  // no copy warp in this role
        attention_role(a, sm, pos);
    } else {
        contraction_role(a, sm, pos);
        if (threadIdx.x >= kCThreads)
            return;  // the copy warp has left
    }
    __shared__ int exit_flag;
    if (exit_ticket(a.sync, &exit_flag)) {
        finish_step(a, pos);
        stamp(a, a.n_layers, 14);
    }
}

}  // namespace step
}  // namespace bnn
