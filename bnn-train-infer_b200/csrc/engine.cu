// engine.cu - device-resident Qwen3 / bnn-mlp engine (BNND_*, include/bnn_b200_engine.h).
//
// Load path mirrors the reference's (bnn-sw-v2/engine.c:16-78, qwen3.c:144-274,
// bnn-mlp.c:62-151): the same GGUF keys and tensor names, the same shape
// checks and status codes, Q1_0 decoded as bnne_q1_0_read does
// (linear.c:26-62) and uploaded through the BNN_* matrix path (repacked on
// the device). Linears that share an input are concatenated by rows
// (q|k|v, gate|up): every output row is computed independently, so this is
// bit-identical to separate calls.
//
// A decode step (qwen3_step, qwen3.c:396-512) is a fixed kernel sequence over
// device-resident state, captured once per context as a CUDA graph; the
// position and input token live in device memory so one graph serves every
// step. Per layer:
//   W1A8(RMSNorm -> q|k|v) -> qk_norm_rope(+KV append) -> attention
//   -> W1A8(quantise y -> o, x += o) -> W1A8(RMSNorm -> gate|up -> SwiGLU h)
//   -> W1A8(quantise h -> down, x += d)
// then W1A8(RMSNorm -> lm_head) -> argmax -> step_end. The RMSNorm and the
// row quantisation run inside each linear's prologue; the W1A8 linears are
// launched with programmatic dependent launch so their weight streaming
// overlaps the preceding kernel.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <memory>
#include <new>
#include <string>
#include <vector>

#include <nccl.h>

#include "bnn_b200_engine.h"
#include "bnn_b200_ext.h"
#include "bnn_internal.h"
#include "bpe_tokenizer.h"
#include "decode_step.cuh"
#include "engine_kernels.cuh"
#include "gguf_reader.h"
#include "mlp_fused.cuh"
#include "prefill_kernels.cuh"
#include "w1a8_gemv.cuh"
#include "w1a8_mma.cuh"
#include "w1a8_prep.cuh"

namespace {

constexpr uint32_t kStepRowsPrep = 4;  // decode steps of this many context rows prepare each row in its own CTA
constexpr size_t kAttnSmemBudget = 227u * 1024u;  // dynamic shared memory of one attention block (the sm_100 maximum)

thread_local std::string g_last_error;

BNND_Status fail(BNND_Status st, const char* fmt, ...) {
    char buf[256];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return st;
}

BNND_Status from_accel(BNN_Status st, const char* what) {
    if (st == BNN_OK)
        return BNND_OK;
    BNND_Status r = BNND_ECOMPUTE;
    if (st == BNN_ENOMEM) r = BNND_ENOMEM;
    else if (st == BNN_ENOTSUP) r = BNND_ENOTSUP;
    else if (st == BNN_ERANGE) r = BNND_ERANGE;
    else if (st == BNN_EIO || st == BNN_ETIMEOUT) r = BNND_EIO;
    return fail(r, "%s: %s", what, BNN_StatusString(st));
}



// Timestamps between launches while capturing an instrumented step.
struct StepRecorder {
    cudaStream_t stream = nullptr;
    std::vector<cudaEvent_t> events;  // events[i] precedes launch i
    std::vector<std::string> names;   // names[i] labels launch i
    std::vector<double> bytes;        // algorithmic bytes of launch i
    size_t next = 0;
    bool overflow = false;
    void mark(const char* name, double b) {
        if (next + 1 >= events.size()) {
            overflow = true;
            return;
        }
        names[next] = name;
        bytes[next] = b;
        ++next;
        cudaEventRecordWithFlags(events[next], stream, cudaEventRecordExternal);
    }
};
thread_local StepRecorder* g_rec = nullptr;
thread_local double g_next_bytes = 0.0;  // bytes of the launch being reported

// First failing launch of an enqueue sequence (name + error), for diagnostics.
struct LaunchCheck {
    const char* what = nullptr;
    cudaError_t err = cudaSuccess;
    void operator()(const char* name, cudaError_t e = cudaGetLastError()) {
        if (e != cudaSuccess && err == cudaSuccess) {
            err = e;
            what = name;
        }
        ++launches;
        if (g_rec)
            g_rec->mark(name, g_next_bytes);
        g_next_bytes = 0.0;
    }
    uint32_t launches = 0;
};
thread_local LaunchCheck* g_check = nullptr;

#define CUDA_OR(expr, status)                                                              \
    do {                                                                                   \
        cudaError_t e_ = (expr);                                                           \
        if (e_ != cudaSuccess) {                                                           \
            cudaGetLastError();                                                            \
            return fail(status, "%s: %s", #expr, cudaGetErrorString(e_));                  \
        }                                                                                  \
    } while (0)

// Device allocation owned by a model or context.
struct DevMem {
    void* p = nullptr;
    ~DevMem() {
        if (p)
            cudaFree(p);
    }
    template <typename T>
    T* as() const { return static_cast<T*>(p); }
};

BNND_Status dev_alloc(DevMem& m, size_t bytes) {
    if (bytes == 0)
        bytes = 16;
    if (cudaMalloc(&m.p, bytes) != cudaSuccess) {
        cudaGetLastError();
        m.p = nullptr;
        return fail(BNND_ENOMEM, "device allocation of %zu bytes failed", bytes);
    }
    return BNND_OK;
}

float half_bits_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, mant = h & 0x3ffu;
    int exp = (h >> 10) & 0x1f;
    uint32_t bits;
    if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            int e = 1;
            while ((mant & 0x400u) == 0) {
                mant <<= 1;
                --e;
            }
            bits = sign | ((uint32_t)(e + 112) << 23) | ((mant & 0x3ffu) << 13);
        }
    } else {
        bits = sign | ((uint32_t)(exp + 112) << 23) | (mant << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// A W1 linear on the device: matrix handle plus its launch plan.
struct Linear {
    BNN_Matrix m = nullptr;
    uint32_t in = 0, out = 0;
    ~Linear() { BNN_MatrixDestroy(m); }
};

BNND_Status read_f32(const bnn::GgufFile& g, const std::string& name, size_t count, DevMem* dst,
                     std::vector<float>* host = nullptr) {
    const bnn::GgufTensor* t = g.tensor(name);
    if (!t || (t->type != 0 && t->type != 1))
        return fail(BNND_EFORMAT, "missing or invalid F32/F16 tensor '%s'", name.c_str());
    size_t n = 1;
    for (uint64_t d : t->dims)
        n *= (size_t)d;
    if (n != count)
        return fail(BNND_EFORMAT, "tensor '%s' has %zu elements, expected %zu", name.c_str(), n, count);
    std::vector<float> v(n);
    for (size_t i = 0; i < n; ++i) {
        if (t->type == 0) {
            std::memcpy(&v[i], t->data + 4 * i, 4);
        } else {
            uint16_t h = (uint16_t)(t->data[2 * i] | (t->data[2 * i + 1] << 8));
            v[i] = half_bits_to_float(h);
        }
        if (!std::isfinite(v[i]))
            return fail(BNND_EFORMAT, "non-finite value in tensor '%s'", name.c_str());
    }
    BNND_Status st = dev_alloc(*dst, n * 4);
    if (st != BNND_OK)
        return st;
    CUDA_OR(cudaMemcpy(dst->p, v.data(), n * 4, cudaMemcpyHostToDevice), BNND_EIO);
    if (host)
        *host = std::move(v);
    return BNND_OK;
}

struct QwenLayer {
    Linear qkv, o, gu, down;
    DevMem attn_norm, ffn_norm, q_norm, k_norm;
};

struct MlpLayer {
    Linear w;
    DevMem post_scale, post_bias;
    int relu = 0;
};

}  // namespace

struct bnnd_model {
    BNN_Device dev = nullptr;
    BNND_ModelInfo info{};
    // qwen3
    float eps = 0, rope_base = 0, rope_freq_scale = 1, rope_mscale = 1;
    int32_t rope_corr0 = 0, rope_corr1 = 0;
    int rope_yarn = 0;
    std::vector<std::unique_ptr<QwenLayer>> layers;
    Linear lm_head;        // this rank's lm_head rows (all of them when world == 1)
    Linear embed;          // world > 1: the whole tied embedding, for embed_kernel
    DevMem out_norm;
    BNND_ShardInfo shard{};  // world 1: every range is the whole matrix
    std::unique_ptr<bnn::BpeTokenizer> tok;  // qwen3: the GGUF's text tokenizer
    // bnn-mlp
    std::vector<std::unique_ptr<MlpLayer>> mlp;
    uint32_t mlp_max_dim = 0;
    uint32_t mlp_max_in = 0;  // widest layer input
    uint32_t mlp_max_wbytes = 0;  // largest layer's packed weights
    DevMem mlp_desc;          // bnn::eng::MlpLayerDev per layer, for mlp_fused_kernel
};

// BNND_TokenizerLoad: a tokenizer without a model or a device.
struct bnnd_tokenizer {
    bnn::BpeTokenizer tok;
};

// BNND_GenerateStream keeps up to kStreamAhead decode steps queued ahead of
// the token the host is handing out; each step's token is copied into its own
// pinned slot, so kStreamSlots covers the steps in flight plus the one read.
constexpr uint32_t kStreamAhead = 4;
constexpr uint32_t kStreamSlots = 2 * kStreamAhead + 2;

struct bnnd_context {
    BNND_Model model = nullptr;
    BNND_ContextParams params{};
    uint32_t rows = 1, n_ctx = 0, pos = 0;
    cudaStream_t stream = nullptr;
    DevMem x, qkv, y, h, logits, kcache, vcache, rope_cos, rope_sin, scores;
    DevMem pos_d, tok_in, tok_next, tok_seq, hist, hist_count, status;
    DevMem best;  // [rows] packed greedy pick of the lm_head epilogue ([world][rows] when sharded)
    // tensor parallelism (model shard with world > 1)
    uint32_t world = 1, rank = 0;
    ncclComm_t comm = nullptr;
    DevMem y_st, x_st, h_st, lg_st;  // rank-major all-gather buffers [world][rows][slice]
    DevMem mlp_a, mlp_b;
    DevMem mlp_asw, mlp_rs;  // classify batches of kMmaMinRows+ rows: tensor-core operand, row scales
    size_t tok_seq_cap = 0;
    uint32_t hist_cap = 0;
    bnn::GemvLaunch plan_qkv{}, plan_o{}, plan_gu{}, plan_down{}, plan_head{};
    size_t attn_smem = 0;  // dynamic shared memory of the attention kernel
    uint32_t attn_resident = 0;  // positions whose whole K/V history the attention kernel holds in shared memory
    std::vector<bnn::GemvLaunch> plan_mlp;
    bool pdl = true;  // launch the W1A8 linears with programmatic dependent launch
    cudaGraphExec_t graph_logits = nullptr, graph_prefill = nullptr, graph_profile = nullptr;
    StepRecorder recorder;
    uint32_t step_launches = 0;
    int* h_status = nullptr;
    float* h_mlp_in = nullptr;     // pinned staging of a fused classify call's samples / logits
    float* h_mlp_out = nullptr;
    size_t mlp_fused_smem = 0;     // 0: no fused classify (mlp_fused.cuh) in this context
    int32_t* h_tokens = nullptr;   // pinned staging of input ids
    size_t h_tokens_cap = 0;
    int32_t* h_next = nullptr;     // pinned staging of greedy picks
    bool have_logits = false;
    // batched prefill: activation rows = prompt positions of every row
    DevMem pf_x, pf_qkv, pf_y, pf_h, pf_a, pf_rs, pf_scores, pf_meta;
    DevMem dm_act, dm_tot, dm_rs;  // steps of kStepRowsPrep+ rows: sliced rows, group totals, row scales
    DevMem lg_pos;                 // BNND_DecodeLogitsAll: one position's logits
    // persistent step kernel (decode_step.cuh): one launch per decode step
    DevMem st_sync, st_sched, st_sched_len, st_layers, st_xt, st_qkvt, st_yt, st_ht;
    bnn::step::StepArgs st_args{};
    uint32_t st_positions = 0;     // steps at positions below this use it (0: never)
    cudaGraphExec_t graph_step = nullptr;
    bnn::GemvLaunch plan_qkv_s{}, plan_o_s{}, plan_gu_s{}, plan_down_s{}, plan_head_s{};  // their contractions
    uint32_t pf_rows = 0;          // activation rows the pf_* buffers hold
    size_t pf_meta_cap = 0;        // entries of pf_meta (ids, positions, cache rows)
    uint32_t* h_meta = nullptr;    // pinned staging of pf_meta
    size_t h_meta_cap = 0;
    // BNND_GenerateStream: token copies on a side stream, one slot per step in flight
    cudaStream_t aux = nullptr;
    cudaEvent_t sv_step[kStreamSlots] = {}, sv_copy[kStreamSlots] = {};
    int32_t* h_stream = nullptr;   // pinned [kStreamSlots]

    ~bnnd_context() {
        // graphs that hold NCCL work go before the communicator
        if (graph_logits)
            cudaGraphExecDestroy(graph_logits);
        if (graph_prefill)
            cudaGraphExecDestroy(graph_prefill);
        if (graph_profile)
            cudaGraphExecDestroy(graph_profile);
        if (graph_step)
            cudaGraphExecDestroy(graph_step);
        if (comm)
            ncclCommDestroy(comm);
        for (cudaEvent_t e : recorder.events)
            cudaEventDestroy(e);
        if (h_status)
            cudaFreeHost(h_status);
        if (h_mlp_in)
            cudaFreeHost(h_mlp_in);
        if (h_mlp_out)
            cudaFreeHost(h_mlp_out);
        if (h_tokens)
            cudaFreeHost(h_tokens);
        if (h_next)
            cudaFreeHost(h_next);
        if (h_meta)
            cudaFreeHost(h_meta);
        for (uint32_t i = 0; i < kStreamSlots; ++i) {
            if (sv_step[i])
                cudaEventDestroy(sv_step[i]);
            if (sv_copy[i])
                cudaEventDestroy(sv_copy[i]);
        }
        if (h_stream)
            cudaFreeHost(h_stream);
        if (aux)
            cudaStreamDestroy(aux);
    }
};

namespace {

// qwen3_init_rope_params (qwen3.c:116-142): same formulas, same types.
BNND_Status rope_params(const bnn::GgufFile& g, bnnd_model* m) {
    float factor = 0.0f;
    g.get_f32("qwen3.rope.scaling.factor", &factor);
    if (factor <= 0.0f)
        factor = 1.0f;
    std::string type;
    g.get_str("qwen3.rope.scaling.type", &type);
    uint64_t original = 0;
    g.get_u64("qwen3.rope.scaling.original_context_length", &original);
    if (original == 0)
        original = m->info.n_ctx_train;
    const float freq_scale = 1.0f / factor;
    const int yarn = type == "yarn";
    int32_t corr0 = 0, corr1 = (int32_t)(m->info.head_dim - 1);
    float mscale = 1.0f;
    if (yarn && original) {
        const double base = m->rope_base, orig = (double)original, pi = 3.14159265358979323846;
        const double start = std::floor((double)m->info.head_dim * std::log(orig / (32.0 * 2.0 * pi)) /
                                        (2.0 * std::log(base)));
        const double end = std::ceil((double)m->info.head_dim * std::log(orig / (2.0 * pi)) /
                                     (2.0 * std::log(base)));
        auto clamp = [&](double v) {
            const int32_t hi = (int32_t)m->info.head_dim - 1;
            if (v <= 0.0) return (int32_t)0;
            if (v >= (double)hi) return hi;
            return (int32_t)v;
        };
        corr0 = clamp(start);
        corr1 = clamp(end);
        mscale = 1.0f + 0.1f * logf(1.0f / freq_scale);
    }
    if (!(freq_scale > 0.0f) || !std::isfinite(mscale))
        return fail(BNND_EFORMAT, "invalid Qwen3 rope scaling");
    m->rope_freq_scale = freq_scale;
    m->rope_mscale = mscale;
    m->rope_corr0 = corr0;
    m->rope_corr1 = corr1;
    m->rope_yarn = yarn;
    return BNND_OK;
}

// Row ranges of one rank's column shard (see BNND_ShardInfo).
BNND_Status shard_plan(const BNND_ModelInfo& in, uint32_t world, uint32_t rank, BNND_ShardInfo* out) {
    if (world == 0 || rank >= world)
        return fail(BNND_EINVAL, "rank %u outside world %u", rank, world);
    if (in.heads % world || in.kv_heads % world || in.hidden % (8 * world) || in.ffn % (8 * world))
        return fail(BNND_ENOTSUP, "heads %u / kv_heads %u / hidden %u / ffn %u do not split over %u ranks",
                    in.heads, in.kv_heads, in.hidden, in.ffn, world);
    BNND_ShardInfo sh{};
    sh.world = world;
    sh.rank = rank;
    sh.q_rows = in.heads / world * in.head_dim;
    sh.q_begin = rank * sh.q_rows;
    sh.kv_rows = in.kv_heads / world * in.head_dim;
    sh.kv_begin = rank * sh.kv_rows;
    sh.c_rows = in.hidden / world;
    sh.c_begin = rank * sh.c_rows;
    sh.f_rows = in.ffn / world;
    sh.f_begin = rank * sh.f_rows;
    sh.v_stride = ((in.n_vocab + world - 1) / world + 7) / 8 * 8;
    sh.v_begin = std::min(rank * sh.v_stride, in.n_vocab);
    sh.v_rows = std::min(sh.v_stride, in.n_vocab - sh.v_begin);
    *out = sh;
    return BNND_OK;
}

// ---- GGUF -> device loader: Q1_0 tensors are uploaded as they are in the
// file and repacked into the contraction's layout by q1_0_pack_kernel.
struct DeviceLoader {
    BNN_Device dev = nullptr;
    DevMem stage, bad;  // raw Q1_0 rows of one tensor; the scale check word
    size_t cap = 0;
};

BNND_Status w1_alloc(DeviceLoader* ld, uint32_t in, uint32_t out, Linear* l) {
    l->in = in;
    l->out = out;
    return from_accel(bnn_b200_matrix_alloc(ld->dev, in, out, &l->m), "matrix allocation");
}

// Rows row0 .. row0 + rows - 1 of Q1_0 tensor `name` ([out_total][in]) into
// l's rows from dst_row0 (half < 0), or interleaved as gate (half 0) or up
// (half 1) blocks.
BNND_Status w1_add(DeviceLoader* ld, const bnn::GgufFile& g, const std::string& name, uint32_t in,
                   uint32_t out_total, Linear* l, uint32_t dst_row0, int half, uint32_t row0 = 0,
                   uint32_t rows = UINT32_MAX) {
    const bnn::GgufTensor* t = g.tensor(name);
    if (!t || t->type != 41 || t->dims.size() != 2 || t->dims[0] != in || t->dims[1] != out_total ||
        in % 128 != 0 || l->in != in)
        return fail(BNND_EFORMAT, "unexpected Q1_0 tensor '%s' shape or type", name.c_str());
    if (rows == UINT32_MAX)
        rows = out_total - row0;
    if (row0 > out_total || rows > out_total - row0)
        return fail(BNND_EINVAL, "row range of '%s' outside the tensor", name.c_str());
    const uint32_t groups = in / 128;
    const size_t bytes = (size_t)rows * groups * 18u;
    BNND_Status st;
    if (ld->cap < bytes) {
        ld->stage = DevMem();
        ld->cap = 0;
        if ((st = dev_alloc(ld->stage, bytes)))
            return st;
        ld->cap = bytes;
    }
    if (!ld->bad.p && (st = dev_alloc(ld->bad, 4)))
        return st;
    const cudaStream_t s = ld->dev->stream;
    CUDA_OR(cudaMemsetAsync(ld->bad.p, 0, 4, s), BNND_EIO);
    CUDA_OR(cudaMemcpyAsync(ld->stage.p, t->data + (size_t)row0 * groups * 18u, bytes, cudaMemcpyHostToDevice, s),
            BNND_EIO);
    const size_t units = (size_t)rows * groups;
    const unsigned grid = (unsigned)std::min<size_t>((units + 255) / 256, 148u * 16u);
    bnn::eng::q1_0_pack_kernel<<<grid, 256, 0, s>>>(ld->stage.as<uint8_t>(), rows, groups, dst_row0, half,
                                                   l->m->wblocks, ld->bad.as<int>());
    int bad = 0;
    CUDA_OR(cudaGetLastError(), BNND_EIO);
    CUDA_OR(cudaMemcpyAsync(&bad, ld->bad.p, 4, cudaMemcpyDeviceToHost, s), BNND_EIO);
    CUDA_OR(cudaStreamSynchronize(s), BNND_EIO);
    if (bad)
        return fail(BNND_EFORMAT, "Q1_0 scale in '%s' is not finite", name.c_str());
    return BNND_OK;
}

BNND_Status load_qwen3(const bnn::GgufFile& g, bnnd_model* m) {
    uint64_t L = 0, C = 0, FF = 0, H = 0, Hk = 0, kl = 0, vl = 0, ctx = 0;
    g.get_u64("qwen3.block_count", &L);
    g.get_u64("qwen3.embedding_length", &C);
    g.get_u64("qwen3.feed_forward_length", &FF);
    g.get_u64("qwen3.attention.head_count", &H);
    g.get_u64("qwen3.attention.head_count_kv", &Hk);
    g.get_u64("qwen3.attention.key_length", &kl);
    g.get_u64("qwen3.attention.value_length", &vl);
    g.get_u64("qwen3.context_length", &ctx);
    float eps = 0.0f, base = 0.0f;
    g.get_f32("qwen3.attention.layer_norm_rms_epsilon", &eps);
    g.get_f32("qwen3.rope.freq_base", &base);
    const bnn::GgufTensor* emb = g.tensor("token_embd.weight");
    if (!emb || emb->type != 41 || emb->dims.size() != 2)
        return fail(BNND_EFORMAT, "missing token_embd.weight");
    // Same admissible ranges as qwen3_load (qwen3.c:155-189).
    if (L == 0 || L > 128 || C == 0 || C > UINT32_MAX || FF == 0 || FF > UINT32_MAX || H == 0 ||
        H > 256 || Hk == 0 || Hk > 256 || kl == 0 || kl > UINT32_MAX || kl != vl || ctx == 0 ||
        ctx > UINT32_MAX || eps <= 0.0f || base <= 0.0f || emb->dims[0] != C || emb->dims[1] == 0 ||
        emb->dims[1] > (1u << 20))
        return fail(BNND_EFORMAT, "unsupported Qwen3 dimensions");
    const uint32_t HD = (uint32_t)kl, V = (uint32_t)emb->dims[1];
    if (HD > C || H * HD != C || H % Hk != 0 || C % 128 != 0 || FF % 128 != 0 || HD % 2 != 0)
        return fail(BNND_EFORMAT, "inconsistent Qwen3 dimensions");
    const uint32_t KV = (uint32_t)(Hk * HD);
    if (KV % 128 != 0)
        return fail(BNND_EFORMAT, "Qwen3 KV width is not group aligned");
    if (HD > 1024)
        return fail(BNND_ENOTSUP, "head_dim above 1024 is not supported");
    if (C > bnn::kMaxPrologueK || FF > bnn::kMaxPrologueK)
        return fail(BNND_ENOTSUP, "hidden or ffn width above %u is not supported", bnn::kMaxPrologueK);
    BNND_ModelInfo& info = m->info;
    info.task = BNND_TASK_LLM;
    info.n_layers = (uint32_t)L;
    info.hidden = (uint32_t)C;
    info.ffn = (uint32_t)FF;
    info.heads = (uint32_t)H;
    info.kv_heads = (uint32_t)Hk;
    info.head_dim = HD;
    info.n_vocab = V;
    info.n_ctx_train = (uint32_t)ctx;
    uint64_t eos = 0;
    info.eos_token = g.get_u64("tokenizer.ggml.eos_token_id", &eos) ? (int32_t)eos : -1;
    {
        const uint32_t world = m->shard.world ? m->shard.world : 1, rank = m->shard.rank;
        const BNND_Status sst = shard_plan(info, world, rank, &m->shard);
        if (sst != BNND_OK)
            return sst;
    }
    const BNND_ShardInfo& sh = m->shard;
    m->eps = eps;
    m->rope_base = base;
    BNND_Status st = rope_params(g, m);
    if (st != BNND_OK)
        return st;
    st = read_f32(g, "output_norm.weight", C, &m->out_norm);
    if (st != BNND_OK)
        return st;
    DeviceLoader ld;
    ld.dev = m->dev;
    {
        Linear* full = sh.world > 1 ? &m->embed : &m->lm_head;
        if ((st = w1_alloc(&ld, (uint32_t)C, V, full)) != BNND_OK ||
            (st = w1_add(&ld, g, "token_embd.weight", (uint32_t)C, V, full, 0, -1)) != BNND_OK)
            return st;
        if (sh.world > 1 &&
            ((st = w1_alloc(&ld, (uint32_t)C, sh.v_rows, &m->lm_head)) != BNND_OK ||
             (st = w1_add(&ld, g, "token_embd.weight", (uint32_t)C, V, &m->lm_head, 0, -1, sh.v_begin, sh.v_rows)) !=
                 BNND_OK))
            return st;
    }
    uint64_t weights = (uint64_t)C * V;
    for (uint32_t l = 0; l < L; ++l) {
        auto layer = std::make_unique<QwenLayer>();
        const std::string p = "blk." + std::to_string(l) + ".";
        if ((st = read_f32(g, p + "attn_norm.weight", C, &layer->attn_norm)) != BNND_OK ||
            (st = read_f32(g, p + "ffn_norm.weight", C, &layer->ffn_norm)) != BNND_OK ||
            (st = read_f32(g, p + "attn_q_norm.weight", HD, &layer->q_norm)) != BNND_OK ||
            (st = read_f32(g, p + "attn_k_norm.weight", HD, &layer->k_norm)) != BNND_OK)
            return st;
        // this rank's rows (all of them for world 1): whole GQA groups of
        // q|k|v, matching gate and up ranges (interleaved by 8-row blocks for
        // the SwiGLU epilogue), o and down output ranges
        const uint32_t Cq = sh.q_rows, Ck = sh.kv_rows;
        if ((st = w1_alloc(&ld, C, Cq + 2 * Ck, &layer->qkv)) != BNND_OK ||
            (st = w1_add(&ld, g, p + "attn_q.weight", C, C, &layer->qkv, 0, -1, sh.q_begin, Cq)) != BNND_OK ||
            (st = w1_add(&ld, g, p + "attn_k.weight", C, KV, &layer->qkv, Cq, -1, sh.kv_begin, Ck)) != BNND_OK ||
            (st = w1_add(&ld, g, p + "attn_v.weight", C, KV, &layer->qkv, Cq + Ck, -1, sh.kv_begin, Ck)) !=
                BNND_OK ||
            (st = w1_alloc(&ld, C, sh.c_rows, &layer->o)) != BNND_OK ||
            (st = w1_add(&ld, g, p + "attn_output.weight", C, C, &layer->o, 0, -1, sh.c_begin, sh.c_rows)) !=
                BNND_OK ||
            (st = w1_alloc(&ld, C, 2 * sh.f_rows, &layer->gu)) != BNND_OK ||
            (st = w1_add(&ld, g, p + "ffn_gate.weight", C, FF, &layer->gu, 0, 0, sh.f_begin, sh.f_rows)) !=
                BNND_OK ||
            (st = w1_add(&ld, g, p + "ffn_up.weight", C, FF, &layer->gu, 0, 1, sh.f_begin, sh.f_rows)) != BNND_OK ||
            (st = w1_alloc(&ld, FF, sh.c_rows, &layer->down)) != BNND_OK ||
            (st = w1_add(&ld, g, p + "ffn_down.weight", FF, C, &layer->down, 0, -1, sh.c_begin, sh.c_rows)) !=
                BNND_OK)
            return st;
        weights += (uint64_t)C * (C + 2 * KV) + (uint64_t)C * C + 3ull * C * FF;
        m->layers.push_back(std::move(layer));
    }
    info.weight_count = weights;
    return BNND_OK;
}

BNND_Status load_mlp(const bnn::GgufFile& g, bnnd_model* m) {
    DeviceLoader ld;
    ld.dev = m->dev;
    uint64_t blocks = 0, in = 0, classes = 0, pixels = 0;
    float stdv = 1.0f;
    g.get_u64("bnn-mlp.block_count", &blocks);
    g.get_u64("bnn-mlp.input_features", &in);
    g.get_u64("bnn-mlp.class_count", &classes);
    g.get_u64("bnn-mlp.input_pixels", &pixels);
    if (!g.get_f32("bnn-mlp.input_std", &stdv))
        stdv = 0.0f;
    // Same checks as bnn_mlp_load (bnn-mlp.c:62-70).
    if (blocks == 0 || blocks > 64 || in == 0 || in > UINT32_MAX || in % 128 != 0 || classes == 0 ||
        classes > UINT32_MAX || (pixels && pixels > in) || !(stdv > 0.0f))
        return fail(BNND_EFORMAT, "unsupported bnn-mlp metadata");
    if (in > bnn::kMaxPrologueK)
        return fail(BNND_ENOTSUP, "bnn-mlp input width above %u is not supported", bnn::kMaxPrologueK);
    uint32_t expected = (uint32_t)in, max_dim = (uint32_t)in;
    uint64_t weights = 0;
    for (uint32_t i = 0; i < blocks; ++i) {
        auto layer = std::make_unique<MlpLayer>();
        const std::string p = "blk." + std::to_string(i) + ".";
        const bnn::GgufTensor* t = g.tensor(p + "weight");
        if (!t || t->dims.size() != 2 || t->dims[0] == 0 || t->dims[1] == 0 || t->dims[0] > UINT32_MAX ||
            t->dims[1] > UINT32_MAX)
            return fail(BNND_EFORMAT, "missing or invalid Q1_0 tensor '%sweight'", p.c_str());
        const uint32_t lin = (uint32_t)t->dims[0], lout = (uint32_t)t->dims[1];
        if (lout > bnn::kMaxPrologueK && i + 1 < blocks)
            return fail(BNND_ENOTSUP, "bnn-mlp hidden width above %u is not supported", bnn::kMaxPrologueK);
        if (lin != expected)
            return fail(BNND_EFORMAT, "layer %u input width %u does not match previous output %u", i, lin,
                        expected);
        if (lin % 128 != 0)
            return fail(BNND_EFORMAT, "unexpected Q1_0 tensor '%sweight' shape or type", p.c_str());
        BNND_Status st = w1_alloc(&ld, lin, lout, &layer->w);
        if (st == BNND_OK)
            st = w1_add(&ld, g, p + "weight", lin, lout, &layer->w, 0, -1);
        if (st == BNND_OK)
            st = read_f32(g, p + "post_scale", lout, &layer->post_scale);
        if (st == BNND_OK)
            st = read_f32(g, p + "post_bias", lout, &layer->post_bias);
        if (st != BNND_OK)
            return st;
        std::string act;
        if (!g.get_str("bnn-mlp.block." + std::to_string(i) + ".activation", &act) || act.empty())
            layer->relu = i + 1 < blocks;
        else if (act == "relu")
            layer->relu = 1;
        else if (act == "none")
            layer->relu = 0;
        else
            return fail(BNND_EFORMAT, "invalid activation for bnn-mlp block %u", i);
        max_dim = std::max(max_dim, lout);
        expected = lout;
        weights += (uint64_t)lin * lout;
        m->mlp.push_back(std::move(layer));
    }
    if (expected != classes)
        return fail(BNND_EFORMAT, "last bnn-mlp layer width %u does not match class_count %u", expected,
                    (uint32_t)classes);
    m->info.task = BNND_TASK_CLASSIFY;
    m->info.input_size = (uint32_t)in;
    m->info.n_classes = (uint32_t)classes;
    m->info.eos_token = -1;
    m->info.weight_count = weights;
    m->mlp_max_dim = max_dim;
    // the layers as the fused classifier kernel reads them
    std::vector<bnn::eng::MlpLayerDev> desc;
    for (const auto& layer : m->mlp) {
        bnn::eng::MlpLayerDev d = {};
        d.wblocks = layer->w.m->wblocks;
        d.post_scale = layer->post_scale.as<float>();
        d.post_bias = layer->post_bias.as<float>();
        d.in = layer->w.in;
        d.out = layer->w.out;
        d.relu = layer->relu;
        desc.push_back(d);
        m->mlp_max_in = std::max(m->mlp_max_in, layer->w.in);
        m->mlp_max_wbytes = std::max(m->mlp_max_wbytes, bnn::eng::mlp_layer_wbytes(layer->w.in, layer->w.out));
    }
    BNND_Status st = dev_alloc(m->mlp_desc, desc.size() * sizeof(desc[0]));
    if (st != BNND_OK)
        return st;
    if (cudaMemcpy(m->mlp_desc.p, desc.data(), desc.size() * sizeof(desc[0]), cudaMemcpyHostToDevice) != cudaSuccess)
        return fail(BNND_EIO, "bnn-mlp layer table upload failed");
    return BNND_OK;
}

// qwen3_init_rope_tables (qwen3.c:298-319), computed on the host with the
// same libm calls so the tables are bit-identical.
void rope_tables(const bnnd_model* m, uint32_t n_ctx, std::vector<float>* cs, std::vector<float>* sn) {
    const uint32_t hd = m->info.head_dim, half = hd / 2;
    cs->resize((size_t)n_ctx * half);
    sn->resize((size_t)n_ctx * half);
    for (uint32_t pos = 0; pos < n_ctx; ++pos) {
        for (uint32_t j = 0; j < half; ++j) {
            const float theta_extrap = (float)pos * powf(m->rope_base, -2.0f * (float)j / (float)hd);
            float theta = m->rope_freq_scale * theta_extrap;
            if (m->rope_yarn) {
                const float span = (float)(m->rope_corr1 - m->rope_corr0);
                const float denom = span > 0.001f ? span : 0.001f;
                const float y = ((float)j - (float)m->rope_corr0) / denom;
                const float ramp = 1.0f - fminf(1.0f, fmaxf(0.0f, y));
                theta = (m->rope_freq_scale * theta_extrap) * (1.0f - ramp) + theta_extrap * ramp;
            }
            (*cs)[(size_t)pos * half + j] = cosf(theta) * m->rope_mscale;
            (*sn)[(size_t)pos * half + j] = sinf(theta) * m->rope_mscale;
        }
    }
}

// One W1A8 linear: FP32 input rows x (stride l.in), RMSNorm gains when the
// plan's prologue normalises, output rows of `out_stride` bytes.

// Attention instantiations: head_dim 64/128 x 1/2/4/8 query heads per KV head.
using AttnFn = void (*)(bnn::eng::AttnArgs);
AttnFn attention_fn(uint32_t hd, uint32_t kv_mul, bool sc_smem) {
    using namespace bnn::eng;
#define BNN_ATTN_CASE(H, Q) \
    if (hd == H && kv_mul == Q)  \
        return sc_smem ? attention_kernel<H, Q, true> : attention_kernel<H, Q, false>;
    BNN_ATTN_CASE(128, 1) BNN_ATTN_CASE(128, 2) BNN_ATTN_CASE(128, 4) BNN_ATTN_CASE(128, 8)
    BNN_ATTN_CASE(64, 1) BNN_ATTN_CASE(64, 2) BNN_ATTN_CASE(64, 4) BNN_ATTN_CASE(64, 8)
#undef BNN_ATTN_CASE
    return nullptr;
}

// The attention kernel, launched like the linears (programmatic dependent
// launch: it streams K/V tiles of earlier steps while the q|k|v projection
// finishes).
// A one-argument kernel on the context's stream, with programmatic dependent
// launch when the context uses it (the kernel waits for its predecessor
// before it reads what earlier kernels wrote).
template <typename Arg>
cudaError_t launch_on(const bnnd_context* c, void (*fn)(Arg), dim3 grid, dim3 block, size_t smem, const Arg& arg) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = c->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = c->pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, fn, arg);
}

cudaError_t launch_attention(bnnd_context* c, const bnn::eng::AttnArgs& a) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.kv_heads, c->rows);
    cfg.blockDim = dim3(bnn::eng::kAttnThreads);
    cfg.dynamicSmemBytes = c->attn_smem;
    cfg.stream = c->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = c->pdl ? 1 : 0;
    const AttnFn fn = attention_fn(a.hd, a.heads / a.kv_heads, a.scores == nullptr);
    return fn ? cudaLaunchKernelEx(&cfg, fn, a) : cudaErrorInvalidValue;
}
cudaError_t launch_linear(const bnnd_context* c, const bnn::GemvLaunch& cl, const Linear& l, const float* x,
                          const float* gain, uint32_t rows, float* out, size_t out_stride, int* status,
                          unsigned long long* best = nullptr, uint32_t index_base = 0, const float* res = nullptr,
                          size_t res_stride = 0) {
    bnn::GemvArgs a = {};
    a.wblocks = l.m->wblocks;
    a.n = l.out;
    a.groups = l.in / 128;
    a.m = rows;
    a.tiles = cl.tiles;
    a.stages = cl.stages;
    a.blocks_per_tile = cl.blocks_per_tile;
    a.x = x;
    a.x_stride = l.in;
    a.gain = gain;
    a.eps = c->model->eps;
    a.exact = c->params.exact;
    a.out = reinterpret_cast<unsigned char*>(out);
    a.out_stride = out_stride;
    a.status = status;
    a.best = best;
    a.index_base = index_base;
    a.res = reinterpret_cast<const unsigned char*>(res);
    a.res_stride = res_stride;
    g_next_bytes = ((double)l.out * l.in * 0.140625 + 4.0 * l.in + 4.0 * l.out) * rows;
    return bnn::launch_gemv(cl, rows, a, c->stream, c->pdl);
}

// All-gather of the rank-major buffer st ([world][rows][slice]; this rank's
// part written in place) and its reordering into dst [rows][width].
cudaError_t all_gather_rows(bnnd_context* c, float* st, uint32_t slice, float* dst, uint32_t width) {
    const uint32_t R = c->rows;
    const size_t count = (size_t)R * slice;
    if (ncclAllGather(st + (size_t)c->rank * count, st, count, ncclFloat32, c->comm, c->stream) != ncclSuccess)
        return cudaErrorUnknown;
    const size_t total = (size_t)R * width;
    const uint32_t blocks = (uint32_t)std::min<size_t>((total + 255) / 256, 1024);
    bnn::eng::gather_rows_kernel<<<blocks, 256, 0, c->stream>>>(st, dst, c->world, R, slice, width, width);
    return cudaGetLastError();
}

// RMSNorm (gain non-null) or plain quantisation of `rows` rows of width k
// into the pre-tiled tensor-core operand.
cudaError_t prefill_prep(bnnd_context* c, unsigned char* a_sw, float* rs, const float* x, uint32_t k, const float* gain,
                         uint32_t rows) {
    bnn::eng::RowsPrepArgs a = {};
    a.x = x;
    a.x_stride = k;
    a.gain = gain;
    a.eps = c->model->eps;
    a.exact = c->params.exact;
    a.k = k;
    a.m = rows;
    a.a_sw = a_sw;
    a.row_scale = rs;
    a.status = c->status.as<int>();
    a.early_next = c->pdl ? 1 : 0;
    const size_t smem = bnn::eng::rows_prep_smem(k, c->params.exact != 0);
    cudaError_t e = cudaFuncSetAttribute(bnn::eng::rows_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess)
        return e;
    return launch_on(c, bnn::eng::rows_prep_kernel, dim3(rows), dim3(bnn::eng::kRowsPrepThreads), smem, a);
}

// The linear l over the prepared rows on the tensor cores; epi kEpiView,
// kEpiResidual (out += Y) or kEpiSwiGLU.
cudaError_t prefill_linear(bnnd_context* c, const unsigned char* a_sw, const float* rs, const Linear& l, uint32_t rows,
                           float* out, size_t out_stride, int epi) {
    bnn::MmaArgs a = {};
    a.wblocks = l.m->wblocks;
    a.n = l.out;
    a.groups = l.in / 128;
    a.m = rows;
    a.a_sw = a_sw;
    a.row_scale = rs;
    a.out = reinterpret_cast<unsigned char*>(out);
    a.out_stride = out_stride;
    a.epi = epi;
    a.status = c->status.as<int>();
    g_next_bytes = (double)l.out * l.in * 0.140625 + (double)rows * (l.in + 4.0 * l.out);
    return bnn::launch_mma(a, c->model->dev->sm_count, c->stream, c->pdl);
}

// Multi-row steps: RMSNorm (gain non-null) + QuantizeRow of every row in its
// own CTA, written in the contraction's sliced layout.
cudaError_t step_prep(bnnd_context* c, const float* x, uint32_t k, const float* gain, uint32_t rows) {
    bnn::eng::RowsPrepArgs a = {};
    a.x = x;
    a.x_stride = k;
    a.gain = gain;
    a.eps = c->model->eps;
    a.exact = c->params.exact;
    a.k = k;
    a.m = rows;
    a.act = c->dm_act.as<uint32_t>();
    a.totals = c->dm_tot.as<int32_t>();
    a.row_scale = c->dm_rs.as<float>();
    a.status = c->status.as<int>();
    const size_t smem = bnn::eng::rows_prep_smem(k, c->params.exact != 0);
    cudaError_t e = cudaFuncSetAttribute(bnn::eng::rows_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess)
        return e;
    // a plain launch that lets no successor start early: in the multi-row
    // step graph an overlapped row preparation measured slower (4.2 vs 4.4 K
    // tokens/s at 8 rows)
    bnn::eng::rows_prep_kernel<<<rows, bnn::eng::kRowsPrepThreads, smem, c->stream>>>(a);
    return cudaGetLastError();
}

// The contraction over the rows step_prep prepared (kProSliced prologue).
cudaError_t step_linear(const bnnd_context* c, const bnn::GemvLaunch& cl, const Linear& l, uint32_t rows, float* out,
                        size_t out_stride, unsigned long long* best = nullptr, uint32_t index_base = 0,
                        const float* res = nullptr, size_t res_stride = 0) {
    bnn::GemvArgs a = {};
    a.wblocks = l.m->wblocks;
    a.n = l.out;
    a.groups = l.in / 128;
    a.m = rows;
    a.tiles = cl.tiles;
    a.stages = cl.stages;
    a.blocks_per_tile = cl.blocks_per_tile;
    a.act = c->dm_act.as<uint32_t>();
    a.totals = c->dm_tot.as<int32_t>();
    a.row_scale = c->dm_rs.as<float>();
    a.out = reinterpret_cast<unsigned char*>(out);
    a.out_stride = out_stride;
    a.status = c->status.as<int>();
    a.best = best;
    a.index_base = index_base;
    a.res = reinterpret_cast<const unsigned char*>(res);
    a.res_stride = res_stride;
    g_next_bytes = ((double)l.out * l.in * 0.140625 + 4.0 * l.in + 4.0 * l.out) * rows;
    return bnn::launch_gemv(cl, rows, a, c->stream, c->pdl);
}

// Enqueues one decode step for every row (tokens already in tok_in).
cudaError_t enqueue_step(bnnd_context* c, bool with_logits) {
    LaunchCheck local;
    LaunchCheck& ck = g_check ? *g_check : local;
    const bnnd_model* m = c->model;
    const BNND_ModelInfo& in = m->info;
    const BNND_ShardInfo& sh = m->shard;
    const bool tp = c->world > 1;
    const uint32_t C = in.hidden, F = in.ffn, HD = in.head_dim, R = c->rows;
    cudaStream_t s = c->stream;
    int* status = c->status.as<int>();
    const int exact = c->params.exact;
    unsigned long long* best = c->best.as<unsigned long long>() + (size_t)c->rank * R;
    float* x = c->x.as<float>();
    bnn::eng::embed_kernel<<<R, 256, 0, s>>>(c->tok_in.as<int32_t>(), (tp ? m->embed : m->lm_head).m->wblocks, C, x,
                                             best);
    ck("embed_kernel");
    const uint32_t qkv_width = sh.q_rows + 2 * sh.kv_rows;
    // Steps of several context rows (one GPU) prepare every row in its own
    // CTA (the RMSNorm sums in parallel) and hand the contraction sliced rows,
    // instead of a contraction whose every CTA prepares the rows one after
    // another. Same arithmetic either way.
    const bool rows_prepped = c->dm_act.p != nullptr;
    // One linear: row prep + sliced contraction, or the contraction with the
    // RMSNorm/quantise prologue in every CTA.
    auto lin = [&](const char* prep_name, const char* name, const bnn::GemvLaunch& plan,
                   const bnn::GemvLaunch& plan_s, const Linear& l, const float* xin, uint32_t k, const float* gain,
                   float* out, size_t out_stride, unsigned long long* bst = nullptr, uint32_t ib = 0,
                   const float* res = nullptr, size_t res_stride = 0) {
        if (rows_prepped) {
            ck(prep_name, step_prep(c, xin, k, gain, R));
            ck(name, step_linear(c, plan_s, l, R, out, out_stride, bst, ib, res, res_stride));
        } else {
            ck(name, launch_linear(c, plan, l, xin, gain, R, out, out_stride, status, bst, ib, res, res_stride));
        }
    };
    for (uint32_t l = 0; l < in.n_layers; ++l) {
        const QwenLayer& L = *m->layers[l];
        // attn_norm + q|k|v projections of this rank's heads (prologue: RMSNorm + quantise)
        lin("rows_prep:qkv", "w1a8_gemv:qkv", c->plan_qkv, c->plan_qkv_s, L.qkv, x, C, L.attn_norm.as<float>(),
            c->qkv.as<float>(), (size_t)qkv_width * 4u);
        // q/k norm + rope + KV append + attention, one block per (KV head, row)
        bnn::eng::AttnArgs aa = {};
        aa.qkv = c->qkv.as<float>();
        aa.q_norm = L.q_norm.as<float>();
        aa.k_norm = L.k_norm.as<float>();
        aa.rope_cos = c->rope_cos.as<float>();
        aa.rope_sin = c->rope_sin.as<float>();
        aa.pos = c->pos_d.as<uint32_t>();
        const size_t layer_cache = (size_t)R * c->n_ctx * sh.kv_rows;
        aa.kcache = c->kcache.as<float>() + (size_t)l * (layer_cache / HD * bnn::eng::kcache_row(HD));
        aa.vcache = c->vcache.as<float>() + (size_t)l * layer_cache;
        aa.scores = c->scores.p ? c->scores.as<float>() : nullptr;
        aa.y = tp ? c->y_st.as<float>() + (size_t)c->rank * R * sh.q_rows : c->y.as<float>();
        aa.y_stride = tp ? sh.q_rows : C;
        aa.c = sh.q_rows;
        aa.kv = sh.kv_rows;
        aa.hd = HD;
        aa.heads = in.heads / c->world;
        aa.kv_heads = in.kv_heads / c->world;
        aa.n_ctx = c->n_ctx;
        aa.eps = m->eps;
        aa.scale = 1.0f / sqrtf((float)HD);
        aa.exact = exact;
        aa.status = status;
        aa.resident_max = c->attn_resident;
        ck("attention_kernel", launch_attention(c, aa));
        if (tp)
            ck("all_gather:y", all_gather_rows(c, c->y_st.as<float>(), sh.q_rows, c->y.as<float>(), C));
        // attn_output, x += o (prologue: quantise the attention output)
        if (tp) {
            float* xs = c->x_st.as<float>() + (size_t)c->rank * R * sh.c_rows;
            lin("rows_prep:o", "w1a8_gemv:o", c->plan_o, c->plan_o_s, L.o, c->y.as<float>(), C, nullptr, xs,
                (size_t)sh.c_rows * 4u, nullptr, 0, x + sh.c_begin, (size_t)C * 4u);
            ck("all_gather:x", all_gather_rows(c, c->x_st.as<float>(), sh.c_rows, x, C));
        } else {
            lin("rows_prep:o", "w1a8_gemv:o", c->plan_o, c->plan_o_s, L.o, c->y.as<float>(), C, nullptr, x,
                (size_t)C * 4u);
        }
        // ffn_norm + gate|up + SwiGLU -> h
        if (tp) {
            lin("rows_prep:gate_up", "w1a8_gemv:gate_up", c->plan_gu, c->plan_gu_s, L.gu, x, C,
                L.ffn_norm.as<float>(), c->h_st.as<float>() + (size_t)c->rank * R * sh.f_rows, (size_t)sh.f_rows * 4u);
            ck("all_gather:h", all_gather_rows(c, c->h_st.as<float>(), sh.f_rows, c->h.as<float>(), F));
        } else {
            lin("rows_prep:gate_up", "w1a8_gemv:gate_up", c->plan_gu, c->plan_gu_s, L.gu, x, C,
                L.ffn_norm.as<float>(), c->h.as<float>(), (size_t)F * 4u);
        }
        // ffn_down, x += d (prologue: quantise h)
        if (tp) {
            float* xs = c->x_st.as<float>() + (size_t)c->rank * R * sh.c_rows;
            lin("rows_prep:down", "w1a8_gemv:down", c->plan_down, c->plan_down_s, L.down, c->h.as<float>(), F, nullptr,
                xs, (size_t)sh.c_rows * 4u, nullptr, 0, x + sh.c_begin, (size_t)C * 4u);
            ck("all_gather:x", all_gather_rows(c, c->x_st.as<float>(), sh.c_rows, x, C));
        } else {
            lin("rows_prep:down", "w1a8_gemv:down", c->plan_down, c->plan_down_s, L.down, c->h.as<float>(), F, nullptr,
                x, (size_t)C * 4u);
        }
    }
    if (with_logits) {
        // out_norm + lm_head; the epilogue also takes the greedy pick
        if (tp) {
            lin("rows_prep:lm_head", "w1a8_gemv:lm_head", c->plan_head, c->plan_head_s, m->lm_head, x, C,
                m->out_norm.as<float>(), c->lg_st.as<float>() + (size_t)c->rank * R * sh.v_stride,
                (size_t)sh.v_stride * 4u, best, sh.v_begin);
            ck("all_gather:logits",
               all_gather_rows(c, c->lg_st.as<float>(), sh.v_stride, c->logits.as<float>(), in.n_vocab));
            ck("all_gather:pick", ncclAllGather(best, c->best.p, R, ncclUint64, c->comm, s) == ncclSuccess
                                      ? cudaSuccess
                                      : cudaErrorUnknown);
        } else {
            lin("rows_prep:lm_head", "w1a8_gemv:lm_head", c->plan_head, c->plan_head_s, m->lm_head, x, C,
                m->out_norm.as<float>(), c->logits.as<float>(), (size_t)in.n_vocab * 4u, best);
        }
    }
    bnn::eng::step_end_kernel<<<1, 32 * ((R + 31) / 32), 0, s>>>(
        R, c->pos_d.as<uint32_t>(), c->tok_in.as<int32_t>(), c->tok_next.as<int32_t>(),
        c->best.as<unsigned long long>(), c->world, c->hist.as<int32_t>(), c->hist_count.as<uint32_t>(),
        c->hist_cap, with_logits ? 1 : 0);
    ck("step_end_kernel");
    const cudaError_t tail = cudaGetLastError();
    if (tail != cudaSuccess && ck.err == cudaSuccess)
        ck.err = tail;
    if (with_logits)
        c->step_launches = ck.launches;
    return ck.err;
}

BNND_Status capture_step(bnnd_context* c, bool with_logits, cudaGraphExec_t* out) {
    cudaGraph_t graph = nullptr;
    CUDA_OR(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal), BNND_EIO);
    LaunchCheck ck;
    g_check = &ck;
    if (g_rec)
        cudaEventRecordWithFlags(g_rec->events[0], c->stream, cudaEventRecordExternal);
    cudaError_t e = enqueue_step(c, with_logits);
    g_check = nullptr;
    cudaError_t e2 = cudaStreamEndCapture(c->stream, &graph);
    if (e != cudaSuccess || e2 != cudaSuccess) {
        if (graph)
            cudaGraphDestroy(graph);
        cudaGetLastError();
        return fail(BNND_EIO, "decode step capture failed at %s: %s", ck.what ? ck.what : "end",
                    cudaGetErrorString(e != cudaSuccess ? e : e2));
    }
    e = cudaGraphInstantiate(out, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(BNND_EIO, "decode graph instantiation failed: %s", cudaGetErrorString(e));
    }
    return BNND_OK;
}

// One cooperative launch of the step kernel (one CTA per SM) on the context's stream.
cudaError_t launch_step_kernel(bnnd_context* c, const bnn::step::StepArgs& a) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_attn + a.n_gemv);
    cfg.blockDim = dim3(bnn::step::kThreads);
    cfg.dynamicSmemBytes = bnn::step::kSmemBudget;
    cfg.stream = c->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, bnn::step::decode_step_kernel, a);
}

// The persistent step kernel for one-row, single-GPU, exact-mode contexts
// with 128-wide heads (decode_step.cuh). Leaves c->graph_step null, and the
// per-kernel step graph in charge, when the shape or the device does not
// allow it or BNN_STEP_KERNEL=0; failures here are not errors.
void setup_step_kernel(bnnd_context* c) {
    namespace st = bnn::step;
    const bnnd_model* m = c->model;
    const BNND_ModelInfo& in = m->info;
    const char* env = std::getenv("BNN_STEP_KERNEL");
    if (env && env[0] == '0')
        return;
    const bool say = std::getenv("BNN_STEP_KERNEL_DEBUG") != nullptr;
    auto why = [&](const char* what) {
        if (say)
            std::fprintf(stderr, "step kernel off: %s (%s)\n", what, cudaGetErrorString(cudaGetLastError()));
        cudaGetLastError();
    };
    const int sms = m->dev->sm_count;
    int coop = 0;
    if (c->rows != 1 || c->world != 1 || !c->params.exact || in.head_dim != st::kHD || in.hidden % 128 ||
        in.ffn % 128 || in.heads % in.kv_heads || (int)in.heads + 1 >= sms ||
        (in.hidden / 8 + (sms - in.heads) - 1) / (sms - in.heads) * 8 > st::kOwnRowsMax ||
        in.hidden > 16384 || in.ffn > 16384 ||
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, m->dev->ordinal) != cudaSuccess || !coop) {
        why("shape or device");
        return;
    }
    const uint32_t C = in.hidden, F = in.ffn, L = in.n_layers, HD = in.head_dim;
    const uint32_t n_attn = in.heads, n_gemv = (uint32_t)sms - n_attn;
    const uint32_t qkv_rows = C + 2 * in.kv_heads * HD;
    const uint32_t GC = C / 128, GF = F / 128;
    auto ceil_div = [](uint32_t a, uint32_t b) { return (a + b - 1) / b; };
    // the integer-D buffer holds the largest copy's blocks x 8 rows x groups
    const uint32_t nb_v = ceil_div(in.n_vocab, 8);
    uint32_t dsm_units = std::max({ceil_div(qkv_rows / 8, n_gemv) * GC, ceil_div(C / 8, n_gemv) * GF,
                                   2 * ceil_div(F / 8, n_gemv) * GC,
                                   std::min(st::kLmChunkBlocks, ceil_div(nb_v, n_gemv)) * GC});
    const uint32_t dsm_bytes = dsm_units * 8u * 2u;
    const st::GemvPlan gp = st::gemv_plan(C, F, dsm_bytes);
    if (gp.ring >= st::kSmemBudget) {
        why("shared memory");
        return;
    }
    const uint32_t ring = (uint32_t)((st::kSmemBudget - gp.ring) & ~(size_t)127);
    st::ScheduleShape shape{L, C, F, qkv_rows, in.n_vocab, n_gemv, ring};
    std::vector<st::LayerSrc> srcs(L);
    for (uint32_t l = 0; l < L; ++l) {
        const QwenLayer& Q = *m->layers[l];
        srcs[l] = st::LayerSrc{(uint64_t)(uintptr_t)Q.qkv.m->wblocks, (uint64_t)(uintptr_t)Q.o.m->wblocks,
                               (uint64_t)(uintptr_t)Q.gu.m->wblocks, (uint64_t)(uintptr_t)Q.down.m->wblocks,
                               (uint64_t)(uintptr_t)Q.attn_norm.p, (uint64_t)(uintptr_t)Q.ffn_norm.p};
    }
    std::vector<std::vector<st::Copy>> scheds(n_gemv);
    uint32_t stride = 1;
    for (uint32_t j = 0; j < n_gemv; ++j) {
        if (!st::build_schedule(shape, srcs, (uint64_t)(uintptr_t)m->lm_head.m->wblocks,
                                (uint64_t)(uintptr_t)m->out_norm.p, j, &scheds[j])) {
            why("schedule");
            return;
        }
        stride = std::max<uint32_t>(stride, (uint32_t)scheds[j].size());
    }
    if (stride > st::kSchedMax) {
        why("too many copies per step");
        return;
    }
    std::vector<st::Copy> flat((size_t)n_gemv * stride);
    std::vector<uint32_t> lens(n_gemv);
    for (uint32_t j = 0; j < n_gemv; ++j) {
        std::copy(scheds[j].begin(), scheds[j].end(), flat.begin() + (size_t)j * stride);
        lens[j] = (uint32_t)scheds[j].size();
    }
    const BNND_ShardInfo& sh = m->shard;
    const size_t layer_cache = (size_t)c->n_ctx * sh.kv_rows;
    std::vector<st::LayerPtrs> lp(L);
    for (uint32_t l = 0; l < L; ++l) {
        const QwenLayer& Q = *m->layers[l];
        lp[l] = st::LayerPtrs{Q.q_norm.as<float>(), Q.k_norm.as<float>(),
                              c->kcache.as<float>() + (size_t)l * (layer_cache / HD * bnn::eng::kcache_row(HD)),
                              c->vcache.as<float>() + (size_t)l * layer_cache};
    }
    const uint32_t sync_init[2] = {0u, 1u};  // exit ticket, step generation
    if (L > st::kMaxStepLayers) {
        why("too many layers");
        return;
    }
    // hand-off rows as (value, generation) pairs, cleared to a generation no step stamps
    if (dev_alloc(c->st_xt, (size_t)C * 8) || dev_alloc(c->st_qkvt, (size_t)qkv_rows * 8) ||
        dev_alloc(c->st_yt, (size_t)C * 8) || dev_alloc(c->st_ht, (size_t)F * 8) ||
        cudaMemset(c->st_xt.p, 0xff, (size_t)C * 8) != cudaSuccess ||
        cudaMemset(c->st_qkvt.p, 0xff, (size_t)qkv_rows * 8) != cudaSuccess ||
        cudaMemset(c->st_yt.p, 0xff, (size_t)C * 8) != cudaSuccess ||
        cudaMemset(c->st_ht.p, 0xff, (size_t)F * 8) != cudaSuccess) {
        why("allocation");
        g_last_error.clear();
        return;
    }
    if (dev_alloc(c->st_sync, sizeof sync_init) || dev_alloc(c->st_sched, flat.size() * sizeof(st::Copy)) ||
        dev_alloc(c->st_sched_len, lens.size() * 4) || dev_alloc(c->st_layers, lp.size() * sizeof(st::LayerPtrs)) ||
        cudaMemcpy(c->st_sync.p, sync_init, sizeof sync_init, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(c->best.p, 0, 8) != cudaSuccess ||
        cudaMemcpy(c->st_sched.p, flat.data(), flat.size() * sizeof(st::Copy), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(c->st_sched_len.p, lens.data(), lens.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(c->st_layers.p, lp.data(), lp.size() * sizeof(st::LayerPtrs), cudaMemcpyHostToDevice) !=
            cudaSuccess) {
        why("allocation");
        g_last_error.clear();
        return;
    }
    st::StepArgs& a = c->st_args;
    a.layers = c->st_layers.as<st::LayerPtrs>();
    a.n_layers = L;
    a.C = C;
    a.F = F;
    a.V = in.n_vocab;
    a.qkv_rows = qkv_rows;
    a.heads = in.heads;
    a.kv_heads = in.kv_heads;
    a.n_ctx = c->n_ctx;
    a.n_attn = n_attn;
    a.n_gemv = n_gemv;
    a.sched = c->st_sched.as<st::Copy>();
    a.sched_len = c->st_sched_len.as<uint32_t>();
    a.sched_stride = stride;
    a.ring_bytes = ring;
    a.dsm_bytes = dsm_bytes;
    a.kv_resident = std::min<uint32_t>(st::attn_resident_max(), c->n_ctx);
    a.lm_head = m->lm_head.m->wblocks;
    a.tok_in = c->tok_in.as<int32_t>();
    a.pos = c->pos_d.as<uint32_t>();
    a.tok_next = c->tok_next.as<int32_t>();
    a.hist = c->hist.as<int32_t>();
    a.hist_count = c->hist_count.as<uint32_t>();
    a.hist_cap = c->hist_cap;
    a.logits = c->logits.as<float>();
    a.best = c->best.as<unsigned long long>();
    a.rope_cos = c->rope_cos.as<float>();
    a.rope_sin = c->rope_sin.as<float>();
    a.sync = c->st_sync.as<uint32_t>();
    a.epoch = c->st_sync.as<uint32_t>() + 1;
    a.xt = c->st_xt.as<unsigned long long>();
    a.qkvt = c->st_qkvt.as<unsigned long long>();
    a.yt = c->st_yt.as<unsigned long long>();
    a.ht = c->st_ht.as<unsigned long long>();
    a.status = c->status.as<int>();
    a.eps = m->eps;
    a.scale = 1.0f / sqrtf((float)HD);
    const char* pn = std::getenv("BNN_STEP_POLL_NS");
    a.poll_ns = pn ? (uint32_t)std::strtoul(pn, nullptr, 10) : 4u;  // measured: shorter pauses are faster (8 vs 512 ns: 1186 vs 929 tok/s)
    int occ = 0;
    if (cudaFuncSetAttribute(st::decode_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)st::kSmemBudget) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, st::decode_step_kernel, st::kThreads, st::kSmemBudget) !=
            cudaSuccess ||
        occ < 1) {
        why("occupancy");
        return;
    }
    // one cooperative launch per step, captured once; where capturing it is
    // refused (some profilers), the kernel is launched directly instead
    c->st_positions = a.kv_resident;
    cudaGraph_t graph = nullptr;
    if (cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        why("capture");
        return;
    }
    const cudaError_t e1 = launch_step_kernel(c, a);
    const cudaError_t e2 = cudaStreamEndCapture(c->stream, &graph);
    cudaGraphExec_t exec = nullptr;
    const cudaError_t e3 = (e1 == cudaSuccess && e2 == cudaSuccess) ? cudaGraphInstantiate(&exec, graph, 0) : e1;
    if (graph)
        cudaGraphDestroy(graph);
    if (e1 != cudaSuccess || e2 != cudaSuccess || e3 != cudaSuccess)
        why("graph (direct launches instead)");
    else
        c->graph_step = exec;
    if (say)
        std::fprintf(stderr, "step kernel on below position %u (%s)\n", c->st_positions,
                     c->graph_step ? "graph" : "direct launches");
}

// Enqueues the decode step at position `pos` (with logits and the greedy
// pick when want): the persistent step kernel while the K/V history fits
// it, else the per-kernel step graph.
cudaError_t run_step(bnnd_context* c, uint32_t pos, bool want) {
    if (!want)
        return cudaGraphLaunch(c->graph_prefill, c->stream);
    if (c->st_positions && pos < c->st_positions)
        return c->graph_step ? cudaGraphLaunch(c->graph_step, c->stream) : launch_step_kernel(c, c->st_args);
    return cudaGraphLaunch(c->graph_logits, c->stream);
}

BNND_Status create_llm_context(bnnd_context* c) {
    const bnnd_model* m = c->model;
    const BNND_ModelInfo& in = m->info;
    const BNND_ShardInfo& sh = m->shard;
    const uint32_t C = in.hidden, F = in.ffn, R = c->rows;
    BNND_Status st;
    c->world = sh.world;
    c->rank = sh.rank;
    if (c->world > 1) {
        // collective over the ranks: every rank creates its context
        if (!c->params.comm_id)
            return fail(BNND_EINVAL, "a sharded model needs comm_id in the context parameters");
        ncclUniqueId id;
        std::memcpy(&id, c->params.comm_id, sizeof id);
        const ncclResult_t r = ncclCommInitRank(&c->comm, (int)c->world, id, (int)c->rank);
        if (r != ncclSuccess) {
            c->comm = nullptr;
            return fail(BNND_EIO, "ncclCommInitRank: %s", ncclGetErrorString(r));
        }
    }
    const uint32_t P = c->world;
    // V: [layers][rows][kv heads][n_ctx][HD]; K the same with kcache_row(HD) floats a position
    const size_t cache = (size_t)in.n_layers * R * c->n_ctx * sh.kv_rows * 4u;
    const size_t kcache = cache / in.head_dim * bnn::eng::kcache_row(in.head_dim);
    if ((st = dev_alloc(c->x, (size_t)R * C * 4)) ||
        (st = dev_alloc(c->qkv, (size_t)R * (sh.q_rows + 2 * sh.kv_rows) * 4)) ||
        (st = dev_alloc(c->y, (size_t)R * C * 4)) || (st = dev_alloc(c->h, (size_t)R * F * 4)) ||
        (st = dev_alloc(c->logits, (size_t)R * in.n_vocab * 4)) || (st = dev_alloc(c->kcache, kcache)) ||
        (st = dev_alloc(c->vcache, cache)) || (st = dev_alloc(c->pos_d, (size_t)R * 4)) ||
        (st = dev_alloc(c->tok_in, (size_t)R * 4)) || (st = dev_alloc(c->tok_next, (size_t)R * 4)) ||
        (st = dev_alloc(c->hist_count, 4)) || (st = dev_alloc(c->status, 4)) ||
        (st = dev_alloc(c->best, (size_t)P * R * 8)))
        return st;
    if (P > 1 && ((st = dev_alloc(c->y_st, (size_t)P * R * sh.q_rows * 4)) ||
                  (st = dev_alloc(c->x_st, (size_t)P * R * sh.c_rows * 4)) ||
                  (st = dev_alloc(c->h_st, (size_t)P * R * sh.f_rows * 4)) ||
                  (st = dev_alloc(c->lg_st, (size_t)P * R * sh.v_stride * 4))))
        return st;
    c->hist_cap = c->n_ctx;
    if ((st = dev_alloc(c->hist, (size_t)c->hist_cap * R * 4)))
        return st;
    std::vector<float> cs, sn;
    rope_tables(m, c->n_ctx, &cs, &sn);
    if ((st = dev_alloc(c->rope_cos, cs.size() * 4)) || (st = dev_alloc(c->rope_sin, sn.size() * 4)))
        return st;
    CUDA_OR(cudaMemcpy(c->rope_cos.p, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice), BNND_EIO);
    CUDA_OR(cudaMemcpy(c->rope_sin.p, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice), BNND_EIO);
    CUDA_OR(cudaMemset(c->pos_d.p, 0, (size_t)R * 4), BNND_EIO);
    CUDA_OR(cudaMemset(c->tok_in.p, 0, (size_t)R * 4), BNND_EIO);
    CUDA_OR(cudaMemset(c->hist_count.p, 0, 4), BNND_EIO);
    CUDA_OR(cudaMemset(c->status.p, 0, 4), BNND_EIO);
    const int sms = m->dev->sm_count;
    if (R >= kStepRowsPrep) {
        const uint32_t gmax = std::max(C, F) / 128;
        if ((st = dev_alloc(c->dm_act, (size_t)R * gmax * bnn::kWordsPerGroup * 4)) ||
            (st = dev_alloc(c->dm_tot, (size_t)R * gmax * 4)) || (st = dev_alloc(c->dm_rs, (size_t)R * 4)))
            return st;
        c->plan_qkv_s = bnn::plan_gemv(m->dev->sm_count, sh.q_rows + 2 * sh.kv_rows, C / 128, R, bnn::kProSliced,
                                       bnn::kEpiView);
        c->plan_o_s = bnn::plan_gemv(m->dev->sm_count, sh.c_rows, C / 128, R, bnn::kProSliced, bnn::kEpiResidual);
        c->plan_gu_s = bnn::plan_gemv(m->dev->sm_count, 2 * sh.f_rows, C / 128, R, bnn::kProSliced, bnn::kEpiSwiGLU);
        c->plan_down_s = bnn::plan_gemv(m->dev->sm_count, sh.c_rows, F / 128, R, bnn::kProSliced, bnn::kEpiResidual);
        c->plan_head_s = bnn::plan_gemv(m->dev->sm_count, sh.v_rows, C / 128, R, bnn::kProSliced, bnn::kEpiView);
    }
    c->plan_qkv = bnn::plan_gemv(sms, sh.q_rows + 2 * sh.kv_rows, C / 128, R, bnn::kProRmsNorm, bnn::kEpiView);
    c->plan_o = bnn::plan_gemv(sms, sh.c_rows, C / 128, R, bnn::kProQuant, bnn::kEpiResidual);
    c->plan_gu = bnn::plan_gemv(sms, 2 * sh.f_rows, C / 128, R, bnn::kProRmsNorm, bnn::kEpiSwiGLU);
    c->plan_down = bnn::plan_gemv(sms, sh.c_rows, F / 128, R, bnn::kProQuant, bnn::kEpiResidual);
    c->plan_head = bnn::plan_gemv(sms, sh.v_rows, C / 128, R, bnn::kProRmsNorm, bnn::kEpiView);
    for (const bnn::GemvLaunch* p : {&c->plan_qkv, &c->plan_o, &c->plan_gu, &c->plan_down, &c->plan_head})
        if (p->smem > bnn::kGemvSmemBudget)
            return fail(BNND_ENOTSUP, "hidden/ffn width too large for the contraction kernel");
    const uint32_t kv_mul = in.heads / in.kv_heads;
    if (attention_fn(in.head_dim, kv_mul, true) == nullptr)
        return fail(BNND_ENOTSUP, "attention shape (head_dim %u, %u query heads per KV head) not supported",
                    in.head_dim, kv_mul);
    // scores of a block's query heads in shared memory when they fit, else in
    // a device scratch [rows][heads][n_ctx]
    bnn::eng::AttnSmem ap = bnn::eng::attn_smem_plan(in.head_dim, kv_mul, c->n_ctx, true);
    if (ap.total > kAttnSmemBudget) {
        ap = bnn::eng::attn_smem_plan(in.head_dim, kv_mul, c->n_ctx, false);
        if ((st = dev_alloc(c->scores, (size_t)R * in.heads * bnn::eng::attn_sc_stride(c->n_ctx) * 4)))
            return st;
    }
    // past the ring, the rest of the budget holds whole K/V histories of up to
    // attn_resident positions (the kernel's tile-free path)
    c->attn_resident = std::min<uint32_t>(bnn::eng::attn_resident_rows(in.head_dim, kAttnSmemBudget - ap.ring),
                                          c->n_ctx);
    c->attn_smem = c->attn_resident > 0 ? kAttnSmemBudget : ap.total;
    CUDA_OR(cudaFuncSetAttribute(attention_fn(in.head_dim, kv_mul, c->scores.p == nullptr),
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kAttnSmemBudget),
            BNND_EIO);
    if ((st = capture_step(c, true, &c->graph_logits)) || (st = capture_step(c, false, &c->graph_prefill)))
        return st;
    setup_step_kernel(c);
    return BNND_OK;
}

BNND_Status create_mlp_context(bnnd_context* c) {
    const bnnd_model* m = c->model;
    const uint32_t R = c->rows, D = m->mlp_max_dim;
    BNND_Status st;
    if ((st = dev_alloc(c->mlp_a, (size_t)R * D * 4)) || (st = dev_alloc(c->mlp_b, (size_t)R * D * 4)) ||
        (st = dev_alloc(c->status, 4)))
        return st;
    CUDA_OR(cudaMemset(c->status.p, 0, 4), BNND_EIO);
    if (R >= bnn::kMmaMinRows &&
        ((st = dev_alloc(c->mlp_asw, bnn::mma_a_bytes(R, D / 128))) || (st = dev_alloc(c->mlp_rs, (size_t)R * 4))))
        return st;
    for (const auto& l : m->mlp) {
        c->plan_mlp.push_back(
            bnn::plan_gemv(m->dev->sm_count, l->w.out, l->w.in / 128, R, bnn::kProQuant, bnn::kEpiView));
        if (c->plan_mlp.back().smem > bnn::kGemvSmemBudget)
            return fail(BNND_ENOTSUP, "layer width too large for the contraction kernel");
    }
    // calls of up to kMlpFusedMaxSamples samples: one fused launch, pinned staging
    const size_t fused = bnn::eng::mlp_fused_smem(m->mlp_max_in, m->mlp_max_wbytes);
    if (fused <= 200u * 1024u) {
        const size_t rows = std::min<size_t>(R, bnn::eng::kMlpFusedMaxSamples);
        CUDA_OR(cudaFuncSetAttribute(bnn::eng::mlp_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)fused),
                BNND_EIO);
        CUDA_OR(cudaMallocHost(&c->h_mlp_in, rows * m->info.input_size * 4), BNND_ENOMEM);
        CUDA_OR(cudaMallocHost(&c->h_mlp_out, rows * m->info.n_classes * 4), BNND_ENOMEM);
        c->mlp_fused_smem = fused;
    }
    return BNND_OK;
}

// Reads and clears the device status word after the stream drains.
BNND_Status finish(bnnd_context* c, const char* what) {
    CUDA_OR(cudaMemcpyAsync(c->h_status, c->status.p, 4, cudaMemcpyDeviceToHost, c->stream), BNND_EIO);
    CUDA_OR(cudaStreamSynchronize(c->stream), BNND_EIO);
    const int st = *c->h_status;
    if (st) {
        cudaMemsetAsync(c->status.p, 0, 4, c->stream);
        cudaStreamSynchronize(c->stream);
        if (st & bnn::kStatusTimeout)
            return fail(BNND_EIO, "%s: device wait timed out", what);
        if (st & bnn::eng::kStatusInputNotFinite)  // checked on the device (fused classify)
            return fail(BNND_EINVAL, "input contains NaN or Inf");
        if (st == bnn::kStatusBadInput)  // a linear's FP32 input held NaN/Inf (BNN_ERANGE)
            return fail(BNND_ERANGE, "%s: linear input contains NaN or Inf", what);
        return fail(BNND_ECOMPUTE, "%s: model produced NaN or Inf values", what);
    }
    return BNND_OK;
}

BNND_Status set_pos(bnnd_context* c, uint32_t pos) {
    std::vector<uint32_t> p(c->rows, pos);
    CUDA_OR(cudaMemcpyAsync(c->pos_d.p, p.data(), p.size() * 4, cudaMemcpyHostToDevice, c->stream), BNND_EIO);
    CUDA_OR(cudaStreamSynchronize(c->stream), BNND_EIO);
    c->pos = pos;
    return BNND_OK;
}

// ---- batched prefill (prefill_kernels.cuh): rows x positions activation rows

// Prefill buffers for `rows` activation rows (grown on demand).
BNND_Status ensure_prefill(bnnd_context* c, uint32_t rows) {
    if (c->pf_rows >= rows)
        return BNND_OK;
    const BNND_ModelInfo& in = c->model->info;
    const uint32_t C = in.hidden, F = in.ffn, QKV = in.hidden + 2 * in.kv_heads * in.head_dim;
    c->pf_rows = 0;
    for (DevMem* d : {&c->pf_x, &c->pf_qkv, &c->pf_y, &c->pf_h, &c->pf_a, &c->pf_rs, &c->pf_scores})
        *d = DevMem();
    BNND_Status st;
    if ((st = dev_alloc(c->pf_x, (size_t)rows * C * 4)) || (st = dev_alloc(c->pf_qkv, (size_t)rows * QKV * 4)) ||
        (st = dev_alloc(c->pf_y, (size_t)rows * C * 4)) || (st = dev_alloc(c->pf_h, (size_t)rows * F * 4)) ||
        (st = dev_alloc(c->pf_a, bnn::mma_a_bytes(rows, std::max(C, F) / 128))) ||
        (st = dev_alloc(c->pf_rs, (size_t)rows * 4)))
        return st;
    // attention scores of a query tile in shared memory when the whole context fits, else here
    const bnn::eng::PfSmem pf = bnn::eng::pf_smem_plan(in.head_dim, in.heads / in.kv_heads,
                                                       bnn::eng::attn_sc_stride(c->n_ctx), true);
    if (pf.total > bnn::eng::kPfSmemBudget &&
        (st = dev_alloc(c->pf_scores, (size_t)rows * in.heads * bnn::eng::attn_sc_stride(c->n_ctx) * 4)))
        return st;
    c->pf_rows = rows;
    return BNND_OK;
}

using PfAttnFn = void (*)(bnn::eng::PfAttnArgs);
PfAttnFn prefill_attention_fn(uint32_t hd, uint32_t kv_mul, bool sc_smem) {
    using namespace bnn::eng;
#define BNN_PF_CASE(H, Q) \
    if (hd == H && kv_mul == Q) \
        return sc_smem ? prefill_attention_kernel<H, Q, true> : prefill_attention_kernel<H, Q, false>;
    BNN_PF_CASE(128, 1) BNN_PF_CASE(128, 2) BNN_PF_CASE(128, 4) BNN_PF_CASE(128, 8)
    BNN_PF_CASE(64, 1) BNN_PF_CASE(64, 2) BNN_PF_CASE(64, 4) BNN_PF_CASE(64, 8)
#undef BNN_PF_CASE
    return nullptr;
}

using KvAppendFn = void (*)(bnn::eng::KvAppendArgs);
KvAppendFn kv_append_fn(uint32_t hd) {
    if (hd == 128)
        return bnn::eng::kv_append_kernel<128>;
    if (hd == 64)
        return bnn::eng::kv_append_kernel<64>;
    return nullptr;
}

// Every layer over `rows` = context rows x `len` activation rows (positions
// pos_end - len .. pos_end - 1 of each row): meta = [ids][positions][cache rows].
cudaError_t enqueue_prefill_chunk(bnnd_context* c, uint32_t rows, uint32_t len, uint32_t pos_end,
                                  const uint32_t* meta) {
    LaunchCheck local;
    LaunchCheck& ck = g_check ? *g_check : local;
    const bnnd_model* m = c->model;
    const BNND_ModelInfo& in = m->info;
    const uint32_t C = in.hidden, F = in.ffn, HD = in.head_dim, KV = in.kv_heads * HD;
    const uint32_t QKV = C + 2 * KV;
    cudaStream_t s = c->stream;
    int* status = c->status.as<int>();
    const int32_t* ids = reinterpret_cast<const int32_t*>(meta);
    const uint32_t* pos = meta + rows;
    const uint32_t* slot = meta + 2 * (size_t)rows;
    float* x = c->pf_x.as<float>();
    unsigned char* pa_sw = c->pf_a.as<unsigned char>();
    float* pa_rs = c->pf_rs.as<float>();
    float* qkv = c->pf_qkv.as<float>();
    float* y = c->pf_y.as<float>();
    float* h = c->pf_h.as<float>();
    bnn::eng::embed_kernel<<<rows, 256, 0, s>>>(ids, m->lm_head.m->wblocks, C, x, nullptr);
    ck("embed_kernel");
    const KvAppendFn append = kv_append_fn(HD);
    const size_t append_smem = bnn::eng::kv_append_smem(HD, in.kv_heads);
    // tiled causal attention: scores in shared memory up to this chunk's last position
    const uint32_t kv_mul = in.heads / in.kv_heads;
    const uint32_t sc_local = bnn::eng::attn_sc_stride(pos_end);
    bnn::eng::PfSmem pf_plan = bnn::eng::pf_smem_plan(HD, kv_mul, sc_local, true);
    const bool pf_global = pf_plan.total > bnn::eng::kPfSmemBudget;
    if (pf_global)
        pf_plan = bnn::eng::pf_smem_plan(HD, kv_mul, bnn::eng::attn_sc_stride(c->n_ctx), false);
    const PfAttnFn pf_attn = prefill_attention_fn(HD, kv_mul, !pf_global);
    if (!pf_attn || (pf_global && !c->pf_scores.p))
        return cudaErrorInvalidValue;
    {
        const cudaError_t e = cudaFuncSetAttribute(pf_attn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)pf_plan.total);
        if (e != cudaSuccess)
            return e;
    }
    const dim3 pf_grid(in.kv_heads, (rows / len) * ((len + bnn::eng::kPfQT - 1) / bnn::eng::kPfQT));
    for (uint32_t l = 0; l < in.n_layers; ++l) {
        const QwenLayer& L = *m->layers[l];
        const size_t layer_cache = (size_t)c->rows * c->n_ctx * KV;
        float* kc = c->kcache.as<float>() + (size_t)l * (layer_cache / HD * bnn::eng::kcache_row(HD));
        float* vc = c->vcache.as<float>() + (size_t)l * layer_cache;
        ck("rows_prep:qkv", prefill_prep(c, pa_sw, pa_rs, x, C, L.attn_norm.as<float>(), rows));
        ck("w1a8_mma:qkv", prefill_linear(c, pa_sw, pa_rs, L.qkv, rows, qkv, (size_t)QKV * 4u, bnn::kEpiView));
        bnn::eng::KvAppendArgs ka = {};
        ka.qkv = qkv;
        ka.k_norm = L.k_norm.as<float>();
        ka.rope_cos = c->rope_cos.as<float>();
        ka.rope_sin = c->rope_sin.as<float>();
        ka.pos = pos;
        ka.slot = slot;
        ka.kcache = kc;
        ka.vcache = vc;
        ka.c = C;
        ka.kv = KV;
        ka.kv_heads = in.kv_heads;
        ka.n_ctx = c->n_ctx;
        ka.eps = m->eps;
        ka.exact = c->params.exact;
        ka.status = status;
        ck("kv_append_kernel", launch_on(c, append, dim3(rows), dim3(32 * in.kv_heads), append_smem, ka));
        bnn::eng::PfAttnArgs pa = {};
        pa.qkv = qkv;
        pa.q_norm = L.q_norm.as<float>();
        pa.rope_cos = c->rope_cos.as<float>();
        pa.rope_sin = c->rope_sin.as<float>();
        pa.pos = pos;
        pa.slot = slot;
        pa.kcache = kc;
        pa.vcache = vc;
        pa.scores = pf_global ? c->pf_scores.as<float>() : nullptr;
        pa.y = y;
        pa.y_stride = C;
        pa.c = C;
        pa.kv = KV;
        pa.heads = in.heads;
        pa.kv_heads = in.kv_heads;
        pa.n_ctx = c->n_ctx;
        pa.len = len;
        pa.sc_stride = pf_global ? bnn::eng::attn_sc_stride(c->n_ctx) : sc_local;
        pa.eps = m->eps;
        pa.scale = 1.0f / sqrtf((float)HD);
        pa.exact = c->params.exact;
        pa.status = status;
        ck("prefill_attention_kernel", launch_on(c, pf_attn, pf_grid, dim3(bnn::eng::kPfThreads), pf_plan.total, pa));
        ck("rows_prep:o", prefill_prep(c, pa_sw, pa_rs, y, C, nullptr, rows));
        ck("w1a8_mma:o", prefill_linear(c, pa_sw, pa_rs, L.o, rows, x, (size_t)C * 4u, bnn::kEpiResidual));
        ck("rows_prep:gate_up", prefill_prep(c, pa_sw, pa_rs, x, C, L.ffn_norm.as<float>(), rows));
        ck("w1a8_mma:gate_up", prefill_linear(c, pa_sw, pa_rs, L.gu, rows, h, (size_t)F * 4u, bnn::kEpiSwiGLU));
        ck("rows_prep:down", prefill_prep(c, pa_sw, pa_rs, h, F, nullptr, rows));
        ck("w1a8_mma:down", prefill_linear(c, pa_sw, pa_rs, L.down, rows, x, (size_t)C * 4u, bnn::kEpiResidual));
    }
    return ck.err;
}

// The prompt of every row through the batched prefill, then (want) the
// decode step's out_norm + lm_head + greedy pick on each row's last position.
// all (one-row contexts only): every position's logits, [n][n_vocab] on the
// host, each from the prefill's final hidden row through out_norm + lm_head
// (the decode step's own kernel and plan).
BNND_Status prefill(bnnd_context* c, const int32_t* tokens, uint32_t n, bool want, float* all = nullptr) {
    const uint32_t R = c->rows, start = c->pos, chunk = std::min(n, c->params.prefill_chunk);
    const size_t count = (size_t)R * n;
    BNND_Status st = ensure_prefill(c, R * chunk);
    if (st != BNND_OK)
        return st;
    if (c->pf_meta_cap < 3 * count) {
        c->pf_meta = DevMem();
        c->pf_meta_cap = 0;
        if ((st = dev_alloc(c->pf_meta, 3 * count * 4)))
            return st;
        c->pf_meta_cap = 3 * count;
    }
    if (c->h_meta_cap < 3 * count) {
        if (c->h_meta)
            cudaFreeHost(c->h_meta);
        c->h_meta = nullptr;
        c->h_meta_cap = 0;
        CUDA_OR(cudaMallocHost(&c->h_meta, 3 * count * 4), BNND_ENOMEM);
        c->h_meta_cap = 3 * count;
    }
    // chunk j (positions j0 .. j0 + len - 1 of every row): rows r * len + i
    uint32_t* hm = c->h_meta;
    for (uint32_t j0 = 0; j0 < n; j0 += chunk) {
        const uint32_t len = std::min(chunk, n - j0), P = R * len;
        uint32_t* base = hm + 3 * (size_t)R * j0;
        for (uint32_t r = 0; r < R; ++r)
            for (uint32_t i = 0; i < len; ++i) {
                const uint32_t p = r * len + i;
                base[p] = (uint32_t)tokens[(size_t)r * n + j0 + i];
                base[P + p] = start + j0 + i;
                base[2 * P + p] = r;
            }
    }
    cudaStream_t s = c->stream;
    CUDA_OR(cudaMemcpyAsync(c->pf_meta.p, hm, 3 * count * 4, cudaMemcpyHostToDevice, s), BNND_EIO);
    uint32_t last_len = 0;
    const bnnd_model* md = c->model;
    const size_t V = md->info.n_vocab;
    if (all && !c->lg_pos.p && (st = dev_alloc(c->lg_pos, V * 4)))
        return st;
    for (uint32_t j0 = 0; j0 < n; j0 += chunk) {
        last_len = std::min(chunk, n - j0);
        CUDA_OR(enqueue_prefill_chunk(c, R * last_len, last_len, start + j0 + last_len,
                                      c->pf_meta.as<uint32_t>() + 3 * (size_t)R * j0),
                BNND_EIO);
        for (uint32_t i = 0; all && i < last_len; ++i) {
            const float* xi = c->pf_x.as<float>() + (size_t)i * md->info.hidden;
            CUDA_OR(launch_linear(c, c->plan_head, md->lm_head, xi, md->out_norm.as<float>(), 1, c->lg_pos.as<float>(),
                                  V * 4u, c->status.as<int>()),
                    BNND_EIO);
            CUDA_OR(cudaMemcpyAsync(all + (size_t)(j0 + i) * V, c->lg_pos.p, V * 4, cudaMemcpyDeviceToHost,
                                    c->stream),
                    BNND_EIO);
        }
    }
    // device positions: start + n after the call (the tail's step_end adds the last 1)
    std::vector<uint32_t> pv(R, start + n - (want ? 1u : 0u));
    CUDA_OR(cudaMemcpyAsync(c->pos_d.p, pv.data(), (size_t)R * 4, cudaMemcpyHostToDevice, s), BNND_EIO);
    if (!want)
        return BNND_OK;
    const bnnd_model* m = c->model;
    const uint32_t C = m->info.hidden;
    float* x = c->x.as<float>();
    CUDA_OR(cudaMemcpy2DAsync(x, (size_t)C * 4, c->pf_x.as<float>() + (size_t)(last_len - 1) * C,
                              (size_t)last_len * C * 4, (size_t)C * 4, R, cudaMemcpyDeviceToDevice, s),
            BNND_EIO);
    unsigned long long* best = c->best.as<unsigned long long>();
    CUDA_OR(cudaMemsetAsync(best, 0, (size_t)R * 8, s), BNND_EIO);
    CUDA_OR(launch_linear(c, c->plan_head, m->lm_head, x, m->out_norm.as<float>(), R, c->logits.as<float>(),
                          (size_t)m->info.n_vocab * 4u, c->status.as<int>(), best),
            BNND_EIO);
    bnn::eng::step_end_kernel<<<1, 32 * ((R + 31) / 32), 0, s>>>(
        R, c->pos_d.as<uint32_t>(), c->tok_in.as<int32_t>(), c->tok_next.as<int32_t>(), best, 1,
        c->hist.as<int32_t>(), c->hist_count.as<uint32_t>(), c->hist_cap, 1);
    CUDA_OR(cudaGetLastError(), BNND_EIO);
    return BNND_OK;
}

// Shared body of BNND_Decode / BNND_DecodeArgmax.
BNND_Status decode(bnnd_context* c, const int32_t* tokens, uint32_t n, float* logits, int32_t* next,
                   float* all = nullptr) {
    g_last_error.clear();
    if (!c || !tokens || n == 0)
        return BNND_EINVAL;
    const bnnd_model* m = c->model;
    if (m->info.task != BNND_TASK_LLM)
        return fail(BNND_ENOTSUP, "model is not a language model");
    if (c->pos > c->n_ctx || n > c->n_ctx - c->pos)
        return fail(BNND_ERANGE, "decode exceeds context length");
    const size_t count = (size_t)n * c->rows;
    for (size_t i = 0; i < count; ++i)
        if (tokens[i] < 0 || (uint32_t)tokens[i] >= m->info.n_vocab)
            return fail(BNND_ERANGE, "token ID is outside vocabulary");
    bnn::DeviceGuard guard(m->dev->ordinal);
    if (c->tok_seq_cap < count) {
        c->tok_seq = DevMem();
        BNND_Status st = dev_alloc(c->tok_seq, count * 4);
        if (st != BNND_OK)
            return st;
        c->tok_seq_cap = count;
    }
    if (c->h_tokens_cap < count) {
        if (c->h_tokens)
            cudaFreeHost(c->h_tokens);
        c->h_tokens = nullptr;
        c->h_tokens_cap = 0;
        CUDA_OR(cudaMallocHost(&c->h_tokens, count * 4), BNND_ENOMEM);
        c->h_tokens_cap = count;
    }
    // Step-major layout in pinned staging: entry [i][row] is row's i-th token.
    int32_t* seq = c->h_tokens;
    for (uint32_t r = 0; r < c->rows; ++r)
        for (uint32_t i = 0; i < n; ++i)
            seq[(size_t)i * c->rows + r] = tokens[(size_t)r * n + i];
    const uint32_t start = c->pos;
    const bool want = logits || next || all;
    const bool batched = c->params.prefill_chunk > 0 && n >= BNND_PREFILL_MIN_TOKENS && c->world == 1;
    if (batched) {
        BNND_Status pst = prefill(c, tokens, n, want, all);
        if (pst != BNND_OK) {
            cudaStreamSynchronize(c->stream);
            set_pos(c, start);
            return pst;
        }
    } else if (n == 1) {
        // one token per row: straight into the step's input slot
        CUDA_OR(cudaMemcpyAsync(c->tok_in.p, seq, count * 4, cudaMemcpyHostToDevice, c->stream), BNND_EIO);
    } else {
        CUDA_OR(cudaMemcpyAsync(c->tok_seq.p, seq, count * 4, cudaMemcpyHostToDevice, c->stream), BNND_EIO);
    }
    for (uint32_t i = 0; i < (batched ? 0u : n); ++i) {
        if (n > 1)
            CUDA_OR(cudaMemcpyAsync(c->tok_in.p, c->tok_seq.as<int32_t>() + (size_t)i * c->rows, c->rows * 4,
                                    cudaMemcpyDeviceToDevice, c->stream),
                    BNND_EIO);
        const bool last = i + 1 == n;
        CUDA_OR(run_step(c, start + i, (last && want) || all), BNND_EIO);
        if (all)
            CUDA_OR(cudaMemcpyAsync(all + (size_t)i * m->info.n_vocab, c->logits.p, (size_t)m->info.n_vocab * 4,
                                    cudaMemcpyDeviceToHost, c->stream),
                    BNND_EIO);
    }
    if (logits)
        CUDA_OR(cudaMemcpyAsync(logits, c->logits.p, (size_t)c->rows * m->info.n_vocab * 4,
                                cudaMemcpyDeviceToHost, c->stream),
                BNND_EIO);
    if (next)
        CUDA_OR(cudaMemcpyAsync(c->h_next, c->tok_next.p, (size_t)c->rows * 4, cudaMemcpyDeviceToHost, c->stream),
                BNND_EIO);
    BNND_Status st = finish(c, "BNND_Decode");
    if (st == BNND_OK && next)
        std::memcpy(next, c->h_next, (size_t)c->rows * 4);
    if (st != BNND_OK) {
        set_pos(c, start);  // the KV cache returns to the position before the call
        return st;
    }
    c->pos = start + n;
    c->have_logits = want;
    return BNND_OK;
}

BNND_Status tok_status(bnn::TokStatus t) {
    switch (t) {
    case bnn::TokStatus::kOk: return BNND_OK;
    case bnn::TokStatus::kRange: return BNND_ERANGE;
    case bnn::TokStatus::kFormat: return BNND_EFORMAT;
    default: return BNND_EINVAL;
    }
}

// A language model carries its tokenizer; a GGUF without a usable one does
// not load (BNNE_ModelLoad, engine.c:61-67).
BNND_Status load_tokenizer(const bnn::GgufFile& g, bnnd_model* m) {
    auto t = std::unique_ptr<bnn::BpeTokenizer>(new (std::nothrow) bnn::BpeTokenizer());
    if (!t)
        return fail(BNND_ENOMEM, "out of memory");
    std::string why;
    const BNND_Status st = tok_status(t->build(g, &why));
    if (st != BNND_OK)
        return fail(st, "%s", why.c_str());
    m->tok = std::move(t);
    return BNND_OK;
}

}  // namespace

extern "C" {

BNND_Status BNND_ModelLoad(BNN_Device device, const char* gguf_path, BNND_Model* out_model) {
    return BNND_ModelLoadShard(device, gguf_path, 1, 0, out_model);
}

BNND_Status BNND_ModelLoadShard(BNN_Device device, const char* gguf_path, uint32_t world, uint32_t rank,
                                BNND_Model* out_model) {
    if (out_model)
        *out_model = nullptr;
    g_last_error.clear();
    if (!device || !gguf_path || !out_model || world == 0 || rank >= world)
        return BNND_EINVAL;
    bnn::GgufFile g;
    if (!g.open(gguf_path))
        return fail(BNND_EFORMAT, "%s: %s", gguf_path, g.error().c_str());
    std::string arch;
    if (!g.get_str("general.architecture", &arch))
        return fail(BNND_EFORMAT, "%s: missing general.architecture", gguf_path);
    auto* m = new (std::nothrow) bnnd_model();
    if (!m)
        return fail(BNND_ENOMEM, "out of memory");
    m->dev = device;
    m->shard.world = 1;
    bnn::DeviceGuard guard(device->ordinal);
    BNND_Status st;
    if (arch == "qwen3") {
        m->shard.world = world;
        m->shard.rank = rank;
        st = load_qwen3(g, m);
        if (st == BNND_OK)
            st = load_tokenizer(g, m);
    } else if (arch == "bnn-mlp")
        st = load_mlp(g, m);  // whole model: classification is data-parallel
    else
        st = fail(BNND_ENOTSUP, "unsupported GGUF architecture '%s'", arch.c_str());
    if (st != BNND_OK) {
        delete m;
        return st;
    }
    *out_model = m;
    return BNND_OK;
}

void BNND_ModelFree(BNND_Model model) {
    if (!model)
        return;
    bnn::DeviceGuard guard(model->dev->ordinal);
    delete model;
}

BNND_Status BNND_ModelGetInfo(BNND_Model model, BNND_ModelInfo* out_info) {
    if (!model || !out_info)
        return BNND_EINVAL;
    *out_info = model->info;
    return BNND_OK;
}

BNND_Status BNND_ShardPlan(const BNND_ModelInfo* info, uint32_t world, uint32_t rank, BNND_ShardInfo* out) {
    g_last_error.clear();
    if (!info || !out || info->task != BNND_TASK_LLM)
        return BNND_EINVAL;
    return shard_plan(*info, world, rank, out);
}

BNND_Status BNND_ModelGetShard(BNND_Model model, BNND_ShardInfo* out) {
    if (!model || !out)
        return BNND_EINVAL;
    *out = model->shard;
    return BNND_OK;
}

BNND_Status BNND_CommIdCreate(unsigned char id[BNND_COMM_ID_BYTES]) {
    static_assert(sizeof(ncclUniqueId) == BNND_COMM_ID_BYTES, "NCCL unique id size");
    g_last_error.clear();
    if (!id)
        return BNND_EINVAL;
    ncclUniqueId u;
    const ncclResult_t r = ncclGetUniqueId(&u);
    if (r != ncclSuccess)
        return fail(BNND_EIO, "ncclGetUniqueId: %s", ncclGetErrorString(r));
    std::memcpy(id, &u, sizeof u);
    return BNND_OK;
}

void BNND_ContextParamsInit(BNND_ContextParams* params) {
    if (params) {
        params->n_ctx = 0;
        params->n_batch = 1;
        params->exact = 1;
        params->comm_id = nullptr;
        params->prefill_chunk = BNND_PREFILL_CHUNK_DEFAULT;
    }
}

BNND_Status BNND_ContextCreate(BNND_Model model, const BNND_ContextParams* params, BNND_Context* out_ctx) {
    if (out_ctx)
        *out_ctx = nullptr;
    g_last_error.clear();
    if (!model || !out_ctx)
        return BNND_EINVAL;
    auto c = std::unique_ptr<bnnd_context>(new (std::nothrow) bnnd_context());
    if (!c)
        return fail(BNND_ENOMEM, "out of memory");
    c->model = model;
    BNND_ContextParamsInit(&c->params);
    if (params)
        c->params = *params;
    c->rows = c->params.n_batch ? c->params.n_batch : 1;
    if (c->rows > 1024)
        return fail(BNND_ERANGE, "n_batch above 1024 is not supported");
    bnn::DeviceGuard guard(model->dev->ordinal);
    c->stream = model->dev->stream;
    if (cudaMallocHost(&c->h_status, 4) != cudaSuccess ||
        cudaMallocHost(&c->h_next, (size_t)c->rows * 4) != cudaSuccess) {
        cudaGetLastError();
        return fail(BNND_ENOMEM, "pinned allocation failed");
    }
    BNND_Status st;
    if (model->info.task == BNND_TASK_LLM) {
        c->n_ctx = c->params.n_ctx ? c->params.n_ctx : model->info.n_ctx_train;
        if (c->n_ctx == 0 || c->n_ctx > model->info.n_ctx_train)
            return fail(BNND_ERANGE, "context length %u exceeds model capacity %u", c->n_ctx,
                        model->info.n_ctx_train);
        st = create_llm_context(c.get());
    } else {
        st = create_mlp_context(c.get());
    }
    if (st != BNND_OK)
        return st;
    *out_ctx = c.release();
    return BNND_OK;
}

void BNND_ContextFree(BNND_Context ctx) {
    if (!ctx)
        return;
    bnn::DeviceGuard guard(ctx->model->dev->ordinal);
    cudaStreamSynchronize(ctx->stream);
    delete ctx;
}

BNND_Status BNND_Decode(BNND_Context ctx, const int32_t* tokens, uint32_t n_tokens, float* logits) {
    return decode(ctx, tokens, n_tokens, logits, nullptr);
}

BNND_Status BNND_DecodeLogitsAll(BNND_Context ctx, const int32_t* tokens, uint32_t n_tokens, float* logits_all) {
    g_last_error.clear();
    if (!ctx || !logits_all)
        return BNND_EINVAL;
    if (ctx->rows != 1 || ctx->world != 1)
        return fail(BNND_ENOTSUP, "per-position logits need a one-row, single-GPU context");
    return decode(ctx, tokens, n_tokens, nullptr, nullptr, logits_all);
}

BNND_Status BNND_DecodeArgmax(BNND_Context ctx, const int32_t* tokens, uint32_t n_tokens,
                              int32_t* next_tokens) {
    if (!next_tokens)
        return BNND_EINVAL;
    return decode(ctx, tokens, n_tokens, nullptr, next_tokens);
}

BNND_Status BNND_Generate(BNND_Context c, uint32_t steps, int32_t* out_tokens) {
    g_last_error.clear();
    if (!c || steps == 0)
        return BNND_EINVAL;
    if (c->model->info.task != BNND_TASK_LLM)
        return fail(BNND_ENOTSUP, "model is not a language model");
    if (!c->have_logits)
        return fail(BNND_EINVAL, "BNND_Generate needs a preceding decode with logits");
    // Each step consumes one position; the last generated token is not fed back.
    if (c->pos > c->n_ctx || steps - 1 > c->n_ctx - c->pos)
        return fail(BNND_ERANGE, "generation exceeds context length");
    if (steps > c->hist_cap)
        return fail(BNND_ERANGE, "too many steps for one call");
    bnn::DeviceGuard guard(c->model->dev->ordinal);
    const uint32_t start = c->pos;
    // The first generated token is the argmax already computed.
    CUDA_OR(cudaMemsetAsync(c->hist_count.p, 0, 4, c->stream), BNND_EIO);
    CUDA_OR(cudaMemcpyAsync(c->hist.p, c->tok_next.p, (size_t)c->rows * 4, cudaMemcpyDeviceToDevice, c->stream),
            BNND_EIO);
    CUDA_OR(cudaMemcpyAsync(c->tok_in.p, c->tok_next.p, (size_t)c->rows * 4, cudaMemcpyDeviceToDevice, c->stream),
            BNND_EIO);
    const uint32_t one = 1;
    CUDA_OR(cudaMemcpyAsync(c->hist_count.p, &one, 4, cudaMemcpyHostToDevice, c->stream), BNND_EIO);
    for (uint32_t i = 1; i < steps; ++i)
        CUDA_OR(run_step(c, start + i - 1, true), BNND_EIO);
    if (out_tokens)
        CUDA_OR(cudaMemcpyAsync(out_tokens, c->hist.p, (size_t)steps * c->rows * 4, cudaMemcpyDeviceToHost,
                                c->stream),
                BNND_EIO);
    BNND_Status st = finish(c, "BNND_Generate");
    if (st != BNND_OK) {
        set_pos(c, start);
        return st;
    }
    c->pos = start + steps - 1;
    if (out_tokens) {
        // Device history is step-major; the API returns row-major [rows][steps].
        std::vector<int32_t> tmp(out_tokens, out_tokens + (size_t)steps * c->rows);
        for (uint32_t s = 0; s < steps; ++s)
            for (uint32_t r = 0; r < c->rows; ++r)
                out_tokens[(size_t)r * steps + s] = tmp[(size_t)s * c->rows + r];
    }
    return BNND_OK;
}

// The reference CLI's generation loop (bnn-infer-v2.c:253-282) with the
// device kept busy: the host hands out token s while steps s+1 .. s+kStreamAhead
// already run. The loop it reproduces, from t0 = the preceding decode's pick:
//   for s in 0..steps-1: stop if EOG(t_s); emit t_s;
//                        stop if s+1 == steps or the context is full;
//                        t_{s+1} = argmax(decode(t_s))
// so D decodes are kept, D = the number of emitted tokens, less one unless the
// loop stopped at an EOG token. Steps queued past D are dropped afterwards:
// the position returns to start + D and the pending pick to t_D, the state
// the plain loop leaves (stale K/V rows past the position are rewritten
// before any step reads them).
BNND_Status BNND_GenerateStream(BNND_Context c, uint32_t steps, BNND_PieceFn fn, void* user, int32_t* out_tokens,
                                uint32_t* out_count) {
    if (out_count)
        *out_count = 0;
    g_last_error.clear();
    if (!c || steps == 0)
        return BNND_EINVAL;
    const bnnd_model* m = c->model;
    if (m->info.task != BNND_TASK_LLM || !m->tok)
        return fail(BNND_ENOTSUP, "model has no text tokenizer");
    if (c->rows != 1)
        return fail(BNND_ENOTSUP, "streaming generation needs a one-row context");
    if (!c->have_logits)
        return fail(BNND_EINVAL, "BNND_GenerateStream needs a preceding decode with logits");
    if (c->pos > c->n_ctx)
        return fail(BNND_ERANGE, "context is past its length");
    bnn::DeviceGuard guard(m->dev->ordinal);
    if (!c->aux) {
        CUDA_OR(cudaStreamCreateWithFlags(&c->aux, cudaStreamNonBlocking), BNND_EIO);
        for (uint32_t i = 0; i < kStreamSlots; ++i) {
            CUDA_OR(cudaEventCreateWithFlags(&c->sv_step[i], cudaEventDisableTiming), BNND_EIO);
            CUDA_OR(cudaEventCreateWithFlags(&c->sv_copy[i], cudaEventDisableTiming), BNND_EIO);
        }
        CUDA_OR(cudaMallocHost(&c->h_stream, kStreamSlots * 4), BNND_ENOMEM);
    }
    const uint32_t start = c->pos;
    // decodes the loop can ever run: one fewer than steps, and none past the context
    const uint32_t d_max = std::min(steps - 1, c->n_ctx - start);
    int32_t* tok_next = c->tok_next.as<int32_t>();
    // slot s % kStreamSlots receives t_s: t_0 now, t_{j+1} after decode j
    auto copy_token = [&](uint32_t s) -> cudaError_t {
        const uint32_t k = s % kStreamSlots;
        cudaError_t e = cudaEventRecord(c->sv_step[k], c->stream);
        if (e == cudaSuccess)
            e = cudaStreamWaitEvent(c->aux, c->sv_step[k], 0);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(c->h_stream + k, c->hist.as<int32_t>() + s, 4, cudaMemcpyDeviceToHost, c->aux);
        if (e == cudaSuccess)
            e = cudaEventRecord(c->sv_copy[k], c->aux);
        return e;
    };
    CUDA_OR(cudaMemcpyAsync(c->hist.p, tok_next, 4, cudaMemcpyDeviceToDevice, c->stream), BNND_EIO);
    CUDA_OR(cudaMemcpyAsync(c->tok_in.p, tok_next, 4, cudaMemcpyDeviceToDevice, c->stream), BNND_EIO);
    const uint32_t one = 1;
    CUDA_OR(cudaMemcpyAsync(c->hist_count.p, &one, 4, cudaMemcpyHostToDevice, c->stream), BNND_EIO);
    CUDA_OR(copy_token(0), BNND_EIO);
    uint32_t queued = 0;  // decodes enqueued
    auto queue_to = [&](uint32_t want) -> cudaError_t {
        for (; queued < want; ++queued) {
            cudaError_t e = run_step(c, start + queued, true);
            if (e == cudaSuccess)
                e = copy_token(queued + 1);
            if (e != cudaSuccess)
                return e;
        }
        return cudaSuccess;
    };
    BNND_Status st = BNND_OK;
    uint32_t kept = 0, emitted = 0;  // D, tokens handed out
    int32_t last = 0;                // t_D
    cudaError_t ce = queue_to(std::min(d_max, kStreamAhead));
    for (uint32_t s = 0; ce == cudaSuccess; ++s) {
        ce = cudaEventSynchronize(c->sv_copy[s % kStreamSlots]);
        if (ce != cudaSuccess)
            break;
        const int32_t t = c->h_stream[s % kStreamSlots];
        last = t;
        kept = s;
        if (t < 0 || (uint32_t)t >= m->info.n_vocab) {
            st = fail(BNND_ECOMPUTE, "step produced token %d outside the vocabulary", t);
            break;
        }
        if (m->tok->is_eog(t))
            break;
        if (out_tokens)
            out_tokens[s] = t;
        ++emitted;
        const char* bytes = nullptr;
        size_t len = 0;
        m->tok->piece(t, &bytes, &len);
        const bool stop = fn && fn(user, t, bytes, len) != 0;
        if (stop || s + 1 == steps || start + s >= c->n_ctx)
            break;
        ce = queue_to(std::min(d_max, s + 1 + kStreamAhead));
    }
    if (ce != cudaSuccess)
        st = fail(BNND_EIO, "BNND_GenerateStream: %s", cudaGetErrorString(ce));
    const cudaError_t e1 = cudaStreamSynchronize(c->stream), e2 = cudaStreamSynchronize(c->aux);
    if (st == BNND_OK && (e1 != cudaSuccess || e2 != cudaSuccess))
        st = fail(BNND_EIO, "BNND_GenerateStream: %s", cudaGetErrorString(e1 != cudaSuccess ? e1 : e2));
    if (st == BNND_OK && queued)
        st = finish(c, "BNND_GenerateStream");
    if (out_count)
        *out_count = emitted;
    if (st != BNND_OK) {
        set_pos(c, start);
        c->have_logits = false;
        return st;
    }
    if (queued != kept) {  // drop the steps queued past the loop's end
        c->h_next[0] = last;
        CUDA_OR(cudaMemcpyAsync(tok_next, c->h_next, 4, cudaMemcpyHostToDevice, c->stream), BNND_EIO);
        BNND_Status ps = set_pos(c, start + kept);
        if (ps != BNND_OK)
            return ps;
    }
    c->pos = start + kept;
    return BNND_OK;
}

uint32_t BNND_ContextPos(BNND_Context ctx) { return ctx ? ctx->pos : 0; }

BNND_Status BNND_Tokenize(BNND_Model model, const char* text, int parse_special, int32_t* ids, uint32_t capacity,
                          uint32_t* out_count) {
    if (out_count)
        *out_count = 0;
    g_last_error.clear();
    if (!model || !text || !ids || !out_count || capacity == 0)
        return BNND_EINVAL;
    if (!model->tok)
        return fail(BNND_ENOTSUP, "model has no text tokenizer");
    return tok_status(model->tok->encode(text, std::strlen(text), parse_special != 0, ids, capacity, out_count));
}

BNND_Status BNND_TokenPiece(BNND_Model model, int32_t id, const char** out_bytes, size_t* out_len) {
    if (out_bytes)
        *out_bytes = nullptr;
    if (out_len)
        *out_len = 0;
    g_last_error.clear();
    if (!model || !out_bytes || !out_len)
        return BNND_EINVAL;
    if (!model->tok)
        return fail(BNND_ENOTSUP, "model has no text tokenizer");
    return tok_status(model->tok->piece(id, out_bytes, out_len));
}

int BNND_TokenIsEog(BNND_Model model, int32_t id) {
    if (!model || !model->tok || id < 0 || (uint32_t)id >= model->info.n_vocab)
        return 0;
    return model->tok->is_eog(id) ? 1 : 0;
}

BNND_Status BNND_TokenizerLoad(const char* gguf_path, BNND_Tokenizer* out) {
    if (out)
        *out = nullptr;
    g_last_error.clear();
    if (!gguf_path || !out)
        return BNND_EINVAL;
    bnn::GgufFile g;
    if (!g.open(gguf_path))
        return fail(BNND_EFORMAT, "%s: %s", gguf_path, g.error().c_str());
    auto t = std::unique_ptr<bnnd_tokenizer>(new (std::nothrow) bnnd_tokenizer());
    if (!t)
        return fail(BNND_ENOMEM, "out of memory");
    std::string why;
    const BNND_Status st = tok_status(t->tok.build(g, &why));
    if (st != BNND_OK)
        return fail(st, "%s", why.c_str());
    *out = t.release();
    return BNND_OK;
}

void BNND_TokenizerFree(BNND_Tokenizer tok) { delete tok; }

uint32_t BNND_TokenizerSize(BNND_Tokenizer tok) { return tok ? tok->tok.size() : 0; }

BNND_Status BNND_TokenizerEncode(BNND_Tokenizer tok, const char* text, size_t len, int parse_special, int32_t* ids,
                                 uint32_t capacity, uint32_t* out_count) {
    if (out_count)
        *out_count = 0;
    g_last_error.clear();
    if (!tok || (!text && len) || !ids || !out_count || capacity == 0)
        return BNND_EINVAL;
    return tok_status(tok->tok.encode(text ? text : "", len, parse_special != 0, ids, capacity, out_count));
}

BNND_Status BNND_TokenizerPiece(BNND_Tokenizer tok, int32_t id, const char** out_bytes, size_t* out_len) {
    if (out_bytes)
        *out_bytes = nullptr;
    if (out_len)
        *out_len = 0;
    g_last_error.clear();
    if (!tok || !out_bytes || !out_len)
        return BNND_EINVAL;
    return tok_status(tok->tok.piece(id, out_bytes, out_len));
}

int BNND_TokenizerIsEog(BNND_Tokenizer tok, int32_t id) { return tok && tok->tok.is_eog(id) ? 1 : 0; }

BNND_Status BNND_ContextTruncate(BNND_Context ctx, uint32_t pos) {
    g_last_error.clear();
    if (!ctx)
        return BNND_EINVAL;
    if (pos > ctx->pos)
        return fail(BNND_EINVAL, "truncate position is beyond current position");
    if (ctx->model->info.task != BNND_TASK_LLM) {
        ctx->pos = pos;
        return BNND_OK;
    }
    bnn::DeviceGuard guard(ctx->model->dev->ordinal);
    ctx->have_logits = false;
    return set_pos(ctx, pos);
}

BNND_Status BNND_Classify(BNND_Context c, const float* input, uint32_t n_samples, float* logits) {
    g_last_error.clear();
    if (!c || !input || !logits || n_samples == 0)
        return BNND_EINVAL;
    const bnnd_model* m = c->model;
    if (m->info.task != BNND_TASK_CLASSIFY)
        return fail(BNND_ENOTSUP, "model is not a classifier");
    if (n_samples > c->rows)
        return fail(BNND_ERANGE, "sample count exceeds context batch size");
    const size_t inputs = (size_t)n_samples * m->info.input_size;
    const size_t outputs = (size_t)n_samples * m->info.n_classes;
    bnn::DeviceGuard guard(m->dev->ordinal);
    cudaStream_t s = c->stream;
    float* cur = c->mlp_a.as<float>();
    float* nxt = c->mlp_b.as<float>();
    if (n_samples <= bnn::eng::kMlpFusedMaxSamples && c->mlp_fused_smem) {
        // every layer of a sample in one CTA (mlp_fused.cuh): one launch per
        // call, the input check on the device, copies through pinned staging
        // the kernel reads the samples from, and writes the logits to, the
        // pinned staging buffers directly (device-addressable host memory):
        // no copy operations on the stream
        std::memcpy(c->h_mlp_in, input, inputs * 4);
        bnn::eng::MlpFusedArgs fa = {};
        fa.layers = m->mlp_desc.as<bnn::eng::MlpLayerDev>();
        fa.n_layers = (uint32_t)m->mlp.size();
        fa.max_in = m->mlp_max_in;
        fa.max_wbytes = m->mlp_max_wbytes;
        fa.x = c->h_mlp_in;
        fa.logits = c->h_mlp_out;
        fa.status = c->status.as<int>();
        bnn::eng::mlp_fused_kernel<<<n_samples, bnn::eng::kMlpThreads, c->mlp_fused_smem, s>>>(fa);
        CUDA_OR(cudaGetLastError(), BNND_EIO);
        const BNND_Status st = finish(c, "BNND_Classify");
        if (st == BNND_OK)
            std::memcpy(logits, c->h_mlp_out, outputs * 4);
        return st;
    }
    for (size_t i = 0; i < inputs; ++i)
        if (!std::isfinite(input[i]))
            return fail(BNND_EINVAL, "input contains NaN or Inf");
    CUDA_OR(cudaMemcpyAsync(cur, input, inputs * 4, cudaMemcpyHostToDevice, s), BNND_EIO);
    const bool mma = n_samples >= bnn::kMmaMinRows;  // the batch on the tensor cores (BNN_Execute's threshold)
    for (size_t i = 0; i < m->mlp.size(); ++i) {
        const MlpLayer& L = *m->mlp[i];
        if (mma) {
            // QuantizeRow of every sample into the pre-tiled operand, then GEMM_F32
            bnn::PrepArgs pa = {};
            pa.in = reinterpret_cast<const unsigned char*>(cur);
            pa.in_stride = (size_t)L.w.in * 4u;
            pa.kind = bnn::kInputF32;
            pa.k = L.w.in;
            pa.m = n_samples;
            pa.a_sw = c->mlp_asw.as<unsigned char>();
            pa.row_scale = c->mlp_rs.as<float>();
            pa.status = c->status.as<int>();
            const size_t prep_smem = bnn::prep_smem_bytes(L.w.in);
            CUDA_OR(cudaFuncSetAttribute(bnn::w1a8_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)prep_smem),
                    BNND_EIO);
            bnn::w1a8_prep_kernel<<<n_samples, bnn::kPrepThreads, prep_smem, s>>>(pa);
            bnn::MmaArgs ma = {};
            ma.wblocks = L.w.m->wblocks;
            ma.n = L.w.out;
            ma.groups = L.w.in / 128;
            ma.m = n_samples;
            ma.a_sw = c->mlp_asw.as<unsigned char>();
            ma.row_scale = c->mlp_rs.as<float>();
            ma.out = reinterpret_cast<unsigned char*>(nxt);
            ma.out_stride = (size_t)L.w.out * 4u;
            ma.epi = bnn::kEpiView;
            ma.status = c->status.as<int>();
            CUDA_OR(bnn::launch_mma(ma, m->dev->sm_count, s), BNND_EIO);
        } else {
            CUDA_OR(launch_linear(c, c->plan_mlp[i], L.w, cur, nullptr, n_samples, nxt, (size_t)L.w.out * 4u,
                                  c->status.as<int>()),
                    BNND_EIO);
        }
        bnn::eng::mlp_post_kernel<<<64, 256, 0, s>>>(nxt, L.post_scale.as<float>(), L.post_bias.as<float>(),
                                                     L.w.out, n_samples, L.relu);
        std::swap(cur, nxt);
    }
    bnn::eng::finite_check_kernel<<<16, 256, 0, s>>>(cur, outputs, c->status.as<int>(), bnn::kStatusNonFinite);
    CUDA_OR(cudaMemcpyAsync(logits, cur, outputs * 4, cudaMemcpyDeviceToHost, s), BNND_EIO);
    return finish(c, "BNND_Classify");
}

BNND_Status BNND_ContextProfile(BNND_Context c, uint32_t steps, BNND_KernelStat* stats, uint32_t capacity,
                                uint32_t* count, double* total_ms) {
    g_last_error.clear();
    if (count)
        *count = 0;
    if (!c || steps == 0 || (!stats && capacity))
        return BNND_EINVAL;
    if (c->model->info.task != BNND_TASK_LLM)
        return fail(BNND_ENOTSUP, "model is not a language model");
    if (!c->have_logits)
        return fail(BNND_EINVAL, "BNND_ContextProfile needs a preceding decode with logits");
    if (c->pos > c->n_ctx || steps > c->n_ctx - c->pos)
        return fail(BNND_ERANGE, "profiling exceeds context length");
    bnn::DeviceGuard guard(c->model->dev->ordinal);
    StepRecorder& rec = c->recorder;
    if (!c->graph_profile) {
        const size_t n_events = (size_t)c->step_launches + 2;
        rec.stream = c->stream;
        rec.events.resize(n_events);
        rec.names.assign(n_events, std::string());
        rec.bytes.assign(n_events, 0.0);
        for (cudaEvent_t& e : rec.events)
            CUDA_OR(cudaEventCreate(&e), BNND_EIO);
        rec.next = 0;
        g_rec = &rec;
        BNND_Status st = capture_step(c, true, &c->graph_profile);
        g_rec = nullptr;
        if (st != BNND_OK)
            return st;
        if (rec.overflow)
            return fail(BNND_EIO, "profile recorder overflow");
    }
    const uint32_t start = c->pos;
    CUDA_OR(cudaMemcpyAsync(c->tok_in.p, c->tok_next.p, (size_t)c->rows * 4, cudaMemcpyDeviceToDevice, c->stream),
            BNND_EIO);
    std::vector<std::string> names;
    std::vector<BNND_KernelStat> acc;
    double total = 0.0;
    for (uint32_t step = 0; step < steps; ++step) {
        CUDA_OR(cudaGraphLaunch(c->graph_profile, c->stream), BNND_EIO);
        CUDA_OR(cudaStreamSynchronize(c->stream), BNND_EIO);
        for (size_t i = 0; i < rec.next; ++i) {
            float ms = 0.0f;
            CUDA_OR(cudaEventElapsedTime(&ms, rec.events[i], rec.events[i + 1]), BNND_EIO);
            total += ms;
            size_t k = 0;
            while (k < names.size() && names[k] != rec.names[i])
                ++k;
            if (k == names.size()) {
                names.push_back(rec.names[i]);
                BNND_KernelStat z{};
                std::snprintf(z.name, sizeof z.name, "%s", rec.names[i].c_str());
                acc.push_back(z);
            }
            if (step == 0)
                acc[k].launches += 1;
            acc[k].ms += ms;
            acc[k].bytes += rec.bytes[i];
        }
    }
    BNND_Status st = finish(c, "BNND_ContextProfile");
    if (st != BNND_OK) {
        set_pos(c, start);
        return st;
    }
    c->pos = start + steps;
    const uint32_t n = (uint32_t)std::min<size_t>(acc.size(), capacity);
    for (uint32_t i = 0; i < n; ++i)
        stats[i] = acc[i];
    if (count)
        *count = n;
    if (total_ms)
        *total_ms = total;
    return BNND_OK;
}

uint32_t BNND_StepLaunches(BNND_Context ctx) { return ctx ? ctx->step_launches : 0; }

uint32_t BNND_StepKernelPositions(BNND_Context ctx) { return ctx ? ctx->st_positions : 0; }

BNND_Status BNND_StepKernelTrace(BNND_Context c, uint64_t* stamps, size_t capacity, size_t* count) {
    g_last_error.clear();
    if (!c || !stamps || !count)
        return BNND_EINVAL;
    if (!c->st_positions || c->pos >= c->st_positions || c->pos >= c->n_ctx)
        return fail(BNND_ENOTSUP, "the step kernel does not serve this context or position");
    if (!c->have_logits)
        return fail(BNND_EINVAL, "a step trace needs a preceding decode with logits");
    const uint32_t grid = (uint32_t)c->model->dev->sm_count;
    const size_t words = (size_t)grid * (c->st_args.n_layers + 1) * bnn::step::kTraceSlots;
    *count = words;
    if (capacity < words)
        return fail(BNND_ERANGE, "trace needs %zu entries", words);
    bnn::DeviceGuard guard(c->model->dev->ordinal);
    DevMem tr;
    BNND_Status st = dev_alloc(tr, words * 8);
    if (st != BNND_OK)
        return st;
    CUDA_OR(cudaMemsetAsync(tr.p, 0, words * 8, c->stream), BNND_EIO);
    bnn::step::StepArgs a = c->st_args;
    a.trace = tr.as<unsigned long long>();
    CUDA_OR(launch_step_kernel(c, a), BNND_EIO);
    CUDA_OR(cudaMemcpyAsync(stamps, tr.p, words * 8, cudaMemcpyDeviceToHost, c->stream), BNND_EIO);
    const uint32_t start = c->pos;
    st = finish(c, "BNND_StepKernelTrace");
    if (st != BNND_OK) {
        set_pos(c, start);
        return st;
    }
    c->pos = start + 1;
    return BNND_OK;
}

const char* BNND_LastError(void) { return g_last_error.c_str(); }

void* BNND_ContextStream(BNND_Context ctx) { return ctx ? static_cast<void*>(ctx->stream) : nullptr; }

}  // extern "C"

namespace bnn {
cudaError_t set_test_hooks_engine(unsigned long long limit_ns, int starve) {
    cudaError_t e = cudaMemcpyToSymbol(g_wait_ns_limit, &limit_ns, sizeof limit_ns);
    if (e == cudaSuccess)
        e = cudaMemcpyToSymbol(g_test_starve_producer, &starve, sizeof starve);
    return e;
}
}  // namespace bnn
