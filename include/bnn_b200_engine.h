/*
 * bnn_b200_engine.h - device-resident W1A8 engine (libbnn_b200.so).
 *
 * The reference engine (bnn-sw-v2/bnn-engine.h) runs its model glue on the
 * host and crosses the accelerator boundary once per linear (215 times per
 * Qwen3-1.7B token, bnn-sw-v2/linear.c:161-216). This engine keeps the whole
 * step on the B200: embedding, RMSNorm, the W1A8 linears, q/k-norm, RoPE,
 * the KV cache, attention, SwiGLU, lm_head and the greedy argmax. Its API
 * mirrors BNNE_* (same task model, same status values, same argument and
 * range rules) under a BNND_ prefix so both engines can be linked into one
 * program. A context holds `n_batch` independent rows (sequences) decoded
 * in lockstep; the reference's single-sequence context is n_batch = 1.
 *
 * Numerics: the linears are the bit-exact BNN_* contraction. In the default
 * exact mode the glue reproduces qwen3.c's FP32 operation order (sequential
 * sums, per-op rounding, host-computed RoPE tables) so logits match the
 * reference engine; the one known difference is expf, which is correctly
 * rounded here while glibc's misrounds ~0.004% of inputs by one ulp.
 */
#ifndef BNN_B200_ENGINE_H
#define BNN_B200_ENGINE_H

#include <stddef.h>
#include <stdint.h>

#include "bnn_b200_accel.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct bnnd_model* BNND_Model;
typedef struct bnnd_context* BNND_Context;
typedef struct bnnd_tokenizer* BNND_Tokenizer;

/* Same values as BNNE_Status (bnn-sw-v2/bnn-engine.h:36-45). */
typedef enum {
    BNND_OK = 0,
    BNND_EINVAL = -1,
    BNND_ENOMEM = -2,
    BNND_ENOTSUP = -3,
    BNND_ERANGE = -4,
    BNND_EIO = -5,
    BNND_EFORMAT = -6,
    BNND_ECOMPUTE = -7
} BNND_Status;

typedef enum { BNND_TASK_CLASSIFY = 1, BNND_TASK_LLM = 2 } BNND_Task;

/* Mirrors BNNE_ModelInfo (bnn-engine.h:52-68) plus the Qwen3 shape. */
typedef struct {
    BNND_Task task;
    uint32_t input_size; /* classify: features per sample */
    uint32_t n_classes;
    uint32_t n_vocab;    /* llm */
    uint32_t n_ctx_train;
    int32_t eos_token;   /* -1 if not declared */
    uint32_t n_layers, hidden, heads, kv_heads, head_dim, ffn;
    uint64_t weight_count; /* W1 weights streamed per token (llm) or sample (classify) */
} BNND_ModelInfo;

/* n_ctx: KV capacity (0 = the model's training context); n_batch: rows per
 * call (sequences for llm, samples for classify; 0 = 1); exact: 1 = the
 * reference's operation order for all FP32 glue (default), 0 = parallel
 * reductions for the norm and attention sums. */
typedef struct {
    uint32_t n_ctx;
    uint32_t n_batch;
    int exact;
    /* Sharded models only (BNND_ModelLoadShard with world > 1): the NCCL
     * unique id of BNND_CommIdCreate, the same bytes on every rank; NULL
     * otherwise. Context creation is then collective over the ranks. */
    const unsigned char* comm_id;
    /* Batched prefill (llm, world = 1): a decode call of at least
     * BNND_PREFILL_MIN_TOKENS tokens per row runs its prompt layer by layer
     * over up to prefill_chunk positions of every row at once, each linear a
     * GEMM on the tensor cores; results are bit-identical to one step per
     * token. 0 = one decode step per token (the reference's BNNE_Decode). */
    uint32_t prefill_chunk;
} BNND_ContextParams;
#define BNND_PREFILL_MIN_TOKENS 8
#define BNND_PREFILL_CHUNK_DEFAULT 512

/* Tensor parallelism over `world` GPUs of one node, one process per GPU.
 * Every linear is sharded by out_features (q|k|v by whole GQA groups, so
 * q/k-norm, RoPE, the KV cache and attention stay local to the rank's heads;
 * gate/up by matching row ranges, so SwiGLU is local); each step all-gathers
 * the outputs over NCCL after attention, o, SwiGLU and down, and reduces the
 * greedy pick over the ranks' (value, index) keys. Every output element's
 * arithmetic is unchanged, so results are bit-identical to world = 1. No
 * counterpart in the reference (its accelerator is one device). */
typedef struct {
    uint32_t world, rank;
    uint32_t q_begin, q_rows;   /* q outputs (heads * head_dim) of this rank */
    uint32_t kv_begin, kv_rows; /* k and v outputs each (kv_heads * head_dim) */
    uint32_t c_begin, c_rows;   /* o and down outputs (hidden) */
    uint32_t f_begin, f_rows;   /* gate and up outputs each (ffn) */
    uint32_t v_begin, v_rows;   /* lm_head outputs (vocabulary), clipped */
    uint32_t v_stride;          /* lm_head rows per rank before clipping (multiple of 8) */
} BNND_ShardInfo;
/* Row ranges of `rank` (pure host computation, no device needed). ENOTSUP
 * when the shape does not split (heads, kv_heads, hidden/8 and ffn/8 must
 * be multiples of world). */
BNND_Status BNND_ShardPlan(const BNND_ModelInfo* info, uint32_t world, uint32_t rank, BNND_ShardInfo* out);
/* BNND_ModelLoad of rank `rank`'s shard (qwen3); a bnn-mlp model is loaded
 * whole (classification is data-parallel). world = 1 is BNND_ModelLoad. */
BNND_Status BNND_ModelLoadShard(BNN_Device device, const char* gguf_path, uint32_t world, uint32_t rank,
                                BNND_Model* out_model);
BNND_Status BNND_ModelGetShard(BNND_Model model, BNND_ShardInfo* out);
#define BNND_COMM_ID_BYTES 128
/* A new NCCL unique id, made once (by rank 0) and handed to every rank. */
BNND_Status BNND_CommIdCreate(unsigned char id[BNND_COMM_ID_BYTES]);

/* Replaces BNNE_ModelLoad (bnn-engine.h:95): parses the GGUF (architectures
 * "qwen3" and "bnn-mlp") and uploads every tensor to the device of `device`,
 * Q1_0 weights repacked into the contraction kernel's layout. */
BNND_Status BNND_ModelLoad(BNN_Device device, const char* gguf_path, BNND_Model* out_model);
void BNND_ModelFree(BNND_Model model);
BNND_Status BNND_ModelGetInfo(BNND_Model model, BNND_ModelInfo* out_info);

void BNND_ContextParamsInit(BNND_ContextParams* params);
BNND_Status BNND_ContextCreate(BNND_Model model, const BNND_ContextParams* params, BNND_Context* out_ctx);
void BNND_ContextFree(BNND_Context ctx);

/* Replaces BNNE_Decode (bnn-engine.h:139): appends n_tokens per row
 * (tokens [n_batch][n_tokens], row-major) at the current position, one step
 * per token; logits (NULL for prefill only) receive [n_batch][n_vocab] of the
 * last token. Range and finiteness rules of BNNE_Decode apply. */
BNND_Status BNND_Decode(BNND_Context ctx, const int32_t* tokens, uint32_t n_tokens, float* logits);

/* Like BNND_Decode but returns only the greedy next token of each row
 * (first maximum, lowest index on ties, as bnn-infer-v2.c:48-54). */
BNND_Status BNND_DecodeArgmax(BNND_Context ctx, const int32_t* tokens, uint32_t n_tokens,
                              int32_t* next_tokens);

/* BNND_Decode that returns the logits of every fed position, logits_all
 * [n_tokens][n_vocab], as tools/precision/dump-logits.c collects them with
 * one BNNE_Decode per token (dump-logits.c:295-306); a prompt of
 * BNND_PREFILL_MIN_TOKENS or more still runs as one batched prefill. One-row
 * (n_batch 1), single-GPU contexts; BNND_ENOTSUP otherwise. */
BNND_Status BNND_DecodeLogitsAll(BNND_Context ctx, const int32_t* tokens, uint32_t n_tokens, float* logits_all);

/* Greedy generation entirely on the device: feeds each row's last argmax
 * back as input for `steps` steps (one CUDA graph launch per step) and writes
 * the generated ids to out_tokens [n_batch][steps] (host) when non-NULL.
 * Requires a preceding BNND_Decode/BNND_DecodeArgmax. */
BNND_Status BNND_Generate(BNND_Context ctx, uint32_t steps, int32_t* out_tokens);

/* Receives one generated token and its piece (BNND_TokenPiece bytes, valid
 * until the model is freed). A non-zero return stops the generation after
 * this token. */
typedef int (*BNND_PieceFn)(void* user, int32_t id, const char* bytes, size_t len);

/* The reference CLI's text generation loop (bnn-infer-v2.c:253-282) with
 * the device kept busy: starting from the argmax of the preceding
 * BNND_Decode/BNND_DecodeArgmax, hands out up to `steps` tokens in order to
 * fn (may be NULL) and out_tokens (may be NULL, [steps]); stops before an EOG
 * token (BNND_TokenIsEog), after `steps` tokens, when the context is full,
 * or when fn returns non-zero. Decode steps run up to four tokens ahead of
 * the host; on return the context is exactly where the plain loop leaves it
 * (position = start + tokens handed out, less one unless it stopped at an
 * EOG token; the next pick is the token after the last one decoded).
 * *out_count = tokens handed out. One-row contexts (n_batch 1). */
BNND_Status BNND_GenerateStream(BNND_Context ctx, uint32_t steps, BNND_PieceFn fn, void* user,
                                int32_t* out_tokens, uint32_t* out_count);

uint32_t BNND_ContextPos(BNND_Context ctx);
/* Replaces BNNE_ContextTruncate (bnn-engine.h:144). */
BNND_Status BNND_ContextTruncate(BNND_Context ctx, uint32_t pos);

/* Replaces BNNE_Classify (bnn-engine.h:131) for bnn-mlp: input
 * [n_samples][input_size], logits [n_samples][n_classes]. */
BNND_Status BNND_Classify(BNND_Context ctx, const float* input, uint32_t n_samples, float* logits);

/* ---- text: the qwen3 GGUF's byte-level BPE tokenizer (host) ----
 * Replace BNNE_Tokenize / BNNE_TokenPiece / BNNE_TokenIsEog
 * (bnn-engine.h:106-116; behaviour of bnn-sw-v2/tokenizer/tokenizer-bpe.c).
 * BNND_Tokenize: parse_special != 0 matches special tokens (types 3 and 4)
 * as literals. *out_count always receives the ids written: on BNND_ERANGE
 * (capacity too small) that is `capacity`, the ids written so far, as the
 * reference engine does; text outside special tokens that is not valid UTF-8
 * gives BNND_EINVAL. BNND_ENOTSUP for a model without a tokenizer (bnn-mlp).
 * BNND_TokenPiece: the token's raw bytes (possibly a partial UTF-8 sequence),
 * NUL-terminated, borrowed until BNND_ModelFree; BNND_ERANGE for a bad id.
 * BNND_TokenIsEog: 1 for eos_token_id, <|endoftext|> and <|im_end|>; 0 for
 * other ids, ids outside the vocabulary and models without a tokenizer. */
BNND_Status BNND_Tokenize(BNND_Model model, const char* text, int parse_special, int32_t* ids, uint32_t capacity,
                          uint32_t* out_count);
BNND_Status BNND_TokenPiece(BNND_Model model, int32_t id, const char** out_bytes, size_t* out_len);
int BNND_TokenIsEog(BNND_Model model, int32_t id);

/* The same tokenizer read straight from a GGUF, without a model or a device
 * (host text pipelines, tests). BNND_TokenizerEncode takes an explicit byte
 * length; otherwise the rules above apply. */
BNND_Status BNND_TokenizerLoad(const char* gguf_path, BNND_Tokenizer* out);
void BNND_TokenizerFree(BNND_Tokenizer tok);
uint32_t BNND_TokenizerSize(BNND_Tokenizer tok);
BNND_Status BNND_TokenizerEncode(BNND_Tokenizer tok, const char* text, size_t len, int parse_special, int32_t* ids,
                                 uint32_t capacity, uint32_t* out_count);
BNND_Status BNND_TokenizerPiece(BNND_Tokenizer tok, int32_t id, const char** out_bytes, size_t* out_len);
int BNND_TokenizerIsEog(BNND_Tokenizer tok, int32_t id);

/* Thread-local text of the last failure (BNNE_LastError, bnn-engine.h:157). */
const char* BNND_LastError(void);

/* Device time per kernel of the decode step, for measurement. Has no
 * counterpart in the reference (its BNNE_Stats splits host wall time only,
 * bnn-engine.h:76-87). */
typedef struct {
    char name[32];      /* kernel (W1A8 linears as "w1a8_gemv:<linear>") */
    uint32_t launches;  /* launches per step */
    double ms;          /* device time summed over the profiled steps */
    double bytes;       /* algorithmic bytes summed over the profiled steps; for
                           a linear N*K*0.140625 + 4K + 4N per launch and row */
} BNND_KernelStat;

/* Runs `steps` greedy decode steps (as BNND_Generate, advancing the context)
 * through an instrumented copy of the step graph with a timestamp between
 * every pair of launches, and returns one entry per kernel name (at most
 * `capacity`, *count set to the number written) plus the summed step time. */
BNND_Status BNND_ContextProfile(BNND_Context ctx, uint32_t steps, BNND_KernelStat* stats,
                                uint32_t capacity, uint32_t* count, double* total_ms);

/* Number of kernel launches in one decode step with logits (the per-kernel
 * step graph). */
uint32_t BNND_StepLaunches(BNND_Context ctx);

/* Decode steps with logits at positions below the returned value run as ONE
 * persistent kernel launch (one-row, single-GPU, exact-mode contexts with
 * 128-wide heads; the whole K/V history of a head must fit one SM's shared
 * memory); later positions, and other contexts (return 0), use the
 * per-kernel step graph. Both give the same bits. Setting the environment
 * variable BNN_STEP_KERNEL=0 before BNND_ContextCreate turns it off. */
uint32_t BNND_StepKernelPositions(BNND_Context ctx);

/* Runs ONE greedy decode step (as BNND_Generate's next step) through the
 * step kernel with %globaltimer stamps at its phase boundaries, for
 * measurement; no counterpart in the reference. stamps receives
 * [SMs][n_layers + 1][16] nanosecond stamps (0 where a CTA has no such
 * phase): *count is set to that size, BNND_ERANGE if capacity is smaller.
 * Per layer, contraction CTAs: 0 phase start, 1 x ready, 2 RMSNorm +
 * quantise done, 3 q|k|v rows done, 4 y ready, 5 quantised, 6 o done,
 * 7 x ready, 8 RMSNorm done, 9 gate|up done, 10 h ready, 11 quantised,
 * 12 down done, 13 and 14 the two RMSNorm sums done, 15 x loaded; attention CTAs: 0 q|k|v ready, 1 norms + RoPE, 2 K/V
 * history in, 3 scores, 4 softmax, 5 y written. Last record: 0 x ready,
 * 1 RMSNorm done, 2 lm_head done, 14 step end (last CTA), 15 CTA start. */
BNND_Status BNND_StepKernelTrace(BNND_Context ctx, uint64_t* stamps, size_t capacity, size_t* count);

/* The CUDA stream the context's work runs on (cudaStream_t as void*). */
void* BNND_ContextStream(BNND_Context ctx);

#ifdef __cplusplus
}
#endif

#endif
