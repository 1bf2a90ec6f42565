/*
 * opure_engine.h -- C ABI of libopure_engine.so, the C++20 host engine.
 *
 * Wraps engine::VoxelEngine (the reference's src/engine/Opure_VoxelEngine.h:114-335)
 * for callers that bind C: the reference's HTTP server and harness call Generate,
 * ForwardLogits and RunLayersTraced on the class directly (Opure_Server.cpp:305,
 * Opure_TestHarness.cpp:624,956-987); these entry points expose the same operations
 * with token ids in and out. C++ exceptions never cross the ABI: each call returns an
 * opure_status and opure_engine_last_error() holds the message of the last failure.
 *
 * Also exported: the seeded synthetic-input generators that the benchmark
 * configurations use in place of the reference's downloaded checkpoint.
 */
#ifndef OPURE_ENGINE_H
#define OPURE_ENGINE_H

#include <stddef.h>
#include <stdint.h>

#include "opure_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct opure_engine opure_engine;

/* EngineOptions (Opure_VoxelEngine.h:54-65) plus the B200 engine's own settings. */
typedef struct opure_engine_options {
    uint32_t max_new_tokens;  /* EngineOptions.maxNewTokens (0: 256)                   */
    uint32_t max_batch;       /* independent sequences per step (0: 1)                 */
    uint32_t max_len;         /* tokens per sequence incl. prompt (0: min(max_pos, 4096)) */
    uint32_t page_size;       /* KV page size in tokens: 16/32/64/128 (0: 64)          */
    uint64_t page_seed;       /* seeded shuffle of the KV free list (0: in order)      */
    uint32_t use_graphs;      /* 1: capture each step into a CUDA graph                */
    float attn_scale;         /* attention score scale (0: 1.0, the reference's)       */
    uint32_t path;            /* OPURE_PATH_*: which step kernels to record            */
    uint32_t phase_trace;     /* 1: the persistent step records per-CTA phase stamps   */
    uint32_t prefill_chunk;   /* >0: prefill prompts as steps of up to this many token
                                 vectors (tensor-core GEMMs, causal within the step)
                                 instead of one token per step (0: the reference's way) */
    uint32_t kv_window;       /* >0: sliding-window KV cache of this many tokens, a multiple
                                 of page_size (>= 2 pages): each sequence keeps that many
                                 tokens of pages as a ring (opure_kv_layout.ring) and a
                                 position attends to the last kv_window / page_size - 1 whole
                                 pages and its own; 0: every position up to max_len */
    uint32_t tp_allreduce;    /* tensor parallel: OPURE_TP_* (0: OPURE_TP_AUTO)          */
} opure_engine_options;

enum {
    OPURE_TP_AUTO = 0,        /* the peer kernels (measured faster than NCCL at 2, 4 and
                                 8 ranks) when every pair of GPUs maps each other's memory,
                                 else NCCL                                                 */
    OPURE_TP_NCCL = 1,        /* NCCL all-reduces between the per-op kernels             */
    OPURE_TP_PEER = 2         /* opure_gemv_allreduce / opure_peer_argmax over NVLink peer
                                 memory at any rank count (NCCL if it cannot be mapped)    */
};

enum {
    OPURE_PATH_AUTO = 0,      /* fused latency kernels when eligible, else per-op kernels */
    OPURE_PATH_UNFUSED = 1,   /* per-op kernels: GEMV, RoPE+KV, attention, GEMV, ...      */
    OPURE_PATH_FUSED = 2,     /* opure_decode_fused; creation fails when not eligible     */
    OPURE_PATH_FUSED_LAYERS = 3 /* opure_decode_fused as three kernels per layer (never the
                                   persistent single-kernel step)                        */
};

typedef struct opure_engine_info {
    uint32_t vocab, hidden, inter, layers, heads, kv_heads, head_dim, max_pos;
    uint32_t max_len, max_batch, page_size, w_dtype;
    uint64_t weight_bytes;        /* resident weight arena                              */
    uint64_t stream_bytes;        /* weight bytes one decode step reads                 */
    uint64_t kv_bytes_per_token;  /* fp16 K+V, all layers, one sequence                 */
    uint32_t tp_ranks;            /* tensor-parallel ranks (1 without a communicator)     */
    uint32_t tp_peer;             /* 1: collectives run as NVLink peer kernels, 0: NCCL   */
} opure_engine_info;

typedef struct opure_generate_timing {
    double prefill_ms;            /* device time of the prefill steps                   */
    double decode_ms;             /* device time of the decode steps                    */
    uint32_t prefill_steps, decode_steps;
} opure_generate_timing;

opure_status opure_engine_create(const char *model_dir, int device,
                                 const opure_engine_options *opts, opure_engine **out);
opure_status opure_engine_destroy(opure_engine *e);
const char *opure_engine_last_error(opure_engine *e);
opure_status opure_engine_get_info(opure_engine *e, opure_engine_info *info);
opure_ctx *opure_engine_ctx(opure_engine *e);

/* Generate (Opure_VoxelEngine.cpp:894-958) for n_seq independent prompts: prompts are
 * concatenated in `prompts`, prompt_lens[n_seq] gives each length; each sequence gets up
 * to `budget` greedy tokens in out_tokens[n_seq][budget]. Prefill and decode run on the
 * device with no per-token host round trip. The reference's stop rules hold per sequence:
 * generation ends after the stop id (config.json's eos_token_id; the reference uses its
 * tokenizer's <|endoftext|>, :904,925-930), which is kept as the last token, or once
 * prompt + generated tokens reach max_position_embeddings (:932); entries after a
 * sequence's last token are -1. timing may be NULL. */
opure_status opure_engine_generate(opure_engine *e, const int32_t *prompts, const uint32_t *prompt_lens,
                                   uint32_t n_seq, uint32_t budget, int32_t *out_tokens,
                                   opure_generate_timing *timing);
/* opure_engine_generate that also reports each sequence's token count (counts[n_seq]) and
 * whether the stop id ended it (hit_stop[n_seq]: GenerateResult.hitStop, :103-104); either
 * may be NULL. */
opure_status opure_engine_generate_stop(opure_engine *e, const int32_t *prompts, const uint32_t *prompt_lens,
                                        uint32_t n_seq, uint32_t budget, int32_t *out_tokens, uint32_t *counts,
                                        uint32_t *hit_stop, opure_generate_timing *timing);

/* Prefill of one sequence (slot 0) ahead of host-driven decode steps (:682-710); `next`
 * (may be NULL) receives the argmax of the last prompt position (ArgMaxFrom, :962-988). */
opure_status opure_engine_prefill(opure_engine *e, const int32_t *tokens, uint32_t n, int32_t *next);
/* One host-driven step for sequences 0..n-1: tokens[i] at positions[i] in, next[i] out
 * (DecodeStep, Opure_VoxelEngine.cpp:765-800: copy in, one step, 8-byte readback). */
opure_status opure_engine_decode_step(opure_engine *e, const int32_t *tokens, const int32_t *positions,
                                      uint32_t n, int32_t *next);

/* Device-resident decoding after opure_engine_generate: enqueues `steps` replays of the
 * step graph for sequences 0..n-1 (self-driving greedy, no host round trip) and returns
 * without waiting; opure_engine_set_positions rewinds positions (tokens already in the
 * history are then re-fed rather than re-chosen); opure_engine_sync waits for the stream
 * and reports any device-side failure. */
opure_status opure_engine_run_steps(opure_engine *e, uint32_t n, uint32_t steps);
opure_status opure_engine_set_positions(opure_engine *e, const int32_t *positions, uint32_t n);
opure_status opure_engine_sync(opure_engine *e);

/* ForwardLogits / ForwardArgMax (Opure_VoxelEngine.cpp:803-821, :879-891). */
opure_status opure_engine_forward_logits(opure_engine *e, const int32_t *tokens, uint32_t n, float *logits);
opure_status opure_engine_forward_argmax(opure_engine *e, const int32_t *tokens, uint32_t n, int32_t *out);

/* RunLayersTraced (Opure_VoxelEngine.cpp:546-587): residual after each of the first
 * n_layers layers for `token` at position 0, into trace[n_layers][hidden]. */
opure_status opure_engine_trace(opure_engine *e, int32_t token, uint32_t n_layers, float *trace);

/* Fills the activation buffers with `value` (PoisonBanks, :625-636). */
opure_status opure_engine_poison(opure_engine *e, float value);

/* Loads precomputed fp16 K/V [layers][2][kv_heads][len][head_dim] into sequence slot `seq`
 * (synthetic long contexts for the large-model configuration). */
opure_status opure_engine_load_kv(opure_engine *e, uint32_t seq, const uint16_t *kv, uint32_t len);

/* Synthetic long contexts (config 4's 4096-token contexts without a prefill): slots
 * 0..n-1 get `len` cached positions of seeded KV values (opure_kv_synth), `reserve`
 * positions of KV pages, and continue self-driving (opure_engine_run_steps) from position
 * len with first_tokens[v] as input. opure_engine_read_tokens copies `count` tokens of a
 * slot's history from position `pos`. */
opure_status opure_engine_synth_context(opure_engine *e, uint32_t n, uint32_t len, uint32_t reserve,
                                        uint64_t seed, const int32_t *first_tokens);
opure_status opure_engine_read_tokens(opure_engine *e, uint32_t slot, uint32_t pos, uint32_t count,
                                      int32_t *out);

/* Tensor-parallel shard (the large-model configuration's 8-way TP at batch 1): the
 * engine enqueues on `ctx` (which the caller created and keeps) and is rank r of n of
 * `comm` (opure_comm_init on the same ctx). It holds q/k/v and gate/up rows, o_proj and
 * down_proj columns and lm_head vocabulary rows of its shard, caches its KV heads, and
 * each step all-reduces the o_proj and down_proj partial sums (fp32 sum) and the argmax
 * keys (u64 max) over NCCL. Every rank must make the same calls in the same order.
 * stream_bytes and kv_bytes_per_token of opure_engine_get_info are the shard's. */
opure_status opure_engine_create_tp(const char *model_dir, opure_ctx *ctx, opure_comm *comm,
                                    const opure_engine_options *opts, opure_engine **out);

/* VoxelEngine::SnapshotMetrics (Opure_VoxelEngine.h MetricsSnapshot, Opure_VoxelEngine.cpp:
 * 640-670): KV page occupancy, tokens/s of the last generation's decode steps, memory
 * pressure (0: the KV pool is fixed at creation), and the speculative acceptance rate of the
 * last opure_engine_spec_generate this engine was the target of (-1 before any; the
 * reference fixes it at -1, :666); `position` is CurrentPosition(). */
typedef struct opure_engine_metrics {
    float kv_occupancy, tokens_per_sec, memory_pressure, speculative_acceptance;
    uint32_t position;
} opure_engine_metrics;
opure_status opure_engine_snapshot_metrics(opure_engine *e, opure_engine_metrics *m);

/* The last persistent decode step's per-CTA %globaltimer stamps (layout of
 * opure_fused_step.trace: [sm_count][3 layers + 2][2]); needs options.phase_trace = 1.
 * Copies at most `cap` words; *written gets the count (0 without tracing). */
opure_status opure_engine_phase_trace(opure_engine *e, uint64_t *out, size_t cap, size_t *written);

/* ---- speculative decoding (no reference counterpart: the reference's verify shader,
 *      Opure_SpeculativeDecode.usf:60-189, is never dispatched and it has no draft loop
 *      or accept rule; speculativeAcceptance is fixed at -1, Opure_VoxelEngine.cpp:666) */

/* An engine that enqueues on `share`'s ctx (stream) instead of its own, so a draft and a
 * target engine can hand data to each other in stream order. `share` must outlive it. */
opure_status opure_engine_create_shared(const char *model_dir, opure_engine *share,
                                        const opure_engine_options *opts, opure_engine **out);

typedef struct opure_spec_options {
    uint32_t k;               /* draft tokens per round (1..64)                         */
    uint32_t mode;            /* OPURE_SPEC_GREEDY or OPURE_SPEC_REJECTION (temperature 1) */
    uint64_t seed;            /* sequence s draws uniforms from Rng(seed ^ s * 0x9E3779B97F4A7C15) */
    int32_t *draft_log;       /* NULL, or [draft_log_rounds][n_seq][k]: each round's drafted
                                 tokens d_1..d_k per sequence (-1 for a finished sequence;
                                 rounds past the last are filled with -2)               */
    uint32_t draft_log_rounds;
} opure_spec_options;

typedef struct opure_spec_stats {
    uint32_t rounds;
    uint64_t drafted, accepted;   /* proposals to still-generating sequences, accepted   */
    double draft_ms, verify_ms, total_ms;   /* device time of draft steps, verify + accept */
} opure_spec_stats;

/* Speculative decoding of n_seq prompts of length prompt_len (concatenated in `prompts`)
 * into out_tokens[n_seq][budget]: per round the draft engine proposes k tokens per
 * sequence, the target verifies the k+1 positions of all sequences in one batched step,
 * and opure_spec_accept keeps the accepted prefix plus one target token. `draft` must be
 * created with opure_engine_create_shared(…, target, …); target max_batch >= n_seq (k+1),
 * draft max_batch >= n_seq, both max_len >= prompt_len + budget + k + 2. accept_log
 * (may be NULL) receives up to accept_log_rounds rounds of n_seq accepted counts (-1 for
 * a finished sequence); stats may be NULL. */
opure_status opure_engine_spec_generate(opure_engine *target, opure_engine *draft, const int32_t *prompts,
                                        uint32_t prompt_len, uint32_t n_seq, uint32_t budget,
                                        const opure_spec_options *o, int32_t *out_tokens,
                                        int32_t *accept_log, uint32_t accept_log_rounds,
                                        opure_spec_stats *stats);

typedef struct opure_sample_options {
    float temperature;        /* <= 0: greedy                                           */
    uint32_t top_k;           /* 0: off                                                 */
    float top_p;              /* (0, 1]; 1: off                                         */
    float rep_penalty;        /* > 0; 1: off                                            */
    uint64_t seed;            /* sequence s draws uniforms from Rng(seed ^ s * 0x9E3779B97F4A7C15) */
} opure_sample_options;

/* Sampled generation of n_seq prompts of length prompt_len (concatenated in `prompts`) into
 * out_tokens[n_seq][budget]: after the prompt, each token is drawn on the device by
 * opure_sample_filtered (temperature, top-k, top-p, repetition penalty over the sequence so
 * far; the reference declares these in GenerationConfig, src/proto/opure.proto:35-46,
 * without implementing them) from its position's logits with the next uniform of the
 * sequence's stream, and is the next step's input. stats (may be NULL) receives
 * [n_seq][budget][4] opure_logit_stats of those logits: max, L2 norm, entropy (nats),
 * log-sum-exp (the reference's RefreshLogitStats, Opure_VoxelEngine.cpp:832-876); logits
 * (may be NULL; costly) the logits themselves, [n_seq][budget][vocab].
 * max_batch >= n_seq, max_len >= prompt_len + budget + 1. */
opure_status opure_engine_sample_generate(opure_engine *e, const int32_t *prompts, uint32_t prompt_len, uint32_t n_seq,
                                          uint32_t budget, const opure_sample_options *o, int32_t *out_tokens,
                                          float *stats, float *logits);

/* Parses config.json, maps model.safetensors, resolves tensor roles and plans the device
 * layout without touching a GPU (the reference's opure_inspect tool, Opure_Inspect.cpp).
 * On failure the reason is copied to err (err_len bytes, may be NULL). */
opure_status opure_model_inspect(const char *model_dir, opure_engine_info *info, char *err, size_t err_len);

/* ---- serving front end (the reference's HTTP server, src/app/Opure_Server.cpp) ---------
 * GET /health, POST /generate, GET /metrics on 127.0.0.1:port (0: any free port), with one
 * engine per listed device serving requests concurrently (the reference serves one at a
 * time on its one device, :21-25). /generate takes {"tokens": [ids], "max_tokens": n
 * (clamped to 1..2048), "temperature": t (> 0: sampled), "seed": s} and answers
 * {"tokens": [...], "prompt_tokens", "generated_tokens", "ms_per_token", "total_ms",
 * "hit_stop", "engine"}; there is no tokenizer, so a text "prompt" is refused with 400.
 * Bodies over 1 MiB: 413; unknown routes 404; wrong methods 405; chunked bodies 400;
 * /generate with no engine (n_devices 0): 503. */
typedef struct opure_server opure_server;
opure_status opure_server_start(const char *model_dir, const int *devices, uint32_t n_devices, uint16_t port,
                                const opure_engine_options *opts, opure_server **out);
uint16_t opure_server_port(const opure_server *s);
/* Stops accepting, finishes the requests in hand, joins the workers, frees the engines. */
opure_status opure_server_stop(opure_server *s);
/* The /generate body parser on its own: token ids into tokens[cap] (n_tokens gets the
 * count), the clamped max_tokens and temperature; on a malformed body returns
 * OPURE_ERR_INVALID_ARG with the client-facing message in err. vocab 0: ids unchecked. */
opure_status opure_server_parse_generate(const char *body, size_t len, uint32_t vocab, int32_t *tokens,
                                         uint32_t cap, uint32_t *n_tokens, uint32_t *max_tokens,
                                         float *temperature, char *err, size_t err_len);

/* ---- seeded synthetic inputs (the reference downloads a checkpoint instead,
 *      scripts/fetch_model.ps1) ---------------------------------------------- */
typedef struct opure_synth_spec {
    uint32_t vocab, hidden, inter, layers, heads, kv_heads, max_pos;
    float eps;
    double theta;
    uint32_t tied;            /* 1: lm_head is the embedding                          */
    uint64_t seed;            /* weights N(0, std), xorshift64 + Box-Muller, fp16 RNE  */
    float std;
    uint32_t int8;            /* 1: matrices as per-tensor int8 + "scale" header key   */
    uint64_t noise_seed;      /* draft models: + N(0, noise_std) per matrix element    */
    float noise_std;
} opure_synth_spec;

opure_status opure_synth_model(const char *dir, const opure_synth_spec *spec);
opure_status opure_synth_normal_f16(uint64_t seed, float stddev, uint64_t n, uint16_t *out);
opure_status opure_synth_prompt(uint64_t seed, uint32_t vocab, uint32_t n, int32_t *out);
opure_status opure_synth_permutation(uint64_t seed, uint32_t n, int32_t *out);
opure_status opure_synth_uniforms(uint64_t seed, uint64_t n, float *out);
/* Host form of opure_kv_synth for one slot: [layers][2][n_kv][len][head_dim] fp16. */
opure_status opure_synth_kv(uint64_t seed, uint32_t slot, uint32_t layers, uint32_t n_kv, uint32_t len,
                            uint32_t head_dim, uint16_t *out);

#ifdef __cplusplus
}
#endif
#endif /* OPURE_ENGINE_H */
