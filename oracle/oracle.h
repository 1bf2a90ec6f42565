/*
 * oracle.h -- CPU restatement of Opure-VoxelEngine's decode path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA
 * path: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
 * reference legs may load it. Nothing in the product links it or calls it.
 *
 * Every function restates the reference's scalar C++ CPU path
 * (src/engine/Opure_CpuReference.cpp) or, where that file has no counterpart,
 * the semantics of the reference shader named beside it. Citations are
 * path:line inside the reference project.
 *
 * Pinning: the reference ships no golden files. Its known-answer tests are the
 * seeded generated kernel tests of src/app/Opure_TestHarness.cpp, whose expected
 * values the harness computes inline in fp32. tests/test_oracle_pin.py checks this
 * oracle against a restatement of those inline computations on the same seeded
 * inputs (committed as .npz fixtures under tests/golden), using the harness's own pass criterion
 * (Compare, :70-101). The reference's CpuReference translation units include
 * <windows.h> and cannot be compiled here, so there is no oracle/_ref build.
 * Semantics the reference does not define at all -- the paged KV layout, the int8
 * quantiser, speculative accept/reject and softmax sampling -- are "parity unpinned":
 * they are restated from the published methods named at each function.
 */
#ifndef OPURE_ORACLE_H
#define OPURE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- deterministic data ------------------------------------------------ */

/* xorshift64 stream of NextU32() values, Opure_TestHarness.cpp:36-47 (seed 0 -> 1). */
void orc_rng_u32_stream(uint64_t seed, uint64_t n, uint32_t *out);

/* ---- IEEE binary16 ------------------------------------------------------ */
uint16_t orc_f32_to_f16(float f);           /* round to nearest even */
float    orc_f16_to_f32(uint16_t h);        /* exact, Opure_Streamer.cpp:49-84 */
void     orc_f32_to_f16_n(const float *src, uint16_t *dst, uint64_t n);
void     orc_f16_to_f32_n(const uint16_t *src, float *dst, uint64_t n);

/* ---- kernels ------------------------------------------------------------ */

/* y[v][o] = float(sum_i double(W[o][i]) * double(x[v][i])), Opure_CpuReference.cpp:151-161.
 * W is row-major [rows, cols] fp16; x is [nvec][cols]; y is [nvec][rows]. */
void orc_gemv_f16(const uint16_t *w, const float *x, float *y,
                  uint32_t rows, uint32_t cols, uint32_t nvec);
void orc_gemv_f32(const float *w, const float *x, float *y,
                  uint32_t rows, uint32_t cols, uint32_t nvec);

/* y = scaleW * scaleX * sum q[o][i] * x[i], shaders/Opure_GEMV_Quant.usf:52-93, with the
 * sum in double as the CPU reference accumulates. q is row-major int8 [rows, cols];
 * packed four to a little-endian word this is the shader's byte order
 * (byte k of word w = element 4w+k, Opure_TestHarness.cpp:1259-1265). */
void orc_gemv_q8(const int8_t *q, float scale_w, float scale_x, const float *x, float *y,
                 uint32_t rows, uint32_t cols, uint32_t nvec);

/* Per-tensor symmetric int8 quantiser. The reference consumes pre-quantised int8 plus a
 * header scale and defines no quantiser (parity unpinned): scale = absmax/127 (1 for an
 * all-zero tensor), q = clamp(round_half_even(w/scale), -127, 127). */
void orc_quantize_q8(const uint16_t *w_f16, uint64_t n, int8_t *q, float *scale);

/* y = float(double(x) * inv * double(g)), inv = 1/sqrt(sum x^2 / d + eps),
 * Opure_CpuReference.cpp:163-169. x and y may alias. */
void orc_rmsnorm(const float *x, const float *g, float *y, uint32_t d, float eps);

/* Interleaved-pair RoPE in place on [nheads][hd], structure Opure_CpuReference.cpp:171-189.
 * Frequency theta^(-2*pair/hd) as shaders/Opure_RoPE.usf:56; cpu_literal=1 uses the CPU
 * file's theta^(-2*i/hd) with i = 2*pair instead. */
void orc_rope(float *vec, uint32_t nheads, uint32_t hd, uint32_t pos, double theta,
              int cpu_literal);

/* h = (g * s) * u, s = 1/(1+exp(-g)) in float, Opure_CpuReference.cpp:191-198. */
void orc_swiglu(const float *g, const float *u, float *h, uint32_t n);

/* Lowest index of the largest value per row; NaN never wins (strict >), as the
 * harness's linear scans, Opure_TestHarness.cpp:990-1002,1443-1448. An all-NaN row
 * yields index 0 and value -inf. */
void orc_argmax(const float *x, uint32_t n, uint32_t rows, uint32_t *idx, float *val);

/* Paged decode attention, exact two-pass softmax in double with the float-rounded
 * running output of Opure_CpuReference.cpp:259-305; GQA kv = h / (nH/nKV); score
 * scaled by `scale` (the reference applies none: 1.0).
 *
 * KV pool layout (one layer; parity unpinned, the reference has no pages):
 *   K(page p, kv head g, slot t, dim d) at ((p*2 + 0)*nKV + g)*P*hd + t*hd + d,
 *   V(page p, kv head g, slot t, dim d) at ((p*2 + 1)*nKV + g)*P*hd + t*hd + d.
 * page_table is [nseq][max_pages]; query j of sequence b (q is [nseq][nq][nH][hd])
 * attends to the first seq_lens[b] + j keys (causal multi-query when nq > 1). */
void orc_attention_paged(const float *q, const uint16_t *pool, const int32_t *page_table,
                         const uint32_t *seq_lens, uint32_t nseq, uint32_t nq,
                         uint32_t max_pages, uint32_t page_size, uint32_t n_heads,
                         uint32_t n_kv, uint32_t hd, float scale, float *out);

/* The same attention over the reference's own fp32 cache layout, one plane each for K
 * and V of [nKV][max_seq][hd] (Opure_CpuReference.h:97, Opure_RoPE.usf:106-108):
 * the form the harness's attention test uses. q and out are [nH][hd]. */
void orc_attention_f32(const float *q, const float *k_plane, const float *v_plane,
                       uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t max_seq,
                       uint32_t seq_len, float scale, float *out);

/* Inverse-CDF draw from softmax(logits) at temperature 1 (parity unpinned): the
 * smallest x with sum_{y<=x} exp(l_y - max) > u * Z, sums in double in index order. */
uint32_t orc_sample_softmax(const float *logits, uint32_t vocab, float u);

/* Filtered sampling (parity unpinned: the reference declares temperature, top_p, top_k
 * and repetition_penalty in src/proto/opure.proto:35-46 but implements none of them).
 * Restates, sequentially, the rules of opure_sample_filtered: penalty on tokens of
 * hist[0, hist_len); greedy when T <= 0 or top_k == 1; keys sorted descending (value,
 * then lower index); top-k prefix; masses round(exp(l/T - max) * 2^40) as uint64; top-p
 * prefix reaching ceil(top_p * Z); draw = smallest index whose running kept mass exceeds
 * floor(u * Z_kept). */
uint32_t orc_sample_filtered(const float *logits, uint32_t vocab, float temperature, uint32_t top_k,
                             float top_p, float rep_penalty, const int32_t *hist, uint32_t hist_len,
                             float u);

/* Logit statistics of VoxelEngine::RefreshLogitStats (src/engine/Opure_VoxelEngine.cpp:
 * 832-876): out = {max, sqrt(sum l^2), entropy in nats, max + log(sum exp(l - max))};
 * NaN logits are skipped for the max. */
void orc_logit_stats(const float *logits, uint32_t vocab, float *out);

/* Speculative accept/reject (the reference has none; parity unpinned).
 * Greedy: accepted = longest prefix with argmax(target_logits[i]) == draft[i]; the
 * token after it is argmax(target_logits[accepted]).
 * Rejection sampling at T=1 (Leviathan, Kalman & Matias 2023; Chen et al. 2023), with
 * p = softmax(target_logits[i]) and q = softmax(draft_logits[i]) in double: draft[i] is
 * accepted when u_accept[i] * q(draft[i]) <= p(draft[i]). At the first rejection the
 * replacement is the inverse-CDF draw from max(0, p - q) with u_final (from p when that
 * residual is all zero); with every draft accepted, the bonus token is the inverse-CDF
 * draw from softmax(target_logits[k]) with u_final.
 * target_logits is [k+1][V], draft_logits [k][V]; out_tokens gets accepted+1 ids.
 * Both return the accepted count. */
int orc_spec_accept_greedy(const float *target_logits, const uint32_t *draft, uint32_t k,
                           uint32_t vocab, uint32_t *out_tokens);
int orc_spec_accept_rejection(const float *target_logits, const float *draft_logits,
                              const uint32_t *draft, const float *u_accept, float u_final,
                              uint32_t k, uint32_t vocab, uint32_t *out_tokens);

/* ---- whole model ------------------------------------------------------- */

typedef struct {
    uint32_t vocab, hidden, inter, layers, heads, kv_heads, max_pos;
    float    eps;
    double   theta;
    float    attn_scale;        /* 1.0 = reference semantics */
    int32_t  rope_cpu_literal;  /* 0 = shader frequencies */
} orc_config;

enum {
    ORC_EMBED = 0, ORC_FINAL_NORM = 1, ORC_LM_HEAD = 2,
    ORC_IN_NORM = 3, ORC_POST_NORM = 4, ORC_WQ = 5, ORC_WK = 6, ORC_WV = 7,
    ORC_WO = 8, ORC_GATE = 9, ORC_UP = 10, ORC_DOWN = 11
};
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_BF16 = 2, ORC_I8 = 3 };

typedef struct orc_model orc_model;
typedef struct orc_state orc_state;

orc_model *orc_model_create(const orc_config *cfg);
/* Copies a tensor in. Role ORC_LM_HEAD is optional (tied to ORC_EMBED when absent).
 * Matrices may be F16, F32, BF16 or I8 (with its per-tensor scale); norm gains and the
 * embedding must be floating point. Returns 0 on success, -1 on a bad role/shape. */
int  orc_model_set_tensor(orc_model *m, int role, int layer, int dtype, const void *data,
                          uint64_t nelem, float scale);
/* 0 when every required tensor is present. */
int  orc_model_ready(const orc_model *m);
void orc_model_free(orc_model *m);

/* One sequence's KV cache (contiguous, [L][K|V][nKV][max_pos][hd] as the reference's
 * Opure_CpuReference.h:97, but holding fp16 values: the CUDA path's cache is fp16, so
 * K and V are rounded to fp16 on append). */
orc_state *orc_state_create(const orc_model *m, uint32_t max_pos);
void       orc_state_free(orc_state *s);
uint32_t   orc_state_len(const orc_state *s);
void       orc_state_truncate(orc_state *s, uint32_t len);
/* Sliding window (parity unpinned: the reference's eviction, EvictOldestKV in
 * Opure_VoxelEngine.cpp:721-763, shifts the cache by one token and is never reached):
 * the token at position t attends to positions [w0, t], w0 = max(0, t / page_size -
 * ring + 1) * page_size, as opure_kv_layout.ring. ring 0: off. */
void       orc_state_set_window(orc_state *s, uint32_t page_size, uint32_t ring);
/* Loads `len` positions of precomputed fp16 K/V, laid out [L][2][nKV][len][hd]. */
int        orc_state_load_kv(orc_state *s, const uint16_t *kv, uint32_t len);

/* One token at position orc_state_len(s), Opure_CpuReference.cpp:219-345.
 * logits [vocab] and trace [layers][hidden] (residual after each layer) may be NULL. */
int orc_forward(const orc_model *m, orc_state *s, uint32_t token, float *logits, float *trace);

/* Greedy Generate, Opure_VoxelEngine.cpp:894-958: prefill, argmax, then `budget`
 * iterations of push/DecodeStep (stop when seqLen + 1 >= max_pos). Returns the number
 * of tokens written to `out`; margins (top1 - top2 logit behind each) may be NULL. */
int orc_generate(const orc_model *m, const uint32_t *prompt, uint32_t n_prompt,
                 uint32_t budget, uint32_t max_pos, uint32_t *out, float *margins);

/* Generate with both of the reference's stop rules (Opure_VoxelEngine.cpp:894-958): the
 * token predicted from the last prompt position is pushed first; after each push the loop
 * ends when that token is `eos` (:925-930; eos < 0: no stop id) or when seqLen + 1 >=
 * max_pos (:932), else one decode step follows. Returns the tokens written (<= budget);
 * *hit_stop (may be NULL) is 1 when the stop id ended it. */
int orc_generate_stop(const orc_model *m, const uint32_t *prompt, uint32_t n_prompt, uint32_t budget,
                      uint32_t max_pos, int64_t eos, uint32_t *out, float *margins, int *hit_stop);

/* orc_generate_stop for n_seq independent sequences (prompts concatenated, prompt_lens
 * each), one sequence per host thread at a time on `threads` threads, each computing
 * serially: out [n_seq][budget], counts [n_seq] tokens each, margins (may be NULL)
 * [n_seq][budget] top-1 minus top-2 logit behind each token, second (may be NULL)
 * [n_seq][budget] the top-2 token (lowest index among equal values). Results equal the
 * one-at-a-time ones. 0 on success. */
int orc_generate_batch(const orc_model *m, const uint32_t *prompts, const uint32_t *prompt_lens,
                       uint32_t n_seq, uint32_t budget, uint32_t max_pos, int64_t eos, int threads,
                       uint32_t *out, uint32_t *counts, float *margins, uint32_t *second);

/* Worker threads for the row loops of GEMV and the head loop of attention. Rows are
 * independent, so results are identical for any thread count. */
void orc_set_threads(int n);
int  orc_get_threads(void);
/* on = 1: the calling thread computes serially and never uses the worker pool (for
 * callers that run independent sequences on threads of their own). */
void orc_thread_serial(int on);

/* ---- seeded synthetic inputs ------------------------------------------------
 * The benchmark configurations' random-init models and inputs, generated here so the
 * CPU side (parity checks, the reference arm of the benchmark) needs nothing of the
 * product: the harness's xorshift64 Rng (Opure_TestHarness.cpp:36-47, seed 0 -> 1);
 * normals by Box-Muller on pairs of open uniforms (NextU32() + 0.5) / 2^32, r cos(a)
 * then r sin(a); fp16 by round-to-nearest-even. tests/ check these bytes against the
 * engine's own generators. */
void orc_synth_normal_f16(uint64_t seed, float stddev, uint64_t n, uint16_t *out);
void orc_synth_prompt(uint64_t seed, uint32_t vocab, uint32_t n, int32_t *out);   /* NextU32() % vocab */
void orc_synth_permutation(uint64_t seed, uint32_t n, int32_t *out);              /* Fisher-Yates */
void orc_synth_uniforms(uint64_t seed, uint64_t n, float *out);                   /* NextU32() / 2^32 */

typedef struct {
    uint64_t seed;        /* matrices N(0, std) in file order                             */
    float    std;
    uint32_t tied;        /* 1: lm_head is the embedding                                   */
    uint32_t int8;        /* 1: matrices (not the embedding / untied head) per-tensor int8 */
    uint64_t noise_seed;  /* draft models: each element + N(0, noise_std), noise_std > 0   */
    float    noise_std;
} orc_synth;

/* A random-init model built in memory: the embedding, then per layer q, k, v, o, gate,
 * up, down (then the untied lm_head) drawn in that order from one normal stream, each
 * element fp16(N(0, std)) (+ the noise stream's N(0, noise_std), re-rounded to fp16);
 * norm gains 1.0. NULL on a bad configuration. */
orc_model *orc_model_create_synth(const orc_config *cfg, const orc_synth *spec);

#ifdef __cplusplus
}
#endif
#endif
