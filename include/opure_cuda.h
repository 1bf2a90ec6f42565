/*
 * opure_cuda.h -- C ABI of libopure_cuda.so, the B200 (sm_100a) kernel layer.
 *
 * This library replaces the reference's GPU layers L1 + L2: the Direct3D 12
 * device (src/core/Opure_Dx12.h:144-337: GpuBuffer, Device upload/readback,
 * CommandScope::{SetPipeline,SetParams,Dispatch,Barrier}) and the HLSL kernel
 * library (src/core/Opure_Shaders.h:23-128, the shaders/ directory). Where the reference
 * addresses tensors as 32-bit word offsets into five bound buffers plus bank ids
 * (shaders/Opure_Common.hlsl:35-96), this ABI takes plain device pointers,
 * element counts and explicit dtypes.
 *
 * Conventions
 *  - Every call returns an opure_status; nothing throws across the ABI.
 *  - One opure_ctx per GPU, owning one CUDA stream. Kernel calls enqueue on that
 *    stream and return immediately; opure_sync() waits with a deadline. A ctx is
 *    not thread-safe: use one host thread per ctx.
 *  - Buffers from opure_alloc are 256-byte aligned (as Opure_Dx12.cpp:113).
 *  - Kernel calls allocate nothing (scratch is caller-provided), so a sequence
 *    of them can be captured into a CUDA graph with opure_graph_begin/end.
 *  - Device-side waits are bounded: a kernel that gives up records
 *    OPURE_ERR_DEVICE_TIMEOUT in the ctx status word (opure_last_error) and
 *    returns; no kernel traps.
 */
#ifndef OPURE_CUDA_H
#define OPURE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum opure_status {
    OPURE_OK = 0,
    OPURE_ERR_INVALID_ARG = 1,    /* bad pointer, size or combination of options   */
    OPURE_ERR_NO_DEVICE = 2,      /* no CUDA device, or not sm_100                  */
    OPURE_ERR_CUDA = 3,           /* a CUDA runtime call failed                     */
    OPURE_ERR_OUT_OF_MEMORY = 4,
    OPURE_ERR_TIMEOUT = 5,        /* host-side bounded wait expired (opure_sync)    */
    OPURE_ERR_DEVICE_TIMEOUT = 6, /* a device-side bounded wait gave up             */
    OPURE_ERR_UNSUPPORTED = 7,    /* shape or option this build has no kernel for   */
    OPURE_ERR_INJECTED = 8,       /* failure injected by opure_debug_inject_failure */
    OPURE_ERR_DEVICE_BOUNDS = 9   /* a kernel's own bounds check refused an index   */
} opure_status;

typedef struct opure_ctx opure_ctx;
typedef struct opure_graph opure_graph;
typedef struct opure_event opure_event;

typedef struct opure_device_info {
    int32_t device;
    int32_t sm_count;
    int32_t cc_major, cc_minor;
    uint64_t hbm_bytes;
    uint64_t l2_bytes;
    uint32_t smem_per_block_optin;
    uint32_t clock_mhz_max;
    char name[96];
} opure_device_info;

/* ---- lifetime (replaces dx12::Device::Initialize/Shutdown, Opure_Dx12.cpp:152-229) */
opure_status opure_init(int device, opure_ctx **out);
opure_status opure_shutdown(opure_ctx *ctx);
opure_status opure_get_device_info(opure_ctx *ctx, opure_device_info *info);
const char *opure_strerror(opure_status s);
/* Reads and clears the device status word that kernels write on a bounds or
 * timeout failure (the reference decodes device-removed reasons instead,
 * Opure_Dx12.cpp:53-81). Synchronises the stream. */
opure_status opure_last_error(opure_ctx *ctx);
/* The same, also returning the failing kernel's site id and offending value (0 if none). */
opure_status opure_last_error_detail(opure_ctx *ctx, uint32_t *where, uint32_t *detail);
/* cudaStream_t of the ctx, for interop. */
void *opure_stream(opure_ctx *ctx);

/* ---- memory (replaces GpuBuffer + UploadToBuffer/ReadbackFromBuffer,
 *      Opure_Dx12.h:144-173, Opure_Dx12.cpp:611-723) ------------------------- */
opure_status opure_alloc(opure_ctx *ctx, size_t bytes, void **dptr);
opure_status opure_free(opure_ctx *ctx, void *dptr);
opure_status opure_alloc_host(opure_ctx *ctx, size_t bytes, void **hptr); /* pinned */
opure_status opure_free_host(opure_ctx *ctx, void *hptr);
opure_status opure_h2d(opure_ctx *ctx, void *dst, const void *src, size_t bytes);
opure_status opure_d2h(opure_ctx *ctx, void *dst, const void *src, size_t bytes);
opure_status opure_d2d(opure_ctx *ctx, void *dst, const void *src, size_t bytes);
/* Byte fill, for poisoning (VoxelEngine::PoisonBanks, Opure_VoxelEngine.cpp:625-636). */
opure_status opure_fill(opure_ctx *ctx, void *dst, uint8_t byte, size_t bytes);
/* Waits for the ctx stream, polling with a deadline (the reference's 30 s fence
 * wait, Opure_Dx12.cpp:459-492, returns OPURE_ERR_TIMEOUT here instead of throwing). */
opure_status opure_sync(opure_ctx *ctx, uint32_t timeout_ms);

/* ---- graphs and timing --------------------------------------------------- */
opure_status opure_graph_begin(opure_ctx *ctx);
opure_status opure_graph_end(opure_ctx *ctx, opure_graph **out);
opure_status opure_graph_launch(opure_ctx *ctx, opure_graph *g);
opure_status opure_graph_free(opure_graph *g);
opure_status opure_event_create(opure_ctx *ctx, opure_event **out);
opure_status opure_event_record(opure_ctx *ctx, opure_event *e);
opure_status opure_event_elapsed_ms(opure_event *start, opure_event *stop, float *ms);
opure_status opure_event_free(opure_event *e);

/* ---- element-wise and reduction kernels ------------------------------------
 * Each mirrors one reference shader; the fused decode path below folds them into
 * GEMV prologues and epilogues, but they stay callable on their own. */

/* out[t][i] = float(embed[tokens[t]][i]); embed fp16 [vocab][d].
 * Replaces EmbeddingMain, shaders/Opure_Embedding.usf:21-35. */
opure_status opure_embedding(opure_ctx *ctx, const uint16_t *embed_f16, uint32_t vocab,
                             const int32_t *tokens, uint32_t n, uint32_t d, float *out);

/* y[v] = x[v] * rsqrt(mean(x[v]^2) + eps) * g, per row of d; g fp16 or NULL (identity).
 * Replaces RMSNormMain, shaders/Opure_RMSNorm.usf:31-79. */
opure_status opure_rmsnorm(opure_ctx *ctx, const float *x, const uint16_t *gain_f16,
                           float *y, uint32_t d, uint32_t rows, float eps);

/* h = silu(g) * u, silu(g) = g * sigmoid(g). Replaces SwiGLUMain, Opure_SwiGLU.usf:19-40. */
opure_status opure_swiglu(opure_ctx *ctx, const float *g, const float *u, float *h, uint32_t n);

/* dst = a + b (dst may alias a or b). Replaces AddResMain, Opure_AddRes.usf:29-43,
 * and AddMain, Opure_Add.usf:14-27. */
opure_status opure_add(opure_ctx *ctx, const float *a, const float *b, float *dst, uint32_t n);

/* Per row: lowest index of the largest value (NaN never wins). Writes the index and
 * value of each of `rows` rows of n logits. Replaces ArgMaxMain, Opure_ArgMax.usf:33-85,
 * with the lowest-index tie rule of the CPU checks (Opure_TestHarness.cpp:990-1002). */
opure_status opure_argmax(opure_ctx *ctx, const float *logits, uint32_t n, uint32_t rows,
                          uint32_t *out_idx, float *out_val);

/* ---- paged KV cache ------------------------------------------------------ *
 * One pool per layer, fp16, laid out [page][K|V][n_kv][page_size][head_dim]: the K
 * (or V) block of one page and kv head is contiguous (page_size*head_dim*2 bytes).
 * page_table is int32 [n_seq][max_pages] of physical page ids. The reference keeps
 * one contiguous fp32 region per layer (Opure_Graph.cpp:396-400) and has no pages. */
typedef struct opure_kv_layout {
    uint16_t *pool;            /* this layer's page pool                          */
    const int32_t *page_table; /* [n_seq][max_pages]                              */
    uint32_t n_pages;          /* pages in the pool (bounds check)                */
    uint32_t max_pages;        /* row length of page_table                        */
    uint32_t page_size;        /* tokens per page: 16, 32, 64 or 128              */
    uint32_t n_kv;             /* KV heads                                        */
    uint32_t head_dim;         /* 64 or 128                                       */
    /* Sliding window (0: off). The first `ring` entries of a sequence's table row are used
     * as a ring: position p lives in page page_table[seq][(p / page_size) % ring], and the
     * attention of a query at position p covers positions [window_begin(p), p] with
     * window_begin(p) = max(0, p / page_size - ring + 1) * page_size, i.e. the last
     * ring - 1 whole pages and the current one; older pages are recycled in place. */
    uint32_t ring;
} opure_kv_layout;

/* Seeded synthetic context: fills positions [0, len) of sequence slots slot0 ..
 * slot0+n_slots-1 of one layer's pool (pages from page_table) with fp16 values
 * v = fp16(4 u - 2), u = (splitmix64(seed ^ slot << 48 ^ i) >> 40) / 2^24, where
 * i = (((layer * 2 + kv_sel) * n_kv + head) * 65536 + pos) * head_dim + d. Lets
 * long-context decode (4096-token contexts) run without a prefill; opure_synth_kv in
 * the engine library produces the same bits on the host. len <= 65536. */
opure_status opure_kv_synth(opure_ctx *ctx, const opure_kv_layout *kv, uint32_t layer,
                            uint32_t slot0, uint32_t n_slots, uint32_t len, uint64_t seed);

/* RoPE + KV append for n token vectors. Row i of `qkv` (row stride `stride` floats) holds
 * [q: n_heads*hd | k: n_kv*hd | v: n_kv*hd], the layout of the fused q;k;v GEMV. q and k are
 * rotated with interleaved-pair RoPE at position pos[i] (frequency theta^(-2*pair/hd) as
 * Opure_RoPE.usf:56; angle, sin/cos and rotation in double as Opure_CpuReference.cpp:171-189);
 * the rotated q goes to q_out [n][n_heads][hd] and the rotated k and raw v are appended as
 * fp16 to the paged cache of sequence seq[i] at slot pos[i].
 * Replaces RoPEMain, shaders/Opure_RoPE.usf:33-115. */
opure_status opure_rope_kv_append(opure_ctx *ctx, const float *qkv, uint32_t stride, float *q_out,
                                  const int32_t *seq, const int32_t *pos, uint32_t n,
                                  uint32_t n_heads, double theta, const opure_kv_layout *kv);

/* Split-K flash-decode attention over the paged fp16 cache, fp32 softmax.
 * Query j of entry i (q is [n][n_q][n_heads][hd] fp32) belongs to sequence seq[i] and
 * attends to keys [0, seq_len[i] + j) -- causal multi-query when n_q > 1 (speculative
 * verify). GQA maps query head h to kv head h / (n_heads / n_kv). Scores are scaled by
 * `scale` (the reference applies none: pass 1.0). Partial results of the key splits are
 * merged inside the kernel by the last CTA of each (entry, kv head).
 * Replaces AttentionMain{32..256}, shaders/Opure_FlashAttention_Decode.usf:58-179.
 *
 * scratch: opure_attention_scratch_bytes(...) bytes of device memory, caller-owned;
 * its counter words must be zero before the first call (opure_fill) and are left
 * zero by every call. */
typedef struct opure_attn_args {
    const float *q;
    float *out;                /* [n][n_q][n_heads][hd] fp32                      */
    const int32_t *seq;        /* [n] sequence index into page_table              */
    const int32_t *seq_len;    /* [n] keys visible to query 0                     */
    uint32_t n, n_q, n_heads;
    float scale;
    uint32_t max_ctx;          /* upper bound of seq_len + n_q - 1 (sizes the grid) */
    uint32_t split_tokens;     /* keys per split; 0 = choose for this device       */
    void *scratch;
    size_t scratch_bytes;
    opure_kv_layout kv;
    /* NULL, or a packed operand (see opure_gemv_args) of the n * n_q output vectors of
     * length n_heads * head_dim, written besides `out`: the o_proj GEMV's x_packed.
     * opure_attention only (opure_attention_static ignores it). */
    uint16_t *out_packed;
} opure_attn_args;
size_t opure_attention_scratch_bytes(uint32_t n, uint32_t n_q, uint32_t n_heads,
                                     uint32_t n_kv, uint32_t head_dim, uint32_t max_ctx,
                                     uint32_t split_tokens);
opure_status opure_attention(opure_ctx *ctx, const opure_attn_args *a);

/* Allocation-free attention. No counterpart in the reference (its attention has no scratch).
 *
 * Same computation and arguments as opure_attention, except that a->scratch and
 * a->scratch_bytes are ignored: the split partials and counters live in a fixed buffer of
 * OPURE_ATTN_STATIC_SCRATCH_BYTES inside this library, which every GPU that loads the
 * library keeps until the process exits. It is for callers that are not allowed to
 * allocate device memory themselves -- for example a plugin inside a host application
 * (the reference plans an engine plugin) whose memory budget is owned by the host, or a
 * real-time decode loop that must never stall on cudaMalloc/cudaFree, which synchronise
 * the device. The call allocates nothing and calls no allocating library routine.
 *
 *  - Returns OPURE_ERR_UNSUPPORTED, without launching, when the call would need more than
 *    OPURE_ATTN_STATIC_SCRATCH_BYTES (compare opure_attention_scratch_bytes for the same
 *    shape against the limit).
 *  - The first call on each device looks up the buffer's device address; make that first
 *    call before capturing a stream into a CUDA graph.
 *  - Every call shares the one buffer and clears the counters it needs on the ctx stream.
 *    Calls that may run at the same time on the GPU (other streams or contexts on the same
 *    device) race on the buffer: serialise them. */
#define OPURE_ATTN_STATIC_SCRATCH_BYTES (8u << 20)
opure_status opure_attention_static(opure_ctx *ctx, const opure_attn_args *a);

/* ---- weight-streaming GEMV --------------------------------------------------
 * y[v][o] = epilogue( sum_i W[o][i] * prologue(x[v])[i] ), W row-major [rows][cols]
 * (the safetensors layout), fp32 accumulation, for nvec in 1..9 input vectors.
 * Replaces GEMVMain (shaders/Opure_GEMV.usf:40-88) and GEMVQuantMain
 * (shaders/Opure_GEMV_Quant.usf:38-94). */
enum {
    OPURE_W_F16 = 0,   /* fp16 weights                                                */
    OPURE_W_Q8 = 1     /* int8 weights, per-tensor scale: y = scale_w*scale_x*sum(q*x) */
};
enum {
    OPURE_PRO_NONE = 0,
    OPURE_PRO_RMSNORM = 1   /* x <- x * rsqrt(mean(x^2) + eps) * gain (fp16 gain)     */
};
enum {
    OPURE_EPI_STORE = 0,    /* y = acc                                                */
    OPURE_EPI_ADD = 1,      /* y = residual + acc (residual may alias y)              */
    OPURE_EPI_SWIGLU = 2,   /* W is [2*rows][cols] = [gate; up]: y = silu(gate) * up  */
    OPURE_EPI_ARGMAX = 3    /* y = acc (if y != NULL) and argmax per vector           */
};
typedef struct opure_gemv_args {
    const void *w;
    uint32_t w_dtype;          /* OPURE_W_F16 / OPURE_W_Q8                      */
    float scale_w, scale_x;    /* OPURE_W_Q8 only                               */
    float scale_w2;            /* OPURE_W_Q8 + OPURE_EPI_SWIGLU: scale of the up half */
    uint32_t rows, cols, nvec;
    const float *x;            /* [nvec][x_stride]                              */
    uint32_t x_stride;
    float *y;                  /* [nvec][y_stride]                              */
    uint32_t y_stride;
    uint32_t prologue;
    const uint16_t *norm_gain; /* [cols] fp16, OPURE_PRO_RMSNORM                */
    float eps;
    uint32_t epilogue;
    const float *residual;     /* OPURE_EPI_ADD: [nvec][y_stride]               */
    /* OPURE_EPI_ARGMAX: packed (value, index) keys, one uint64 per vector, which the
     * caller zeroes first; decode with opure_argmax_decode. */
    unsigned long long *argmax_keys;
    /* Chained tensor-core operands (fp16 weights, 16..256 vectors, cols a multiple of 64;
     * OPURE_ERR_UNSUPPORTED otherwise). A packed operand holds the nvec vectors of length
     * L as fp16 pairs hi = fp16(v), lo = fp16((v - hi) * 2^11): [2][npad][L] halves, hi
     * rows first, npad = nvec rounded up to 16 (opure_packed_bytes). Values must stay
     * below 65504 in magnitude (a larger one is reported as OPURE_ERR_DEVICE_BOUNDS).
     * Zero-initialise new packed buffers once: padding rows are read but never written. */
    const uint16_t *x_packed;  /* non-NULL: the input vectors come from this packed operand
                                  (x may then be NULL). With OPURE_PRO_RMSNORM the packed values
                                  are gain * x, and x_sumsq supplies the norm               */
    const float *x_sumsq;      /* x_packed + OPURE_PRO_RMSNORM: [ceil(cols / 128)][nvec] partial
                                  sums of squares of x (a producer's y_sumsq)               */
    uint16_t *y_packed;        /* non-NULL: also write the output vectors (STORE: y, ADD: the
                                  new residual, SWIGLU: the activation) as a packed operand
                                  [2][npad][rows], each value times y_pack_gain[row] if given */
    const uint16_t *y_pack_gain; /* [rows] fp16 or NULL: the next GEMV's RMSNorm gain        */
    float *y_sumsq;            /* [ceil(rows / 128)][nvec] or NULL: per 128-row block, the sum
                                  of squares of the output vectors (before y_pack_gain)      */
} opure_gemv_args;
/* Bytes of a packed operand of nvec vectors of length len (see opure_gemv_args). */
size_t opure_packed_bytes(uint32_t nvec, uint32_t len);
opure_status opure_gemv(opure_ctx *ctx, const opure_gemv_args *a);
/* Decodes OPURE_EPI_ARGMAX keys into (index, value) on the device. */
opure_status opure_argmax_decode(opure_ctx *ctx, const unsigned long long *keys, uint32_t n,
                                 uint32_t *out_idx, float *out_val);

/* ---- decode-step bookkeeping ----------------------------------------------------
 * A decode step computes one token vector per entry. opure_step_begin / opure_step_end
 * bracket the per-layer kernels of a step so that a captured step graph replays with no
 * host work: begin picks each vector's token (from the token history, or for a
 * self-driving greedy vector past its known tokens, from the previous step's argmax key),
 * records it, clears the key, publishes seq_len = pos + 1 and gathers the embedding row
 * into the residual stream (EmbeddingMain, Opure_Embedding.usf:21-35); end advances the
 * positions of self-driving vectors. This is the reference's DecodeStep/ArgMaxFrom loop
 * (Opure_VoxelEngine.cpp:765-800, :962-988) without the per-token host round trip. */
enum { OPURE_VEC_AUTO = 1 };
typedef struct opure_step_io {
    uint32_t nvec;
    const int32_t *seq;        /* [nvec] sequence slot (page-table / token-history row) */
    int32_t *pos;              /* [nvec] position computed by this step                  */
    int32_t *seq_len;          /* [nvec] written by begin: pos + 1                       */
    int32_t *known;            /* [nvec] tokens[seq][0, known) are valid                 */
    const uint32_t *flags;     /* [nvec] OPURE_VEC_AUTO or 0 (token given by the host)   */
    const int32_t *in_tokens;  /* [nvec] or NULL: token of each non-AUTO vector, recorded
                                  into the history at pos (NULL: read the history)        */
    int32_t *tokens;           /* [slots][max_len] token history                        */
    uint32_t max_len;
    unsigned long long *keys;  /* [nvec] argmax keys of the previous step's lm_head       */
    const uint16_t *embed;     /* fp16 [vocab][hidden]                                   */
    uint32_t vocab, hidden;
    float *x;                  /* [nvec][hidden] residual stream, written by begin        */
} opure_step_io;
opure_status opure_step_begin(opure_ctx *ctx, const opure_step_io *io);
opure_status opure_step_end(opure_ctx *ctx, const opure_step_io *io);

/* ---- fused decode step (latency path, 1..8 token vectors, fp16 weights) ---------------
 * Enqueues the whole per-layer graph of one decode step as three kernels per layer plus
 * the lm_head (Opure_VoxelEngine.cpp:189-536 records 14 dispatches per layer):
 *   A  RMSNorm + q;k;v GEMV + RoPE + fp16 paged-KV append      (one CTA per 8 q;k;v rows)
 *   B  paged attention + o_proj partial sums into the residual (one CTA per kv head and
 *      block of o_proj rows; o_proj stored grouped per kv head)
 *   C  RMSNorm + gate;up GEMV + SwiGLU + down_proj partial sums (one CTA per block of the
 *      intermediate dimension; down_proj stored transposed)
 *   L  final RMSNorm + lm_head GEMV + argmax keys (+ logits when `logits` != NULL)
 * Each kernel copies its whole weight slice into shared memory with a TMA bulk copy before
 * waiting on its predecessor (programmatic dependent launch), so weight streaming overlaps
 * the previous kernel. The residual stream is kept as fp32 base vectors plus 64-bit
 * fixed-point (2^-32) deltas that the B and C partial sums are added to atomically, which
 * makes the sums independent of arrival order; each kernel rebuilds x = base + delta.
 * Input: `x` holds the step's embedding rows (opure_step_begin writes them).
 * Requirements: head_dim 64 or 128, n_heads/n_kv <= 4, hidden % 8 == 0, nvec <= 8. */
typedef struct opure_fused_layer {
    const uint16_t *in_norm, *post_norm; /* fp16 [hidden]                                  */
    const uint16_t *w_qkv;      /* [(n_heads + 2 n_kv) head_dim][hidden]: q, k, v rows     */
    const uint16_t *w_o_blk;    /* [n_kv][hidden][G head_dim]: (g, o, c) = Wo[o][g G hd + c] */
    const uint16_t *w_gate_up;  /* [2 inter][hidden]: gate rows then up rows               */
    const uint16_t *w_down_t;   /* [inter][hidden]: down_proj transposed                   */
    uint16_t *kv_pool;          /* this layer's page pool (layout of opure_kv_layout)      */
    /* Per-tensor scales of int8 matrices (opure_fused_step.w_dtype = OPURE_W_Q8; the
     * matrices above then hold int8 in the same layouts): y = scale * sum(q * x). */
    float s_q, s_k, s_v, s_o, s_gate, s_up, s_down;
} opure_fused_layer;

typedef struct opure_fused_step {
    uint32_t nvec, hidden, inter, n_heads, n_kv, head_dim, vocab, n_layers;
    float eps, attn_scale;
    double theta;
    const opure_fused_layer *layers;   /* host array [n_layers], read during the call    */
    const uint16_t *final_norm;        /* fp16 [hidden]                                  */
    const uint16_t *lm_head;           /* fp16 [vocab][hidden]                           */
    const int32_t *page_table;
    uint32_t n_pages, max_pages, page_size;
    const int32_t *seq, *pos;          /* [nvec] (pos = position computed by this step)  */
    float *x;                          /* [nvec][hidden] embedding in, then base buffer 0 */
    float *base1;                      /* [nvec][hidden]                                 */
    long long *delta0, *delta1;        /* [nvec][hidden] fixed-point partial sums         */
    float *q;                          /* [nvec][n_heads head_dim]                        */
    float *logits;                     /* [nvec][vocab] or NULL                          */
    unsigned long long *keys;          /* [nvec] argmax keys (zeroed by opure_step_begin) */
    uint32_t *sync;                    /* [3 n_layers + 1] device words for the persistent
                                          kernel's grid barriers (reset by the call), or NULL */
    uint32_t mode;                     /* OPURE_FUSED_AUTO or OPURE_FUSED_LAYER_KERNELS     */
    unsigned long long *trace;         /* NULL, or [sm_count][3 n_layers + 2][2] words: the
                                          persistent kernel's per-CTA %globaltimer stamps
                                          (row k < 3 n_layers: arrival at / release from grid
                                          barrier k; row 3 n_layers: [1] = kernel start; row
                                          3 n_layers + 1: [0] = end), rewritten every step */
    uint32_t kv_ring;                  /* sliding window of the cache (opure_kv_layout.ring) */
    uint32_t w_dtype;                  /* layer matrices: OPURE_W_F16 (0) or OPURE_W_Q8 (int8
                                          GEMV_Quant, persistent kernel only: head_dim 64,
                                          hidden a multiple of 16, mode AUTO; otherwise
                                          OPURE_ERR_UNSUPPORTED). Embedding, norms and the
                                          lm_head are fp16 either way. */
} opure_fused_step;
/* AUTO: when the model fits (head_dim 64, <= 48 layers, each phase's work in one wave of
 * CTAs, a layer's weight slices of one CTA double-buffered in shared memory) and `sync` is
 * given, the whole step is ONE persistent cooperative kernel (one CTA per SM) whose layer
 * phases meet at bounded grid-wide barriers; otherwise the three kernels per layer above.
 * LAYER_KERNELS: always the three kernels per layer. */
enum { OPURE_FUSED_AUTO = 0, OPURE_FUSED_LAYER_KERNELS = 1 };
opure_status opure_decode_fused(opure_ctx *ctx, const opure_fused_step *s);

/* ---- speculative verify / accept (no reference counterpart: the reference's
 *      SpeculativeVerify pipelines, Opure_SpeculativeDecode.usf:60-189, are never
 *      dispatched and it has no accept logic) ------------------------------- */
enum { OPURE_SPEC_GREEDY = 0, OPURE_SPEC_REJECTION = 1 };
typedef struct opure_spec_args {
    uint32_t mode;
    uint32_t n_seq, k, vocab;
    const float *target_logits; /* [n_seq][k+1][vocab]                          */
    const float *draft_logits;  /* [n_seq][k][vocab]      (rejection only)      */
    const int32_t *draft;       /* [n_seq][k]                                   */
    const float *u_accept;      /* [n_seq][k]             (rejection only)      */
    const float *u_final;       /* [n_seq]                (rejection only)      */
    int32_t *out_tokens;        /* [n_seq][k+1]: accepted drafts + 1 new token  */
    int32_t *out_accepted;      /* [n_seq]                                      */
} opure_spec_args;
opure_status opure_spec_accept(opure_ctx *ctx, const opure_spec_args *a);

/* Inverse-CDF draw per row from softmax(logits) at temperature 1 with uniforms u[row]. */
opure_status opure_sample_softmax(opure_ctx *ctx, const float *logits, uint32_t vocab,
                                  uint32_t rows, const float *u, int32_t *out_tokens);

/* Filtered sampling, one row of logits per sequence (the reference declares temperature,
 * top_p, top_k and repetition_penalty in GenerationConfig, src/proto/opure.proto:35-46,
 * without implementing them). Per row: logits of tokens in hist[seq[row]][0, hist_len[row])
 * are penalised (l / r for l > 0, else l * r); temperature <= 0 or top_k == 1 is greedy
 * (lowest index among the largest); otherwise z = l * (1 / T), top_k keeps the k largest
 * (0: all; ties to the lower index), top_p < 1 keeps the shortest prefix of them, in the
 * same order, whose mass reaches ceil(top_p * Z), and the token is the smallest index whose
 * running kept mass exceeds floor(u[row] * Z_kept). Masses are exp(z - z_max) rounded to
 * nearest in units of 2^-40 and summed as uint64. The token goes to out[row] and/or, as
 * an argmax key, to keys[row] (the next self-driving step's input). vocab <= 2^18. */
typedef struct opure_sample_args {
    const float *logits;       /* [rows][stride]                                        */
    uint32_t vocab, rows;
    size_t stride;             /* floats between rows, >= vocab                         */
    float temperature;
    uint32_t top_k;            /* 0: off                                                */
    float top_p;               /* (0, 1]; 1: off                                        */
    float rep_penalty;         /* > 0; 1: off                                           */
    const int32_t *hist;       /* [slots][max_len] token history, or NULL (no penalty)  */
    uint32_t max_len;
    const int32_t *seq;        /* [rows] history slot of each row, or NULL (slot = row) */
    const int32_t *hist_len;   /* [rows] tokens of the history that count               */
    const float *u;            /* [rows] uniforms in [0, 1) (not read when greedy)      */
    int32_t *out;              /* [rows] or NULL                                        */
    unsigned long long *keys;  /* [rows] or NULL                                        */
} opure_sample_args;
opure_status opure_sample_filtered(opure_ctx *ctx, const opure_sample_args *a);

/* Per row of logits: out[row] = {max logit, L2 norm, softmax entropy (nats), log-sum-exp},
 * as VoxelEngine::RefreshLogitStats (src/engine/Opure_VoxelEngine.cpp:832-876) computes
 * the first three on the host: sqrt(sum l^2) in double; entropy with p = exp(double(l -
 * max)) / sum, accumulated in double. */
opure_status opure_logit_stats(opure_ctx *ctx, const float *logits, uint32_t vocab, uint32_t rows,
                               size_t stride, float *out);

/* The same draw, written as an argmax key into keys[row] so that the next self-driving
 * decode step (OPURE_VEC_AUTO) takes the sampled token as its input: the draft model's
 * sampling step of speculative decoding. With save != NULL row r is also copied to
 * save + r * save_stride (the draft distribution the accept step needs). */
opure_status opure_sample_keys(opure_ctx *ctx, const float *logits, uint32_t vocab, uint32_t rows,
                               const float *u, unsigned long long *keys, float *save,
                               size_t save_stride);

/* Speculative round bookkeeping without a host round trip. For each sequence slot s whose
 * round starts at position base[s]: the draft's proposals d_1..d_k are read from its
 * token history hist[s][base+1 .. base+k-1] (the inputs of its later self-driving steps)
 * and from keys[s] (the last step's result, d_k); writes the target's verify inputs
 * verify_tokens[s][0..k] = (hist[s][base], d_1..d_k) and draft[s][0..k-1] = d_1..d_k. */
opure_status opure_spec_gather(opure_ctx *ctx, const int32_t *hist, uint32_t max_len,
                               const unsigned long long *keys, const int32_t *base, uint32_t n_seq,
                               uint32_t k, int32_t *verify_tokens, int32_t *draft);

/* ---- tensor parallelism (the large-model configuration's 8-way TP at batch 1) --------
 * NCCL communicators over NVLink/NVSwitch, loaded at run time from libnccl.so.2
 * (OPURE_ERR_UNSUPPORTED when absent). One rank calls opure_comm_unique_id and sends the
 * 128-byte id to the others out of band; every rank then calls opure_comm_init with its
 * own ctx. Initialisation is non-blocking and bounded by timeout_ms (OPURE_ERR_TIMEOUT
 * when a rank never joins). Collectives enqueue on the ctx stream (graph-capturable). */
typedef struct opure_comm opure_comm;
#define OPURE_COMM_ID_BYTES 128
opure_status opure_comm_unique_id(uint8_t *id /* [OPURE_COMM_ID_BYTES] */);
opure_status opure_comm_init(opure_ctx *ctx, uint32_t n_ranks, uint32_t rank, const uint8_t *id,
                             uint32_t timeout_ms, opure_comm **out);
opure_status opure_comm_destroy(opure_comm *c);
opure_status opure_comm_info(const opure_comm *c, uint32_t *n_ranks, uint32_t *rank);
/* In-place all-reduce over the communicator's ranks. */
opure_status opure_allreduce_sum_f32(opure_ctx *ctx, opure_comm *c, float *buf, size_t n);
opure_status opure_allreduce_max_u64(opure_ctx *ctx, opure_comm *c, unsigned long long *buf, size_t n);
/* Argmax keys of a vocabulary shard whose first row is `offset`: rewrites each non-zero
 * key's index to the global one (value bits unchanged), ready for a u64 max all-reduce. */
opure_status opure_argmax_key_offset(opure_ctx *ctx, unsigned long long *keys, uint32_t n, uint32_t offset);

/* ---- NVLink peer all-reduce fused into the producing kernel (tensor parallelism) -------
 * The reference has no multi-GPU path at all (one D3D12 device, Opure_Dx12.h:144-337); these
 * replace, on the tensor-parallel step, the pair opure_allreduce_sum_f32 + opure_add after
 * each o_proj / down_proj GEMV and the pair opure_argmax_key_offset + opure_allreduce_max_u64
 * after the lm_head (the reference's serial AddRes / ArgMax dispatches,
 * Opure_VoxelEngine.cpp:451-470,508-532).
 *
 * A peer group gives every rank of `comm` (one process per GPU) a mailbox in its own HBM
 * that every other rank maps through CUDA IPC. Creation is collective over `comm` (same call
 * on every rank, bounded by the communicator's timeout) and returns OPURE_ERR_UNSUPPORTED on
 * every rank when any pair of GPUs cannot map each other's memory (then keep NCCL).
 * `max_rows` bounds the GEMV rows of a collective; device-side waits give up after
 * `timeout_ms` (0: 2000) with OPURE_ERR_DEVICE_TIMEOUT in the status word. Every rank must
 * issue the same sequence of peer collectives with the same shapes. destroy is collective
 * too (pass the communicator, or NULL if the other ranks are known to be done). */
typedef struct opure_peer opure_peer;
#define OPURE_PEER_MAX_RANKS 8
#define OPURE_PEER_MAX_KEYS 256
opure_status opure_peer_create(opure_ctx *ctx, opure_comm *comm, uint32_t max_rows, uint32_t timeout_ms,
                               opure_peer **out);
opure_status opure_peer_destroy(opure_ctx *ctx, opure_comm *comm, opure_peer *peer);
opure_status opure_peer_info(const opure_peer *peer, uint32_t *n_ranks, uint32_t *rank, uint32_t *max_rows);
/* GEMV (as opure_gemv, epilogue OPURE_EPI_STORE or OPURE_EPI_ADD, CUDA-core path for any
 * nvec, in passes of up to 9 vectors) whose partial sums are all-reduced over the group
 * inside the same kernel: y = (residual +) sum over ranks of W_rank x_rank, summed in rank
 * order so every rank gets bit-identical results. One kernel per pass; no scratch. */
opure_status opure_gemv_allreduce(opure_ctx *ctx, opure_peer *peer, const opure_gemv_args *a);
/* In place: keys[i] <- the largest key over all ranks, after rewriting this rank's keys to
 * global indices (its vocabulary shard starts at row `offset`); n <= OPURE_PEER_MAX_KEYS. */
opure_status opure_peer_argmax(opure_ctx *ctx, opure_peer *peer, unsigned long long *keys, uint32_t n,
                               uint32_t offset);

/* ---- fault injection (host side; tests of the error paths) -----------------
 * The next `count` ABI calls after `after_calls` more calls return OPURE_ERR_INJECTED
 * without touching the GPU. count = 0 disarms. */
opure_status opure_debug_inject_failure(opure_ctx *ctx, uint32_t after_calls, uint32_t count);

#ifdef __cplusplus
}
#endif
#endif /* OPURE_CUDA_H */
