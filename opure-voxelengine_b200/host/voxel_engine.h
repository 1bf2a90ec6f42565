// voxel_engine.h -- the decode engine: prefill, decode step and generate loop.
//
// Keeps the API of the reference's engine::VoxelEngine (src/engine/Opure_VoxelEngine.h:
// EngineOptions :54-65, GenerateResult :99-109, Initialize, Generate, ForwardArgMax,
// ForwardLogits, Prefill, DecodeStep, ArgMaxFrom-style readback, RunLayersTraced,
// PoisonBanks, SnapshotMetrics, CurrentPosition), and adds batched generation over
// independent sequences. All device work goes through the C ABI of libopure_cuda
// (include/opure_cuda.h); nothing here computes on the CPU.
//
// One decode step runs, for every active token vector:
//   step_begin (token pick + embedding gather)
//   per layer: q;k;v GEMV with fused RMSNorm prologue -> RoPE + paged fp16 KV append
//              -> split-K paged attention -> o_proj GEMV + residual
//              -> gate;up GEMV with fused RMSNorm prologue and SwiGLU epilogue
//              -> down_proj GEMV + residual
//   lm_head GEMV with fused final RMSNorm and argmax epilogue, step_end.
// The reference records the same graph as ~423 dispatches with a UAV barrier before each
// (Opure_VoxelEngine.cpp:189-536) and waits on a fence every token; here the step is
// captured once into a CUDA graph (kernels chained with programmatic dependent launch)
// and replayed, and the token loop runs on the device without host round trips.
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <utility>
#include <vector>

#include "graph.h"
#include "kv_cache.h"
#include "opure_cuda.h"

namespace opure::engine {

struct EngineOptions {
    bool enablePlasticity = false;  // the SignSGD side feature is not part of this engine
    uint32_t maxNewTokens = 256;
    float temperature = 0.0f;       // 0 = greedy (the only mode Generate uses, as the reference)
    // B200 engine options.
    uint32_t maxBatch = 1;          // token vectors per step
    uint32_t maxLen = 0;            // tokens per sequence (0: min(max_positions, 4096))
    uint32_t pageSize = 64;         // KV page size in tokens
    uint64_t pageSeed = 3;          // free-list shuffle (0: pages in order)
    bool useGraphs = true;
    float attnScale = 1.0f;         // 1.0 = the reference's unscaled scores
    uint32_t path = 0;              // 0 auto, 1 per-op kernels, 2 fused required (persistent kernel
                                    // when eligible), 3 fused as three kernels per layer
    bool phaseTrace = false;        // persistent kernel: record per-CTA phase timestamps
    uint32_t prefillChunk = 0;      // >0: prompts prefilled as steps of up to this many token
                                    // vectors (tensor-core GEMMs) instead of one token per step
    uint32_t kvWindow = 0;          // >0: sliding-window KV cache of this many tokens (a multiple
                                    // of pageSize): a sequence keeps kvWindow / pageSize pages as a
                                    // ring, and a position attends to the last kvWindow / pageSize - 1
                                    // whole pages and its own
    uint32_t tpAllreduce = 0;       // tensor parallel: 0 auto (peer kernels when mappable), 1 NCCL, 2 peer
};

struct GenerateResult {
    std::vector<uint32_t> promptTokens;
    std::vector<uint32_t> generated;
    uint32_t stopToken = 0;
    bool hitStop = false;
    double msPerToken = 0.0;
    double lastMs = 0.0;
};

struct StepTiming {
    double prefillMs = 0.0;   // device time of the prefill steps
    double decodeMs = 0.0;    // device time of the decode steps
    uint32_t prefillSteps = 0, decodeSteps = 0;
};

// Reads the ctx's device status word; throws opure::Error naming the failing kernel site
// and offending value when a kernel recorded a failure.
void CheckDevice(opure_ctx *ctx);

class VoxelEngine {
public:
    VoxelEngine() = default;
    ~VoxelEngine();
    VoxelEngine(const VoxelEngine &) = delete;
    VoxelEngine &operator=(const VoxelEngine &) = delete;

    // Loads the model onto `device`: layout plan, weight upload, KV pool, buffers. With
    // `shared`, the engine enqueues on that existing ctx (stream) instead of creating its
    // own: engines that cooperate on one stream (speculative decoding's draft and target)
    // then need no synchronisation between them. The owner of `shared` must outlive it.
    // With `comm` (created on `shared`'s or this engine's device), the engine is shard
    // rank-of-n of a tensor-parallel model: it holds its slice of the weights and KV heads,
    // and every step all-reduces the o_proj and down_proj partial sums and the vocabulary
    // shards' argmax keys over NCCL. All ranks must step in lockstep.
    void Initialize(const std::string &modelDir, const EngineOptions &opts, int device,
                    opure_ctx *shared = nullptr, opure_comm *comm = nullptr);
    void Shutdown();
    bool IsReady() const { return ready_; }

    const graph::Graph &GraphModel() const { return graph_; }
    bool UsesPeer() const { return peer_ != nullptr; }
    const graph::ModelConfig &Model() const { return graph_.Config(); }
    opure_ctx *Ctx() const { return ctx_; }
    uint32_t MaxLen() const { return maxLen_; }
    const EngineOptions &Options() const { return opts_; }

    // Prefill `tokens`, then `opts.maxNewTokens` greedy steps (Opure_VoxelEngine.cpp:894-958).
    GenerateResult Generate(const std::vector<uint32_t> &tokens, const EngineOptions &opts);
    // Independent sequences, one per token vector (at most maxBatch), same budget each.
    std::vector<GenerateResult> GenerateBatch(const std::vector<std::vector<uint32_t>> &prompts,
                                              uint32_t budget, StepTiming *timing = nullptr);

    uint32_t ForwardArgMax(const std::vector<uint32_t> &tokens);
    void ForwardLogits(const std::vector<uint32_t> &tokens, std::vector<float> &logitsOut);

    // Host-driven steps, the reference's Prefill + DecodeStep contract: each DecodeStep
    // copies the token in, runs one step and reads the 8-byte argmax result back.
    // Returns the argmax of the last prompt position (Prefill + ArgMaxFrom).
    uint32_t Prefill(const std::vector<uint32_t> &tokens);
    uint32_t DecodeStep(uint32_t tokenId, uint32_t position);
    // The same for n sequences at once (slots 0..n-1): tokens/positions in, next tokens out.
    void DecodeStepBatch(const int32_t *tokens, const int32_t *positions, uint32_t n, int32_t *next);

    // Embedding + the first nLayers layers for one token at position 0; the residual
    // after each layer (Opure_VoxelEngine.cpp:546-587).
    void RunLayersTraced(uint32_t tokenId, uint32_t nLayers, std::vector<std::vector<float>> &trace);
    // Fills the activation buffers with `fill` (Opure_VoxelEngine.cpp:625-636).
    void PoisonBanks(float fill);

    // Loads precomputed fp16 K/V [L][2][n_kv][len][hd] for sequence slot `seq` and marks
    // `len` positions as cached (synthetic long contexts).
    void LoadKv(uint32_t seq, const uint16_t *kv, uint32_t len);
    // Synthetic long contexts on the device: slots 0..n-1 get `len` cached positions of
    // seeded KV values (opure_kv_synth), `reserve` positions of pages each, and continue
    // self-driving from position len with first[v] as their next input.
    void PrepareSynthetic(uint32_t n, uint32_t len, uint32_t reserve, uint64_t seed, const int32_t *first);
    // Reads `count` tokens of a slot's token history from position `pos`.
    void ReadHistory(uint32_t slot, uint32_t pos, uint32_t count, int32_t *out);
    // Copies the last persistent step's phase timestamps (layout of opure_fused_step.trace)
    // to `out` (cap words); returns the words written (0 without phaseTrace).
    size_t ReadPhaseTrace(unsigned long long *out, size_t cap);

    struct MetricsSnapshot {
        float kvOccupancy = 0.0f;
        float tokensPerSec = 0.0f;
        float memoryPressure = 0.0f;
        float speculativeAcceptance = -1.0f;
    };
    MetricsSnapshot SnapshotMetrics() const;
    // Acceptance rate of the last speculative generation this engine was the target of.
    void SetSpeculativeAcceptance(float a) { specAcceptance_ = a; }
    uint32_t CurrentPosition() const { return seqLen_; }

    // Enqueues `steps` decode steps for the first n vectors (graph replays when enabled).
    void RunSteps(uint32_t n, uint32_t steps, bool logits);

    // Building blocks of multi-engine loops (speculative decoding):
    // prefill independent prompts of equal length into slots 0..n-1 (reserving `reserve`
    // positions each) and return the greedy next token of each;
    std::vector<uint32_t> PrefillBatch(const std::vector<std::vector<uint32_t>> &prompts, uint32_t reserve,
                                       bool logits);
    // describe the next step's n token vectors: sequence slot, position and token of each
    // (host-driven: no argmax feedback, positions not advanced; tok == NULL leaves the
    // tokens to a device producer writing DeviceInTokens());
    void SetVectors(const int32_t *seq, const int32_t *pos, const int32_t *tok, uint32_t n);
    // or make vectors 0..n-1 self-driving on slots 0..n-1 from positions pos[v]: history
    // tokens below known[v] are re-fed, later inputs are the previous step's result;
    void SetAutoVectors(const int32_t *pos, const int32_t *known, uint32_t n);
    // write `count` tokens into a slot's token history from position `pos`.
    void WriteHistory(uint32_t slot, uint32_t pos, const int32_t *tokens, uint32_t count);
    int32_t *DeviceHistory() const { return buf_.tokens; }      // [maxBatch][maxLen]
    int32_t *DeviceInTokens() const { return buf_.inTokens; }   // [maxBatch]
    float *DeviceLogits() const { return buf_.logits; }       // [maxBatch][vocab]
    unsigned long long *DeviceKeys() const { return buf_.keys; }
    const int32_t *DeviceSeq() const { return buf_.seq; }      // [vectors] slot of each vector
    const int32_t *DevicePos() const { return buf_.pos; }      // [vectors] next position of each
    // Rewinds the positions of vectors 0..n-1 (stream-ordered, no wait).
    void SetPositions(const int32_t *positions, uint32_t n);
    void Sync();

    struct Buffers {
        float *x = nullptr, *qkv = nullptr, *q = nullptr, *attn = nullptr, *h = nullptr;
        float *logits = nullptr;
        unsigned long long *keys = nullptr;
        int32_t *seq = nullptr, *pos = nullptr, *seqLen = nullptr, *known = nullptr;
        uint32_t *flags = nullptr;
        int32_t *inTokens = nullptr;
        int32_t *tokens = nullptr;
        // Fused path: second residual base and the two fixed-point delta buffers.
        float *base1 = nullptr;
        long long *delta0 = nullptr, *delta1 = nullptr;
        float *partial = nullptr;  // tensor parallelism: [maxBatch][hidden] shard partial sums
        uint32_t *sync = nullptr;  // grid-barrier words of the persistent decode kernel
        unsigned long long *trace = nullptr;  // its phase timestamps (EngineOptions.phaseTrace)
        unsigned long long *prefillKeys = nullptr;  // [maxBatch] chunked prefill's last-token keys
        // Chained tensor-core operands (steps of 16..256 vectors, fp16 weights): the packed
        // inputs of the o_proj (attention output), gate;up / next q;k;v / lm_head (gained
        // residual) and down_proj (SwiGLU activation), and the residual's per-tile sums of
        // squares for the consumer's RMSNorm.
        uint16_t *packAttn = nullptr, *packRes = nullptr, *packAct = nullptr;
        float *sumsq = nullptr;
    };
    // True when steps of n vectors run on opure_decode_fused.
    bool UsesFused(uint32_t n) const;
    // True when steps of n vectors run the per-op tensor-core GEMVs with chained operands.
    bool Chained(uint32_t n) const;
    const Buffers &Buf() const { return buf_; }

private:
    void AllocBuffers();
    void RecordStep(uint32_t n, bool logits);
    void RecordLayer(uint32_t layer, uint32_t n);
    void TpGemvAllreduce(const void *w, float scale, uint32_t rows, uint32_t cols, const float *in,
                         uint32_t in_stride, uint32_t n);
    // Split-K attention scratch for batch n (one zeroed buffer per batch size, so its
    // split counters always start at zero).
    void *AttnScratch(uint32_t n, size_t *bytes);
    void ResetSequences(const std::vector<std::vector<uint32_t>> &prompts, uint32_t reserve, bool automatic);
    // Chunked prefill of slots 0..n-1 after ResetSequences(..., false); leaves them
    // self-driving at their prompt lengths. Returns the number of steps it ran.
    uint32_t PrefillChunks(const std::vector<std::vector<uint32_t>> &prompts);
    opure_step_io StepIO(uint32_t n) const;

    opure_ctx *ctx_ = nullptr;
    graph::Graph graph_;
    kv::PagedKvCache kv_;
    EngineOptions opts_{};
    void *weights_ = nullptr;
    Buffers buf_{};
    uint32_t maxLen_ = 0;
    bool ready_ = false;
    uint32_t seqLen_ = 0;
    double lastTokenMs_ = 0.0;
    float specAcceptance_ = -1.0f;
    std::map<std::pair<uint32_t, bool>, opure_graph *> graphs_;
    std::map<uint32_t, std::pair<void *, size_t>> attnScratch_;
    void *hostIo_ = nullptr;  // pinned staging of the host-driven step
    bool hostDriven_ = false; // step flags currently cleared for host-supplied tokens
    bool seqIdentity_ = true; // vector v currently maps to sequence slot v
    bool ownsCtx_ = true;
    opure_comm *comm_ = nullptr;  // tensor-parallel communicator (not owned)
    opure_peer *peer_ = nullptr;  // NVLink peer mailboxes of the tensor-parallel group (owned)
    size_t traceWords_ = 0;
    uint32_t maxVec_ = 1;  // token vectors per step: max(maxBatch, prefillChunk)
};

}  // namespace opure::engine
