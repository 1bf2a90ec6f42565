// graph.h -- model geometry and the device layout plan.
// Keeps the API of the reference's graph::ModelConfig / VramPlan / Graph
// (src/engine/Opure_Graph.h:46-233): Parse, Validate, KvCacheWords-style sizing,
// Graph::{LoadConfigOnly, UploadWeights, IsQuantized, GetQuantizedScale}. The backing
// store is one cudaMalloc'd arena (through the C ABI) holding every weight as fp16 (or
// per-tensor int8), not fp32 words: the reference widens F16/BF16 to F32 on upload
// (Opure_Graph.cpp:509-517); keeping fp16 halves the bytes every decode step streams.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "model_spec.h"
#include "opure_cuda.h"
#include "streamer.h"

namespace opure::graph {

struct ModelConfig {
    std::string modelType = "llama";
    std::string architecture = "LlamaForCausalLM";
    std::string hiddenAct = "silu";
    uint32_t vocabSize = 0, hiddenSize = 0, intermediateSize = 0, numLayers = 0;
    uint32_t numHeads = 0, numKvHeads = 0, maxPositions = 0;
    float rmsNormEps = 1e-5f;
    double ropeTheta = 10000.0;
    bool tieWordEmbeddings = true, attentionBias = false, mlpBias = false;
    std::string torchDtype;
    std::string ropeScalingType = "none";
    double ropeScalingFactor = 1.0;
    // Generation stop id: the reference takes the tokenizer's <|endoftext|> id
    // (Opure_VoxelEngine.cpp:904); this engine loads no tokenizer and takes config.json's
    // eos_token_id (the first entry when it is a list). -1: none.
    int64_t eosTokenId = -1;

    uint32_t HeadDim() const { return numHeads ? hiddenSize / numHeads : 0; }
    uint32_t KvGroupSize() const { return numKvHeads ? numHeads / numKvHeads : 0; }
    uint32_t QkvRows() const { return (numHeads + 2 * numKvHeads) * HeadDim(); }
    // fp16 KV bytes per token per sequence, all layers (K and V).
    uint64_t KvBytesPerToken() const { return 2ull * numLayers * numKvHeads * HeadDim() * 2ull; }
    bool Validate(std::string &err) const;
    static ModelConfig Parse(std::string_view jsonText);
};

struct LayoutOptions {
    bool fusedLayouts = true;  // also store o_proj grouped per kv head and down_proj^T
    // Tensor parallelism: this device holds shard tpRank of tpSize. q/k/v and gate/up are
    // split by rows (whole heads / intermediate rows), o_proj and down_proj by columns (the
    // matching input slice), the lm_head by vocabulary rows; embeddings and norms are whole.
    uint32_t tpSize = 1, tpRank = 0;
};

// The part of the model one tensor-parallel shard computes (the whole model at tpSize 1).
struct LocalGeometry {
    uint32_t heads = 0, kvHeads = 0, inter = 0, vocab = 0, vocabOffset = 0;
    uint32_t tpSize = 1, tpRank = 0;
    uint32_t QkvRows(uint32_t headDim) const { return (heads + 2 * kvHeads) * headDim; }
};

// Byte offsets into the weight arena.
struct VramPlan {
    struct LayerTensors {
        uint64_t inputNorm = 0, postAttNorm = 0;
        uint64_t wqkv = 0;   // [q rows; k rows; v rows][hidden]
        uint64_t wo = 0;     // [hidden][hidden]
        uint64_t woBlk = 0;  // [n_kv][hidden][group*head_dim]: o_proj columns grouped per kv head
        uint64_t wgu = 0;    // [gate rows; up rows][hidden]
        uint64_t wdown = 0;  // [hidden][inter]
        uint64_t wdownT = 0; // [inter][hidden]
        float sq = 1, sk = 1, sv = 1, so = 1, sgate = 1, sup = 1, sdown = 1;  // int8 scales
    };
    std::vector<LayerTensors> layers;
    uint64_t embedTokens = 0, finalNorm = 0, lmHead = 0;
    float slm = 1.0f;
    uint32_t wDtype = OPURE_W_F16;  // matrices: OPURE_W_F16 or OPURE_W_Q8
    bool lmQuantized = false;
    bool hasFused = false;
    uint64_t weightBytes = 0;
};

class Graph {
public:
    Graph() = default;
    Graph(const Graph &) = delete;
    Graph &operator=(const Graph &) = delete;

    // Parses config.json, maps model.safetensors, resolves roles and plans the layout.
    void LoadConfigOnly(const std::string &modelDir, const LayoutOptions &opts = {});
    // Converts and copies every planned tensor into `arena` (device, weightBytes long).
    void UploadWeights(opure_ctx *ctx, void *arena);
    void Release();

    const ModelConfig &Config() const { return cfg_; }
    const VramPlan &Plan() const { return plan_; }
    const LocalGeometry &Local() const { return local_; }
    // Weight bytes one decode step of this shard reads (matrices once, norms, lm_head rows).
    uint64_t StreamBytes() const;
    const ModelSpec &Spec() const { return spec_; }
    bool IsLoaded() const { return loaded_; }
    bool IsQuantized() const { return plan_.wDtype == OPURE_W_Q8; }

private:
    void PlanLayout(const LayoutOptions &opts);

    ModelConfig cfg_;
    VramPlan plan_;
    LocalGeometry local_;
    ModelSpec spec_;
    safetensors::WeightStreamer stream_;
    bool loaded_ = false;
};

std::string ReadSmallFile(const std::string &path);
std::string JoinPath(const std::string &dir, const std::string &leaf);

}  // namespace opure::graph
