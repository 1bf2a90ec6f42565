// model_spec.h -- resolves a .safetensors file into graph roles.
// Same API as the reference's graph::ModelSpec (src/engine/Opure_ModelSpec.h:57-164):
// TensorRef, BlockTensors, SupportIssue, ModelSpec::{Resolve, Check, Supported, Explain,
// Embed, FinalNorm, LmHead, Blocks, ReadSet}.
#pragma once

#include <initializer_list>
#include <string>
#include <vector>

#include "streamer.h"

namespace opure::graph {

struct ModelConfig;

struct TensorRef {
    std::string name;  // empty when absent
    safetensors::Dtype dtype = safetensors::Dtype::F32;
    std::vector<int64_t> shape;
    float scale = 1.0f;
    bool Present() const { return !name.empty(); }
    uint64_t Elements() const;
    bool Matches(std::initializer_list<int64_t> dims) const;
    bool IsQuantized() const {
        return dtype == safetensors::Dtype::I8 || dtype == safetensors::Dtype::U8 ||
               dtype == safetensors::Dtype::I4 || dtype == safetensors::Dtype::U4;
    }
};

struct BlockTensors {
    TensorRef inputNorm, postAttNorm, wq, wk, wv, wo, gate, up, down;
};

struct SupportIssue {
    std::string reason;
    std::string fix;
};

class ModelSpec {
public:
    void Resolve(const ModelConfig &cfg, const safetensors::WeightStreamer &stream);
    void Check(const ModelConfig &cfg);
    bool Supported() const { return issues_.empty(); }
    const std::vector<SupportIssue> &Issues() const { return issues_; }
    std::string Explain() const;

    const std::string &LayerPrefix() const { return layerPrefix_; }
    const TensorRef &Embed() const { return embed_; }
    const TensorRef &FinalNorm() const { return finalNorm_; }
    const TensorRef &LmHead() const { return lmHead_; }
    const std::vector<BlockTensors> &Blocks() const { return blocks_; }
    const std::vector<const TensorRef *> &ReadSet() const { return readSet_; }

private:
    void AddIssue(std::string reason, std::string fix);
    void Require(const TensorRef &t, const std::string &role, std::initializer_list<int64_t> dims);
    void RebuildReadSet();

    TensorRef embed_, finalNorm_, lmHead_;
    std::vector<BlockTensors> blocks_;
    std::string layerPrefix_;
    std::vector<const TensorRef *> readSet_;
    std::vector<SupportIssue> issues_;
};

}  // namespace opure::graph
