// model_spec.cpp -- tensor-role resolution across the Hugging Face naming conventions
// the reference accepts (Opure_ModelSpec.cpp:101-224), and the shape/feature gates of
// its Check (:227-313).
#include "model_spec.h"

#include <algorithm>
#include <sstream>

#include "graph.h"
#include "platform.h"

namespace opure::graph {

uint64_t TensorRef::Elements() const {
    uint64_t n = 1;
    for (int64_t d : shape) n *= uint64_t(d < 0 ? 0 : d);
    return n;
}

bool TensorRef::Matches(std::initializer_list<int64_t> dims) const {
    return shape.size() == dims.size() && std::equal(shape.begin(), shape.end(), dims.begin());
}

namespace {

TensorRef Make(const safetensors::WeightStreamer &s, const std::string &name) {
    const safetensors::Tensor *t = s.TryFind(name);
    if (!t) return {};
    TensorRef r;
    r.name = t->name;
    r.dtype = t->dtype;
    r.shape = t->shape;
    r.scale = t->scale;
    return r;
}

TensorRef Probe(const safetensors::WeightStreamer &s, std::initializer_list<std::string> names) {
    for (const std::string &n : names) {
        TensorRef r = Make(s, n);
        if (r.Present()) return r;
    }
    return {};
}

// The per-block prefix, found from layer 0's query projection, stops before the "0.".
std::string DetectLayerPrefix(const safetensors::WeightStreamer &s) {
    static const char *kCandidates[] = {
        "model.layers.0.self_attn.q_proj.weight",
        "model.layers.0.attention.wq.weight",
        "transformer.h.0.attn.c_attn.wq.weight",
        "model.decoder.layers.0.self_attn.q_proj.weight",
    };
    for (const char *c : kCandidates) {
        if (s.TryFind(c)) {
            const std::string full(c);
            return full.substr(0, full.find("0."));
        }
    }
    return "model.layers.";
}

}  // namespace

void ModelSpec::AddIssue(std::string reason, std::string fix) {
    for (const SupportIssue &i : issues_)
        if (i.reason == reason) return;
    issues_.push_back({std::move(reason), std::move(fix)});
}

std::string ModelSpec::Explain() const {
    if (issues_.empty()) return "supported";
    std::ostringstream os;
    for (size_t i = 0; i < issues_.size(); ++i) {
        os << (i ? "\n  - " : "  - ") << issues_[i].reason;
        if (!issues_[i].fix.empty()) os << "\n      fix: " << issues_[i].fix;
    }
    return os.str();
}

void ModelSpec::Require(const TensorRef &t, const std::string &role,
                        std::initializer_list<int64_t> dims) {
    if (!t.Present()) {
        AddIssue("missing tensor for role '" + role + "'",
                 "check the naming convention; no tensor in the file matched this role");
        return;
    }
    if (!t.Matches(dims)) {
        std::ostringstream want, got;
        for (auto it = dims.begin(); it != dims.end(); ++it) want << (it == dims.begin() ? "" : ", ") << *it;
        for (size_t i = 0; i < t.shape.size(); ++i) got << (i ? ", " : "") << t.shape[i];
        AddIssue("tensor '" + t.name + "' for role '" + role + "' has shape [" + got.str() +
                     "] but the config implies [" + want.str() + "]",
                 "the weights and config.json disagree");
    }
}

void ModelSpec::Resolve(const ModelConfig &cfg, const safetensors::WeightStreamer &s) {
    issues_.clear();
    embed_ = Probe(s, {"model.embed_tokens.weight", "transformer.wte.weight",
                       "model.decoder.embed_tokens.weight"});
    finalNorm_ = Probe(s, {"model.norm.weight", "transformer.ln_f.weight",
                           "model.final_layernorm.weight"});
    lmHead_ = Probe(s, {"lm_head.weight", "model.lm_head.weight", "output.weight"});
    layerPrefix_ = DetectLayerPrefix(s);

    auto pick = [&](const char *canon, const char *alt) {
        if (s.TryFind(layerPrefix_ + "0." + canon)) return std::string(canon);
        if (s.TryFind(layerPrefix_ + "0." + alt)) return std::string(alt);
        return std::string(canon);
    };
    const std::string q = pick("self_attn.q_proj.weight", "attention.wq.weight");
    const std::string k = pick("self_attn.k_proj.weight", "attention.wk.weight");
    const std::string v = pick("self_attn.v_proj.weight", "attention.wv.weight");
    const std::string o = pick("self_attn.o_proj.weight", "attention.wo.weight");

    blocks_.assign(cfg.numLayers, {});
    for (uint32_t l = 0; l < cfg.numLayers; ++l) {
        const std::string p = layerPrefix_ + std::to_string(l) + ".";
        BlockTensors &b = blocks_[l];
        b.inputNorm = Probe(s, {p + "input_layernorm.weight", p + "attention_norm.weight", p + "ln_1.weight"});
        b.postAttNorm = Probe(s, {p + "post_attention_layernorm.weight", p + "ffn_norm.weight", p + "ln_2.weight"});
        b.wq = Make(s, p + q);
        b.wk = Make(s, p + k);
        b.wv = Make(s, p + v);
        b.wo = Make(s, p + o);
        b.gate = Make(s, p + "mlp.gate_proj.weight");
        b.up = Make(s, p + "mlp.up_proj.weight");
        b.down = Make(s, p + "mlp.down_proj.weight");
    }
    RebuildReadSet();
}

void ModelSpec::Check(const ModelConfig &cfg) {
    const int64_t h = cfg.hiddenSize, ff = cfg.intermediateSize, hd = cfg.HeadDim();
    const int64_t kvh = int64_t(cfg.numKvHeads) * hd;
    if (hd != 64 && hd != 128)
        AddIssue("head_dim " + std::to_string(hd) + " has no decode kernel (64 and 128 do)",
                 "the split-K attention kernel also runs 32..256; the fused decode path is 64/128");
    if (cfg.numKvHeads == 0 || cfg.numHeads % cfg.numKvHeads)
        AddIssue("num_heads is not a multiple of num_kv_heads", "GQA needs whole query groups");
    else if (cfg.numHeads / cfg.numKvHeads > 4)
        AddIssue("more than 4 query heads per kv head", "add the group size to the attention kernels");
    if (hd * cfg.numHeads != h) AddIssue("num_heads * head_dim != hidden_size", "config.json is inconsistent");
    if (cfg.hiddenAct != "silu") AddIssue("activation '" + cfg.hiddenAct + "' is not implemented", "SwiGLU only");
    if (cfg.attentionBias || cfg.mlpBias) AddIssue("projection biases are not read", "no bias support");
    if (cfg.ropeScalingType != "none")
        AddIssue("RoPE scaling type '" + cfg.ropeScalingType + "' is not implemented", "");
    Require(embed_, "embed_tokens", {int64_t(cfg.vocabSize), h});
    Require(finalNorm_, "norm", {h});
    if (!cfg.tieWordEmbeddings) Require(lmHead_, "lm_head", {int64_t(cfg.vocabSize), h});
    for (size_t l = 0; l < blocks_.size(); ++l) {
        const BlockTensors &b = blocks_[l];
        const std::string at = "layer " + std::to_string(l) + ": ";
        Require(b.inputNorm, at + "input_layernorm", {h});
        Require(b.postAttNorm, at + "post_attn_layernorm", {h});
        Require(b.wq, at + "q_proj", {h, h});
        Require(b.wk, at + "k_proj", {kvh, h});
        Require(b.wv, at + "v_proj", {kvh, h});
        Require(b.wo, at + "o_proj", {h, h});
        Require(b.gate, at + "gate_proj", {ff, h});
        Require(b.up, at + "up_proj", {ff, h});
        Require(b.down, at + "down_proj", {h, ff});
        for (const TensorRef *t : {&b.wq, &b.wk, &b.wv, &b.wo, &b.gate, &b.up, &b.down}) {
            if (t->Present() && (t->dtype == safetensors::Dtype::U8 || t->dtype == safetensors::Dtype::U4 ||
                                 t->dtype == safetensors::Dtype::I4))
                AddIssue("tensor '" + t->name + "' is " + DtypeName(t->dtype) +
                             "; only F32/F16/BF16 and per-tensor I8 are served",
                         "");
        }
    }
}

void ModelSpec::RebuildReadSet() {
    readSet_.clear();
    auto add = [this](const TensorRef &t) {
        if (t.Present() && std::find(readSet_.begin(), readSet_.end(), &t) == readSet_.end())
            readSet_.push_back(&t);
    };
    add(embed_);
    add(finalNorm_);
    add(lmHead_);
    for (const BlockTensors &b : blocks_)
        for (const TensorRef *t : {&b.inputNorm, &b.postAttNorm, &b.wq, &b.wk, &b.wv, &b.wo, &b.gate, &b.up, &b.down})
            add(*t);
}

}  // namespace opure::graph
