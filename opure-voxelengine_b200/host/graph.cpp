// graph.cpp -- config parsing/validation (Opure_Graph.cpp:74-196), layout planning
// (:307-404) and weight upload (:435-531), for an fp16/int8-resident device arena.
#include "graph.h"

#include <algorithm>
#include <fstream>
#include <sstream>

#include "json.h"
#include "platform.h"

namespace opure::graph {

namespace {

uint64_t Align(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

uint32_t GetU32(const json::Value &root, std::string_view key, std::string_view ctx) {
    const int64_t v = root.GetInt(key, ctx);
    OPURE_CHECK(v >= 0 && v <= int64_t(UINT32_MAX), std::string(ctx) + ": '" + std::string(key) + "' out of range");
    return uint32_t(v);
}

}  // namespace

std::string ReadSmallFile(const std::string &path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) ThrowError("cannot open '" + path + "'");
    std::stringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

std::string JoinPath(const std::string &dir, const std::string &leaf) {
    if (dir.empty() || dir.back() == '/') return dir + leaf;
    return dir + "/" + leaf;
}

ModelConfig ModelConfig::Parse(std::string_view text) {
    const json::Value root = json::ParseObject(text, "config.json");
    constexpr std::string_view ctx = "config.json";
    ModelConfig c;
    if (const json::Value *v = root.Find("model_type"); v && v->IsString()) c.modelType = v->str;
    if (const json::Value *a = root.Find("architectures"); a && a->IsArray() && !a->arr.empty() && a->arr[0].IsString())
        c.architecture = a->arr[0].str;
    c.hiddenAct = root.GetStr("hidden_act", ctx);
    c.vocabSize = GetU32(root, "vocab_size", ctx);
    c.hiddenSize = GetU32(root, "hidden_size", ctx);
    c.intermediateSize = GetU32(root, "intermediate_size", ctx);
    c.numLayers = GetU32(root, "num_hidden_layers", ctx);
    c.numHeads = GetU32(root, "num_attention_heads", ctx);
    c.maxPositions = GetU32(root, "max_position_embeddings", ctx);
    // Absent on MHA models; defaulting to num_attention_heads is the HF convention.
    c.numKvHeads = root.Find("num_key_value_heads") ? GetU32(root, "num_key_value_heads", ctx) : c.numHeads;
    if (const json::Value *v = root.Find("rope_theta"); v && v->IsNumber()) c.ropeTheta = v->num;
    if (const json::Value *v = root.Find("rope_scaling"); v && v->IsObject()) {
        if (const json::Value *t = v->Find("rope_type"); t && t->IsString()) c.ropeScalingType = t->str;
        else if (const json::Value *t2 = v->Find("type"); t2 && t2->IsString()) c.ropeScalingType = t2->str;
        if (const json::Value *f = v->Find("factor"); f && f->IsNumber()) c.ropeScalingFactor = f->num;
    }
    c.rmsNormEps = float(root.GetNum("rms_norm_eps", ctx));
    c.tieWordEmbeddings = root.GetBool("tie_word_embeddings", true, ctx);
    c.attentionBias = root.GetBool("attention_bias", false, ctx);
    c.mlpBias = root.GetBool("mlp_bias", false, ctx);
    if (const json::Value *t = root.Find("torch_dtype"); t && t->IsString()) c.torchDtype = t->str;
    if (const json::Value *e = root.Find("eos_token_id")) {
        const json::Value *id = e->IsArray() ? (e->arr.empty() ? nullptr : &e->arr[0]) : e;
        if (id && id->IsNumber() && id->integral && id->inum >= 0 && id->inum < int64_t(c.vocabSize))
            c.eosTokenId = id->inum;
    }
    return c;
}

bool ModelConfig::Validate(std::string &err) const {
    if (hiddenSize == 0 || numHeads == 0 || numLayers == 0 || vocabSize == 0) {
        err = "config.json is missing a required dimension";
        return false;
    }
    if (hiddenSize % numHeads) {
        err = "hidden_size " + std::to_string(hiddenSize) + " is not divisible by num_attention_heads " +
              std::to_string(numHeads);
        return false;
    }
    if (numKvHeads == 0 || numHeads % numKvHeads) {
        err = "num_attention_heads " + std::to_string(numHeads) + " is not divisible by num_key_value_heads " +
              std::to_string(numKvHeads);
        return false;
    }
    const uint32_t hd = HeadDim();
    if (hd != 64 && hd != 128) {
        err = "head_dim " + std::to_string(hd) + " has no decode kernel (64 and 128 do)";
        return false;
    }
    if (intermediateSize == 0 || maxPositions == 0) {
        err = "intermediate_size and max_position_embeddings must be non-zero";
        return false;
    }
    if (hiddenAct != "silu") {
        err = "hidden_act '" + hiddenAct + "' is not implemented (only silu/SwiGLU is)";
        return false;
    }
    if (attentionBias || mlpBias) {
        err = "bias terms are not implemented by this engine";
        return false;
    }
    if (hiddenSize % 16 || intermediateSize % 16) {
        err = "hidden_size and intermediate_size must be multiples of 16 (16-byte weight chunks)";
        return false;
    }
    return true;
}

void Graph::Release() {
    stream_.Close();
    loaded_ = false;
}

void Graph::LoadConfigOnly(const std::string &modelDir, const LayoutOptions &opts) {
    Release();
    cfg_ = ModelConfig::Parse(ReadSmallFile(JoinPath(modelDir, "config.json")));
    std::string err;
    if (!cfg_.Validate(err)) ThrowError("model configuration rejected: " + err);
    stream_.Open(JoinPath(modelDir, "model.safetensors"));
    spec_.Resolve(cfg_, stream_);
    spec_.Check(cfg_);
    if (!spec_.Supported()) ThrowError("model is not supported by this engine:\n" + spec_.Explain());
    PlanLayout(opts);
    loaded_ = true;
}

void Graph::PlanLayout(const LayoutOptions &opts) {
    plan_ = VramPlan{};
    const uint32_t ts = opts.tpSize;
    OPURE_CHECK(ts >= 1 && opts.tpRank < ts, "tensor-parallel rank out of range");
    OPURE_CHECK(cfg_.numKvHeads % ts == 0, "num_key_value_heads must divide by the tensor-parallel size");
    OPURE_CHECK(cfg_.intermediateSize % (16 * ts) == 0,
                "intermediate_size / tensor-parallel size must be a multiple of 16");
    OPURE_CHECK(cfg_.vocabSize % ts == 0, "vocab_size must divide by the tensor-parallel size");
    local_ = LocalGeometry{};
    local_.tpSize = ts;
    local_.tpRank = opts.tpRank;
    local_.heads = cfg_.numHeads / ts;
    local_.kvHeads = cfg_.numKvHeads / ts;
    local_.inter = cfg_.intermediateSize / ts;
    local_.vocab = cfg_.vocabSize / ts;
    local_.vocabOffset = local_.vocab * opts.tpRank;
    OPURE_CHECK(ts == 1 || (uint64_t(local_.heads) * cfg_.HeadDim()) % 16 == 0,
                "a shard's attention width must be a multiple of 16 elements");
    const uint64_t h = cfg_.hiddenSize, ff = local_.inter;
    const uint64_t qkv = local_.QkvRows(cfg_.HeadDim());
    const uint64_t att = uint64_t(local_.heads) * cfg_.HeadDim();  // o_proj input columns
    // Matrices are all int8 or all floating point; mixing would need per-GEMV dtypes.
    bool anyQ = false, allQ = true;
    for (const BlockTensors &b : spec_.Blocks())
        for (const TensorRef *t : {&b.wq, &b.wk, &b.wv, &b.wo, &b.gate, &b.up, &b.down}) {
            anyQ |= t->IsQuantized();
            allQ &= t->IsQuantized();
        }
    OPURE_CHECK(!anyQ || allQ, "layer matrices mix int8 and floating point");
    plan_.wDtype = allQ ? OPURE_W_Q8 : OPURE_W_F16;
    const uint64_t eb = allQ ? 1 : 2;
    plan_.hasFused = opts.fusedLayouts && ts == 1;

    uint64_t cur = 0;
    auto place = [&](uint64_t bytes) {
        const uint64_t at = cur;
        cur = Align(cur + bytes, 256);
        return at;
    };
    plan_.embedTokens = place(uint64_t(cfg_.vocabSize) * h * 2);  // embeddings stay fp16
    plan_.finalNorm = place(h * 2);
    const TensorRef &lm = spec_.LmHead();
    if (lm.Present() && !cfg_.tieWordEmbeddings) {
        plan_.lmQuantized = lm.IsQuantized();
        plan_.slm = lm.scale;
        plan_.lmHead = place(uint64_t(local_.vocab) * h * (plan_.lmQuantized ? 1 : 2));
    } else {
        // Tied: this shard's vocabulary rows of the (whole) embedding.
        plan_.lmHead = plan_.embedTokens + uint64_t(local_.vocabOffset) * h * 2;
    }
    plan_.layers.resize(cfg_.numLayers);
    for (uint32_t l = 0; l < cfg_.numLayers; ++l) {
        const BlockTensors &b = spec_.Blocks()[l];
        VramPlan::LayerTensors &t = plan_.layers[l];
        t.inputNorm = place(h * 2);
        t.postAttNorm = place(h * 2);
        t.wqkv = place(qkv * h * eb);
        t.wo = place(h * att * eb);
        t.wgu = place(2 * ff * h * eb);
        t.wdown = place(h * ff * eb);
        if (plan_.hasFused) {
            t.woBlk = place(h * h * eb);
            t.wdownT = place(h * ff * eb);
        }
        t.sq = b.wq.scale; t.sk = b.wk.scale; t.sv = b.wv.scale; t.so = b.wo.scale;
        t.sgate = b.gate.scale; t.sup = b.up.scale; t.sdown = b.down.scale;
    }
    plan_.weightBytes = cur;
}

uint64_t Graph::StreamBytes() const {
    const uint64_t eb = plan_.wDtype == OPURE_W_Q8 ? 1 : 2;
    const uint64_t h = cfg_.hiddenSize, ff = local_.inter, hd = cfg_.HeadDim();
    const uint64_t perLayer = (uint64_t(local_.QkvRows(uint32_t(hd))) * h + h * local_.heads * hd + 3 * ff * h) * eb +
                              2 * h * 2;
    return perLayer * cfg_.numLayers + uint64_t(local_.vocab) * h * (plan_.lmQuantized ? 1 : 2) + h * 2;
}

void Graph::UploadWeights(opure_ctx *ctx, void *arena) {
    OPURE_CHECK(loaded_, "UploadWeights before LoadConfigOnly");
    auto *base = static_cast<uint8_t *>(arena);
    const uint64_t h = cfg_.hiddenSize, ff = cfg_.intermediateSize;
    const uint32_t ts = local_.tpSize, tr = local_.tpRank;
    const uint32_t hd = cfg_.HeadDim(), G = cfg_.KvGroupSize(), nkv = cfg_.numKvHeads;
    const bool q8 = plan_.wDtype == OPURE_W_Q8;
    const uint64_t eb = q8 ? 1 : 2;
    std::vector<uint8_t> stage;

    // Host copy of a tensor in the resident format (fp16 bits, or raw int8).
    auto fetch = [&](const TensorRef &r, std::vector<uint8_t> &out, bool allow_q8) {
        const safetensors::Tensor &t = stream_.Find(r.name);
        const uint64_t n = t.ElementCount();
        if (t.dtype == safetensors::Dtype::I8 && allow_q8) {
            out.assign(static_cast<const uint8_t *>(stream_.Data(t)), static_cast<const uint8_t *>(stream_.Data(t)) + n);
        } else {
            out.resize(n * 2);
            safetensors::NarrowToF16(t.dtype, stream_.Data(t), n, reinterpret_cast<uint16_t *>(out.data()));
        }
    };
    auto put = [&](uint64_t off, const std::vector<uint8_t> &bytes) {
        OPURE_CUDA_CHECK(opure_h2d(ctx, base + off, bytes.data(), bytes.size()));
        OPURE_CUDA_CHECK(opure_sync(ctx, 600000));  // staging is reused
    };

    fetch(spec_.Embed(), stage, false);
    put(plan_.embedTokens, stage);
    fetch(spec_.FinalNorm(), stage, false);
    put(plan_.finalNorm, stage);
    const uint64_t lmEb = plan_.lmQuantized ? 1 : 2;
    if (!cfg_.tieWordEmbeddings && spec_.LmHead().Present()) {
        fetch(spec_.LmHead(), stage, true);
        if (ts > 1) {  // this shard's vocabulary rows
            const uint64_t rb = h * lmEb;
            stage = std::vector<uint8_t>(stage.begin() + uint64_t(local_.vocabOffset) * rb,
                                         stage.begin() + uint64_t(local_.vocabOffset + local_.vocab) * rb);
        }
        put(plan_.lmHead, stage);
    }
    // Row block [r0, r0 + nr) of a row-major matrix with `cols` columns.
    auto rows = [&](std::vector<uint8_t> &m, uint64_t cols, uint64_t r0, uint64_t nr) {
        if (ts == 1) return;
        m = std::vector<uint8_t>(m.begin() + r0 * cols * eb, m.begin() + (r0 + nr) * cols * eb);
    };
    // Column block [c0, c0 + nc) of every row of a row-major [nrows][cols] matrix.
    auto cols_of = [&](std::vector<uint8_t> &m, uint64_t nrows, uint64_t cols, uint64_t c0, uint64_t nc) {
        if (ts == 1) return;
        std::vector<uint8_t> out(nrows * nc * eb);
        for (uint64_t r = 0; r < nrows; ++r)
            std::copy_n(m.data() + (r * cols + c0) * eb, nc * eb, out.data() + r * nc * eb);
        m.swap(out);
    };
    const uint64_t hq = uint64_t(local_.heads) * hd, hk = uint64_t(local_.kvHeads) * hd, ffl = local_.inter;
    std::vector<uint8_t> a, b2;
    for (uint32_t l = 0; l < cfg_.numLayers; ++l) {
        const BlockTensors &b = spec_.Blocks()[l];
        const VramPlan::LayerTensors &t = plan_.layers[l];
        fetch(b.inputNorm, stage, false);
        put(t.inputNorm, stage);
        fetch(b.postAttNorm, stage, false);
        put(t.postAttNorm, stage);
        // q; k; v contiguous, so the three projections run as one GEMV over QkvRows().
        uint64_t off = t.wqkv;
        for (const TensorRef *r : {&b.wq, &b.wk, &b.wv}) {
            fetch(*r, stage, q8);
            const uint64_t nr = r == &b.wq ? hq : hk;
            rows(stage, h, uint64_t(tr) * nr, nr);  // this shard's heads
            put(off, stage);
            off += stage.size();
        }
        fetch(b.wo, a, q8);
        cols_of(a, h, h, uint64_t(tr) * hq, hq);  // input columns of this shard's heads
        put(t.wo, a);
        if (plan_.hasFused) {
            // woBlk[g][o][c] = Wo[o][g*G*hd + c]: each kv head's input columns contiguous.
            const uint64_t gw = uint64_t(G) * hd;
            b2.resize(a.size());
            for (uint32_t g = 0; g < nkv; ++g)
                for (uint64_t o = 0; o < h; ++o)
                    std::copy_n(a.data() + (o * h + g * gw) * eb, gw * eb, b2.data() + ((g * h + o) * gw) * eb);
            put(t.woBlk, b2);
        }
        fetch(b.gate, stage, q8);
        rows(stage, h, uint64_t(tr) * ffl, ffl);
        put(t.wgu, stage);
        fetch(b.up, stage, q8);
        rows(stage, h, uint64_t(tr) * ffl, ffl);
        put(t.wgu + ffl * h * eb, stage);
        fetch(b.down, a, q8);
        cols_of(a, h, ff, uint64_t(tr) * ffl, ffl);
        put(t.wdown, a);
        if (plan_.hasFused) {
            b2.resize(a.size());
            for (uint64_t o = 0; o < h; ++o)
                for (uint64_t f = 0; f < ff; ++f)
                    std::copy_n(a.data() + (o * ff + f) * eb, eb, b2.data() + (f * h + o) * eb);
            put(t.wdownT, b2);
        }
    }
}

}  // namespace opure::graph
