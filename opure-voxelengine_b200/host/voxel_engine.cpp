// voxel_engine.cpp -- decode engine on top of the C ABI (see voxel_engine.h).
#include "voxel_engine.h"

#include <algorithm>
#include <cmath>
#include <cstring>

#include "platform.h"

namespace opure::engine {

namespace {

template <typename T>
T *Alloc(opure_ctx *ctx, size_t count) {
    void *p = nullptr;
    OPURE_CUDA_CHECK(opure_alloc(ctx, std::max<size_t>(count * sizeof(T), 16), &p));
    return static_cast<T *>(p);
}

const uint8_t *At(const void *base, uint64_t off) { return static_cast<const uint8_t *>(base) + off; }

}  // namespace

VoxelEngine::~VoxelEngine() { Shutdown(); }

void VoxelEngine::Shutdown() {
    if (!ctx_) return;
    opure_sync(ctx_, 60000);
    for (auto &kv : graphs_) opure_graph_free(kv.second);
    graphs_.clear();
    if (peer_) opure_peer_destroy(ctx_, comm_, peer_);  // collective: every rank shuts down
    peer_ = nullptr;
    kv_.Destroy();
    for (void *p : {static_cast<void *>(buf_.x), static_cast<void *>(buf_.qkv), static_cast<void *>(buf_.q),
                    static_cast<void *>(buf_.attn), static_cast<void *>(buf_.h), static_cast<void *>(buf_.logits),
                    static_cast<void *>(buf_.keys), static_cast<void *>(buf_.seq),
                    static_cast<void *>(buf_.seqLen), static_cast<void *>(buf_.known), static_cast<void *>(buf_.flags),
                    static_cast<void *>(buf_.inTokens), static_cast<void *>(buf_.tokens),
                    static_cast<void *>(buf_.base1), static_cast<void *>(buf_.delta0),
                    static_cast<void *>(buf_.delta1), static_cast<void *>(buf_.partial),
                    static_cast<void *>(buf_.sync), static_cast<void *>(buf_.trace),
                    static_cast<void *>(buf_.prefillKeys), static_cast<void *>(buf_.packAttn),
                    static_cast<void *>(buf_.packRes), static_cast<void *>(buf_.packAct),
                    static_cast<void *>(buf_.sumsq), weights_})
        if (p) opure_free(ctx_, p);
    for (auto &s : attnScratch_) opure_free(ctx_, s.second.first);
    attnScratch_.clear();
    if (hostIo_) opure_free_host(ctx_, hostIo_);
    hostIo_ = nullptr;
    buf_ = Buffers{};
    weights_ = nullptr;
    if (ownsCtx_) opure_shutdown(ctx_);
    ctx_ = nullptr;
    ownsCtx_ = true;
    comm_ = nullptr;
    graph_.Release();
    ready_ = false;
}

void VoxelEngine::Initialize(const std::string &modelDir, const EngineOptions &opts, int device,
                             opure_ctx *shared, opure_comm *comm) {
    Shutdown();
    OPURE_CHECK(!opts.enablePlasticity, "the SignSGD plasticity pass is not part of this engine");
    OPURE_CHECK(opts.maxBatch >= 1, "maxBatch must be at least 1");
    opts_ = opts;
    if (shared) {
        ctx_ = shared;
        ownsCtx_ = false;
    } else {
        OPURE_CUDA_CHECK(opure_init(device, &ctx_));
        ownsCtx_ = true;
    }
    graph::LayoutOptions lo;
    lo.fusedLayouts = opts.path != 1;  // grouped o_proj and transposed down_proj
    comm_ = comm;
    if (comm) {
        OPURE_CUDA_CHECK(opure_comm_info(comm, &lo.tpSize, &lo.tpRank));
        lo.fusedLayouts = false;
        OPURE_CHECK(opts.path != 2, "the fused decode path does not run tensor-parallel");
    }
    graph_.LoadConfigOnly(modelDir, lo);
    const graph::ModelConfig &cfg = graph_.Config();
    const graph::VramPlan &plan = graph_.Plan();

    OPURE_CUDA_CHECK(opure_alloc(ctx_, plan.weightBytes, &weights_));
    graph_.UploadWeights(ctx_, weights_);

    maxLen_ = opts.maxLen ? std::min(opts.maxLen, cfg.maxPositions) : std::min(cfg.maxPositions, 4096u);
    OPURE_CHECK(opts.kvWindow % opts.pageSize == 0, "the KV window must be a multiple of the page size");
    const uint32_t ring = opts.kvWindow / opts.pageSize;
    OPURE_CHECK(ring == 0 || ring >= 2, "the KV window must span at least two pages");
    const uint32_t pagesPerSeq = ring ? ring : (maxLen_ + opts.pageSize - 1) / opts.pageSize;
    graph::ModelConfig kvCfg = cfg;
    kvCfg.numKvHeads = graph_.Local().kvHeads;  // a shard caches only its own KV heads
    kv_.Create(ctx_, kvCfg, opts.pageSize, pagesPerSeq * opts.maxBatch, opts.maxBatch, pagesPerSeq, opts.pageSeed,
               ring);
    maxVec_ = std::max(opts.maxBatch, opts.prefillChunk);
    AllocBuffers();
    // The fused GEMV + peer exchange (one kernel, tagged 8-byte words) took 8.5-9.4 us per
    // o_proj-shaped call at 2, 4 and 8 ranks against 9.3 / 14.9 / 24.9 us for NCCL's 8 KB
    // all-reduce alone (B200, 1.7B shape; 535 vs 473 tok/s at TP-2, 616 vs 482 at TP-4, 664
    // vs 421 at TP-8), so auto takes the peer kernels at every rank count.
    uint32_t tpRanks = 1;
    if (comm) OPURE_CUDA_CHECK(opure_comm_info(comm, &tpRanks, nullptr));
    const bool wantPeer = opts.tpAllreduce == 2 || (opts.tpAllreduce == 0 && tpRanks >= 2);
    if (comm && wantPeer) {
        // NVLink peer mailboxes for the fused all-reduces; every rank falls back to NCCL
        // together when any pair of GPUs cannot map each other's memory.
        const opure_status ps = opure_peer_create(ctx_, comm, cfg.hiddenSize, 2000, &peer_);
        if (ps == OPURE_ERR_UNSUPPORTED)
            peer_ = nullptr;
        else
            OPURE_CUDA_CHECK(ps);
    }
    seqLen_ = 0;
    ready_ = true;
    if ((opts.path == 2 || opts.path == 3) && !UsesFused(opts.maxBatch))
        ThrowError("the fused decode path does not support this model or batch size");
}

bool VoxelEngine::UsesFused(uint32_t n) const {
    const graph::ModelConfig &c = graph_.Config();
    const graph::VramPlan &p = graph_.Plan();
    const uint32_t hd = c.HeadDim(), G = c.KvGroupSize();
    const bool shape = !comm_ && p.hasFused && !p.lmQuantized && G >= 1 && G <= 4 &&
                       (n == 1 || n == 2 || n == 4 || n == 8) && 3ull * c.hiddenSize * 2 <= 160 * 1024;
    if (p.wDtype == OPURE_W_Q8)  // GEMV_Quant weights: the persistent kernel only
        return shape && opts_.path != 1 && opts_.path != 3 && hd == 64 && c.numLayers <= 48 &&
               c.hiddenSize % 16 == 0 && (G * hd) % 16 == 0;
    return shape && opts_.path != 1 && (hd == 64 || hd == 128);
}

bool VoxelEngine::Chained(uint32_t n) const {
    const graph::ModelConfig &c = graph_.Config();
    const graph::VramPlan &p = graph_.Plan();
    const uint32_t att = c.numHeads * c.HeadDim();
    return !comm_ && p.wDtype == OPURE_W_F16 && !p.lmQuantized && n >= 16 && n <= 256 && n <= maxVec_ &&
           (c.HeadDim() == 64 || c.HeadDim() == 128) &&  // the attention kernel with packed output
           c.hiddenSize % 64 == 0 && c.intermediateSize % 64 == 0 && att % 64 == 0 && c.hiddenSize <= 16384 &&
           c.intermediateSize <= 16384 && att <= 16384 && buf_.packRes != nullptr;
}

void VoxelEngine::AllocBuffers() {
    const graph::ModelConfig &c = graph_.Config();
    const uint32_t B = maxVec_;  // token vectors per step (sequence slots: opts_.maxBatch)
    buf_.x = Alloc<float>(ctx_, size_t(B) * c.hiddenSize);
    buf_.qkv = Alloc<float>(ctx_, size_t(B) * c.QkvRows());
    buf_.q = Alloc<float>(ctx_, size_t(B) * c.numHeads * c.HeadDim());
    buf_.attn = Alloc<float>(ctx_, size_t(B) * c.hiddenSize);
    buf_.h = Alloc<float>(ctx_, size_t(B) * c.intermediateSize);
    buf_.logits = Alloc<float>(ctx_, size_t(B) * c.vocabSize);
    buf_.keys = Alloc<unsigned long long>(ctx_, B);
    buf_.seq = Alloc<int32_t>(ctx_, B);
    buf_.seqLen = Alloc<int32_t>(ctx_, B);
    buf_.known = Alloc<int32_t>(ctx_, B);
    buf_.flags = Alloc<uint32_t>(ctx_, B);
    // Host-given tokens and positions side by side, as in the pinned staging buffer, so the
    // host-driven step copies both with one H2D (buf_.pos is not a separate allocation).
    buf_.inTokens = Alloc<int32_t>(ctx_, 2 * size_t(B));
    buf_.pos = buf_.inTokens + B;
    buf_.tokens = Alloc<int32_t>(ctx_, size_t(opts_.maxBatch) * maxLen_);
    buf_.prefillKeys = Alloc<unsigned long long>(ctx_, opts_.maxBatch);
    buf_.base1 = Alloc<float>(ctx_, size_t(B) * c.hiddenSize);
    buf_.delta0 = Alloc<long long>(ctx_, size_t(B) * c.hiddenSize);
    buf_.delta1 = Alloc<long long>(ctx_, size_t(B) * c.hiddenSize);
    if (!comm_ && B >= 16) {
        const uint32_t nv = std::min<uint32_t>(B, 256);
        const uint32_t att = c.numHeads * c.HeadDim();
        auto packed = [&](uint32_t len) {
            const size_t bytes = opure_packed_bytes(nv, len);
            void *ptr = nullptr;
            OPURE_CUDA_CHECK(opure_alloc(ctx_, bytes, &ptr));
            OPURE_CUDA_CHECK(opure_fill(ctx_, ptr, 0, bytes));  // padding rows stay zero
            return static_cast<uint16_t *>(ptr);
        };
        buf_.packAttn = packed(att);
        buf_.packRes = packed(c.hiddenSize);
        buf_.packAct = packed(c.intermediateSize);
        buf_.sumsq = Alloc<float>(ctx_, size_t((c.hiddenSize + 127) / 128) * nv);
    }
    if (comm_) buf_.partial = Alloc<float>(ctx_, size_t(B) * c.hiddenSize);
    buf_.sync = Alloc<uint32_t>(ctx_, 3 * size_t(c.numLayers) + 1);
    if (opts_.phaseTrace) {
        opure_device_info di{};
        OPURE_CUDA_CHECK(opure_get_device_info(ctx_, &di));
        traceWords_ = size_t(di.sm_count) * (3 * size_t(c.numLayers) + 2) * 2;
        buf_.trace = Alloc<unsigned long long>(ctx_, traceWords_);
        OPURE_CUDA_CHECK(opure_fill(ctx_, buf_.trace, 0, traceWords_ * 8));
    }
    OPURE_CUDA_CHECK(opure_fill(ctx_, buf_.keys, 0, sizeof(unsigned long long) * B));
    // Per-vector step state starts defined (no self-driving vector, nothing known).
    OPURE_CUDA_CHECK(opure_fill(ctx_, buf_.flags, 0, sizeof(uint32_t) * B));
    OPURE_CUDA_CHECK(opure_fill(ctx_, buf_.known, 0, sizeof(int32_t) * B));
    OPURE_CUDA_CHECK(opure_fill(ctx_, buf_.tokens, 0, sizeof(int32_t) * size_t(opts_.maxBatch) * maxLen_));
    // Pinned staging for the host-driven step: [in_tokens B][positions B][keys B (u64)], B =
    // token vectors per step (the device's inTokens / pos layout).
    OPURE_CUDA_CHECK(opure_alloc_host(ctx_, size_t(B) * 16, &hostIo_));
    OPURE_CUDA_CHECK(opure_sync(ctx_, 60000));
}

void *VoxelEngine::AttnScratch(uint32_t n, size_t *bytes) {
    auto it = attnScratch_.find(n);
    if (it == attnScratch_.end()) {
        const graph::ModelConfig &c = graph_.Config();
        const size_t b = opure_attention_scratch_bytes(n, 1, c.numHeads, c.numKvHeads, c.HeadDim(), maxLen_, 0);
        OPURE_CHECK(b > 0, "attention scratch size query failed");
        void *p = nullptr;
        OPURE_CUDA_CHECK(opure_alloc(ctx_, b, &p));
        OPURE_CUDA_CHECK(opure_fill(ctx_, p, 0, b));  // split counters start at zero
        it = attnScratch_.emplace(n, std::make_pair(p, b)).first;
    }
    *bytes = it->second.second;
    return it->second.first;
}

opure_step_io VoxelEngine::StepIO(uint32_t n) const {
    const graph::ModelConfig &c = graph_.Config();
    opure_step_io io{};
    io.nvec = n;
    io.seq = buf_.seq;
    io.pos = buf_.pos;
    io.seq_len = buf_.seqLen;
    io.known = buf_.known;
    io.flags = buf_.flags;
    io.in_tokens = buf_.inTokens;
    io.tokens = buf_.tokens;
    io.max_len = maxLen_;
    io.keys = buf_.keys;
    io.embed = reinterpret_cast<const uint16_t *>(At(weights_, graph_.Plan().embedTokens));
    io.vocab = c.vocabSize;
    io.hidden = c.hiddenSize;
    io.x = buf_.x;
    return io;
}

void VoxelEngine::RecordLayer(uint32_t L, uint32_t n) {
    const graph::ModelConfig &c = graph_.Config();
    const graph::VramPlan &plan = graph_.Plan();
    const graph::VramPlan::LayerTensors &t = plan.layers[L];
    const graph::LocalGeometry &lg = graph_.Local();  // the whole model unless tensor-parallel
    const uint32_t h = c.hiddenSize, ff = lg.inter, hd = c.HeadDim();
    const uint32_t qkvRows = lg.QkvRows(hd), att = lg.heads * hd;
    const bool q8 = plan.wDtype == OPURE_W_Q8;
    const uint64_t eb = q8 ? 1 : 2;

    // Chained tensor-core operands: each GEMV's epilogue (and the attention kernel) writes the
    // next GEMV's packed fp16 input, and the residual's sums of squares for its RMSNorm, so
    // no pack kernel runs between them (the first layer's q;k;v packs the embedding rows).
    const bool ch = Chained(n);
    struct Chain {
        const uint16_t *in = nullptr;
        const float *inSumsq = nullptr;
        uint16_t *out = nullptr;
        const void *outGain = nullptr;
        float *outSumsq = nullptr;
    };
    auto gemv = [&](const void *w, float scale, float scale2, uint32_t rows, uint32_t cols,
                    const float *x, uint32_t xs, float *y, uint32_t ys, uint32_t pro,
                    const void *gain, uint32_t epi, const float *res, const Chain &chain = Chain{}) {
        opure_gemv_args a{};
        a.w = w;
        a.w_dtype = plan.wDtype;
        a.scale_w = scale;
        a.scale_x = 1.0f;  // activations stay fp32 (Opure_VoxelEngine.cpp:200-206)
        a.scale_w2 = scale2;
        a.rows = rows;
        a.cols = cols;
        a.nvec = n;
        a.x = x;
        a.x_stride = xs;
        a.y = y;
        a.y_stride = ys;
        a.prologue = pro;
        a.norm_gain = static_cast<const uint16_t *>(gain);
        a.eps = c.rmsNormEps;
        a.epilogue = epi;
        a.residual = res;
        a.x_packed = chain.in;
        a.x_sumsq = chain.inSumsq;
        a.y_packed = chain.out;
        a.y_pack_gain = static_cast<const uint16_t *>(chain.outGain);
        a.y_sumsq = chain.outSumsq;
        OPURE_CUDA_CHECK(opure_gemv(ctx_, &a));
    };
    const void *inNorm = At(weights_, t.inputNorm), *postNorm = At(weights_, t.postAttNorm);
    // The gain of the RMSNorm after this layer: the next layer's input norm, or the final norm.
    const void *nextNorm =
        L + 1 < c.numLayers ? At(weights_, plan.layers[L + 1].inputNorm) : At(weights_, plan.finalNorm);
    Chain qkvIn, oChain, guChain, downChain;
    if (ch) {
        if (L > 0) {
            qkvIn.in = buf_.packRes;
            qkvIn.inSumsq = buf_.sumsq;
        }
        oChain.in = buf_.packAttn;
        oChain.out = buf_.packRes;
        oChain.outGain = postNorm;
        oChain.outSumsq = buf_.sumsq;
        guChain.in = buf_.packRes;
        guChain.inSumsq = buf_.sumsq;
        guChain.out = buf_.packAct;
        downChain.in = buf_.packAct;
        downChain.out = buf_.packRes;
        downChain.outGain = nextNorm;
        downChain.outSumsq = buf_.sumsq;
    }

    // q;k;v in one pass over the concatenated rows (three passes for int8, whose
    // per-tensor scales differ).
    if (!q8) {
        gemv(At(weights_, t.wqkv), 1.f, 1.f, qkvRows, h, buf_.x, h, buf_.qkv, qkvRows, OPURE_PRO_RMSNORM,
             inNorm, OPURE_EPI_STORE, nullptr, qkvIn);
    } else {
        const uint32_t qr = lg.heads * hd, kr = lg.kvHeads * hd;
        gemv(At(weights_, t.wqkv), t.sq, t.sq, qr, h, buf_.x, h, buf_.qkv, qkvRows, OPURE_PRO_RMSNORM,
             inNorm, OPURE_EPI_STORE, nullptr);
        gemv(At(weights_, t.wqkv + uint64_t(qr) * h * eb), t.sk, t.sk, kr, h, buf_.x, h, buf_.qkv + qr, qkvRows,
             OPURE_PRO_RMSNORM, inNorm, OPURE_EPI_STORE, nullptr);
        gemv(At(weights_, t.wqkv + uint64_t(qr + kr) * h * eb), t.sv, t.sv, kr, h, buf_.x, h, buf_.qkv + qr + kr,
             qkvRows, OPURE_PRO_RMSNORM, inNorm, OPURE_EPI_STORE, nullptr);
    }
    const opure_kv_layout kv = kv_.Layout(L);
    OPURE_CUDA_CHECK(opure_rope_kv_append(ctx_, buf_.qkv, qkvRows, buf_.q, buf_.seq, buf_.pos, n, lg.heads,
                                          c.ropeTheta, &kv));
    opure_attn_args a{};
    a.q = buf_.q;
    a.out = buf_.attn;
    a.seq = buf_.seq;
    a.seq_len = buf_.seqLen;
    a.n = n;
    a.n_q = 1;
    a.n_heads = lg.heads;
    a.scale = opts_.attnScale;
    a.max_ctx = maxLen_;
    a.split_tokens = 0;
    a.scratch = AttnScratch(n, &a.scratch_bytes);
    a.kv = kv;
    a.out_packed = ch ? buf_.packAttn : nullptr;
    OPURE_CUDA_CHECK(opure_attention(ctx_, &a));
    if (!comm_) {
        // o_proj + residual, in place on the residual stream.
        gemv(At(weights_, t.wo), t.so, t.so, h, h, buf_.attn, h, buf_.x, h, OPURE_PRO_NONE, nullptr, OPURE_EPI_ADD,
             buf_.x, oChain);
    } else if (peer_) {
        // Tensor parallel over NVLink peer memory: one kernel computes this shard's partial
        // o_proj sum, exchanges it with every rank and adds the total to the residual.
        TpGemvAllreduce(At(weights_, t.wo), t.so, h, att, buf_.attn, h, n);
    } else {
        // Tensor parallel: this shard's heads give a partial o_proj sum over their input
        // columns; the shards' partials are summed over NCCL, then added to the residual.
        gemv(At(weights_, t.wo), t.so, t.so, h, att, buf_.attn, h, buf_.partial, h, OPURE_PRO_NONE, nullptr,
             OPURE_EPI_STORE, nullptr);
        OPURE_CUDA_CHECK(opure_allreduce_sum_f32(ctx_, comm_, buf_.partial, size_t(n) * h));
        OPURE_CUDA_CHECK(opure_add(ctx_, buf_.x, buf_.partial, buf_.x, n * h));
    }
    // gate;up with the post-attention norm, SwiGLU epilogue.
    gemv(At(weights_, t.wgu), t.sgate, t.sup, ff, h, buf_.x, h, buf_.h, ff, OPURE_PRO_RMSNORM, postNorm,
         OPURE_EPI_SWIGLU, nullptr, guChain);
    if (!comm_) {
        // down_proj + residual.
        gemv(At(weights_, t.wdown), t.sdown, t.sdown, h, ff, buf_.h, ff, buf_.x, h, OPURE_PRO_NONE, nullptr,
             OPURE_EPI_ADD, buf_.x, downChain);
    } else if (peer_) {
        TpGemvAllreduce(At(weights_, t.wdown), t.sdown, h, ff, buf_.h, ff, n);
    } else {
        gemv(At(weights_, t.wdown), t.sdown, t.sdown, h, ff, buf_.h, ff, buf_.partial, h, OPURE_PRO_NONE, nullptr,
             OPURE_EPI_STORE, nullptr);
        OPURE_CUDA_CHECK(opure_allreduce_sum_f32(ctx_, comm_, buf_.partial, size_t(n) * h));
        OPURE_CUDA_CHECK(opure_add(ctx_, buf_.x, buf_.partial, buf_.x, n * h));
    }
}

// residual x += sum over the tensor-parallel ranks of W_rank . in_rank (o_proj / down_proj
// shards, `cols` input columns each), reduced over NVLink inside the GEMV kernel.
void VoxelEngine::TpGemvAllreduce(const void *w, float scale, uint32_t rows, uint32_t cols, const float *in,
                                  uint32_t in_stride, uint32_t n) {
    opure_gemv_args a{};
    a.w = w;
    a.w_dtype = graph_.Plan().wDtype;
    a.scale_w = scale;
    a.scale_x = 1.0f;
    a.scale_w2 = scale;
    a.rows = rows;
    a.cols = cols;
    a.nvec = n;
    a.x = in;
    a.x_stride = in_stride;
    a.y = buf_.x;
    a.y_stride = rows;
    a.prologue = OPURE_PRO_NONE;
    a.epilogue = OPURE_EPI_ADD;
    a.residual = buf_.x;
    OPURE_CUDA_CHECK(opure_gemv_allreduce(ctx_, peer_, &a));
}

void VoxelEngine::RecordStep(uint32_t n, bool logits) {
    const graph::ModelConfig &c = graph_.Config();
    const graph::VramPlan &plan = graph_.Plan();
    const opure_step_io io = StepIO(n);
    OPURE_CUDA_CHECK(opure_step_begin(ctx_, &io));
    if (UsesFused(n)) {
        std::vector<opure_fused_layer> layers(c.numLayers);
        for (uint32_t L = 0; L < c.numLayers; ++L) {
            const graph::VramPlan::LayerTensors &t = plan.layers[L];
            opure_fused_layer &f = layers[L];
            f.in_norm = reinterpret_cast<const uint16_t *>(At(weights_, t.inputNorm));
            f.post_norm = reinterpret_cast<const uint16_t *>(At(weights_, t.postAttNorm));
            f.w_qkv = reinterpret_cast<const uint16_t *>(At(weights_, t.wqkv));
            f.w_o_blk = reinterpret_cast<const uint16_t *>(At(weights_, t.woBlk));
            f.w_gate_up = reinterpret_cast<const uint16_t *>(At(weights_, t.wgu));
            f.w_down_t = reinterpret_cast<const uint16_t *>(At(weights_, t.wdownT));
            f.kv_pool = kv_.Pool(L);
            f.s_q = t.sq;
            f.s_k = t.sk;
            f.s_v = t.sv;
            f.s_o = t.so;
            f.s_gate = t.sgate;
            f.s_up = t.sup;
            f.s_down = t.sdown;
        }
        opure_fused_step fs{};
        fs.nvec = n;
        fs.hidden = c.hiddenSize;
        fs.inter = c.intermediateSize;
        fs.n_heads = c.numHeads;
        fs.n_kv = c.numKvHeads;
        fs.head_dim = c.HeadDim();
        fs.vocab = c.vocabSize;
        fs.n_layers = c.numLayers;
        fs.eps = c.rmsNormEps;
        fs.attn_scale = opts_.attnScale;
        fs.theta = c.ropeTheta;
        fs.layers = layers.data();
        fs.final_norm = reinterpret_cast<const uint16_t *>(At(weights_, plan.finalNorm));
        fs.lm_head = reinterpret_cast<const uint16_t *>(At(weights_, plan.lmHead));
        fs.page_table = kv_.DeviceTable();
        fs.n_pages = kv_.NumPages();
        fs.max_pages = kv_.MaxPages();
        fs.page_size = kv_.PageSize();
        fs.kv_ring = kv_.Ring();
        fs.seq = buf_.seq;
        fs.pos = buf_.pos;
        fs.x = buf_.x;
        fs.base1 = buf_.base1;
        fs.delta0 = buf_.delta0;
        fs.delta1 = buf_.delta1;
        fs.q = buf_.q;
        fs.logits = logits ? buf_.logits : nullptr;
        fs.keys = buf_.keys;
        fs.sync = buf_.sync;
        fs.trace = buf_.trace;
        fs.mode = opts_.path == 3 ? uint32_t(OPURE_FUSED_LAYER_KERNELS) : uint32_t(OPURE_FUSED_AUTO);
        fs.w_dtype = plan.wDtype;
        OPURE_CUDA_CHECK(opure_decode_fused(ctx_, &fs));
        OPURE_CUDA_CHECK(opure_step_end(ctx_, &io));
        return;
    }
    for (uint32_t L = 0; L < c.numLayers; ++L) RecordLayer(L, n);
    // Final norm + (tied) LM head + argmax (Opure_VoxelEngine.cpp:514-532, ArgMax :783-791).
    opure_gemv_args a{};
    a.w = At(weights_, plan.lmHead);
    a.w_dtype = plan.lmQuantized ? uint32_t(OPURE_W_Q8) : uint32_t(OPURE_W_F16);
    a.scale_w = plan.slm;
    a.scale_x = 1.0f;
    const graph::LocalGeometry &lg = graph_.Local();
    a.rows = lg.vocab;  // tensor parallel: this shard's vocabulary rows
    a.cols = c.hiddenSize;
    a.nvec = n;
    a.x = buf_.x;
    a.x_stride = c.hiddenSize;
    a.y = logits ? buf_.logits : nullptr;
    a.y_stride = lg.vocab;
    a.prologue = OPURE_PRO_RMSNORM;
    a.norm_gain = reinterpret_cast<const uint16_t *>(At(weights_, plan.finalNorm));
    a.eps = c.rmsNormEps;
    a.epilogue = OPURE_EPI_ARGMAX;
    a.argmax_keys = buf_.keys;
    if (Chained(n)) {
        // The last down_proj left the final-norm-gained residual packed.
        a.x_packed = buf_.packRes;
        a.x_sumsq = buf_.sumsq;
    }
    OPURE_CUDA_CHECK(opure_gemv(ctx_, &a));
    if (peer_ && n <= OPURE_PEER_MAX_KEYS) {
        // Vocabulary shards: global indices and the largest key over all shards in one
        // peer kernel (ties keep the lowest global index, as in one unsplit argmax).
        OPURE_CUDA_CHECK(opure_peer_argmax(ctx_, peer_, buf_.keys, n, lg.vocabOffset));
    } else if (comm_) {
        // Vocabulary shards: global indices, then the largest key over all shards (ties
        // keep the lowest global index, as in one unsplit argmax).
        OPURE_CUDA_CHECK(opure_argmax_key_offset(ctx_, buf_.keys, n, lg.vocabOffset));
        OPURE_CUDA_CHECK(opure_allreduce_max_u64(ctx_, comm_, buf_.keys, n));
    }
    OPURE_CUDA_CHECK(opure_step_end(ctx_, &io));
}

void VoxelEngine::RunSteps(uint32_t n, uint32_t steps, bool logits) {
    OPURE_CHECK(ready_, "engine used before Initialize");
    OPURE_CHECK(n >= 1 && n <= maxVec_, "more token vectors than the engine's step capacity");
    if (!opts_.useGraphs) {
        for (uint32_t s = 0; s < steps; ++s) RecordStep(n, logits);
        return;
    }
    const auto key = std::make_pair(n, logits);
    auto it = graphs_.find(key);
    if (it == graphs_.end()) {
        size_t dummy = 0;
        AttnScratch(n, &dummy);  // allocate outside the capture
        OPURE_CUDA_CHECK(opure_sync(ctx_, 60000));
        OPURE_CUDA_CHECK(opure_graph_begin(ctx_));
        try {
            RecordStep(n, logits);
        } catch (...) {
            opure_graph *g = nullptr;
            opure_graph_end(ctx_, &g);
            if (g) opure_graph_free(g);
            throw;
        }
        opure_graph *g = nullptr;
        OPURE_CUDA_CHECK(opure_graph_end(ctx_, &g));
        it = graphs_.emplace(key, g).first;
    }
    for (uint32_t s = 0; s < steps; ++s) OPURE_CUDA_CHECK(opure_graph_launch(ctx_, it->second));
}

void VoxelEngine::SetPositions(const int32_t *positions, uint32_t n) {
    OPURE_CHECK(n >= 1 && n <= opts_.maxBatch, "batch exceeds maxBatch");
    for (uint32_t v = 0; v < n; ++v) {
        OPURE_CHECK(positions[v] >= 0 && uint32_t(positions[v]) < maxLen_, "position exceeds maxLen");
        OPURE_CHECK(kv_.Covers(v, uint32_t(positions[v])), "position beyond the sequence's reserved KV pages");
    }
    // Pageable source: the copy is staged before opure_h2d returns, so the caller's
    // array may be reused immediately.
    OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.pos, positions, n * 4));
}

void VoxelEngine::Sync() {
    OPURE_CUDA_CHECK(opure_sync(ctx_, 600000));
    CheckDevice(ctx_);
}

void CheckDevice(opure_ctx *ctx) {
    uint32_t where = 0, detail = 0;
    const opure_status st = opure_last_error_detail(ctx, &where, &detail);
    if (st != OPURE_OK)
        ThrowError(std::string("device reported: ") + opure_strerror(st) + " (kernel site " + std::to_string(where) +
                       ", value " + std::to_string(detail) + ")",
                   st);
}

void VoxelEngine::ResetSequences(const std::vector<std::vector<uint32_t>> &prompts, uint32_t reserve,
                                 bool automatic) {
    const uint32_t n = uint32_t(prompts.size());
    OPURE_CHECK(n >= 1 && n <= opts_.maxBatch, "batch exceeds maxBatch");
    OPURE_CHECK(reserve <= maxLen_, "sequence exceeds the engine's maxLen");
    const graph::ModelConfig &c = graph_.Config();
    std::vector<int32_t> seq(n), pos(n, 0), known(n);
    // Flags of every vector slot: the n sequences' vectors self-drive or not, and no other
    // slot self-drives (a chunked prefill step uses more vectors than there are sequences).
    std::vector<uint32_t> flags(maxVec_, 0u);
    std::fill(flags.begin(), flags.begin() + n, automatic ? uint32_t(OPURE_VEC_AUTO) : 0u);
    for (uint32_t v = 0; v < n; ++v) {
        OPURE_CHECK(!prompts[v].empty(), "empty prompt");
        OPURE_CHECK(prompts[v].size() <= reserve, "prompt exceeds the reserved length");
        for (uint32_t t : prompts[v]) OPURE_CHECK(t < c.vocabSize, "token id out of vocabulary range");
        seq[v] = int32_t(v);
        known[v] = int32_t(prompts[v].size());
        kv_.Release(v);
        OPURE_CHECK(kv_.Reserve(v, reserve), "KV cache has no room for the sequence");
        std::vector<int32_t> row(prompts[v].begin(), prompts[v].end());
        OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.tokens + size_t(v) * maxLen_, row.data(), row.size() * 4));
        OPURE_CUDA_CHECK(opure_sync(ctx_, 60000));
    }
    kv_.SyncTable();
    OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.seq, seq.data(), n * 4));
    OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.pos, pos.data(), n * 4));
    OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.known, known.data(), n * 4));
    OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.flags, flags.data(), flags.size() * 4));
    hostDriven_ = !automatic;
    seqIdentity_ = true;
    OPURE_CUDA_CHECK(opure_fill(ctx_, buf_.keys, 0, n * 8));
    OPURE_CUDA_CHECK(opure_sync(ctx_, 60000));
}

uint32_t VoxelEngine::PrefillChunks(const std::vector<std::vector<uint32_t>> &prompts) {
    // Every prompt position of every sequence becomes one token vector; chunks of up to
    // prefillChunk vectors run as single steps (each vector's attention covers exactly the
    // KV rows before it, including the ones appended by the same step), so a chunk's
    // projections run as tensor-core GEMMs over all its tokens at once.
    const uint32_t n = uint32_t(prompts.size()), C = opts_.prefillChunk;
    std::vector<int32_t> seq, pos, tok;
    std::vector<int32_t> known(n), start(n);
    for (uint32_t s = 0; s < n; ++s) {
        // With a KV window every prompt position must still have its own page: a step's
        // later vectors would otherwise overwrite pages its earlier vectors attend to.
        OPURE_CHECK(!kv_.Ring() || prompts[s].size() <= kv_.Ring() * kv_.PageSize(),
                    "chunked prefill needs the prompt to fit the KV window");
        for (uint32_t t = 0; t < prompts[s].size(); ++t) {
            seq.push_back(int32_t(s));
            pos.push_back(int32_t(t));
            tok.push_back(int32_t(prompts[s][t]));
        }
        known[s] = start[s] = int32_t(prompts[s].size());
    }
    uint32_t steps = 0;
    for (size_t i0 = 0; i0 < seq.size(); i0 += C) {
        const uint32_t m = uint32_t(std::min<size_t>(C, seq.size() - i0));
        SetVectors(seq.data() + i0, pos.data() + i0, tok.data() + i0, m);
        RunSteps(m, 1, false);
        ++steps;
        // The argmax after each sequence's last prompt token: its first generated token.
        for (uint32_t j = 0; j < m; ++j) {
            const uint32_t s = uint32_t(seq[i0 + j]);
            if (pos[i0 + j] + 1 == known[s])
                OPURE_CUDA_CHECK(opure_d2d(ctx_, buf_.prefillKeys + s, buf_.keys + j, 8));
        }
    }
    // Continue self-driving: vector s at position len_s takes the saved key as its input.
    OPURE_CUDA_CHECK(opure_d2d(ctx_, buf_.keys, buf_.prefillKeys, size_t(n) * 8));
    SetAutoVectors(start.data(), known.data(), n);
    return steps;
}

std::vector<GenerateResult> VoxelEngine::GenerateBatch(const std::vector<std::vector<uint32_t>> &prompts,
                                                       uint32_t budget, StepTiming *timing) {
    OPURE_CHECK(ready_, "engine used before Initialize");
    const uint32_t n = uint32_t(prompts.size());
    const uint32_t maxPos = graph_.Config().maxPositions;
    const int64_t eos = graph_.Config().eosTokenId;
    uint32_t maxP = 0;
    for (const auto &p : prompts) maxP = std::max<uint32_t>(maxP, uint32_t(p.size()));
    // The reference's stop rules (Opure_VoxelEngine.cpp:918-933): after pushing a token the
    // loop ends when seqLen + 1 >= maxPos, so a prompt of length len gets at most
    // maxPos - len tokens; and it ends on the stop id, kept as the last token.
    // A step at position p writes the token of position p into the history (the previous
    // step's argmax). After the prefill, vector v stands at start[v]: its prompt length
    // (chunked prefill) or the longest prompt's (one token per step: shorter prompts
    // generate meanwhile); after k decode steps its history holds positions < start + k.
    const bool chunked = opts_.prefillChunk > 0;
    std::vector<uint32_t> limit(n), start(n);
    uint32_t steps = 0;
    for (uint32_t v = 0; v < n; ++v) {
        const uint32_t len = uint32_t(prompts[v].size());
        OPURE_CHECK(len < maxPos, "prompt reaches max_position_embeddings");
        limit[v] = std::min(budget, maxPos - len);
        start[v] = chunked ? len : maxP;
        if (len + limit[v] > start[v]) steps = std::max(steps, len + limit[v] - start[v]);
    }
    OPURE_CHECK(maxP + steps <= maxLen_ && maxP + steps > 0, "prompt + budget exceeds the engine's maxLen");
    ResetSequences(prompts, maxP + steps, !chunked);

    opure_event *e0 = nullptr, *e1 = nullptr, *e2 = nullptr;
    OPURE_CUDA_CHECK(opure_event_create(ctx_, &e0));
    OPURE_CUDA_CHECK(opure_event_create(ctx_, &e1));
    OPURE_CUDA_CHECK(opure_event_create(ctx_, &e2));
    OPURE_CUDA_CHECK(opure_event_record(ctx_, e0));
    uint32_t prefillSteps = maxP;
    if (chunked)
        prefillSteps = PrefillChunks(prompts);
    else
        RunSteps(n, maxP, false);
    OPURE_CUDA_CHECK(opure_event_record(ctx_, e1));
    std::vector<int32_t> rows(size_t(n) * maxLen_);
    // Index of each sequence's last token: limit - 1, or its first stop id.
    std::vector<uint32_t> end(n);
    auto scan = [&](uint32_t upto) {  // after `upto` decode steps
        bool all = true;
        for (uint32_t v = 0; v < n; ++v) {
            const uint32_t len = uint32_t(prompts[v].size());
            end[v] = limit[v] ? limit[v] - 1 : 0;
            bool found = false;
            for (uint32_t k = 0; eos >= 0 && k < limit[v] && len + k < start[v] + upto; ++k)
                if (rows[size_t(v) * maxLen_ + len + k] == int32_t(eos)) {
                    end[v] = k;
                    found = true;
                    break;
                }
            all = all && (found || len + limit[v] <= start[v] + upto);
        }
        return all;
    };
    uint32_t done = 0;
    if (eos < 0) {
        RunSteps(n, steps, false);
        done = steps;
    } else {
        // With a stop id the steps run in chunks, and the loop ends early once every
        // sequence has produced it (one token-row readback per chunk).
        constexpr uint32_t kChunk = 16;
        for (;;) {
            OPURE_CUDA_CHECK(opure_d2h(ctx_, rows.data(), buf_.tokens, rows.size() * 4));
            OPURE_CUDA_CHECK(opure_sync(ctx_, 600000));
            if (scan(done) || done == steps) break;
            const uint32_t c = std::min(kChunk, steps - done);
            RunSteps(n, c, false);
            done += c;
        }
    }
    OPURE_CUDA_CHECK(opure_event_record(ctx_, e2));
    Sync();
    float pre = 0.f, dec = 0.f;
    OPURE_CUDA_CHECK(opure_event_elapsed_ms(e0, e1, &pre));
    OPURE_CUDA_CHECK(opure_event_elapsed_ms(e1, e2, &dec));
    opure_event_free(e0);
    opure_event_free(e1);
    opure_event_free(e2);

    OPURE_CUDA_CHECK(opure_d2h(ctx_, rows.data(), buf_.tokens, rows.size() * 4));
    OPURE_CUDA_CHECK(opure_sync(ctx_, 60000));
    scan(done);
    std::vector<GenerateResult> out(n);
    for (uint32_t v = 0; v < n; ++v) {
        GenerateResult &r = out[v];
        r.promptTokens = prompts[v];
        const uint32_t count = limit[v] ? end[v] + 1 : 0;
        const size_t b = size_t(v) * maxLen_ + prompts[v].size();
        r.generated.assign(rows.begin() + b, rows.begin() + b + count);
        if (count && eos >= 0 && r.generated.back() == uint32_t(eos)) {
            r.hitStop = true;
            r.stopToken = uint32_t(eos);
        }
        r.msPerToken = count ? double(dec) / count : 0.0;
        r.lastMs = done ? double(dec) / done : 0.0;
    }
    if (timing) {
        timing->prefillMs = pre;
        timing->decodeMs = dec;
        timing->prefillSteps = prefillSteps;
        timing->decodeSteps = done;
    }
    seqLen_ = maxP + done;
    lastTokenMs_ = done ? double(dec) / done : 0.0;
    return out;
}

std::vector<uint32_t> VoxelEngine::PrefillBatch(const std::vector<std::vector<uint32_t>> &prompts,
                                                uint32_t reserve, bool logits) {
    OPURE_CHECK(ready_, "engine used before Initialize");
    const uint32_t n = uint32_t(prompts.size());
    const size_t len = prompts.front().size();
    for (const auto &p : prompts) OPURE_CHECK(p.size() == len, "PrefillBatch needs prompts of equal length");
    ResetSequences(prompts, reserve, true);
    RunSteps(n, uint32_t(len), logits);
    Sync();
    std::vector<unsigned long long> keys(n);
    OPURE_CUDA_CHECK(opure_d2h(ctx_, keys.data(), buf_.keys, n * 8));
    OPURE_CUDA_CHECK(opure_sync(ctx_, 60000));
    std::vector<uint32_t> next(n);
    for (uint32_t v = 0; v < n; ++v) next[v] = 0xffffffffu - uint32_t(keys[v] & 0xffffffffull);
    return next;
}

void VoxelEngine::SetVectors(const int32_t *seq, const int32_t *pos, const int32_t *tok, uint32_t n) {
    OPURE_CHECK(n >= 1 && n <= maxVec_, "more token vectors than the engine's step capacity");
    const uint32_t V = graph_.Config().vocabSize;
    for (uint32_t v = 0; v < n; ++v) {
        OPURE_CHECK(seq[v] >= 0 && uint32_t(seq[v]) < opts_.maxBatch, "sequence slot out of range");
        OPURE_CHECK(pos[v] >= 0 && uint32_t(pos[v]) < maxLen_, "position exceeds the engine's maxLen");
        OPURE_CHECK(!tok || (tok[v] >= 0 && uint32_t(tok[v]) < V), "token id out of vocabulary range");
        OPURE_CHECK(kv_.Reserve(uint32_t(seq[v]), uint32_t(pos[v]) + 1), "KV cache has no room for the sequence");
    }
    kv_.SyncTable();
    // Pageable sources: staged before the calls return, so the arrays may be reused.
    OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.seq, seq, n * 4));
    OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.pos, pos, n * 4));
    if (tok) OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.inTokens, tok, n * 4));
    seqIdentity_ = false;
    // Every vector of the step takes its token from the host: clear the self-driving flag of
    // all n (earlier calls may have set flags for fewer vectors, e.g. one per prompt).
    const std::vector<uint32_t> zero(n, 0u);
    OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.flags, zero.data(), n * 4));
    hostDriven_ = true;
}

void VoxelEngine::SetAutoVectors(const int32_t *pos, const int32_t *known, uint32_t n) {
    OPURE_CHECK(ready_, "engine used before Initialize");
    OPURE_CHECK(n >= 1 && n <= opts_.maxBatch, "more token vectors than maxBatch");
    std::vector<int32_t> seq(n);
    std::vector<uint32_t> flags(n, uint32_t(OPURE_VEC_AUTO));
    for (uint32_t v = 0; v < n; ++v) {
        OPURE_CHECK(pos[v] >= 0 && uint32_t(pos[v]) < maxLen_, "position exceeds the engine's maxLen");
        OPURE_CHECK(known[v] >= 0 && uint32_t(known[v]) <= maxLen_, "known length exceeds the engine's maxLen");
        OPURE_CHECK(kv_.Covers(v, uint32_t(pos[v])), "position beyond the sequence's reserved KV pages");
        seq[v] = int32_t(v);
    }
    OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.seq, seq.data(), n * 4));
    OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.pos, pos, n * 4));
    OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.known, known, n * 4));
    OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.flags, flags.data(), n * 4));
    seqIdentity_ = true;
    hostDriven_ = false;
}

void VoxelEngine::WriteHistory(uint32_t slot, uint32_t pos, const int32_t *tokens, uint32_t count) {
    OPURE_CHECK(slot < opts_.maxBatch && uint64_t(pos) + count <= maxLen_, "history write out of range");
    const uint32_t V = graph_.Config().vocabSize;
    for (uint32_t i = 0; i < count; ++i)
        OPURE_CHECK(tokens[i] >= 0 && uint32_t(tokens[i]) < V, "token id out of vocabulary range");
    OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.tokens + size_t(slot) * maxLen_ + pos, tokens, size_t(count) * 4));
}

GenerateResult VoxelEngine::Generate(const std::vector<uint32_t> &tokens, const EngineOptions &opts) {
    GenerateResult r;
    r.promptTokens = tokens;
    if (tokens.empty()) return r;
    // Stops on config.json's eos_token_id (no tokenizer is loaded) and at max_position_embeddings.
    const uint32_t budget = std::min(opts.maxNewTokens, opts_.maxNewTokens);
    return GenerateBatch({tokens}, budget).front();
}

uint32_t VoxelEngine::Prefill(const std::vector<uint32_t> &tokens) {
    OPURE_CHECK(!tokens.empty(), "Prefill called with no tokens");
    const bool chunked = opts_.prefillChunk > 0;
    ResetSequences({tokens}, uint32_t(tokens.size()), !chunked);
    if (chunked)
        PrefillChunks({tokens});
    else
        RunSteps(1, uint32_t(tokens.size()), false);
    Sync();
    unsigned long long key = 0;
    OPURE_CUDA_CHECK(opure_d2h(ctx_, &key, buf_.keys, 8));
    OPURE_CUDA_CHECK(opure_sync(ctx_, 60000));
    seqLen_ = uint32_t(tokens.size());
    return 0xffffffffu - uint32_t(key & 0xffffffffull);  // ArgMaxFrom (:962-988)
}

uint32_t VoxelEngine::ForwardArgMax(const std::vector<uint32_t> &tokens) {
    OPURE_CHECK(!tokens.empty(), "ForwardArgMax called with no tokens");
    ResetSequences({tokens}, uint32_t(tokens.size()), true);
    RunSteps(1, uint32_t(tokens.size()), false);
    Sync();
    unsigned long long key = 0;
    OPURE_CUDA_CHECK(opure_d2h(ctx_, &key, buf_.keys, 8));
    OPURE_CUDA_CHECK(opure_sync(ctx_, 60000));
    seqLen_ = uint32_t(tokens.size());
    return 0xffffffffu - uint32_t(key & 0xffffffffull);
}

void VoxelEngine::ForwardLogits(const std::vector<uint32_t> &tokens, std::vector<float> &logitsOut) {
    OPURE_CHECK(!tokens.empty(), "ForwardLogits called with no tokens");
    OPURE_CHECK(!comm_, "ForwardLogits is not available on a tensor-parallel shard (logits are split)");
    ResetSequences({tokens}, uint32_t(tokens.size()), true);
    RunSteps(1, uint32_t(tokens.size()), true);
    Sync();
    logitsOut.assign(graph_.Config().vocabSize, 0.f);
    OPURE_CUDA_CHECK(opure_d2h(ctx_, logitsOut.data(), buf_.logits, logitsOut.size() * 4));
    OPURE_CUDA_CHECK(opure_sync(ctx_, 60000));
    seqLen_ = uint32_t(tokens.size());
}

void VoxelEngine::DecodeStepBatch(const int32_t *tokens, const int32_t *positions, uint32_t n, int32_t *next) {
    OPURE_CHECK(n >= 1 && n <= opts_.maxBatch, "batch exceeds maxBatch");
    auto *io = static_cast<int32_t *>(hostIo_);
    for (uint32_t v = 0; v < n; ++v) {
        OPURE_CHECK(positions[v] >= 0 && uint32_t(positions[v]) < maxLen_,
                    "decode position exceeds the engine's maxLen");
        OPURE_CHECK(tokens[v] >= 0 && uint32_t(tokens[v]) < graph_.Config().vocabSize,
                    "token id out of vocabulary range");
        OPURE_CHECK(kv_.Reserve(v, uint32_t(positions[v]) + 1), "KV cache has no room for the sequence");
        io[v] = tokens[v];
        io[maxVec_ + v] = positions[v];
    }
    kv_.SyncTable();
    if (!seqIdentity_) {
        // SetVectors may have pointed vectors at other slots; vector v is slot v here.
        std::vector<int32_t> ident(opts_.maxBatch);
        for (uint32_t v = 0; v < opts_.maxBatch; ++v) ident[v] = int32_t(v);
        OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.seq, ident.data(), ident.size() * 4));
        seqIdentity_ = true;
    }
    if (!hostDriven_) {
        // Token and position now come from the host: clear the self-driving flag.
        const std::vector<uint32_t> zero(opts_.maxBatch, 0u);
        OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.flags, zero.data(), zero.size() * 4));
        hostDriven_ = true;
    }
    // One H2D of tokens and positions (pinned; the tokens of vectors n.. are unused by this
    // step and rewritten before any step reads them), one step, one 8-byte-per-sequence
    // readback: the reference's DecodeStep round trip (Opure_VoxelEngine.cpp:765-800).
    OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.inTokens, io, (size_t(maxVec_) + n) * 4));
    RunSteps(n, 1, false);
    auto *keys = reinterpret_cast<unsigned long long *>(io + 2 * size_t(maxVec_));
    OPURE_CUDA_CHECK(opure_d2h(ctx_, keys, buf_.keys, n * 8));
    OPURE_CUDA_CHECK(opure_sync(ctx_, 600000));
    for (uint32_t v = 0; v < n; ++v) next[v] = int32_t(0xffffffffu - uint32_t(keys[v] & 0xffffffffull));
}

uint32_t VoxelEngine::DecodeStep(uint32_t tokenId, uint32_t position) {
    OPURE_CHECK(position < graph_.Config().maxPositions, "decode position exceeds max_position_embeddings");
    const int32_t t = int32_t(tokenId), p = int32_t(position);
    int32_t next = 0;
    DecodeStepBatch(&t, &p, 1, &next);
    seqLen_ = position + 1;
    return uint32_t(next);
}

void VoxelEngine::RunLayersTraced(uint32_t tokenId, uint32_t nLayers, std::vector<std::vector<float>> &trace) {
    OPURE_CHECK(ready_, "engine used before Initialize");
    const graph::ModelConfig &c = graph_.Config();
    nLayers = std::min(nLayers, c.numLayers);
    ResetSequences({{tokenId}}, 1, true);
    const opure_step_io io = StepIO(1);
    OPURE_CUDA_CHECK(opure_step_begin(ctx_, &io));
    trace.assign(nLayers, std::vector<float>(c.hiddenSize));
    for (uint32_t L = 0; L < nLayers; ++L) {
        RecordLayer(L, 1);
        OPURE_CUDA_CHECK(opure_d2h(ctx_, trace[L].data(), buf_.x, c.hiddenSize * 4));
    }
    Sync();
}

void VoxelEngine::PoisonBanks(float fill) {
    const graph::ModelConfig &c = graph_.Config();
    const uint32_t B = maxVec_;
    auto poison = [&](float *p, size_t n) {
        std::vector<float> pat(n, fill);
        OPURE_CUDA_CHECK(opure_h2d(ctx_, p, pat.data(), n * 4));
        OPURE_CUDA_CHECK(opure_sync(ctx_, 60000));
    };
    poison(buf_.x, size_t(B) * c.hiddenSize);
    poison(buf_.qkv, size_t(B) * c.QkvRows());
    poison(buf_.q, size_t(B) * c.numHeads * c.HeadDim());
    poison(buf_.attn, size_t(B) * c.hiddenSize);
    poison(buf_.h, size_t(B) * c.intermediateSize);
    poison(buf_.logits, size_t(B) * c.vocabSize);
    {
        // Step state the host sets: every slot self-driving with nothing known, so a step
        // whose vectors the host did not set up would take tokens from stale keys.
        const std::vector<uint32_t> autoFlags(B, uint32_t(OPURE_VEC_AUTO));
        const std::vector<int32_t> none(B, 0);
        OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.flags, autoFlags.data(), B * 4));
        OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.known, none.data(), B * 4));
        OPURE_CUDA_CHECK(opure_sync(ctx_, 60000));
    }
    if (buf_.packRes) {
        // Chained tensor-core operands: fp16 pairs (the fill's fp16 bits) and the sums of squares.
        const uint32_t nv = std::min<uint32_t>(B, 256), att = c.numHeads * c.HeadDim();
        const uint16_t h = std::isnan(fill) ? uint16_t(0x7e00) : uint16_t(0x3c00);  // NaN, or 1.0
        auto poison16 = [&](uint16_t *p, size_t bytes) {
            std::vector<uint16_t> pat(bytes / 2, h);
            OPURE_CUDA_CHECK(opure_h2d(ctx_, p, pat.data(), bytes));
            OPURE_CUDA_CHECK(opure_sync(ctx_, 60000));
        };
        poison16(buf_.packAttn, opure_packed_bytes(nv, att));
        poison16(buf_.packRes, opure_packed_bytes(nv, c.hiddenSize));
        poison16(buf_.packAct, opure_packed_bytes(nv, c.intermediateSize));
        poison(buf_.sumsq, size_t((c.hiddenSize + 127) / 128) * nv);
    }
}

void VoxelEngine::LoadKv(uint32_t seq, const uint16_t *kvData, uint32_t len) {
    const graph::ModelConfig &c = graph_.Config();
    OPURE_CHECK(seq < opts_.maxBatch && len <= maxLen_, "LoadKv: sequence or length out of range");
    OPURE_CHECK(!kv_.Ring() || len <= kv_.Ring() * kv_.PageSize(), "LoadKv: context longer than the KV window");
    OPURE_CHECK(kv_.Reserve(seq, std::max(len, 1u)), "KV cache has no room for the sequence");
    kv_.SyncTable();
    const uint32_t P = kv_.PageSize(), hd = c.HeadDim(), nkv = c.numKvHeads;
    const std::vector<int32_t> &table = kv_.HostTable();
    for (uint32_t L = 0; L < c.numLayers; ++L) {
        uint8_t *pool = reinterpret_cast<uint8_t *>(kv_.Pool(L));
        for (uint32_t sel = 0; sel < 2; ++sel)
            for (uint32_t g = 0; g < nkv; ++g)
                for (uint32_t lp = 0; lp * P < len; ++lp) {
                    const uint32_t ntok = std::min(P, len - lp * P);
                    const int32_t page = table[size_t(seq) * kv_.MaxPages() + lp];
                    const uint16_t *src = kvData + ((((size_t(L) * 2 + sel) * nkv + g) * len) + size_t(lp) * P) * hd;
                    uint8_t *dst = pool + ((size_t(page) * 2 + sel) * nkv + g) * size_t(P) * hd * 2;
                    OPURE_CUDA_CHECK(opure_h2d(ctx_, dst, src, size_t(ntok) * hd * 2));
                }
        OPURE_CUDA_CHECK(opure_sync(ctx_, 600000));
    }
}

void VoxelEngine::PrepareSynthetic(uint32_t n, uint32_t len, uint32_t reserve, uint64_t seed,
                                   const int32_t *first) {
    OPURE_CHECK(ready_, "engine used before Initialize");
    OPURE_CHECK(n >= 1 && n <= opts_.maxBatch, "batch exceeds maxBatch");
    OPURE_CHECK(len >= 1 && len < reserve && reserve <= maxLen_, "need 1 <= len < reserve <= maxLen");
    const graph::ModelConfig &c = graph_.Config();
    std::vector<int32_t> seq(n), pos(n, int32_t(len)), known(n, int32_t(len) + 1);
    std::vector<uint32_t> flags(n, uint32_t(OPURE_VEC_AUTO));
    for (uint32_t v = 0; v < n; ++v) {
        OPURE_CHECK(first[v] >= 0 && uint32_t(first[v]) < c.vocabSize, "token id out of vocabulary range");
        seq[v] = int32_t(v);
        kv_.Release(v);
        OPURE_CHECK(kv_.Reserve(v, reserve), "KV cache has no room for the sequence");
    }
    kv_.SyncTable();
    for (uint32_t L = 0; L < c.numLayers; ++L) {
        const opure_kv_layout l = kv_.Layout(L);
        OPURE_CUDA_CHECK(opure_kv_synth(ctx_, &l, L, 0, n, len, seed));
    }
    for (uint32_t v = 0; v < n; ++v)
        OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.tokens + size_t(v) * maxLen_ + len, first + v, 4));
    OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.seq, seq.data(), n * 4));
    OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.pos, pos.data(), n * 4));
    OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.known, known.data(), n * 4));
    OPURE_CUDA_CHECK(opure_h2d(ctx_, buf_.flags, flags.data(), n * 4));
    OPURE_CUDA_CHECK(opure_fill(ctx_, buf_.keys, 0, size_t(n) * 8));
    hostDriven_ = false;
    seqIdentity_ = true;
    Sync();
}

void VoxelEngine::ReadHistory(uint32_t slot, uint32_t pos, uint32_t count, int32_t *out) {
    OPURE_CHECK(slot < opts_.maxBatch && uint64_t(pos) + count <= maxLen_, "history read out of range");
    OPURE_CUDA_CHECK(opure_d2h(ctx_, out, buf_.tokens + size_t(slot) * maxLen_ + pos, size_t(count) * 4));
    OPURE_CUDA_CHECK(opure_sync(ctx_, 60000));
}

size_t VoxelEngine::ReadPhaseTrace(unsigned long long *out, size_t cap) {
    if (!buf_.trace) return 0;
    const size_t n = std::min(cap, traceWords_);
    OPURE_CUDA_CHECK(opure_d2h(ctx_, out, buf_.trace, n * 8));
    OPURE_CUDA_CHECK(opure_sync(ctx_, 60000));
    return n;
}

VoxelEngine::MetricsSnapshot VoxelEngine::SnapshotMetrics() const {
    MetricsSnapshot m;
    if (kv_.NumPages()) m.kvOccupancy = 1.0f - float(kv_.FreePages()) / float(kv_.NumPages());
    m.tokensPerSec = lastTokenMs_ > 0 ? float(1000.0 / lastTokenMs_) : 0.0f;
    m.memoryPressure = 0.0f;
    m.speculativeAcceptance = specAcceptance_;
    return m;
}

}  // namespace opure::engine
