// sample_decode.cpp -- the sampled generation loop (see sample_decode.h).
#include "sample_decode.h"

#include <algorithm>

#include "platform.h"
#include "synth.h"

namespace opure::engine {

std::vector<std::vector<uint32_t>> SampleGenerate(VoxelEngine &eng, const std::vector<std::vector<uint32_t>> &prompts,
                                                  const SampleOptions &o, std::vector<float> *stats,
                                                  std::vector<float> *logits) {
    OPURE_CHECK(eng.IsReady(), "engine used before Initialize");
    const uint32_t n = uint32_t(prompts.size()), V = eng.Model().vocabSize;
    OPURE_CHECK(n >= 1 && n <= eng.Options().maxBatch, "prompts must number 1..maxBatch");
    OPURE_CHECK(o.maxNew >= 1, "maxNew must be at least 1");
    OPURE_CHECK(o.topP > 0.0f && o.topP <= 1.0f, "top_p must be in (0, 1]");
    OPURE_CHECK(o.repPenalty > 0.0f, "repetition penalty must be positive");
    const size_t P0 = prompts[0].size();
    for (const auto &p : prompts) OPURE_CHECK(!p.empty() && p.size() == P0, "prompts must be non-empty and of equal length");
    const uint32_t reserve = uint32_t(P0) + o.maxNew + 1;
    OPURE_CHECK(reserve <= eng.MaxLen(), "maxLen must be >= prompt + maxNew + 1");

    opure_ctx *ctx = eng.Ctx();
    struct Bufs {
        opure_ctx *ctx;
        float *u = nullptr, *stats = nullptr, *logits = nullptr;
        int32_t *out = nullptr;
        ~Bufs() {
            opure_free(ctx, u);
            opure_free(ctx, stats);
            opure_free(ctx, logits);
            opure_free(ctx, out);
        }
    } b{ctx};
    const size_t cells = size_t(o.maxNew) * n;
    OPURE_CUDA_CHECK(opure_alloc(ctx, cells * 4, reinterpret_cast<void **>(&b.u)));
    OPURE_CUDA_CHECK(opure_alloc(ctx, cells * 4, reinterpret_cast<void **>(&b.out)));
    if (stats) OPURE_CUDA_CHECK(opure_alloc(ctx, cells * 16, reinterpret_cast<void **>(&b.stats)));
    if (logits) OPURE_CUDA_CHECK(opure_alloc(ctx, cells * V * 4, reinterpret_cast<void **>(&b.logits)));

    // Uniforms [j][s]: draw j of sequence s's stream.
    std::vector<float> u(cells);
    for (uint32_t s = 0; s < n; ++s) {
        synth::Rng rng(o.seed ^ (uint64_t(s) * 0x9E3779B97F4A7C15ull));
        for (uint32_t j = 0; j < o.maxNew; ++j) u[size_t(j) * n + s] = float(double(rng.NextU32()) / 4294967296.0);
    }
    OPURE_CUDA_CHECK(opure_h2d(ctx, b.u, u.data(), cells * 4));

    opure_sample_args a{};
    a.vocab = V;
    a.rows = n;
    a.stride = V;
    a.temperature = o.temperature;
    a.top_k = o.topK;
    a.top_p = o.topP;
    a.rep_penalty = o.repPenalty;
    a.hist = eng.DeviceHistory();
    a.max_len = eng.MaxLen();
    a.seq = eng.DeviceSeq();
    a.hist_len = eng.DevicePos();  // after a step: its position + 1 = the tokens so far
    a.keys = eng.DeviceKeys();     // the next self-driving step's input

    // The prompt, then one self-driving step per further token; every step leaves its
    // last-position logits in DeviceLogits() and positions advanced past it.
    eng.PrefillBatch(prompts, reserve, true);
    for (uint32_t j = 0; j < o.maxNew; ++j) {
        if (j) eng.RunSteps(n, 1, true);
        a.logits = eng.DeviceLogits();
        a.u = b.u + size_t(j) * n;
        a.out = b.out + size_t(j) * n;
        if (stats) OPURE_CUDA_CHECK(opure_logit_stats(ctx, a.logits, V, n, V, b.stats + size_t(j) * n * 4));
        if (logits) OPURE_CUDA_CHECK(opure_d2d(ctx, b.logits + size_t(j) * n * V, a.logits, size_t(n) * V * 4));
        OPURE_CUDA_CHECK(opure_sample_filtered(ctx, &a));
    }
    std::vector<int32_t> tok(cells);
    OPURE_CUDA_CHECK(opure_d2h(ctx, tok.data(), b.out, cells * 4));
    std::vector<float> st(stats ? cells * 4 : 0);
    if (stats) OPURE_CUDA_CHECK(opure_d2h(ctx, st.data(), b.stats, cells * 16));
    std::vector<float> lg(logits ? cells * V : 0);
    if (logits) OPURE_CUDA_CHECK(opure_d2h(ctx, lg.data(), b.logits, cells * V * 4));
    OPURE_CUDA_CHECK(opure_sync(ctx, 600000));
    CheckDevice(ctx);

    std::vector<std::vector<uint32_t>> res(n, std::vector<uint32_t>(o.maxNew));
    for (uint32_t s = 0; s < n; ++s)
        for (uint32_t j = 0; j < o.maxNew; ++j) res[s][j] = uint32_t(tok[size_t(j) * n + s]);
    if (stats) {
        stats->assign(cells * 4, 0.f);
        for (uint32_t s = 0; s < n; ++s)
            for (uint32_t j = 0; j < o.maxNew; ++j)
                std::copy_n(st.data() + (size_t(j) * n + s) * 4, 4, stats->data() + (size_t(s) * o.maxNew + j) * 4);
    }
    if (logits) {
        logits->assign(cells * V, 0.f);
        for (uint32_t s = 0; s < n; ++s)
            for (uint32_t j = 0; j < o.maxNew; ++j)
                std::copy_n(lg.data() + (size_t(j) * n + s) * V, V, logits->data() + (size_t(s) * o.maxNew + j) * V);
    }
    return res;
}

}  // namespace opure::engine
