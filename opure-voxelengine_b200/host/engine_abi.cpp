// engine_abi.cpp -- extern "C" surface of the host engine (include/opure_engine.h).
#include <algorithm>
#include <cstring>
#include <exception>
#include <new>
#include <string>

#include "opure_engine.h"
#include "platform.h"
#include "sample_decode.h"
#include "server.h"
#include "spec_decode.h"
#include "synth.h"
#include "voxel_engine.h"

struct opure_engine {
    opure::engine::VoxelEngine eng;
    std::string err;
};

namespace {

thread_local std::string g_create_error;

// Runs `fn`, turning exceptions into a status and a stored message.
template <class F>
opure_status Guard(opure_engine *e, F &&fn) {
    try {
        fn();
        return OPURE_OK;
    } catch (const opure::Error &x) {
        if (e) e->err = x.what();
        return x.status() != OPURE_OK ? x.status() : OPURE_ERR_INVALID_ARG;
    } catch (const std::bad_alloc &) {
        if (e) e->err = "host out of memory";
        return OPURE_ERR_OUT_OF_MEMORY;
    } catch (const std::exception &x) {
        if (e) e->err = x.what();
        return OPURE_ERR_INVALID_ARG;
    }
}

std::vector<uint32_t> ToU32(const int32_t *t, uint32_t n) {
    std::vector<uint32_t> v(n);
    for (uint32_t i = 0; i < n; ++i) {
        OPURE_CHECK(t[i] >= 0, "negative token id");
        v[i] = uint32_t(t[i]);
    }
    return v;
}

}  // namespace

extern "C" {

namespace {

opure::engine::EngineOptions ToOptions(const opure_engine_options *o) {
    opure::engine::EngineOptions opts;
    if (o) {
        if (o->max_new_tokens) opts.maxNewTokens = o->max_new_tokens;
        if (o->max_batch) opts.maxBatch = o->max_batch;
        opts.maxLen = o->max_len;
        if (o->page_size) opts.pageSize = o->page_size;
        opts.pageSeed = o->page_seed;
        opts.useGraphs = o->use_graphs != 0;
        if (o->attn_scale != 0.f) opts.attnScale = o->attn_scale;
        opts.path = o->path;
        opts.phaseTrace = o->phase_trace != 0;
        opts.prefillChunk = o->prefill_chunk;
        opts.kvWindow = o->kv_window;
        opts.tpAllreduce = o->tp_allreduce;
    }
    return opts;
}

opure_status Create(const char *model_dir, int device, opure_ctx *shared, const opure_engine_options *o,
                    opure_engine **out, opure_comm *comm = nullptr) {
    if (!model_dir || !out) return OPURE_ERR_INVALID_ARG;
    *out = nullptr;
    auto *e = new (std::nothrow) opure_engine;
    if (!e) return OPURE_ERR_OUT_OF_MEMORY;
    const opure_status s = Guard(e, [&] { e->eng.Initialize(model_dir, ToOptions(o), device, shared, comm); });
    if (s != OPURE_OK) {
        g_create_error = e->err;
        delete e;
        return s;
    }
    *out = e;
    return OPURE_OK;
}

}  // namespace

opure_status opure_engine_create(const char *model_dir, int device, const opure_engine_options *o,
                                 opure_engine **out) {
    return Create(model_dir, device, nullptr, o, out);
}

opure_status opure_engine_create_tp(const char *model_dir, opure_ctx *ctx, opure_comm *comm,
                                    const opure_engine_options *o, opure_engine **out) {
    if (!ctx || !comm) return OPURE_ERR_INVALID_ARG;
    opure_device_info di{};
    const opure_status s = opure_get_device_info(ctx, &di);
    if (s != OPURE_OK) return s;
    return Create(model_dir, di.device, ctx, o, out, comm);
}

opure_status opure_engine_create_shared(const char *model_dir, opure_engine *share,
                                        const opure_engine_options *o, opure_engine **out) {
    if (!share || !share->eng.IsReady()) return OPURE_ERR_INVALID_ARG;
    opure_device_info di{};
    const opure_status s = opure_get_device_info(share->eng.Ctx(), &di);
    if (s != OPURE_OK) return s;
    return Create(model_dir, di.device, share->eng.Ctx(), o, out);
}

opure_status opure_engine_phase_trace(opure_engine *e, uint64_t *out, size_t cap, size_t *written) {
    if (!e || !out || !written) return OPURE_ERR_INVALID_ARG;
    return Guard(e, [&] { *written = e->eng.ReadPhaseTrace(reinterpret_cast<unsigned long long *>(out), cap); });
}

opure_status opure_engine_synth_context(opure_engine *e, uint32_t n, uint32_t len, uint32_t reserve,
                                        uint64_t seed, const int32_t *first_tokens) {
    if (!e || !first_tokens) return OPURE_ERR_INVALID_ARG;
    return Guard(e, [&] { e->eng.PrepareSynthetic(n, len, reserve, seed, first_tokens); });
}

opure_status opure_engine_read_tokens(opure_engine *e, uint32_t slot, uint32_t pos, uint32_t count,
                                      int32_t *out) {
    if (!e || !out) return OPURE_ERR_INVALID_ARG;
    return Guard(e, [&] { e->eng.ReadHistory(slot, pos, count, out); });
}

opure_status opure_synth_kv(uint64_t seed, uint32_t slot, uint32_t layers, uint32_t n_kv, uint32_t len,
                            uint32_t head_dim, uint16_t *out) {
    if (!out || len > 65536) return OPURE_ERR_INVALID_ARG;
    return Guard(nullptr, [&] {
        const auto v = opure::synth::SynthKv(seed, slot, layers, n_kv, len, head_dim);
        std::copy(v.begin(), v.end(), out);
    });
}

opure_status opure_engine_spec_generate(opure_engine *target, opure_engine *draft, const int32_t *prompts,
                                        uint32_t prompt_len, uint32_t n_seq, uint32_t budget,
                                        const opure_spec_options *o, int32_t *out_tokens,
                                        int32_t *accept_log, uint32_t accept_log_rounds,
                                        opure_spec_stats *stats) {
    if (!target || !draft || !prompts || !o || !out_tokens || n_seq == 0 || prompt_len == 0 || budget == 0)
        return OPURE_ERR_INVALID_ARG;
    return Guard(target, [&] {
        std::vector<std::vector<uint32_t>> ps(n_seq);
        for (uint32_t s = 0; s < n_seq; ++s) ps[s] = ToU32(prompts + size_t(s) * prompt_len, prompt_len);
        opure::engine::SpecOptions so;
        so.k = o->k;
        so.mode = o->mode;
        so.seed = o->seed;
        so.maxNew = budget;
        opure::engine::SpecStats st;
        std::vector<int32_t> log, dlog;
        const auto res = opure::engine::SpecGenerate(target->eng, draft->eng, ps, so, &st, accept_log ? &log : nullptr,
                                                     o->draft_log ? &dlog : nullptr);
        if (o->draft_log) {
            const size_t cap = size_t(o->draft_log_rounds) * n_seq * o->k;
            const size_t m = std::min(dlog.size(), cap);
            std::copy_n(dlog.begin(), m, o->draft_log);
            std::fill(o->draft_log + m, o->draft_log + cap, -2);
        }
        for (uint32_t s = 0; s < n_seq; ++s)
            for (uint32_t i = 0; i < budget; ++i) out_tokens[size_t(s) * budget + i] = int32_t(res[s][i]);
        if (accept_log) {
            const size_t m = std::min<size_t>(log.size(), size_t(accept_log_rounds) * n_seq);
            std::copy_n(log.begin(), m, accept_log);
            std::fill(accept_log + m, accept_log + size_t(accept_log_rounds) * n_seq, -2);
        }
        if (stats) {
            stats->rounds = st.rounds;
            stats->drafted = st.drafted;
            stats->accepted = st.accepted;
            stats->draft_ms = st.draftMs;
            stats->verify_ms = st.verifyMs;
            stats->total_ms = st.totalMs;
        }
    });
}

opure_status opure_engine_sample_generate(opure_engine *e, const int32_t *prompts, uint32_t prompt_len, uint32_t n_seq,
                                          uint32_t budget, const opure_sample_options *o, int32_t *out_tokens,
                                          float *stats, float *logits) {
    if (!e || !prompts || !o || !out_tokens || n_seq == 0 || prompt_len == 0 || budget == 0)
        return OPURE_ERR_INVALID_ARG;
    return Guard(e, [&] {
        std::vector<std::vector<uint32_t>> ps(n_seq);
        for (uint32_t s = 0; s < n_seq; ++s) ps[s] = ToU32(prompts + size_t(s) * prompt_len, prompt_len);
        opure::engine::SampleOptions so;
        so.temperature = o->temperature;
        so.topK = o->top_k;
        so.topP = o->top_p;
        so.repPenalty = o->rep_penalty;
        so.seed = o->seed;
        so.maxNew = budget;
        std::vector<float> st, lg;
        const auto res = opure::engine::SampleGenerate(e->eng, ps, so, stats ? &st : nullptr, logits ? &lg : nullptr);
        for (uint32_t s = 0; s < n_seq; ++s)
            for (uint32_t i = 0; i < budget; ++i) out_tokens[size_t(s) * budget + i] = int32_t(res[s][i]);
        if (stats) std::copy(st.begin(), st.end(), stats);
        if (logits) std::copy(lg.begin(), lg.end(), logits);
    });
}

opure_status opure_engine_destroy(opure_engine *e) {
    if (!e) return OPURE_ERR_INVALID_ARG;
    delete e;
    return OPURE_OK;
}

const char *opure_engine_last_error(opure_engine *e) { return e ? e->err.c_str() : g_create_error.c_str(); }

opure_ctx *opure_engine_ctx(opure_engine *e) { return e ? e->eng.Ctx() : nullptr; }

namespace {

void FillInfo(const opure::graph::Graph &g, opure_engine_info *info) {
    const auto &c = g.Config();
    const auto &p = g.Plan();
    std::memset(info, 0, sizeof(*info));
    info->vocab = c.vocabSize;
    info->hidden = c.hiddenSize;
    info->inter = c.intermediateSize;
    info->layers = c.numLayers;
    info->heads = c.numHeads;
    info->kv_heads = c.numKvHeads;
    info->head_dim = c.HeadDim();
    info->max_pos = c.maxPositions;
    info->w_dtype = p.wDtype;
    info->weight_bytes = p.weightBytes;
    info->stream_bytes = g.StreamBytes();
    info->kv_bytes_per_token = c.KvBytesPerToken() / g.Local().tpSize;  // this shard's KV heads
    info->tp_ranks = g.Local().tpSize;
}

}  // namespace

opure_status opure_engine_get_info(opure_engine *e, opure_engine_info *info) {
    if (!e || !info) return OPURE_ERR_INVALID_ARG;
    return Guard(e, [&] {
        FillInfo(e->eng.GraphModel(), info);
        info->max_len = e->eng.MaxLen();
        info->max_batch = e->eng.Options().maxBatch;
        info->page_size = e->eng.Options().pageSize;
        info->tp_peer = e->eng.UsesPeer() ? 1 : 0;
    });
}

opure_status opure_engine_snapshot_metrics(opure_engine *e, opure_engine_metrics *m) {
    if (!e || !m) return OPURE_ERR_INVALID_ARG;
    return Guard(e, [&] {
        const auto s = e->eng.SnapshotMetrics();
        m->kv_occupancy = s.kvOccupancy;
        m->tokens_per_sec = s.tokensPerSec;
        m->memory_pressure = s.memoryPressure;
        m->speculative_acceptance = s.speculativeAcceptance;
        m->position = e->eng.CurrentPosition();
    });
}

opure_status opure_model_inspect(const char *model_dir, opure_engine_info *info, char *err, size_t err_len) {
    if (!model_dir || !info) return OPURE_ERR_INVALID_ARG;
    opure_engine scratch;
    const opure_status s = Guard(&scratch, [&] {
        opure::graph::Graph g;
        g.LoadConfigOnly(model_dir);
        FillInfo(g, info);
    });
    if (s != OPURE_OK && err && err_len) {
        std::strncpy(err, scratch.err.c_str(), err_len - 1);
        err[err_len - 1] = 0;
    }
    return s;
}

opure_status opure_engine_generate(opure_engine *e, const int32_t *prompts, const uint32_t *lens,
                                   uint32_t n_seq, uint32_t budget, int32_t *out, opure_generate_timing *t) {
    return opure_engine_generate_stop(e, prompts, lens, n_seq, budget, out, nullptr, nullptr, t);
}

opure_status opure_engine_generate_stop(opure_engine *e, const int32_t *prompts, const uint32_t *lens,
                                        uint32_t n_seq, uint32_t budget, int32_t *out, uint32_t *counts,
                                        uint32_t *hit_stop, opure_generate_timing *t) {
    if (!e || !prompts || !lens || !out || n_seq == 0) return OPURE_ERR_INVALID_ARG;
    return Guard(e, [&] {
        std::vector<std::vector<uint32_t>> ps(n_seq);
        size_t off = 0;
        for (uint32_t i = 0; i < n_seq; ++i) {
            ps[i] = ToU32(prompts + off, lens[i]);
            off += lens[i];
        }
        opure::engine::StepTiming st;
        const auto res = e->eng.GenerateBatch(ps, budget, &st);
        for (uint32_t i = 0; i < n_seq; ++i) {
            const size_t m = res[i].generated.size();
            for (uint32_t k = 0; k < budget; ++k) out[size_t(i) * budget + k] = k < m ? int32_t(res[i].generated[k]) : -1;
            if (counts) counts[i] = uint32_t(m);
            if (hit_stop) hit_stop[i] = res[i].hitStop ? 1u : 0u;
        }
        if (t) {
            t->prefill_ms = st.prefillMs;
            t->decode_ms = st.decodeMs;
            t->prefill_steps = st.prefillSteps;
            t->decode_steps = st.decodeSteps;
        }
    });
}

opure_status opure_engine_prefill(opure_engine *e, const int32_t *tokens, uint32_t n, int32_t *next) {
    if (!e || !tokens || n == 0) return OPURE_ERR_INVALID_ARG;
    return Guard(e, [&] {
        const uint32_t t = e->eng.Prefill(ToU32(tokens, n));
        if (next) *next = int32_t(t);
    });
}

opure_status opure_engine_decode_step(opure_engine *e, const int32_t *tokens, const int32_t *positions,
                                      uint32_t n, int32_t *next) {
    if (!e || !tokens || !positions || !next || n == 0) return OPURE_ERR_INVALID_ARG;
    return Guard(e, [&] { e->eng.DecodeStepBatch(tokens, positions, n, next); });
}

opure_status opure_engine_run_steps(opure_engine *e, uint32_t n, uint32_t steps) {
    if (!e) return OPURE_ERR_INVALID_ARG;
    return Guard(e, [&] { e->eng.RunSteps(n, steps, false); });
}

opure_status opure_engine_set_positions(opure_engine *e, const int32_t *positions, uint32_t n) {
    if (!e || !positions) return OPURE_ERR_INVALID_ARG;
    return Guard(e, [&] { e->eng.SetPositions(positions, n); });
}

opure_status opure_engine_sync(opure_engine *e) {
    if (!e) return OPURE_ERR_INVALID_ARG;
    return Guard(e, [&] { e->eng.Sync(); });
}

opure_status opure_engine_forward_logits(opure_engine *e, const int32_t *tokens, uint32_t n, float *logits) {
    if (!e || !tokens || !logits || n == 0) return OPURE_ERR_INVALID_ARG;
    return Guard(e, [&] {
        std::vector<float> l;
        e->eng.ForwardLogits(ToU32(tokens, n), l);
        std::memcpy(logits, l.data(), l.size() * 4);
    });
}

opure_status opure_engine_forward_argmax(opure_engine *e, const int32_t *tokens, uint32_t n, int32_t *out) {
    if (!e || !tokens || !out || n == 0) return OPURE_ERR_INVALID_ARG;
    return Guard(e, [&] { *out = int32_t(e->eng.ForwardArgMax(ToU32(tokens, n))); });
}

opure_status opure_engine_trace(opure_engine *e, int32_t token, uint32_t n_layers, float *trace) {
    if (!e || !trace || token < 0) return OPURE_ERR_INVALID_ARG;
    return Guard(e, [&] {
        std::vector<std::vector<float>> tr;
        e->eng.RunLayersTraced(uint32_t(token), n_layers, tr);
        for (size_t l = 0; l < tr.size(); ++l) std::memcpy(trace + l * tr[l].size(), tr[l].data(), tr[l].size() * 4);
    });
}

opure_status opure_engine_poison(opure_engine *e, float value) {
    if (!e) return OPURE_ERR_INVALID_ARG;
    return Guard(e, [&] { e->eng.PoisonBanks(value); });
}

opure_status opure_engine_load_kv(opure_engine *e, uint32_t seq, const uint16_t *kv, uint32_t len) {
    if (!e || !kv) return OPURE_ERR_INVALID_ARG;
    return Guard(e, [&] { e->eng.LoadKv(seq, kv, len); });
}

// ---- synthetic inputs -------------------------------------------------------
opure_status opure_synth_model(const char *dir, const opure_synth_spec *s) {
    if (!dir || !s) return OPURE_ERR_INVALID_ARG;
    return Guard(nullptr, [&] {
        opure::synth::ModelSpec m;
        m.vocab = s->vocab;
        m.hidden = s->hidden;
        m.inter = s->inter;
        m.layers = s->layers;
        m.heads = s->heads;
        m.kv_heads = s->kv_heads;
        m.max_pos = s->max_pos;
        m.eps = s->eps;
        m.theta = s->theta;
        m.tied = s->tied != 0;
        m.seed = s->seed;
        m.std = s->std;
        m.int8 = s->int8 != 0;
        m.noise_seed = s->noise_seed;
        m.noise_std = s->noise_std;
        opure::synth::WriteModel(dir, m);
    });
}

opure_status opure_synth_normal_f16(uint64_t seed, float stddev, uint64_t n, uint16_t *out) {
    if (!out) return OPURE_ERR_INVALID_ARG;
    return Guard(nullptr, [&] {
        const auto v = opure::synth::NormalF16(seed, stddev, n);
        std::memcpy(out, v.data(), n * 2);
    });
}

opure_status opure_synth_prompt(uint64_t seed, uint32_t vocab, uint32_t n, int32_t *out) {
    if (!out || vocab == 0) return OPURE_ERR_INVALID_ARG;
    return Guard(nullptr, [&] {
        const auto v = opure::synth::Prompt(seed, vocab, n);
        std::memcpy(out, v.data(), size_t(n) * 4);
    });
}

opure_status opure_synth_permutation(uint64_t seed, uint32_t n, int32_t *out) {
    if (!out) return OPURE_ERR_INVALID_ARG;
    return Guard(nullptr, [&] {
        const auto v = opure::synth::Permutation(seed, n);
        std::memcpy(out, v.data(), size_t(n) * 4);
    });
}

opure_status opure_synth_uniforms(uint64_t seed, uint64_t n, float *out) {
    if (!out) return OPURE_ERR_INVALID_ARG;
    return Guard(nullptr, [&] {
        const auto v = opure::synth::Uniforms(seed, n);
        std::memcpy(out, v.data(), n * 4);
    });
}

}  // extern "C"

// ---- serving front end (server.h) -----------------------------------------------------
struct opure_server {
    std::unique_ptr<opure::server::Server> srv;
};

extern "C" {

opure_status opure_server_start(const char *model_dir, const int *devices, uint32_t n_devices, uint16_t port,
                                const opure_engine_options *opts, opure_server **out) {
    if (!out || (n_devices && (!model_dir || !devices))) return OPURE_ERR_INVALID_ARG;
    *out = nullptr;
    opure_engine scratch;
    const opure_status s = Guard(&scratch, [&] {
        std::vector<std::unique_ptr<opure::engine::VoxelEngine>> engines;
        for (uint32_t i = 0; i < n_devices; ++i) {
            auto e = std::make_unique<opure::engine::VoxelEngine>();
            e->Initialize(model_dir, ToOptions(opts), devices[i]);
            engines.push_back(std::move(e));
        }
        auto *h = new opure_server;
        try {
            h->srv = std::make_unique<opure::server::Server>(std::move(engines), port);
        } catch (...) {
            delete h;
            throw;
        }
        *out = h;
    });
    if (s != OPURE_OK) g_create_error = scratch.err;
    return s;
}

uint16_t opure_server_port(const opure_server *s) { return s && s->srv ? s->srv->Port() : 0; }

opure_status opure_server_stop(opure_server *s) {
    if (!s) return OPURE_ERR_INVALID_ARG;
    delete s;  // stops the threads, then the engines are destroyed
    return OPURE_OK;
}

opure_status opure_server_parse_generate(const char *body, size_t len, uint32_t vocab, int32_t *tokens,
                                         uint32_t cap, uint32_t *n_tokens, uint32_t *max_tokens,
                                         float *temperature, char *err, size_t err_len) {
    if (!body || !n_tokens || !max_tokens || !temperature) return OPURE_ERR_INVALID_ARG;
    opure::server::GenerateRequest r;
    std::string e;
    if (!opure::server::ParseGenerate(std::string_view(body, len), vocab, r, e)) {
        if (err && err_len) {
            std::strncpy(err, e.c_str(), err_len - 1);
            err[err_len - 1] = 0;
        }
        return OPURE_ERR_INVALID_ARG;
    }
    *n_tokens = uint32_t(r.tokens.size());
    for (uint32_t i = 0; i < std::min<uint32_t>(cap, *n_tokens); ++i) tokens[i] = int32_t(r.tokens[i]);
    *max_tokens = r.maxTokens;
    *temperature = r.temperature;
    return OPURE_OK;
}

}  // extern "C"
