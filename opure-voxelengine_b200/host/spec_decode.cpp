// spec_decode.cpp -- the speculative decoding loop (see spec_decode.h).
#include "spec_decode.h"

#include <algorithm>

#include "platform.h"
#include "synth.h"

namespace opure::engine {

namespace {

// Device buffers of the round, freed on every exit path.
class DeviceArena {
public:
    explicit DeviceArena(opure_ctx *ctx) : ctx_(ctx) {}
    ~DeviceArena() {
        for (void *p : bufs_) opure_free(ctx_, p);
        for (opure_event *e : events_) opure_event_free(e);
    }
    template <class T>
    T *Alloc(size_t n) {
        void *p = nullptr;
        OPURE_CUDA_CHECK(opure_alloc(ctx_, std::max<size_t>(n, 1) * sizeof(T), &p));
        bufs_.push_back(p);
        return static_cast<T *>(p);
    }
    opure_event *Event() {
        opure_event *e = nullptr;
        OPURE_CUDA_CHECK(opure_event_create(ctx_, &e));
        events_.push_back(e);
        return e;
    }

private:
    opure_ctx *ctx_;
    std::vector<void *> bufs_;
    std::vector<opure_event *> events_;
};

double Elapsed(opure_event *a, opure_event *b) {
    float ms = 0.f;
    OPURE_CUDA_CHECK(opure_event_elapsed_ms(a, b, &ms));
    return ms;
}

}  // namespace

std::vector<std::vector<uint32_t>> SpecGenerate(VoxelEngine &target, VoxelEngine &draft,
                                                const std::vector<std::vector<uint32_t>> &prompts,
                                                const SpecOptions &o, SpecStats *stats,
                                                std::vector<int32_t> *acceptLog, std::vector<int32_t> *draftLog) {
    OPURE_CHECK(target.IsReady() && draft.IsReady(), "engine used before Initialize");
    // A rolled-back position may need a page its ring has already recycled.
    OPURE_CHECK(!target.Options().kvWindow && !draft.Options().kvWindow,
                "speculative decoding does not run with a sliding-window KV cache");
    OPURE_CHECK(target.Ctx() == draft.Ctx(), "the draft engine must share the target engine's ctx");
    const uint32_t V = target.Model().vocabSize;
    OPURE_CHECK(draft.Model().vocabSize == V, "draft and target vocabularies differ");
    const uint32_t n = uint32_t(prompts.size()), k = o.k;
    OPURE_CHECK(n >= 1, "no prompts");
    OPURE_CHECK(k >= 1 && k <= 64, "draft length k must be in 1..64");
    OPURE_CHECK(o.mode == OPURE_SPEC_GREEDY || o.mode == OPURE_SPEC_REJECTION, "unknown acceptance mode");
    OPURE_CHECK(o.maxNew >= 1, "maxNew must be at least 1");
    const size_t P0 = prompts[0].size();
    for (const auto &p : prompts) OPURE_CHECK(!p.empty() && p.size() == P0, "prompts must be non-empty and of equal length");
    OPURE_CHECK(target.Options().maxBatch >= n * (k + 1), "the target engine needs maxBatch >= n_seq * (k + 1)");
    OPURE_CHECK(draft.Options().maxBatch >= n, "the draft engine needs maxBatch >= n_seq");
    const uint32_t reserve = uint32_t(P0) + o.maxNew + k + 2;
    OPURE_CHECK(reserve <= target.MaxLen() && reserve <= draft.MaxLen(),
                "maxLen of both engines must be >= prompt + maxNew + k + 2");

    opure_ctx *ctx = target.Ctx();
    const bool rej = o.mode == OPURE_SPEC_REJECTION;
    DeviceArena arena(ctx);
    int32_t *dBase = arena.Alloc<int32_t>(n);
    int32_t *dDraft = arena.Alloc<int32_t>(size_t(n) * k);
    int32_t *dOut = arena.Alloc<int32_t>(size_t(n) * (k + 1));
    int32_t *dAcc = arena.Alloc<int32_t>(n);
    float *dDraftLogits = rej ? arena.Alloc<float>(size_t(n) * k * V) : nullptr;
    float *dUDraft = arena.Alloc<float>(size_t(k) * n);   // [j][s]
    float *dUAccept = arena.Alloc<float>(size_t(n) * k);  // [s][j]
    float *dUFinal = arena.Alloc<float>(n);
    opure_event *ev[4] = {arena.Event(), arena.Event(), arena.Event(), arena.Event()};

    std::vector<synth::Rng> rng;
    for (uint32_t s = 0; s < n; ++s) rng.emplace_back(o.seed ^ (uint64_t(s) * 0x9E3779B97F4A7C15ull));
    auto uniform = [&](uint32_t s) { return float(double(rng[s].NextU32()) / 4294967296.0); };

    // Prefill both models; the first generated token comes from the target.
    std::vector<uint32_t> first = target.PrefillBatch(prompts, reserve, rej);
    draft.PrefillBatch(prompts, reserve, false);
    if (rej) {
        std::vector<float> u0(n);
        for (uint32_t s = 0; s < n; ++s) u0[s] = uniform(s);
        OPURE_CUDA_CHECK(opure_h2d(ctx, dUFinal, u0.data(), n * 4));
        OPURE_CUDA_CHECK(opure_sample_softmax(ctx, target.DeviceLogits(), V, n, dUFinal, dAcc));
        std::vector<int32_t> t0(n);
        OPURE_CUDA_CHECK(opure_d2h(ctx, t0.data(), dAcc, n * 4));
        OPURE_CUDA_CHECK(opure_sync(ctx, 60000));
        for (uint32_t s = 0; s < n; ++s) first[s] = uint32_t(t0[s]);
    }

    std::vector<std::vector<uint32_t>> out(n);
    std::vector<int32_t> p(n, int32_t(P0)), t(n), prev(n);
    for (uint32_t s = 0; s < n; ++s) {
        t[s] = int32_t(first[s]);
        prev[s] = int32_t(prompts[s].back());
        out[s].push_back(first[s]);
    }
    auto done = [&](uint32_t s) { return out[s].size() >= o.maxNew; };

    std::vector<int32_t> pos(n), known(n), seqv(size_t(n) * (k + 1)), posv(size_t(n) * (k + 1));
    std::vector<int32_t> hOut(size_t(n) * (k + 1)), hAcc(n), hDraft(size_t(n) * k);
    std::vector<float> ud(size_t(k) * n), ua(size_t(n) * k), uf(n);
    SpecStats st;
    while (true) {
        bool all = true;
        for (uint32_t s = 0; s < n; ++s) all = all && done(s);
        if (all) break;

        // Draft: k+1 self-driving steps from p-1.
        for (uint32_t s = 0; s < n; ++s) {
            const int32_t hist[2] = {prev[s], t[s]};
            draft.WriteHistory(s, uint32_t(p[s] - 1), hist, 2);
            pos[s] = p[s] - 1;
            known[s] = p[s] + 1;
        }
        draft.SetAutoVectors(pos.data(), known.data(), n);
        OPURE_CUDA_CHECK(opure_h2d(ctx, dBase, p.data(), n * 4));
        if (rej) {
            for (uint32_t s = 0; s < n; ++s) {
                for (uint32_t j = 0; j < k; ++j) ud[size_t(j) * n + s] = uniform(s);
                for (uint32_t j = 0; j < k; ++j) ua[size_t(s) * k + j] = uniform(s);
                uf[s] = uniform(s);
            }
            OPURE_CUDA_CHECK(opure_h2d(ctx, dUDraft, ud.data(), ud.size() * 4));
            OPURE_CUDA_CHECK(opure_h2d(ctx, dUAccept, ua.data(), ua.size() * 4));
            OPURE_CUDA_CHECK(opure_h2d(ctx, dUFinal, uf.data(), n * 4));
        }
        OPURE_CUDA_CHECK(opure_event_record(ctx, ev[0]));
        if (!rej) {
            draft.RunSteps(n, k + 1, false);
        } else {
            draft.RunSteps(n, 1, false);  // position p-1: refreshes the KV row only
            for (uint32_t j = 0; j < k; ++j) {
                draft.RunSteps(n, 1, true);
                OPURE_CUDA_CHECK(opure_sample_keys(ctx, draft.DeviceLogits(), V, n, dUDraft + size_t(j) * n,
                                                   draft.DeviceKeys(), dDraftLogits + size_t(j) * V,
                                                   size_t(k) * V));
            }
        }
        OPURE_CUDA_CHECK(opure_event_record(ctx, ev[1]));

        // Verify: the target runs (t, d_1..d_k) at positions p..p+k of every sequence.
        OPURE_CUDA_CHECK(opure_spec_gather(ctx, draft.DeviceHistory(), draft.MaxLen(), draft.DeviceKeys(), dBase,
                                           n, k, target.DeviceInTokens(), dDraft));
        for (uint32_t s = 0; s < n; ++s)
            for (uint32_t j = 0; j <= k; ++j) {
                seqv[size_t(s) * (k + 1) + j] = int32_t(s);
                posv[size_t(s) * (k + 1) + j] = p[s] + int32_t(j);
            }
        target.SetVectors(seqv.data(), posv.data(), nullptr, n * (k + 1));
        target.RunSteps(n * (k + 1), 1, true);

        // Accept.
        opure_spec_args a{};
        a.mode = o.mode;
        a.n_seq = n;
        a.k = k;
        a.vocab = V;
        a.target_logits = target.DeviceLogits();
        a.draft_logits = dDraftLogits;
        a.draft = dDraft;
        a.u_accept = rej ? dUAccept : nullptr;
        a.u_final = rej ? dUFinal : nullptr;
        a.out_tokens = dOut;
        a.out_accepted = dAcc;
        OPURE_CUDA_CHECK(opure_spec_accept(ctx, &a));
        OPURE_CUDA_CHECK(opure_event_record(ctx, ev[2]));
        OPURE_CUDA_CHECK(opure_d2h(ctx, hOut.data(), dOut, hOut.size() * 4));
        OPURE_CUDA_CHECK(opure_d2h(ctx, hAcc.data(), dAcc, n * 4));
        if (draftLog) OPURE_CUDA_CHECK(opure_d2h(ctx, hDraft.data(), dDraft, hDraft.size() * 4));
        OPURE_CUDA_CHECK(opure_sync(ctx, 60000));
        CheckDevice(ctx);
        st.draftMs += Elapsed(ev[0], ev[1]);
        st.verifyMs += Elapsed(ev[1], ev[2]);
        ++st.rounds;

        for (uint32_t s = 0; s < n; ++s) {
            if (draftLog)
                for (uint32_t j = 0; j < k; ++j) draftLog->push_back(done(s) ? -1 : hDraft[size_t(s) * k + j]);
            if (done(s)) {
                if (acceptLog) acceptLog->push_back(-1);
                continue;  // finished sequences keep their position: no KV growth
            }
            const int32_t acc = hAcc[s];
            OPURE_CHECK(acc >= 0 && uint32_t(acc) <= k, "accept step returned an invalid count");
            if (acceptLog) acceptLog->push_back(acc);
            st.drafted += k;
            st.accepted += uint32_t(acc);
            const int32_t *row = hOut.data() + size_t(s) * (k + 1);
            for (int32_t i = 0; i <= acc && !done(s); ++i) out[s].push_back(uint32_t(row[i]));
            prev[s] = acc > 0 ? row[acc - 1] : t[s];
            t[s] = row[acc];
            p[s] += acc + 1;
        }
    }
    st.totalMs = st.draftMs + st.verifyMs;
    // MetricsSnapshot.speculativeAcceptance, which the reference fixes at -1
    // (Opure_VoxelEngine.cpp:666): accepted / drafted over this call.
    if (st.drafted) target.SetSpeculativeAcceptance(float(double(st.accepted) / double(st.drafted)));
    if (stats) *stats = st;
    return out;
}

}  // namespace opure::engine
