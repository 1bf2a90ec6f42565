// spec_decode.h -- speculative decoding: a draft engine proposes k tokens per round, the
// target engine verifies all k+1 positions of every sequence in one batched pass, and
// opure_spec_accept keeps the longest acceptable prefix plus one token of the target.
//
// The reference declares the verify shader (shaders/Opure_SpeculativeDecode.usf:60-189,
// Library::SpecVerifyFor, src/engine/Opure_Shaders.h:110-124) but never dispatches it and
// has no draft loop or accept rule (MetricsSnapshot.speculativeAcceptance is fixed at -1,
// src/engine/Opure_VoxelEngine.cpp:666). This is the loop that shader was meant for.
#pragma once

#include <cstdint>
#include <vector>

#include "voxel_engine.h"

namespace opure::engine {

struct SpecOptions {
    uint32_t k = 4;                 // draft tokens per round
    uint32_t mode = 0;              // OPURE_SPEC_GREEDY or OPURE_SPEC_REJECTION (temperature 1)
    uint64_t seed = 0;              // uniform streams: sequence s uses Rng(seed ^ s * 0x9E3779B97F4A7C15)
    uint32_t maxNew = 256;          // generated tokens per sequence
};

struct SpecStats {
    uint32_t rounds = 0;
    uint64_t drafted = 0;           // draft tokens proposed to sequences still generating
    uint64_t accepted = 0;          // of those, accepted
    double draftMs = 0.0;           // device time of the draft steps
    double verifyMs = 0.0;          // device time of the verify pass + accept
    double totalMs = 0.0;           // device time of all rounds
};

// Generates o.maxNew tokens for every prompt (equal lengths; slots 0..n-1 of both engines).
// Requirements: both engines on one ctx (draft created with target.Ctx() as `shared`),
// the same vocabulary, target maxBatch >= n (k + 1), draft maxBatch >= n, and maxLen of
// both >= prompt + maxNew + k + 2.
//
// Per round, for every sequence with next input t at position p:
//   draft   k+1 self-driving steps at positions p-1 .. p+k-1 (p-1 recomputes the KV row the
//           previous round may not have written), proposing d_1..d_k: greedy argmax, or
//           with `mode` rejection, draws from the draft's softmax (opure_sample_keys) with
//           the sequence's uniforms u_draft[0..k-1];
//   verify  the target runs the n(k+1) vectors (t, d_1..d_k) at positions p..p+k of each
//           sequence as one decode step with logits (their KV rows are appended
//           speculatively; a position's attention sees exactly the rows before it);
//   accept  opure_spec_accept with u_accept[0..k-1], u_final: a drafts accepted, then the
//           target's own token; the sequence continues at p + a + 1, whose KV rows in both
//           engines are all accepted ones (later rows are overwritten before being read).
// The first generated token is the target's greedy argmax after the prompt (rejection
// mode: a draw from its softmax with the sequence's first uniform). Uniform draws per
// sequence and round are always u_draft[k], u_accept[k], u_final, in that order.
// acceptLog, when given, receives per round n entries: the accepted count of each
// sequence, or -1 once that sequence has all its tokens. draftLog, when given, receives
// per round n * k entries: the drafted tokens d_1..d_k of each sequence (-1 once it has
// all its tokens).
std::vector<std::vector<uint32_t>> SpecGenerate(VoxelEngine &target, VoxelEngine &draft,
                                                const std::vector<std::vector<uint32_t>> &prompts,
                                                const SpecOptions &o, SpecStats *stats = nullptr,
                                                std::vector<int32_t> *acceptLog = nullptr,
                                                std::vector<int32_t> *draftLog = nullptr);

}  // namespace opure::engine
