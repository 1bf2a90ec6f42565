// sample_decode.h -- generation with temperature / top-k / top-p / repetition-penalty
// sampling and per-token logit statistics, all on the device.
//
// The reference declares these options (GenerationConfig, src/proto/opure.proto:35-46;
// EngineOptions.temperature, src/engine/Opure_VoxelEngine.h:64) but its Generate is
// greedy, and its entropy / norm statistics are host readbacks of the whole logit vector
// (VoxelEngine::RefreshLogitStats, src/engine/Opure_VoxelEngine.cpp:832-876). Here each
// step's logits stay on the device: opure_logit_stats and opure_sample_filtered read them
// and the sampled token becomes the next self-driving step's input.
#pragma once

#include <cstdint>
#include <vector>

#include "voxel_engine.h"

namespace opure::engine {

struct SampleOptions {
    float temperature = 1.0f;   // <= 0: greedy
    uint32_t topK = 0;          // 0: off
    float topP = 1.0f;          // 1: off
    float repPenalty = 1.0f;    // 1: off; applied to every token of the sequence so far
    uint64_t seed = 0;          // sequence s draws uniforms from Rng(seed ^ s * 0x9E3779B97F4A7C15)
    uint32_t maxNew = 16;       // generated tokens per sequence
};

// Generates o.maxNew tokens for each prompt (equal lengths; slots 0..n-1). Token j of
// sequence s is drawn by opure_sample_filtered from the logits of its position with the
// j-th uniform of the sequence's stream. stats, when given, receives [n][maxNew][4]:
// opure_logit_stats of the logits each token was drawn from; logits, when given, those
// logits themselves, [n][maxNew][vocab] (for verification; costly).
std::vector<std::vector<uint32_t>> SampleGenerate(VoxelEngine &eng, const std::vector<std::vector<uint32_t>> &prompts,
                                                  const SampleOptions &o, std::vector<float> *stats,
                                                  std::vector<float> *logits = nullptr);

}  // namespace opure::engine
