// synth.h -- seeded synthetic inputs: model directories (config.json + model.safetensors),
// prompts, page permutations, uniforms and fp16 normals. The reference fetches a real
// checkpoint instead (scripts/fetch_model.ps1); the benchmark configurations use
// random-init weights, generated here from the harness's xorshift64 Rng
// (Opure_TestHarness.cpp:36-47) so the CUDA path and the CPU oracle read identical bytes.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace opure::synth {

// xorshift64 of Opure_TestHarness.cpp:36-47 (seed 0 behaves as seed 1).
struct Rng {
    uint64_t s;
    explicit Rng(uint64_t seed) : s(seed ? seed : 1) {}
    uint32_t NextU32() {
        s ^= s << 13;
        s ^= s >> 7;
        s ^= s << 17;
        return uint32_t(s >> 32);
    }
    // Uniform in (0, 1): (NextU32() + 0.5) / 2^32.
    double NextOpen() { return (double(NextU32()) + 0.5) / 4294967296.0; }
};

// Standard normals by the Box-Muller transform (Box & Muller 1958) on pairs of open
// uniforms: z0 = r cos(2 pi u2), z1 = r sin(2 pi u2), r = sqrt(-2 ln u1); z0 then z1.
class Normal {
public:
    explicit Normal(uint64_t seed) : rng_(seed) {}
    double Next();
    // out[i] = float(Next() * scale) for the next n normals of the stream, on host threads
    // when n is large: the same values and the same stream state afterwards as n calls.
    void Fill(uint64_t n, double scale, float *out);
    // Continue from a raw xorshift state (at a pair boundary of the stream).
    void SetState(uint64_t s) {
        rng_.s = s;
        has_ = false;
    }

private:
    Rng rng_;
    double spare_ = 0.0;
    bool has_ = false;
};

struct ModelSpec {
    uint32_t vocab = 49152, hidden = 576, inter = 1536, layers = 30, heads = 9, kv_heads = 3;
    uint32_t max_pos = 2048;
    float eps = 1e-5f;
    double theta = 10000.0;
    bool tied = true;
    uint64_t seed = 0;         // weights N(0, std) in file order
    float std = 0.02f;
    bool int8 = false;         // matrices stored as per-tensor int8 with a "scale" key
    uint64_t noise_seed = 0;   // draft models: each matrix element + N(0, noise_std)
    float noise_std = 0.0f;
};

// Writes dir/config.json and dir/model.safetensors. Draw order: embed_tokens, then per
// layer q, k, v, o, gate, up, down (and lm_head last when untied); norm gains are 1.0.
void WriteModel(const std::string &dir, const ModelSpec &spec);

std::vector<uint16_t> NormalF16(uint64_t seed, float stddev, uint64_t n);
std::vector<int32_t> Prompt(uint64_t seed, uint32_t vocab, uint32_t n);      // NextU32() % vocab
std::vector<int32_t> Permutation(uint64_t seed, uint32_t n);                 // Fisher-Yates
std::vector<float> Uniforms(uint64_t seed, uint64_t n);                      // NextU32() / 2^32

// Synthetic KV context values (the host form of opure_kv_synth): element i of a slot is
// fp16(4u - 2) with u = (splitmix64(seed ^ slot << 48 ^ i) >> 40) / 2^24 and
// i = (((layer * 2 + kv_sel) * n_kv + head) * 65536 + pos) * head_dim + d.
uint16_t KvValue(uint64_t seed, uint32_t slot, uint64_t i);
// [layers][2][n_kv][len][head_dim] for one slot (the layout VoxelEngine::LoadKv takes).
std::vector<uint16_t> SynthKv(uint64_t seed, uint32_t slot, uint32_t layers, uint32_t n_kv, uint32_t len,
                              uint32_t head_dim);

}  // namespace opure::synth
