// synth.cpp -- seeded synthetic model and input generation.
#include "synth.h"

#include <sys/stat.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>
#include <thread>

#include "platform.h"
#include "streamer.h"

namespace opure::synth {

double Normal::Next() {
    if (has_) {
        has_ = false;
        return spare_;
    }
    const double u1 = rng_.NextOpen(), u2 = rng_.NextOpen();
    const double r = std::sqrt(-2.0 * std::log(u1));
    const double a = 2.0 * M_PI * u2;
    spare_ = r * std::sin(a);
    has_ = true;
    return r * std::cos(a);
}

namespace {
// Runs fn(i) for i in [0, n) on the host's threads, in contiguous chunks of at least
// `grain` indices.
template <class F>
void ParallelChunks(uint64_t n, uint64_t grain, F &&fn) {
    const uint64_t nt = std::min<uint64_t>(std::max(1u, std::thread::hardware_concurrency()), (n + grain - 1) / grain);
    if (nt <= 1) {
        for (uint64_t i = 0; i < n; ++i) fn(i);
        return;
    }
    std::vector<std::thread> ts;
    for (uint64_t t = 0; t < nt; ++t)
        ts.emplace_back([&, t] {
            for (uint64_t i = n * t / nt; i < n * (t + 1) / nt; ++i) fn(i);
        });
    for (auto &th : ts) th.join();
}
}  // namespace

void Normal::Fill(uint64_t n, double scale, float *out) {
    uint64_t i = 0;
    if (has_ && n) {  // the spare of a pair drawn earlier comes first
        out[i++] = float(spare_ * scale);
        has_ = false;
    }
    // Whole pairs: each block's generator state is found by stepping the xorshift alone,
    // then the blocks (the transcendentals) run on host threads.
    constexpr uint64_t kPairs = uint64_t(1) << 16;
    const uint64_t pairs = (n - i) / 2, blocks = (pairs + kPairs - 1) / kPairs;
    std::vector<uint64_t> starts(blocks);
    for (uint64_t b = 0; b < blocks; ++b) {
        starts[b] = rng_.s;
        const uint64_t m = std::min(kPairs, pairs - b * kPairs);
        for (uint64_t k = 0; k < 2 * m; ++k) rng_.NextU32();
    }
    float *o = out + i;
    ParallelChunks(blocks, 1, [&](uint64_t b) {
        Normal g(1);
        g.rng_.s = starts[b];
        const uint64_t m = std::min(kPairs, pairs - b * kPairs);
        for (uint64_t k = 0; k < 2 * m; ++k) o[2 * b * kPairs + k] = float(g.Next() * scale);
    });
    i += 2 * pairs;
    if (i < n) out[i] = float(Next() * scale);  // an odd count leaves the pair's spare
}

std::vector<uint16_t> NormalF16(uint64_t seed, float stddev, uint64_t n) {
    // Normals come in pairs from pairs of draws, so the stream splits into blocks of whole
    // pairs: each block's generator state is found by stepping the xorshift alone, and the
    // blocks (sqrt/log/sin/cos) run on host threads. The values equal the serial stream's.
    constexpr uint64_t kBlock = uint64_t(1) << 17;  // normals per block (even)
    std::vector<uint16_t> out(n);
    const uint64_t blocks = (n + kBlock - 1) / kBlock;
    std::vector<uint64_t> starts(blocks);
    Rng r(seed);
    for (uint64_t b = 0; b < blocks; ++b) {
        starts[b] = r.s;
        for (uint64_t i = 0; i < kBlock; ++i) r.NextU32();
    }
    auto run = [&](uint64_t b0, uint64_t step) {
        for (uint64_t b = b0; b < blocks; b += step) {
            Normal g(1);
            g.SetState(starts[b]);
            const uint64_t i1 = std::min(n, (b + 1) * kBlock);
            for (uint64_t i = b * kBlock; i < i1; ++i) out[i] = safetensors::F32ToF16(float(g.Next() * stddev));
        }
    };
    const uint64_t nt = std::min<uint64_t>(blocks, std::max(1u, std::thread::hardware_concurrency()));
    std::vector<std::thread> ts;
    for (uint64_t t = 1; t < nt; ++t) ts.emplace_back(run, t, nt);
    run(0, nt ? nt : 1);
    for (auto &t : ts) t.join();
    return out;
}

std::vector<int32_t> Prompt(uint64_t seed, uint32_t vocab, uint32_t n) {
    Rng r(seed);
    std::vector<int32_t> out(n);
    for (uint32_t i = 0; i < n; ++i) out[i] = int32_t(r.NextU32() % vocab);
    return out;
}

std::vector<int32_t> Permutation(uint64_t seed, uint32_t n) {
    std::vector<int32_t> p(n);
    for (uint32_t i = 0; i < n; ++i) p[i] = int32_t(i);
    Rng r(seed);
    for (uint32_t i = n; i > 1; --i) {
        const uint32_t j = r.NextU32() % i;
        std::swap(p[i - 1], p[j]);
    }
    return p;
}

uint16_t KvValue(uint64_t seed, uint32_t slot, uint64_t i) {
    // SplitMix64 finaliser (Steele, Lea & Flood 2014).
    uint64_t z = (seed ^ (uint64_t(slot) << 48) ^ i) + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    const float u = float(uint32_t(z >> 40)) * (1.0f / 16777216.0f);
    return safetensors::F32ToF16(u * 4.0f - 2.0f);
}

std::vector<uint16_t> SynthKv(uint64_t seed, uint32_t slot, uint32_t layers, uint32_t n_kv, uint32_t len,
                              uint32_t head_dim) {
    std::vector<uint16_t> out(size_t(layers) * 2 * n_kv * len * head_dim);
    size_t o = 0;
    for (uint32_t L = 0; L < layers; ++L)
        for (uint32_t sel = 0; sel < 2; ++sel)
            for (uint32_t h = 0; h < n_kv; ++h)
                for (uint32_t p = 0; p < len; ++p)
                    for (uint32_t d = 0; d < head_dim; ++d)
                        out[o++] = KvValue(seed, slot, (((uint64_t(L) * 2 + sel) * n_kv + h) * 65536 + p) * head_dim + d);
    return out;
}

std::vector<float> Uniforms(uint64_t seed, uint64_t n) {
    Rng r(seed);
    std::vector<float> out(n);
    for (uint64_t i = 0; i < n; ++i) out[i] = float(double(r.NextU32()) / 4294967296.0);
    return out;
}

namespace {

struct Entry {
    std::string name;
    std::string dtype;
    std::vector<uint64_t> shape;
    std::vector<uint8_t> bytes;
    float scale = 1.0f;
    bool has_scale = false;
};

// Per-tensor symmetric int8: scale = absmax / 127, round half to even, clamp +-127.
void Quantize(const std::vector<uint16_t> &w, std::vector<uint8_t> &q, float &scale) {
    float amax = 0.f;
    for (uint16_t h : w) amax = std::fmax(amax, std::fabs(safetensors::F16ToF32(h)));
    scale = amax > 0.f ? amax / 127.0f : 1.0f;
    q.resize(w.size());
    for (size_t i = 0; i < w.size(); ++i) {
        float r = std::nearbyint(safetensors::F16ToF32(w[i]) / scale);
        r = std::fmin(127.f, std::fmax(-127.f, r));
        q[i] = uint8_t(int8_t(r));
    }
}

void MkDirs(const std::string &dir) {
    std::string cur;
    std::stringstream ss(dir);
    std::string part;
    if (!dir.empty() && dir[0] == '/') cur = "/";
    while (std::getline(ss, part, '/')) {
        if (part.empty()) continue;
        cur += part + "/";
        ::mkdir(cur.c_str(), 0755);
    }
}

}  // namespace

void WriteModel(const std::string &dir, const ModelSpec &s) {
    OPURE_CHECK(s.heads && s.kv_heads && s.hidden % s.heads == 0 && s.heads % s.kv_heads == 0,
                "synthetic model: inconsistent head counts");
    MkDirs(dir);
    const uint64_t h = s.hidden, ff = s.inter, hd = s.hidden / s.heads, kvh = uint64_t(s.kv_heads) * hd;
    Normal g(s.seed);
    Normal noise(s.noise_seed);
    std::vector<Entry> entries;

    std::vector<float> draws, noises;
    auto matrix = [&](const std::string &name, uint64_t rows, uint64_t cols, bool quantizable) {
        // Element i: fp16(fp16(N_i * std) + noise_i * noise_std), both streams in element order.
        const uint64_t n = rows * cols;
        std::vector<uint16_t> w(n);
        draws.resize(n);
        g.Fill(n, double(s.std), draws.data());
        if (s.noise_std > 0.f) {
            noises.resize(n);
            noise.Fill(n, double(s.noise_std), noises.data());
        }
        ParallelChunks(n, 4096, [&](uint64_t i) {
            float v = safetensors::F16ToF32(safetensors::F32ToF16(draws[i]));
            if (s.noise_std > 0.f) v = v + noises[i];
            w[i] = safetensors::F32ToF16(v);
        });
        Entry e;
        e.name = name;
        e.shape = {rows, cols};
        if (s.int8 && quantizable) {
            e.dtype = "I8";
            Quantize(w, e.bytes, e.scale);
            e.has_scale = true;
        } else {
            e.dtype = "F16";
            e.bytes.resize(w.size() * 2);
            std::memcpy(e.bytes.data(), w.data(), e.bytes.size());
        }
        entries.push_back(std::move(e));
    };
    auto ones = [&](const std::string &name, uint64_t n) {
        Entry e;
        e.name = name;
        e.dtype = "F16";
        e.shape = {n};
        std::vector<uint16_t> w(n, 0x3C00);  // 1.0
        e.bytes.resize(n * 2);
        std::memcpy(e.bytes.data(), w.data(), e.bytes.size());
        entries.push_back(std::move(e));
    };

    matrix("model.embed_tokens.weight", s.vocab, h, false);
    for (uint32_t l = 0; l < s.layers; ++l) {
        const std::string p = "model.layers." + std::to_string(l) + ".";
        ones(p + "input_layernorm.weight", h);
        matrix(p + "self_attn.q_proj.weight", h, h, true);
        matrix(p + "self_attn.k_proj.weight", kvh, h, true);
        matrix(p + "self_attn.v_proj.weight", kvh, h, true);
        matrix(p + "self_attn.o_proj.weight", h, h, true);
        ones(p + "post_attention_layernorm.weight", h);
        matrix(p + "mlp.gate_proj.weight", ff, h, true);
        matrix(p + "mlp.up_proj.weight", ff, h, true);
        matrix(p + "mlp.down_proj.weight", h, ff, true);
    }
    ones("model.norm.weight", h);
    if (!s.tied) matrix("lm_head.weight", s.vocab, h, false);

    // Header JSON with payload-relative offsets.
    std::ostringstream hdr;
    hdr << "{\"__metadata__\":{\"format\":\"pt\"}";
    uint64_t off = 0;
    for (const Entry &e : entries) {
        hdr << ",\"" << e.name << "\":{\"dtype\":\"" << e.dtype << "\",\"shape\":[";
        for (size_t i = 0; i < e.shape.size(); ++i) hdr << (i ? "," : "") << e.shape[i];
        hdr << "],\"data_offsets\":[" << off << "," << off + e.bytes.size() << "]";
        if (e.has_scale) {
            char buf[64];
            std::snprintf(buf, sizeof(buf), "%.9g", double(e.scale));
            hdr << ",\"scale\":" << buf;
        }
        hdr << "}";
        off += e.bytes.size();
    }
    hdr << "}";
    std::string header = hdr.str();
    while (header.size() % 8) header += ' ';  // payload 8-byte aligned

    const std::string tmp = dir + "/model.safetensors.tmp";
    {
        std::ofstream f(tmp, std::ios::binary);
        OPURE_CHECK(bool(f), "cannot write " + tmp);
        const uint64_t hl = header.size();
        f.write(reinterpret_cast<const char *>(&hl), 8);
        f.write(header.data(), std::streamsize(header.size()));
        for (const Entry &e : entries) f.write(reinterpret_cast<const char *>(e.bytes.data()), std::streamsize(e.bytes.size()));
        OPURE_CHECK(bool(f), "short write to " + tmp);
    }
    OPURE_CHECK(std::rename(tmp.c_str(), (dir + "/model.safetensors").c_str()) == 0, "rename failed");

    std::ostringstream cfg;
    char eps[32], theta[32];
    std::snprintf(eps, sizeof(eps), "%.9g", double(s.eps));
    std::snprintf(theta, sizeof(theta), "%.17g", s.theta);
    cfg << "{\n  \"architectures\": [\"LlamaForCausalLM\"],\n  \"model_type\": \"llama\",\n"
        << "  \"hidden_act\": \"silu\",\n  \"vocab_size\": " << s.vocab << ",\n  \"hidden_size\": " << s.hidden
        << ",\n  \"intermediate_size\": " << s.inter << ",\n  \"num_hidden_layers\": " << s.layers
        << ",\n  \"num_attention_heads\": " << s.heads << ",\n  \"num_key_value_heads\": " << s.kv_heads
        << ",\n  \"max_position_embeddings\": " << s.max_pos << ",\n  \"rms_norm_eps\": " << eps
        << ",\n  \"rope_theta\": " << theta << ",\n  \"tie_word_embeddings\": " << (s.tied ? "true" : "false")
        << ",\n  \"torch_dtype\": \"float16\"\n}\n";
    std::ofstream c(dir + "/config.json");
    c << cfg.str();
    OPURE_CHECK(bool(c), "cannot write config.json");
}

}  // namespace opure::synth
