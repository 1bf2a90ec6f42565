// kv_synth.cu -- opure_kv_synth: seeded synthetic KV contexts written straight into the
// paged pool, so long-context decode (the 4096-token contexts of the large-model
// configuration) can be measured without a 4096-step prefill per sequence.
// The value of element (slot, layer, K|V, kv head, pos, d) is a pure function of its
// coordinates; the host restatement (synth::KvValue) produces the same fp16 bits.
#include <algorithm>

#include "ctx.cuh"

namespace opure {
namespace {

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    // SplitMix64 finaliser (Steele, Lea & Flood 2014).
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Uniform on [-2, 2) with 24-bit resolution (exact in fp32), rounded to fp16.
__device__ __forceinline__ __half kv_value(uint64_t seed, uint32_t slot, uint64_t idx) {
    const uint64_t h = splitmix64(seed ^ (uint64_t(slot) << 48) ^ idx);
    const float u = float(uint32_t(h >> 40)) * (1.0f / 16777216.0f);
    return __float2half_rn(u * 4.0f - 2.0f);
}

struct SynthParams {
    uint16_t *pool;
    const int32_t *page_table;
    uint32_t n_pages, max_pages, page_size, n_kv, hd;
    uint32_t layer, slot0, n_slots, len;
    uint64_t seed;
    DeviceStatus *st;
};

// One thread per 8 consecutive head-dim elements of one (slot, K|V, head, pos) row.
__global__ void kv_synth_kernel(SynthParams p) {
    const uint32_t groups = p.hd / 8;
    const uint64_t per_slot = uint64_t(2) * p.n_kv * p.len * groups;
    const uint64_t total = per_slot * p.n_slots;
    for (uint64_t t = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
         t += uint64_t(gridDim.x) * blockDim.x) {
        const uint32_t slot = p.slot0 + uint32_t(t / per_slot);
        uint64_t r = t % per_slot;
        const uint32_t g = uint32_t(r % groups);
        r /= groups;
        const uint32_t pos = uint32_t(r % p.len);
        r /= p.len;
        const uint32_t head = uint32_t(r % p.n_kv);
        const uint32_t sel = uint32_t(r / p.n_kv);
        const uint32_t lp = pos / p.page_size;
        const int32_t page = lp < p.max_pages ? p.page_table[size_t(slot) * p.max_pages + lp] : -1;
        if (page < 0 || uint32_t(page) >= p.n_pages) {
            report(p.st, OPURE_ERR_DEVICE_BOUNDS, 80, pos);
            continue;
        }
        const uint64_t base = ((((uint64_t(p.layer) * 2 + sel) * p.n_kv + head) * 65536 + pos) * p.hd) + g * 8;
        __align__(16) __half v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = kv_value(p.seed, slot, base + e);
        __half *dst = reinterpret_cast<__half *>(p.pool) +
                      ((size_t(page) * 2 + sel) * p.n_kv + head) * size_t(p.page_size) * p.hd +
                      size_t(pos % p.page_size) * p.hd + g * 8;
        *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(v);
    }
}

}  // namespace
}  // namespace opure

using namespace opure;

extern "C" opure_status opure_kv_synth(opure_ctx *ctx, const opure_kv_layout *kv, uint32_t layer,
                                       uint32_t slot0, uint32_t n_slots, uint32_t len, uint64_t seed) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!kv || !kv->pool || !kv->page_table || !kv->page_size || !kv->n_kv || !kv->head_dim)
        return OPURE_ERR_INVALID_ARG;
    if (kv->head_dim % 8 || len > 65536 || uint64_t(len) > uint64_t(kv->max_pages) * kv->page_size ||
        (kv->ring && uint64_t(len) > uint64_t(kv->ring) * kv->page_size))
        return OPURE_ERR_INVALID_ARG;
    if (n_slots == 0 || len == 0) return OPURE_OK;
    SynthParams p{kv->pool, kv->page_table, kv->n_pages, kv->max_pages, kv->page_size, kv->n_kv, kv->head_dim,
                  layer, slot0, n_slots, len, seed, ctx->status};
    const uint64_t total = uint64_t(2) * kv->n_kv * len * (kv->head_dim / 8) * n_slots;
    const uint32_t blocks = uint32_t(std::min<uint64_t>((total + 255) / 256, uint64_t(ctx->sm_count) * 16));
    return launch(ctx, kv_synth_kernel, dim3(blocks), dim3(256), 0, false, p);
}
