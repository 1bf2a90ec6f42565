// attention.cu -- split-K flash-decode attention over the paged fp16 KV cache.
//
// Replaces AttentionMain{32..256} (shaders/Opure_FlashAttention_Decode.usf:58-179): the
// reference runs one 64-thread group per query head, serial over every key with two
// barriers per key, and reads each KV head once per query head. Here one CTA owns a
// (query entry, kv head, key split) triple and serves all G = n_heads / n_kv query heads
// of that kv head from a single read of its keys and values.
//
// The per-lane online-softmax loop lives in attn_core.cuh. States are merged across
// lane groups (shuffles), warps (shared memory) and finally across key splits: each CTA
// writes its partial (m, l, acc) to caller-provided scratch and the last CTA of an
// (entry, kv head) to finish -- found with an atomic ticket, no waiting -- merges them
// and writes the output. With a single split the CTA writes its output directly.
#include <algorithm>
#include <type_traits>

#include "attn_core.cuh"
#include "ctx.cuh"
#include "tma.cuh"

namespace opure {
namespace {

constexpr int kWarps = 4;

template <int HD>
constexpr uint32_t cta_block_tokens() { return AttnShape<HD>::TB * kWarps; }

struct AttnParams {
    const float *q;          // [entries][n_heads][HD] (entry = (i, j) flattened)
    float *out;
    const int32_t *seq;      // [n]
    const int32_t *seq_len;  // [n]
    uint32_t n, n_q, n_heads;
    float scale_log2;        // scale * log2(e)
    uint32_t split_tokens, n_splits;
    float *partials;         // [entries * n_kv * n_splits][G][HD + 2]
    uint32_t *counters;      // [entries * n_kv]
    opure_kv_layout kv;
    DeviceStatus *st;
};

// The TMA-staged kernel's parameters when it also writes the next GEMV's packed operand. A
// separate type: two more fields in AttnParams itself made the kernel ~10% slower on long
// contexts even with them unused (measured, B=64 x 8192 and 32768 tokens).
struct AttnPackedParams : AttnParams {
    __half *out_packed;      // [2][pk_npad][n_heads * HD] (store_packed)
    uint32_t pk_npad;
};
template <bool PK>
using AttnP = std::conditional_t<PK, AttnPackedParams, AttnParams>;

// Output element i (= head * HD + dim) of an entry: fp32, and with PK also the scale-free
// fp16 pair of the next GEMV's packed operand.
template <int HD, bool PK>
__device__ __forceinline__ void store_out(const AttnP<PK> &p, uint32_t entry, uint32_t i, float v) {
    const uint32_t len = p.n_heads * HD;
    p.out[size_t(entry) * len + i] = v;
    if constexpr (PK) store_packed(p.out_packed, p.pk_npad, len, entry, i, v, p.st, 15);
}

template <int HD, int G>
__global__ void __launch_bounds__(kWarps * 32) attn_kernel(AttnParams p) {
    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t n_kv = p.kv.n_kv;
    const uint32_t eg = blockIdx.x;              // (entry, kv head)
    const uint32_t entry = eg / n_kv, g = eg % n_kv;
    const uint32_t split = blockIdx.y;
    const uint32_t i = entry / p.n_q, j = entry % p.n_q;

    grid_dependency_wait();
    grid_dependents_launch();

    const int32_t sidx = p.seq[i];
    const int32_t len = p.seq_len[i] + int32_t(j);
    const uint32_t t_split = split * p.split_tokens;
    const uint32_t t_end = min(uint32_t(max(len, 0)), t_split + p.split_tokens);
    const uint32_t t_begin = max(t_split, window_begin(len - 1, p.kv.page_size, p.kv.ring));
    // Keys past the last split (a caller that understated max_ctx) would be dropped: refuse.
    if (threadIdx.x == 0 && split + 1 == p.n_splits && len > 0 && uint32_t(len) > t_split + p.split_tokens)
        report(p.st, OPURE_ERR_DEVICE_BOUNDS, 14, uint32_t(len));

    float qv[G][AttnShape<HD>::E];
    load_q_slice<HD, G>(p.q + size_t(entry) * p.n_heads * HD, g, p.scale_log2, qv);
    AttnState<HD, G> st;
    st.init();
    KvView kv{reinterpret_cast<const __half *>(p.kv.pool),
              p.kv.page_table + size_t(max(sidx, 0)) * p.kv.max_pages,
              p.kv.max_pages, p.kv.n_pages, p.kv.page_size, n_kv, g, sidx >= 0, p.kv.ring};
    attend_range<HD, G>(st, qv, kv, t_begin, t_end, warp, kWarps, p.st);
    merge_lane_groups<HD, G>(st);

    __shared__ WarpStates<HD, G, kWarps> ws;
    store_warp_state<HD, G, kWarps>(st, ws, warp);
    __syncthreads();

    // CTA partial -> scratch; one thread per (head, dim) plus the (m, l) pair.
    const uint32_t n_splits = p.n_splits;
    if (n_splits == 1) {
        // One split: the CTA's merged state is the result (the split merge below would
        // multiply it by exp2(0) = 1), so no partials, no ticket.
        for (uint32_t idx = threadIdx.x; idx < uint32_t(G) * HD; idx += blockDim.x) {
            const uint32_t h = idx / HD, d = idx % HD;
            float a, mn, ls;
            merge_warps<HD, G, kWarps>(ws, h, d, a, mn, ls);
            p.out[(size_t(entry) * p.n_heads + g * G + h) * HD + d] = a / fmaxf(ls, 1e-30f);
        }
        return;
    }
    float *part = p.partials + (size_t(eg) * n_splits + split) * G * (HD + 2);
    for (uint32_t idx = threadIdx.x; idx < uint32_t(G) * HD; idx += blockDim.x) {
        const uint32_t h = idx / HD, d = idx % HD;
        float a, mn, ls;
        merge_warps<HD, G, kWarps>(ws, h, d, a, mn, ls);
        part[h * (HD + 2) + d] = a;
        if (d == 0) {
            part[h * (HD + 2) + HD] = mn;
            part[h * (HD + 2) + HD + 1] = ls;
        }
    }
    __threadfence();
    __syncthreads();
    __shared__ uint32_t ticket;
    if (threadIdx.x == 0) ticket = atomicAdd(p.counters + eg, 1u);
    __syncthreads();
    if (ticket != n_splits - 1) return;

    // Last CTA of this (entry, kv head): merge every split.
    __threadfence();
    const float *parts = p.partials + size_t(eg) * n_splits * G * (HD + 2);
    for (uint32_t idx = threadIdx.x; idx < uint32_t(G) * HD; idx += blockDim.x) {
        const uint32_t h = idx / HD, d = idx % HD;
        float mn = -INFINITY;
        for (uint32_t sp = 0; sp < n_splits; ++sp)
            mn = fmaxf(mn, __ldcg(parts + (size_t(sp) * G + h) * (HD + 2) + HD));
        float a = 0.f, lsum = 0.f;
        for (uint32_t sp = 0; sp < n_splits; ++sp) {
            const float *pp = parts + (size_t(sp) * G + h) * (HD + 2);
            const float ms = __ldcg(pp + HD);
            const float f = (mn == -INFINITY || ms == -INFINITY) ? 0.f : fast_exp2(ms - mn);
            a += __ldcg(pp + d) * f;
            lsum += __ldcg(pp + HD + 1) * f;
        }
        // acc / max(sum, 1e-30) as the reference's epilogue
        // (Opure_FlashAttention_Decode.usf:235-239).
        p.out[(size_t(entry) * p.n_heads + g * G + h) * HD + d] = a / fmaxf(lsum, 1e-30f);
    }
    if (threadIdx.x == 0) p.counters[eg] = 0u;  // ready for the next call
}

// ---- TMA-staged variant (head_dim 64 and 128) ----------------------------------------
// The register-fed loop above issues one block of K/V loads per warp, then computes on it
// before the next block's addresses (page-table entry, then the rows) are even known: two
// dependent memory latencies per block and nothing in flight while it computes. Here a
// producer warp walks the split's pages ahead of the consumers and copies each page's K
// block and V block (page_size x HD fp16 each, contiguous in the pool) into a ring of
// shared-memory stages with bulk copies that complete on an mbarrier; four consumer warps
// run the same per-lane online softmax out of shared memory and release each stage with
// one arrival per warp. The page-table entries are read 32 at a time by the producer warp.
// All waits are bounded (1 s); a timed-out CTA records OPURE_ERR_DEVICE_TIMEOUT, and the
// producer waits (bounded) for every copy it issued before the CTA exits.
constexpr int kMaxStages = 8;
constexpr uint32_t kStageBudget = 64 * 1024;  // bytes of K/V stages per CTA

__host__ __device__ inline uint32_t stage_count(uint32_t page_bytes_kv) {
    const uint32_t n = kStageBudget / page_bytes_kv;
    return n < 2 ? 2u : (n > uint32_t(kMaxStages) ? uint32_t(kMaxStages) : n);
}

// One staged page through this warp's rounds (round rr covers page rows rr*TPW ..
// rr*TPW + TPW-1; warp w takes rounds w, w + kWarps, ...), R rounds per softmax block.
// CHECK masks rows outside [t_begin, t_end) (an empty range masks the whole page). The
// running state is rescaled only when a block raises the running max (the factor would be
// exactly 1 otherwise).
template <int HD, int G, int R, bool CHECK>
__device__ __forceinline__ void consume_page(AttnState<HD, G> &st, const float (&qv)[G][AttnShape<HD>::E],
                                             const __half *ks, const __half *vs, uint32_t warp, uint32_t rounds,
                                             uint32_t tok0, uint32_t t_begin, uint32_t t_end) {
    using S = AttnShape<HD>;
    constexpr int LPT = S::LPT, CH = S::CH, TPW = S::TPW, E = S::E;
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t grp = lane / LPT, sub = lane % LPT;
    for (uint32_t r0 = warp; r0 < rounds; r0 += kWarps * R) {
        uint4 kr[R][CH], vr[R][CH];
        bool valid[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const uint32_t rr = r0 + r * kWarps;
            const uint32_t row = rr * TPW + grp;
            valid[r] = rr < rounds;
            if (CHECK) valid[r] = valid[r] && tok0 + row >= t_begin && tok0 + row < t_end;
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                kr[r][c] = valid[r] ? *reinterpret_cast<const uint4 *>(ks + size_t(row) * HD + sub * E + c * 8)
                                    : make_uint4(0, 0, 0, 0);
                vr[r][c] = valid[r] ? *reinterpret_cast<const uint4 *>(vs + size_t(row) * HD + sub * E + c * 8)
                                    : make_uint4(0, 0, 0, 0);
            }
        }
        float sc[R][G];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            float kf[E];
#pragma unroll
            for (int c = 0; c < CH; ++c) unpack8(kr[r][c], kf + 8 * c);
#pragma unroll
            for (int h = 0; h < G; ++h) {
                // Packed fp32x2 FMAs (sm_100): even and odd dims in two accumulators.
                float2 d2 = make_float2(0.f, 0.f);
#pragma unroll
                for (int e = 0; e < E; e += 2)
                    d2 = __ffma2_rn(make_float2(qv[h][e], qv[h][e + 1]), make_float2(kf[e], kf[e + 1]), d2);
                float d = d2.x + d2.y;
#pragma unroll
                for (int o = LPT / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
                sc[r][h] = valid[r] ? d : -INFINITY;
            }
        }
#pragma unroll
        for (int h = 0; h < G; ++h) {
            float mb = sc[0][h];
#pragma unroll
            for (int r = 1; r < R; ++r) mb = fmaxf(mb, sc[r][h]);
            if (mb > st.m[h]) {  // also the first valid block (m = -inf)
                const float corr = fast_exp2(st.m[h] - mb);
                st.l[h] *= corr;
                const float2 c2 = make_float2(corr, corr);
#pragma unroll
                for (int e = 0; e < E; e += 2) {
                    const float2 a = __fmul2_rn(make_float2(st.acc[h][e], st.acc[h][e + 1]), c2);
                    st.acc[h][e] = a.x;
                    st.acc[h][e + 1] = a.y;
                }
                st.m[h] = mb;
            }
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            if (!valid[r]) continue;
            float vf[E];
#pragma unroll
            for (int c = 0; c < CH; ++c) unpack8(vr[r][c], vf + 8 * c);
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const float pr = fast_exp2(sc[r][h] - st.m[h]);
                st.l[h] += pr;
                const float2 p2 = make_float2(pr, pr);
#pragma unroll
                for (int e = 0; e < E; e += 2) {
                    const float2 a = __ffma2_rn(p2, make_float2(vf[e], vf[e + 1]), make_float2(st.acc[h][e], st.acc[h][e + 1]));
                    st.acc[h][e] = a.x;
                    st.acc[h][e + 1] = a.y;
                }
            }
        }
    }
}

template <int HD, int G, bool PK>
__global__ void __launch_bounds__((kWarps + 1) * 32) attn_tma_kernel(AttnP<PK> p) {
    using S = AttnShape<HD>;
    constexpr int TPW = S::TPW, E = S::E;
    constexpr int R = 4;  // rounds per consumer block
    extern __shared__ __align__(128) uint8_t stage_mem[];
    __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages];
    __shared__ int stage_ok[kMaxStages];
    __shared__ WarpStates<HD, G, kWarps> ws;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t n_kv = p.kv.n_kv;
    const uint32_t eg = blockIdx.x;
    const uint32_t entry = eg / n_kv, g = eg % n_kv;
    const uint32_t split = blockIdx.y;
    const uint32_t i = entry / p.n_q, j = entry % p.n_q;
    const uint32_t P = p.kv.page_size;
    const uint32_t page_elems = P * HD;
    const uint32_t page_bytes = page_elems * 2;
    const uint32_t n_stages = stage_count(2 * page_bytes);

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < n_stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarps);
        }
    }
    __syncthreads();

    grid_dependency_wait();
    grid_dependents_launch();

    const int32_t sidx = p.seq[i];
    const int32_t len = p.seq_len[i] + int32_t(j);
    const uint32_t t_split = split * p.split_tokens;
    const uint32_t t_end = min(uint32_t(max(len, 0)), t_split + p.split_tokens);
    const uint32_t t_begin = max(t_split, window_begin(len - 1, P, p.kv.ring));
    // Keys past the last split (a caller that understated max_ctx) would be dropped: refuse.
    if (threadIdx.x == 0 && split + 1 == p.n_splits && len > 0 && uint32_t(len) > t_split + p.split_tokens)
        report(p.st, OPURE_ERR_DEVICE_BOUNDS, 14, uint32_t(len));
    const bool any = sidx >= 0 && t_end > t_begin;
    const uint32_t pg_begin = t_begin / P;
    const uint32_t n_pg = any ? (t_end + P - 1) / P - pg_begin : 0u;

    AttnState<HD, G> st;
    st.init();

    if (warp == kWarps) {
        // Producer warp: page-table entries 32 at a time, lane 0 issues the copies.
        const int32_t *pt = p.kv.page_table + size_t(max(sidx, 0)) * p.kv.max_pages;
        const __half *pool = reinterpret_cast<const __half *>(p.kv.pool);
        bool ok = true;
        uint32_t issued = 0;  // iterations whose stage was armed (lane 0)
        for (uint32_t c0 = 0; c0 < n_pg && ok; c0 += 32) {
            int32_t mine = -1;
            if (c0 + lane < n_pg) {
                const uint32_t lp = ring_slot(pg_begin + c0 + lane, p.kv.ring);
                mine = lp < p.kv.max_pages ? pt[lp] : -1;
            }
            const uint32_t cnt = min(32u, n_pg - c0);
            for (uint32_t k = 0; k < cnt; ++k) {
                const int32_t page = __shfl_sync(0xffffffffu, mine, k);
                if (lane == 0 && ok) {
                    const uint32_t it = c0 + k, s = it % n_stages, use = it / n_stages;
                    if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1u)) {
                        report(p.st, OPURE_ERR_DEVICE_TIMEOUT, 12, blockIdx.x);
                        ok = false;
                    } else if (page < 0 || uint32_t(page) >= p.kv.n_pages) {
                        report(p.st, OPURE_ERR_DEVICE_BOUNDS, 11, uint32_t(page));
                        stage_ok[s] = 0;
                        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(&full[s])) : "memory");
                        ++issued;
                    } else {
                        stage_ok[s] = 1;
                        const __half *kp = pool + (size_t(page) * 2 * n_kv + g) * page_elems;
                        uint8_t *dst = stage_mem + size_t(s) * 2 * page_bytes;
                        // Only the page's rows below t_end (a prefix of the K and V blocks):
                        // a sequence's last page is usually partly filled.
                        const uint32_t rows = min(P, t_end - (pg_begin + it) * P);
                        const uint32_t bytes = rows * HD * 2;
                        mbar_expect_tx(&full[s], 2 * bytes);
                        bulk_load_keep(dst, kp, bytes, &full[s]);
                        bulk_load_keep(dst + page_bytes, kp + size_t(n_kv) * page_elems, bytes, &full[s]);
                        ++issued;
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
                if (!ok) break;
            }
        }
        // No copy may still be landing in shared memory when the CTA exits.
        if (lane == 0) {
            // The last use of each slot is the only phase that can still be pending.
            for (uint32_t s = 0; s < n_stages && s < issued; ++s) {
                const uint32_t last = issued - 1 - ((issued - 1 - s) % n_stages);  // last iteration on slot s
                (void)mbar_wait(&full[s], (last / n_stages) & 1u);
            }
        }
    } else {
        float qv[G][E];
        load_q_slice<HD, G>(p.q + size_t(entry) * p.n_heads * HD, g, p.scale_log2, qv);
        const uint32_t rounds = P / TPW;  // token rounds per page
        for (uint32_t it = 0; it < n_pg; ++it) {
            const uint32_t s = it % n_stages;
            if (!mbar_wait(&full[s], (it / n_stages) & 1u)) {
                if (lane == 0) report(p.st, OPURE_ERR_DEVICE_TIMEOUT, 13, blockIdx.x);
                break;
            }
            const bool page_ok = stage_ok[s] != 0;
            const __half *ks = reinterpret_cast<const __half *>(stage_mem + size_t(s) * 2 * page_bytes);
            const __half *vs = ks + page_elems;
            const uint32_t tok0 = (pg_begin + it) * P;
            // Pages wholly inside the split skip the per-row range checks.
            if (page_ok && tok0 >= t_begin && tok0 + P <= t_end)
                consume_page<HD, G, R, false>(st, qv, ks, vs, warp, rounds, tok0, t_begin, t_end);
            else
                consume_page<HD, G, R, true>(st, qv, ks, vs, warp, rounds, tok0, page_ok ? t_begin : t_end, t_end);
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(&empty[s])) : "memory");
        }
        merge_lane_groups<HD, G>(st);
        store_warp_state<HD, G, kWarps>(st, ws, warp);
    }
    __syncthreads();

    const uint32_t n_splits = p.n_splits;
    if (n_splits == 1) {
        // One split: the CTA's merged state is the result (the split merge below would
        // multiply it by exp2(0) = 1), so no partials, no ticket.
        for (uint32_t idx = threadIdx.x; idx < uint32_t(G) * HD; idx += blockDim.x) {
            const uint32_t h = idx / HD, d = idx % HD;
            float a, mn, ls;
            merge_warps<HD, G, kWarps>(ws, h, d, a, mn, ls);
            store_out<HD, PK>(p, entry, (g * G + h) * HD + d, a / fmaxf(ls, 1e-30f));
        }
        if constexpr (PK) asm volatile("fence.proxy.async.global;" ::: "memory");  // read by TMA next
        return;
    }
    float *part = p.partials + (size_t(eg) * n_splits + split) * G * (HD + 2);
    for (uint32_t idx = threadIdx.x; idx < uint32_t(G) * HD; idx += blockDim.x) {
        const uint32_t h = idx / HD, d = idx % HD;
        float a, mn, ls;
        merge_warps<HD, G, kWarps>(ws, h, d, a, mn, ls);
        part[h * (HD + 2) + d] = a;
        if (d == 0) {
            part[h * (HD + 2) + HD] = mn;
            part[h * (HD + 2) + HD + 1] = ls;
        }
    }
    __threadfence();
    __syncthreads();
    __shared__ uint32_t ticket;
    if (threadIdx.x == 0) ticket = atomicAdd(p.counters + eg, 1u);
    __syncthreads();
    if (ticket != n_splits - 1) return;

    __threadfence();
    const float *parts = p.partials + size_t(eg) * n_splits * G * (HD + 2);
    for (uint32_t idx = threadIdx.x; idx < uint32_t(G) * HD; idx += blockDim.x) {
        const uint32_t h = idx / HD, d = idx % HD;
        float mn = -INFINITY;
#pragma unroll 8  // independent loads: several splits in flight
        for (uint32_t sp = 0; sp < n_splits; ++sp)
            mn = fmaxf(mn, __ldcg(parts + (size_t(sp) * G + h) * (HD + 2) + HD));
        float a = 0.f, lsum = 0.f;
#pragma unroll 8  // independent loads: several splits in flight
        for (uint32_t sp = 0; sp < n_splits; ++sp) {
            const float *pp = parts + (size_t(sp) * G + h) * (HD + 2);
            const float ms = __ldcg(pp + HD);
            const float f = (mn == -INFINITY || ms == -INFINITY) ? 0.f : fast_exp2(ms - mn);
            a += __ldcg(pp + d) * f;
            lsum += __ldcg(pp + HD + 1) * f;
        }
        store_out<HD, PK>(p, entry, (g * G + h) * HD + d, a / fmaxf(lsum, 1e-30f));
    }
    if constexpr (PK) asm volatile("fence.proxy.async.global;" ::: "memory");  // read by TMA next
    if (threadIdx.x == 0) p.counters[eg] = 0u;
}

using AttnKernel = void (*)(AttnParams);

template <int HD>
AttnKernel pick_g(uint32_t G) {
    switch (G) {
        case 1: return attn_kernel<HD, 1>;
        case 2: return attn_kernel<HD, 2>;
        case 3: return attn_kernel<HD, 3>;
        case 4: return attn_kernel<HD, 4>;
    }
    return nullptr;
}

template <int HD, bool PK>
void (*pick_tma_g(uint32_t G))(AttnP<PK>) {
    switch (G) {
        case 1: return attn_tma_kernel<HD, 1, PK>;
        case 2: return attn_tma_kernel<HD, 2, PK>;
        case 3: return attn_tma_kernel<HD, 3, PK>;
        case 4: return attn_tma_kernel<HD, 4, PK>;
    }
    return nullptr;
}

// Head dims served by the TMA-staged kernel.
bool tma_path(uint32_t hd) { return hd == 64 || hd == 128; }

AttnKernel pick(uint32_t hd, uint32_t G) {
    switch (hd) {
        case 32: return pick_g<32>(G);
        case 64: return pick_g<64>(G);
        case 96: return pick_g<96>(G);
        case 128: return pick_g<128>(G);
        case 160: return pick_g<160>(G);
        case 192: return pick_g<192>(G);
        case 224: return pick_g<224>(G);
        case 256: return pick_g<256>(G);
    }
    return nullptr;
}

uint32_t cta_tokens(uint32_t hd) {
    switch (hd) {
        case 32: return cta_block_tokens<32>();
        case 64: return cta_block_tokens<64>();
        case 96: return cta_block_tokens<96>();
        case 128: return cta_block_tokens<128>();
        case 160: return cta_block_tokens<160>();
        case 192: return cta_block_tokens<192>();
        case 224: return cta_block_tokens<224>();
        case 256: return cta_block_tokens<256>();
    }
    return 0;
}

// Keys per split: a whole number of CTA blocks, with enough splits to put several
// CTAs on every SM (sm_count 148 on B200) without splitting below one block.
uint32_t choose_split(uint32_t entries, uint32_t n_kv, uint32_t hd, uint32_t max_ctx,
                      uint32_t requested, int sm_count) {
    if (tma_path(hd)) {
        // Splits are whole multiples of 128 tokens, so pages of 16..128 tokens never straddle
        // two splits. Enough splits for about one wave of three CTAs per SM (at most 32: the
        // last CTA of each (entry, kv head) merges every split). When that leaves fewer than
        // three waves and splits of at most 3072 tokens would give three or more, those are
        // taken instead: many mid-sized CTAs even out the SMs' shares of a large batch, while
        // a grid between one and three waves loses more to its partial last wave than it
        // gains. Measured on B200 over split sizes 256..16384 for 1, 8 and 64 sequences at
        // 8192 and 32768 tokens, and on the 1.7B model's 2048 (sequence, kv head) pairs.
        const uint32_t unit = 128;
        if (requested) return ((requested + unit - 1) / unit) * unit;
        const uint64_t pairs = uint64_t(entries) * n_kv;
        const uint64_t wave = uint64_t(sm_count > 0 ? sm_count : 148) * 3;
        uint64_t want = std::min<uint64_t>(32, std::max<uint64_t>(1, (wave + pairs / 2) / pairs));
        const uint64_t by_len = (uint64_t(max_ctx) + 3071) / 3072;
        if (pairs * want < 3 * wave && pairs * by_len >= 3 * wave) want = by_len;
        want = std::min<uint64_t>(want, std::max<uint64_t>(1, max_ctx / unit));
        const uint64_t per = (uint64_t(std::max(max_ctx, 1u)) + want - 1) / want;
        return uint32_t(std::max<uint64_t>(unit, ((per + unit - 1) / unit) * unit));
    }
    const uint32_t unit = cta_tokens(hd);
    if (requested) return ((requested + unit - 1) / unit) * unit;
    // About four CTAs per SM, but no split shorter than 128 tokens: a short context is one
    // CTA's work, and each split adds a combine.
    const uint64_t pairs = uint64_t(entries) * n_kv;
    const uint64_t target = uint64_t(sm_count > 0 ? sm_count : 148) * 4;
    const uint64_t want_splits = std::max<uint64_t>(
        1, std::min<uint64_t>((target + pairs - 1) / pairs, std::max<uint64_t>(1, max_ctx / 128)));
    const uint64_t per = (uint64_t(std::max(max_ctx, 1u)) + want_splits - 1) / want_splits;
    return uint32_t(std::max<uint64_t>(unit, ((per + unit - 1) / unit) * unit));
}

opure_status launch_attention(opure_ctx *ctx, const AttnParams &p, uint32_t hd, uint32_t G, uint32_t pairs,
                              uint32_t n_splits, __half *out_packed = nullptr, uint32_t pk_npad = 0) {
    if (tma_path(hd)) {
        const uint32_t page_bytes = p.kv.page_size * hd * 2;
        const size_t smem = size_t(stage_count(2 * page_bytes)) * 2 * page_bytes;
        // Always: the dynamic stages plus the kernel's static shared memory may pass the
        // default 48 KB per-block limit even when the stages alone do not.
        auto go = [&](auto k, const auto &params) -> opure_status {
            if (!k) return OPURE_ERR_UNSUPPORTED;
            const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
            if (e != cudaSuccess) return cuda_status(e);
            return launch(ctx, k, dim3(pairs, n_splits), dim3((kWarps + 1) * 32), smem, true, params);
        };
        if (out_packed) {
            AttnPackedParams pp;
            static_cast<AttnParams &>(pp) = p;
            pp.out_packed = out_packed;
            pp.pk_npad = pk_npad;
            return go(hd == 64 ? pick_tma_g<64, true>(G) : pick_tma_g<128, true>(G), pp);
        }
        return go(hd == 64 ? pick_tma_g<64, false>(G) : pick_tma_g<128, false>(G), p);
    }
    AttnKernel k = pick(hd, G);
    if (!k || out_packed) return OPURE_ERR_UNSUPPORTED;  // packed output: head_dim 64 / 128 only
    return launch(ctx, k, dim3(pairs, n_splits), dim3(kWarps * 32), 0, true, p);
}

size_t scratch_layout(uint32_t entries, uint32_t n_kv, uint32_t G, uint32_t hd, uint32_t n_splits,
                      size_t *counters_off) {
    const size_t part = size_t(entries) * n_kv * n_splits * G * (hd + 2) * sizeof(float);
    const size_t off = (part + 255) & ~size_t(255);
    if (counters_off) *counters_off = off;
    return off + size_t(entries) * n_kv * sizeof(uint32_t);
}

}  // namespace
}  // namespace opure

using namespace opure;

extern "C" size_t opure_attention_scratch_bytes(uint32_t n, uint32_t n_q, uint32_t n_heads,
                                                uint32_t n_kv, uint32_t hd, uint32_t max_ctx,
                                                uint32_t split_tokens) {
    if (!n || !n_q || !n_kv || !hd || n_heads % n_kv || !cta_tokens(hd)) return 0;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint32_t entries = n * n_q;
    const uint32_t st = choose_split(entries, n_kv, hd, max_ctx, split_tokens, sms);
    const uint32_t n_splits = std::max(1u, (max_ctx + st - 1) / st);
    return scratch_layout(entries, n_kv, n_heads / n_kv, hd, n_splits, nullptr);
}

extern "C" opure_status opure_attention(opure_ctx *ctx, const opure_attn_args *a) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!a || !a->q || !a->out || !a->seq || !a->seq_len || !a->scratch) return OPURE_ERR_INVALID_ARG;
    const opure_kv_layout &kv = a->kv;
    if (!kv.pool || !kv.page_table || !kv.n_kv || !kv.page_size || !kv.max_pages || kv.ring > kv.max_pages)
        return OPURE_ERR_INVALID_ARG;
    if (a->n_heads % kv.n_kv) return OPURE_ERR_INVALID_ARG;
    if (a->n == 0 || a->n_q == 0) return OPURE_OK;
    const uint32_t G = a->n_heads / kv.n_kv;
    if (!pick(kv.head_dim, G)) return OPURE_ERR_UNSUPPORTED;
    if (reinterpret_cast<uintptr_t>(kv.pool) % 16) return OPURE_ERR_UNSUPPORTED;
    const uint32_t entries = a->n * a->n_q;
    const uint32_t st = choose_split(entries, kv.n_kv, kv.head_dim, a->max_ctx, a->split_tokens,
                                     ctx->sm_count);
    const uint32_t n_splits = std::max(1u, (a->max_ctx + st - 1) / st);
    size_t counters_off = 0;
    const size_t need = scratch_layout(entries, kv.n_kv, G, kv.head_dim, n_splits, &counters_off);
    if (a->scratch_bytes < need || (reinterpret_cast<uintptr_t>(a->scratch) % 16))
        return OPURE_ERR_INVALID_ARG;
    if (uint64_t(entries) * kv.n_kv > 0x7fffffffu || n_splits > 65535) return OPURE_ERR_UNSUPPORTED;

    AttnParams p{};
    p.q = a->q;
    p.out = a->out;
    p.seq = a->seq;
    p.seq_len = a->seq_len;
    p.n = a->n;
    p.n_q = a->n_q;
    p.n_heads = a->n_heads;
    p.scale_log2 = a->scale * 1.4426950408889634f;
    p.split_tokens = st;
    p.n_splits = n_splits;
    p.partials = static_cast<float *>(a->scratch);
    p.counters = reinterpret_cast<uint32_t *>(static_cast<char *>(a->scratch) + counters_off);
    p.kv = kv;
    p.st = ctx->status;
    return launch_attention(ctx, p, kv.head_dim, G, entries * kv.n_kv, n_splits,
                            reinterpret_cast<__half *>(a->out_packed), (entries + 15) & ~15u);
}

// ---- Allocation-free variant (opure_attention_static) ---------------------------------
// For callers that may not allocate device memory (a plugin whose host owns the GPU memory
// budget, or a real-time loop that cannot afford cudaMalloc's device synchronisation): the
// split partials and counters live in this fixed array instead of caller scratch. Every
// GPU that loads the library holds it until the process exits.
static __device__ __align__(256) unsigned char g_attn_static_scratch[OPURE_ATTN_STATIC_SCRATCH_BYTES];

#include <mutex>

namespace {
// Device address of g_attn_static_scratch per device, looked up once. In host code the
// array's name is only a host-side stand-in, never a device pointer.
constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
void *g_static_ptr[kMaxDevices] = {};

opure_status static_scratch(int device, void **out) {
    if (device < 0 || device >= kMaxDevices) return OPURE_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (!g_static_ptr[device]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_static_scratch);  // device is current
        if (e != cudaSuccess || !p) return cuda_status(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
        g_static_ptr[device] = p;
    }
    *out = g_static_ptr[device];
    return OPURE_OK;
}
}  // namespace

extern "C" opure_status opure_attention_static(opure_ctx *ctx, const opure_attn_args *a) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!a || !a->q || !a->out || !a->seq || !a->seq_len) return OPURE_ERR_INVALID_ARG;
    const opure_kv_layout &kv = a->kv;
    if (!kv.pool || !kv.page_table || !kv.n_kv || !kv.page_size || !kv.max_pages || kv.ring > kv.max_pages)
        return OPURE_ERR_INVALID_ARG;
    if (a->n_heads % kv.n_kv) return OPURE_ERR_INVALID_ARG;
    if (a->n == 0 || a->n_q == 0) return OPURE_OK;
    const uint32_t G = a->n_heads / kv.n_kv;
    if (!pick(kv.head_dim, G)) return OPURE_ERR_UNSUPPORTED;
    if (reinterpret_cast<uintptr_t>(kv.pool) % 16) return OPURE_ERR_UNSUPPORTED;
    const uint32_t entries = a->n * a->n_q;
    const uint32_t st = choose_split(entries, kv.n_kv, kv.head_dim, a->max_ctx, a->split_tokens,
                                     ctx->sm_count);
    const uint32_t n_splits = std::max(1u, (a->max_ctx + st - 1) / st);
    size_t counters_off = 0;
    const size_t need = scratch_layout(entries, kv.n_kv, G, kv.head_dim, n_splits, &counters_off);
    if (need > OPURE_ATTN_STATIC_SCRATCH_BYTES) return OPURE_ERR_UNSUPPORTED;
    if (uint64_t(entries) * kv.n_kv > 0x7fffffffu || n_splits > 65535) return OPURE_ERR_UNSUPPORTED;
    void *scratch = nullptr;
    if ((s = static_scratch(ctx->device, &scratch))) return s;
    uint32_t *counters = reinterpret_cast<uint32_t *>(static_cast<char *>(scratch) + counters_off);
    // The buffer keeps the previous call's bytes: the split counters must start at zero.
    OPURE_CUDA_TRY(cudaMemsetAsync(counters, 0, size_t(entries) * kv.n_kv * sizeof(uint32_t), ctx->stream));

    AttnParams p{};
    p.q = a->q;
    p.out = a->out;
    p.seq = a->seq;
    p.seq_len = a->seq_len;
    p.n = a->n;
    p.n_q = a->n_q;
    p.n_heads = a->n_heads;
    p.scale_log2 = a->scale * 1.4426950408889634f;
    p.split_tokens = st;
    p.n_splits = n_splits;
    p.partials = static_cast<float *>(scratch);
    p.counters = counters;
    p.kv = kv;
    p.st = ctx->status;
    return launch_attention(ctx, p, kv.head_dim, G, entries * kv.n_kv, n_splits);
}
