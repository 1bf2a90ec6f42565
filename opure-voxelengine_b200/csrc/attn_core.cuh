// attn_core.cuh -- the paged flash-decode inner loop, shared by the split-K attention
// kernel (attention.cu) and the fused attention + o_proj decode kernel (decode.cu).
//
// Lane mapping: a token's head_dim is covered by LPT lanes, each owning CH 16-byte chunks
// (8 fp16 each); for hd 64 eight lanes read one 128-byte K row and one warp load
// instruction covers four consecutive tokens (512 contiguous bytes of a page block).
// Every lane keeps its own online-softmax state (running max m, sum l, output acc) for
// the tokens of its lane group, processed in blocks of R tokens per group so the
// rescale happens once per block. Scores are kept in log2 units (q is pre-scaled by
// scale * log2(e)) and exponentiated with ex2.approx; all softmax arithmetic is fp32.
#pragma once

#include "common.cuh"

namespace opure {

template <int HD>
struct AttnShape {
    static constexpr int kChunks = HD / 8;  // 16-byte chunks per row
    static constexpr int LPT = (kChunks % 32 == 0) ? 32
                             : (kChunks % 16 == 0) ? 16
                             : (kChunks % 8 == 0) ? 8 : 4;  // lanes per token
    static constexpr int CH = kChunks / LPT;                // chunks per lane
    static constexpr int E = CH * 8;                        // dims owned by a lane
    static constexpr int TPW = 32 / LPT;                    // tokens per warp round
    // Rounds per block: 8 with one chunk per lane (hd 32/64/128/256); fewer for the head
    // dims needing several chunks per lane, to bound registers.
    static constexpr int R = CH == 1 ? 8 : (CH <= 3 ? 2 : 1);
    static constexpr int TB = TPW * R;                      // tokens per warp block
    static_assert(kChunks % LPT == 0 && HD % 8 == 0, "head_dim must be a multiple of 8");
};

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int HD, int G>
struct AttnState {
    static constexpr int E = AttnShape<HD>::E;
    float m[G], l[G], acc[G][E];
    __device__ __forceinline__ void init() {
#pragma unroll
        for (int h = 0; h < G; ++h) {
            m[h] = -INFINITY;
            l[h] = 0.f;
#pragma unroll
            for (int e = 0; e < E; ++e) acc[h][e] = 0.f;
        }
    }
};

// Where one sequence's keys for one kv head live.
struct KvView {
    const __half *pool;        // layer pool
    const int32_t *pt;         // this sequence's page-table row
    uint32_t max_pages, n_pages, page_size, n_kv, g;
    bool ok;                   // false: the sequence index was invalid
    uint32_t ring;             // sliding window: table entries used as a ring (0: off)
};


// Rows [0, n) of one sequence's keys and values for one kv head, copied into shared
// memory ([n][HD] each); tokens from n on are read from the pool.
struct KvStage {
    const __half *k, *v;
    uint32_t n;
};

// This lane's slice of the G query rows of kv head g, pre-scaled by scale*log2(e).
template <int HD, int G>
__device__ __forceinline__ void load_q_slice(const float *q_heads /* [n_heads][HD] */, uint32_t g,
                                             float scale_log2, float (&qv)[G][AttnShape<HD>::E]) {
    using S = AttnShape<HD>;
    const uint32_t sub = (threadIdx.x & 31u) % S::LPT;
#pragma unroll
    for (int h = 0; h < G; ++h) {
        const float *qr = q_heads + (size_t(g) * G + h) * HD + sub * S::E;
#pragma unroll
        for (int e = 0; e < S::E; ++e) qv[h][e] = qr[e] * scale_log2;
    }
}

// Accumulates keys [t_begin, t_end) into the lane state. The calling warp processes
// blocks base = t_begin + warp_idx*TB, advancing by warp_count*TB; STRIDED instead
// interleaves the warps round by round (round r of warp w covers tokens base +
// (r*warp_count + w)*TPW ..), so a context shorter than warp_count*TB still spreads over
// every warp. Rounds past t_end are skipped (warp-uniform). COHERENT reads K/V through
// L2 (for caches written earlier in the same kernel). STAGED reads tokens below stg.n
// from shared memory. RB rounds per softmax block (default AttnShape's R): fewer keep
// fewer K/V rows in registers, for callers whose keys mostly come from shared memory.
template <int HD, int G, bool COHERENT = false, bool STRIDED = false, bool STAGED = false,
          int RB = AttnShape<HD>::R>
__device__ __forceinline__ void attend_range(AttnState<HD, G> &st, const float (&qv)[G][AttnShape<HD>::E],
                                             const KvView &kv, uint32_t t_begin, uint32_t t_end,
                                             uint32_t warp_idx, uint32_t warp_count,
                                             DeviceStatus *status, const KvStage &stg = KvStage{nullptr, nullptr, 0}) {
    using S = AttnShape<HD>;
    constexpr int LPT = S::LPT, CH = S::CH, TPW = S::TPW, R = RB, E = S::E;
    constexpr uint32_t TB = uint32_t(TPW) * R;  // tokens per warp block
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t grp = lane / LPT, sub = lane % LPT;
    const size_t blk = size_t(kv.page_size) * HD;  // elements per page block

    for (uint32_t base = t_begin + (STRIDED ? 0u : warp_idx * TB); base < t_end; base += warp_count * TB) {
        uint4 kr[R][CH], vr[R][CH];
        bool valid[R], live[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const uint32_t t0 = STRIDED ? base + (r * warp_count + warp_idx) * TPW : base + r * TPW;
            live[r] = t0 < t_end;  // the same for every lane of the warp
            const uint32_t t = t0 + grp;
            valid[r] = t < t_end && kv.ok;
            const __half *kp = nullptr;
            if (STAGED && valid[r] && t < stg.n) {
                const size_t o = size_t(t) * HD + sub * E;
#pragma unroll
                for (int c = 0; c < CH; ++c) {
                    kr[r][c] = lds128(stg.k + o + c * 8);
                    vr[r][c] = lds128(stg.v + o + c * 8);
                }
                continue;
            }
            if (valid[r]) {
                const uint32_t lp = ring_slot(t / kv.page_size, kv.ring);
                const int32_t page = lp < kv.max_pages ? kv.pt[lp] : -1;
                if (page < 0 || uint32_t(page) >= kv.n_pages) {
                    report(status, OPURE_ERR_DEVICE_BOUNDS, 10, uint32_t(page));
                    valid[r] = false;
                } else {
                    kp = kv.pool + (size_t(page) * 2 * kv.n_kv + kv.g) * blk +
                         size_t(t % kv.page_size) * HD + sub * E;
                }
            }
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                if (COHERENT) {
                    kr[r][c] = valid[r] ? ldcg_v4(kp + c * 8) : make_uint4(0, 0, 0, 0);
                    vr[r][c] = valid[r] ? ldcg_v4(kp + size_t(kv.n_kv) * blk + c * 8) : make_uint4(0, 0, 0, 0);
                } else {
                    kr[r][c] = valid[r] ? ldg_stream(kp + c * 8) : make_uint4(0, 0, 0, 0);
                    vr[r][c] = valid[r] ? ldg_stream(kp + size_t(kv.n_kv) * blk + c * 8) : make_uint4(0, 0, 0, 0);
                }
            }
        }
        float s[R][G];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            if (!live[r]) {
#pragma unroll
                for (int h = 0; h < G; ++h) s[r][h] = -INFINITY;
                continue;
            }
            float kf[E];
#pragma unroll
            for (int c = 0; c < CH; ++c) unpack8(kr[r][c], kf + 8 * c);
#pragma unroll
            for (int h = 0; h < G; ++h) {
                float d = 0.f;
#pragma unroll
                for (int e = 0; e < E; ++e) d = fmaf(qv[h][e], kf[e], d);
#pragma unroll
                for (int o = LPT / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
                s[r][h] = valid[r] ? d : -INFINITY;
            }
        }
#pragma unroll
        for (int h = 0; h < G; ++h) {
            float mb = s[0][h];
#pragma unroll
            for (int r = 1; r < R; ++r) mb = fmaxf(mb, s[r][h]);
            const float mn = fmaxf(st.m[h], mb);
            if (mn == -INFINITY) continue;  // nothing valid seen yet
            const float corr = fast_exp2(st.m[h] - mn);  // exp2(-inf) = 0 on the first block
            st.l[h] *= corr;
#pragma unroll
            for (int e = 0; e < E; ++e) st.acc[h][e] *= corr;
            st.m[h] = mn;
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            if (!live[r]) continue;
            float vf[E];
#pragma unroll
            for (int c = 0; c < CH; ++c) unpack8(vr[r][c], vf + 8 * c);
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const float pr = valid[r] ? fast_exp2(s[r][h] - st.m[h]) : 0.f;
                st.l[h] += pr;
#pragma unroll
                for (int e = 0; e < E; ++e) st.acc[h][e] = fmaf(pr, vf[e], st.acc[h][e]);
            }
        }
    }
}

// Merges the lane groups of a warp: afterwards every group holds the warp's state.
template <int HD, int G>
__device__ __forceinline__ void merge_lane_groups(AttnState<HD, G> &st) {
    using S = AttnShape<HD>;
#pragma unroll
    for (int o = S::LPT; o < 32; o <<= 1) {
#pragma unroll
        for (int h = 0; h < G; ++h) {
            const float mo = __shfl_xor_sync(0xffffffffu, st.m[h], o);
            const float lo = __shfl_xor_sync(0xffffffffu, st.l[h], o);
            const float mn = fmaxf(st.m[h], mo);
            const float a = mn == -INFINITY ? 0.f : fast_exp2(st.m[h] - mn);
            const float b = mn == -INFINITY ? 0.f : fast_exp2(mo - mn);
            st.l[h] = st.l[h] * a + lo * b;
#pragma unroll
            for (int e = 0; e < S::E; ++e) {
                const float ao = __shfl_xor_sync(0xffffffffu, st.acc[h][e], o);
                st.acc[h][e] = st.acc[h][e] * a + ao * b;
            }
            st.m[h] = mn;
        }
    }
}

// Shared-memory image of one state per warp.
template <int HD, int G, int W>
struct WarpStates {
    float m[W][G], l[W][G], acc[W][G][HD];
};

template <int HD, int G, int W>
__device__ __forceinline__ void store_warp_state(const AttnState<HD, G> &st, WarpStates<HD, G, W> &ws,
                                                 uint32_t warp) {
    using S = AttnShape<HD>;
    const uint32_t lane = threadIdx.x & 31u;
    if (lane / S::LPT != 0) return;
    const uint32_t sub = lane % S::LPT;
#pragma unroll
    for (int h = 0; h < G; ++h) {
        if (sub == 0) {
            ws.m[warp][h] = st.m[h];
            ws.l[warp][h] = st.l[h];
        }
#pragma unroll
        for (int e = 0; e < S::E; ++e) ws.acc[warp][h][sub * S::E + e] = st.acc[h][e];
    }
}

// Merged (unnormalised acc, m, l) of the W warp states for head h, dim d.
template <int HD, int G, int W>
__device__ __forceinline__ void merge_warps(const WarpStates<HD, G, W> &ws, uint32_t h, uint32_t d,
                                            float &acc, float &m, float &l) {
    float mn = -INFINITY;
#pragma unroll
    for (int w = 0; w < W; ++w) mn = fmaxf(mn, ws.m[w][h]);
    float a = 0.f, ls = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) {
        const float f = mn == -INFINITY ? 0.f : fast_exp2(ws.m[w][h] - mn);
        a += ws.acc[w][h][d] * f;
        ls += ws.l[w][h] * f;
    }
    acc = a;
    m = mn;
    l = ls;
}

}  // namespace opure
