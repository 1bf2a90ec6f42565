// sample.cu -- token sampling (temperature, top-k, top-p, repetition penalty) and the
// on-device logit statistics of the metrics layer.
//
// The reference only declares the sampling interface: GenerationConfig carries
// temperature, top_p, top_k and repetition_penalty (src/proto/opure.proto:35-46),
// EngineOptions.temperature exists but is never read (src/engine/Opure_VoxelEngine.h:64),
// and Generate is greedy. The rules implemented here are the common ones:
//  - repetition penalty (Keskar et al. 2019, CTRL): a logit l of a token that occurs in
//    the sequence's history becomes l / r when l > 0, else l * r (fp32 arithmetic);
//  - temperature T > 0 divides the (penalised) logits; T <= 0 (or top_k == 1) is greedy:
//    the lowest index among the largest logits;
//  - top-k keeps the k largest logits, ties broken towards the lower index;
//  - top-p (nucleus, Holtzman et al. 2020) keeps, in the same order, the shortest prefix
//    whose probability mass reaches top_p of the mass left by top-k;
//  - the draw is inverse-CDF in index order over the kept tokens.
// Probability masses are exact integers: w_i = exp(l_i / T - max) in double, rounded to
// nearest in units of 2^-40 (a token below 2^-41 of the most likely one has mass 0 and is
// never drawn), summed in uint64. Every comparison (top-p cut-off, draw threshold) is then
// integer arithmetic, so the decisions do not depend on summation order.
//
// Logit statistics follow VoxelEngine::RefreshLogitStats (Opure_VoxelEngine.cpp:832-876):
// L2 norm sqrt(sum l^2) in double; softmax entropy in nats with the fp32 max shift
// exp(double(l - max)), accumulated in double.
#include "ctx.cuh"

namespace opure {
namespace {

constexpr int kThreads = 1024;
constexpr uint32_t kMaxVocab = 1u << 18;  // penalty bitmap: 32 KB of shared memory
constexpr double kMassUnit = 1099511627776.0;  // 2^40

template <typename T>
__device__ T block_sum(T v, T *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : T(0);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const T r = red[0];
    __syncthreads();
    return r;
}

__device__ unsigned long long block_max_key(unsigned long long v, unsigned long long *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xffffffffu, v, o);
        v = t > v ? t : v;
    }
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0ull;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long t = __shfl_xor_sync(0xffffffffu, v, o);
            v = t > v ? t : v;
        }
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const unsigned long long r = red[0];
    __syncthreads();
    return r;
}

constexpr uint32_t kHistBins = 4096;  // top-k pre-select: the keys' leading 12 bits
constexpr uint32_t kCand = 4096;      // candidate keys kept in shared memory
constexpr uint32_t kKeptMax = 1024;   // kept tokens drawn from the candidate list

struct SampleShared {
    uint32_t bits[kMaxVocab / 32];      // tokens in the history (repetition penalty)
    unsigned long long hist[256];       // radix-select bins
    unsigned long long red[32];
    unsigned long long scan[64 + kThreads];  // warp totals, warp offsets, per-thread offsets (draw)
    uint32_t pick;
    uint32_t digit;
    uint32_t n_cand, n_kept;
    uint32_t hist12[kHistBins];         // top-k pre-select histogram
    unsigned long long cand[kCand];     // keys at or above the pre-selected bin
    unsigned long long cmass[kCand];    // their masses (0 below the top-k floor)
    unsigned long long kept[kKeptMax];  // the kept keys, then their masses
    unsigned long long kmass[kKeptMax];
};

// Penalised logit of token i.
__device__ __forceinline__ float pen_logit(const float *l, uint32_t i, const SampleShared &sm, bool pen, float r) {
    float v = l[i];
    if (pen && (sm.bits[i >> 5] >> (i & 31)) & 1u) v = v > 0.f ? v / r : v * r;
    return v;
}

// The key at which the measure of {key >= k}, accumulated from the largest key down,
// first reaches `target`: an 8-bit radix select over the 64-bit keys (unique: value bits,
// then ~index). measure(i, key) >= 0; keys below `floor_key` count nothing. Returns
// floor_key when the total measure is below target.
template <class KeyF, class MeasureF>
__device__ unsigned long long radix_select(uint32_t n, unsigned long long floor_key, unsigned long long target,
                                           KeyF keyf, MeasureF measf, SampleShared &sm) {
    unsigned long long prefix = 0ull, above = 0ull;
    for (int shift = 56; shift >= 0; shift -= 8) {
        const unsigned long long hi_mask = shift == 56 ? 0ull : ~0ull << (shift + 8);
        for (uint32_t b = threadIdx.x; b < 256; b += blockDim.x) sm.hist[b] = 0ull;
        __syncthreads();
        // Warp-aggregated bins: one shared atomic per distinct bin of a warp's 32 keys
        // (most keys of a row share their leading bytes, so per-key atomics would queue).
        const uint32_t lane = threadIdx.x & 31u;
        for (uint32_t base = threadIdx.x - lane; base < n; base += blockDim.x) {
            const uint32_t i = base + lane;
            uint32_t bin = 0;
            unsigned long long m = 0ull;
            if (i < n) {
                const unsigned long long k = keyf(i);
                if (k >= floor_key && (k & hi_mask) == prefix) {
                    m = measf(i, k);
                    bin = uint32_t(k >> shift) & 255u;
                }
            }
            uint32_t rem = __ballot_sync(0xffffffffu, m != 0ull);
            while (rem) {
                const uint32_t lead = __ffs(rem) - 1;
                const uint32_t b = __shfl_sync(0xffffffffu, bin, lead);
                const bool mine = m != 0ull && bin == b;
                unsigned long long v = mine ? m : 0ull;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if (lane == lead) atomicAdd(&sm.hist[b], v);
                rem &= ~__ballot_sync(0xffffffffu, mine);
            }
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            // Warp 0 scans the bins from the top: lane j owns bins 255-8j .. 248-8j.
            unsigned long long h[8], own = 0ull;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                h[q] = sm.hist[255 - 8 * lane - q];
                own += h[q];
            }
            unsigned long long incl = own;  // inclusive prefix over lanes 0..lane
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned long long t = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= uint32_t(o)) incl += t;
            }
            unsigned long long cum = above + incl - own;  // measure above this lane's bins
            uint32_t d = 256;
            unsigned long long cum_d = 0ull;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                if (d == 256 && cum + h[q] >= target) {
                    d = 255 - 8 * lane - q;
                    cum_d = cum;
                }
                cum += h[q];
            }
            // The first lane (from the top) whose bins reach the target decides.
            const uint32_t hit = __ballot_sync(0xffffffffu, d != 256);
            if (hit) {
                const uint32_t src = __ffs(hit) - 1;
                d = __shfl_sync(0xffffffffu, d, src);
                cum_d = __shfl_sync(0xffffffffu, cum_d, src);
            }
            if (lane == 0) {
                sm.digit = hit ? d : 256u;
                sm.red[0] = cum_d;
            }
        }
        __syncthreads();
        if (sm.digit == 256) {
            __syncthreads();
            return floor_key;
        }
        prefix |= (unsigned long long)sm.digit << shift;
        above = sm.red[0];
        __syncthreads();
    }
    return prefix;
}

// Top-k pre-select: a histogram of the keys' leading 12 bits finds the bin holding the k-th
// largest key; every key at or above that bin goes to sm.cand. False (nothing usable) when
// the list would overflow.
template <class KeyF>
__device__ bool compact_top_k(uint32_t n, uint32_t k, KeyF keyf, SampleShared &sm) {
    for (uint32_t b = threadIdx.x; b < kHistBins; b += blockDim.x) sm.hist12[b] = 0u;
    if (threadIdx.x == 0) sm.n_cand = 0u;
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const unsigned long long key = keyf(i);
        if (key) atomicAdd(&sm.hist12[uint32_t(key >> 52)], 1u);
    }
    __syncthreads();
    // Bins from the top: thread t owns bins 4095-4t .. 4092-4t; block-wide inclusive scan.
    constexpr uint32_t kPer = kHistBins / kThreads;
    uint32_t own = 0u;
#pragma unroll
    for (uint32_t q = 0; q < kPer; ++q) own += sm.hist12[kHistBins - 1 - kPer * threadIdx.x - q];
    const uint32_t lane = threadIdx.x & 31u, wid = threadIdx.x >> 5;
    uint32_t incl = own;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= uint32_t(o)) incl += t;
    }
    if (lane == 31) sm.scan[wid] = incl;
    __syncthreads();
    if (wid == 0) {
        const unsigned long long wt = lane < blockDim.x / 32 ? sm.scan[lane] : 0ull;
        unsigned long long wi = wt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long t = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= uint32_t(o)) wi += t;
        }
        sm.scan[32 + lane] = wi - wt;
    }
    if (threadIdx.x == 0) sm.digit = kHistBins;  // bin of the k-th key (none: fewer keys)
    __syncthreads();
    unsigned long long cum = sm.scan[32 + wid] + incl - own;  // keys above this thread's bins
#pragma unroll
    for (uint32_t q = 0; q < kPer; ++q) {
        const uint32_t b = kHistBins - 1 - kPer * threadIdx.x - q;
        const uint32_t h = sm.hist12[b];
        if (cum < k && cum + h >= k) sm.digit = b;  // exactly one bin crosses
        cum += h;
    }
    __syncthreads();
    if (sm.digit == kHistBins) return false;
    const unsigned long long floor_bin = (unsigned long long)sm.digit << 52;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const unsigned long long key = keyf(i);
        if (key >= floor_bin) {
            const uint32_t slot = atomicAdd(&sm.n_cand, 1u);
            if (slot < kCand) sm.cand[slot] = key;
        }
    }
    __syncthreads();
    return sm.n_cand <= kCand;
}

__global__ void __launch_bounds__(kThreads) sample_filtered_kernel(opure_sample_args a) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    SampleShared &sm = *reinterpret_cast<SampleShared *>(smem_raw);
    grid_dependency_wait();
    grid_dependents_launch();
    const uint32_t row = blockIdx.x, V = a.vocab;
    const float *l = a.logits + size_t(row) * a.stride;
    const bool pen = a.rep_penalty != 1.0f && a.hist != nullptr;

    if (pen) {
        for (uint32_t w = threadIdx.x; w < (V + 31) / 32; w += blockDim.x) sm.bits[w] = 0u;
        __syncthreads();
        const int32_t s = a.seq ? a.seq[row] : int32_t(row);
        const int32_t len = a.hist_len ? a.hist_len[row] : 0;
        if (s >= 0 && len > 0) {
            const int32_t *h = a.hist + size_t(s) * a.max_len;
            for (uint32_t i = threadIdx.x; i < min(uint32_t(len), a.max_len); i += blockDim.x) {
                const int32_t t = h[i];
                if (t >= 0 && uint32_t(t) < V) atomicOr(&sm.bits[t >> 5], 1u << (t & 31));
            }
        }
        __syncthreads();
    }
    const float r = a.rep_penalty;
    auto keyf = [&](uint32_t i) { return argmax_key(pen_logit(l, i, sm, pen, r), i); };

    // Greedy: the largest key.
    unsigned long long best = 0ull;
    for (uint32_t i = threadIdx.x; i < V; i += blockDim.x) {
        const unsigned long long k = keyf(i);
        best = k > best ? k : best;
    }
    best = block_max_key(best, sm.red);
    uint32_t token = best ? argmax_key_index(best) : 0u;

    const bool compact = a.temperature > 0.f && a.top_k > 1 && a.top_k <= kKeptMax && a.top_k < V && best &&
                         compact_top_k(V, a.top_k, keyf, sm);
    if (compact) {
        // Top-k survivors and the keys just below them sit in sm.cand: top-k, top-p and the
        // draw run over that list instead of the whole row.
        const double inv_t = 1.0 / double(a.temperature);
        const double zmax = double(argmax_key_value(best)) * inv_t;
        const uint32_t nc = sm.n_cand;
        auto ckey = [&](uint32_t i) { return sm.cand[i]; };
        const unsigned long long kfloor =
            radix_select(nc, 1ull, a.top_k, ckey, [](uint32_t, unsigned long long) { return 1ull; }, sm);
        unsigned long long z = 0ull;
        for (uint32_t i = threadIdx.x; i < nc; i += blockDim.x) {
            const unsigned long long k = sm.cand[i];
            unsigned long long m = 0ull;
            if (k >= kfloor) {
                const double e = exp(double(argmax_key_value(k)) * inv_t - zmax);
                m = e > 0.0 ? __double2ull_rn(e * kMassUnit) : 0ull;
            }
            sm.cmass[i] = m;
            z += m;
        }
        z = block_sum(z, sm.red);  // (syncs: cmass complete)
        unsigned long long floor_key = kfloor;
        if (a.top_p < 1.0f) {
            const double tgt = ceil(double(a.top_p) * double(z));
            const unsigned long long target = tgt < 1.0 ? 1ull : (unsigned long long)tgt;
            if (target < z)
                floor_key = radix_select(nc, kfloor, target, ckey,
                                         [&](uint32_t i, unsigned long long) { return sm.cmass[i]; }, sm);
        }
        // The kept keys (at most top_k), then the draw in index order: each kept token's
        // running mass is the sum over the kept tokens with a lower index.
        if (threadIdx.x == 0) {
            sm.n_kept = 0;
            sm.pick = 0xffffffffu;
        }
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < nc; i += blockDim.x)
            if (sm.cand[i] >= floor_key) {
                const uint32_t slot = atomicAdd(&sm.n_kept, 1u);
                sm.kept[slot] = sm.cand[i];
                sm.kmass[slot] = sm.cmass[i];
            }
        __syncthreads();
        const uint32_t nk = sm.n_kept;
        unsigned long long tot = 0ull;
        for (uint32_t i = threadIdx.x; i < nk; i += blockDim.x) tot += sm.kmass[i];
        tot = block_sum(tot, sm.red);
        if (tot) {
            unsigned long long thr = (unsigned long long)floor(double(a.u[row]) * double(tot));
            if (thr >= tot) thr = tot - 1;
            for (uint32_t i = threadIdx.x; i < nk; i += blockDim.x) {
                const uint32_t idx = argmax_key_index(sm.kept[i]);
                unsigned long long before = 0ull;
                for (uint32_t j = 0; j < nk; ++j)
                    if (argmax_key_index(sm.kept[j]) < idx) before += sm.kmass[j];
                if (before <= thr && thr < before + sm.kmass[i]) sm.pick = idx;
            }
        }
        __syncthreads();
        if (tot) token = sm.pick;
    } else if (a.temperature > 0.f && a.top_k != 1 && best) {
        const double inv_t = 1.0 / double(a.temperature);
        const double zmax = double(argmax_key_value(best)) * inv_t;
        // top-k: the k-th largest key (count measure).
        unsigned long long kfloor = 1ull;  // every non-NaN logit
        if (a.top_k > 1 && a.top_k < V)
            kfloor = radix_select(V, 1ull, a.top_k, keyf, [](uint32_t, unsigned long long) { return 1ull; }, sm);
        auto mass = [&](uint32_t i, unsigned long long k) -> unsigned long long {
            if (k < kfloor) return 0ull;
            const double e = exp(double(argmax_key_value(k)) * inv_t - zmax);
            return e > 0.0 ? __double2ull_rn(e * kMassUnit) : 0ull;  // NaN (inf - inf): 0
        };
        // top-p: the shortest prefix (in key order) reaching ceil(top_p * Z).
        unsigned long long floor_key = kfloor;
        if (a.top_p < 1.0f) {
            unsigned long long z = 0ull;
            for (uint32_t i = threadIdx.x; i < V; i += blockDim.x) z += mass(i, keyf(i));
            z = block_sum(z, sm.red);
            const double tgt = ceil(double(a.top_p) * double(z));
            const unsigned long long target = tgt < 1.0 ? 1ull : (unsigned long long)tgt;
            if (target < z) floor_key = radix_select(V, kfloor, target, keyf, mass, sm);
        }
        // Inverse-CDF draw in index order over {key >= floor_key}: the smallest i whose
        // running mass exceeds floor(u * Z).
        const uint32_t seg = (V + blockDim.x - 1) / blockDim.x;
        const uint32_t b0 = threadIdx.x * seg, b1 = min(V, b0 + seg);
        auto kept_mass = [&](uint32_t i) {
            const unsigned long long k = keyf(i);
            return k >= floor_key ? mass(i, k) : 0ull;
        };
        unsigned long long local = 0ull;
        for (uint32_t i = b0; i < b1; ++i) local += kept_mass(i);
        // Exclusive scan of the segment masses in thread order: within warps, then over
        // the warp totals.
        const uint32_t lane = threadIdx.x & 31u, wid = threadIdx.x >> 5;
        unsigned long long incl = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= uint32_t(o)) incl += t;
        }
        if (lane == 31) sm.scan[wid] = incl;
        if (threadIdx.x == 0) sm.pick = 0xffffffffu;
        __syncthreads();
        if (wid == 0) {
            const unsigned long long wt = lane < blockDim.x / 32 ? sm.scan[lane] : 0ull;
            unsigned long long wi = wt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned long long t = __shfl_up_sync(0xffffffffu, wi, o);
                if (lane >= uint32_t(o)) wi += t;
            }
            sm.scan[32 + lane] = wi - wt;  // mass of the warps before this one
            if (lane == 31) sm.red[0] = wi;
        }
        __syncthreads();
        sm.scan[64 + threadIdx.x] = sm.scan[32 + wid] + incl - local;
        __syncthreads();
        const unsigned long long total = sm.red[0];
        const double uu = double(a.u[row]);
        unsigned long long thr = (unsigned long long)floor(uu * double(total));
        if (thr >= total) thr = total - 1;  // u in [0, 1): only reachable through rounding
        unsigned long long c = sm.scan[64 + threadIdx.x];
        if (total && c <= thr && c + local > thr) {
            for (uint32_t i = b0; i < b1; ++i) {
                c += kept_mass(i);
                if (c > thr) {
                    sm.pick = i;
                    break;
                }
            }
        }
        __syncthreads();
        if (total) token = sm.pick;  // no mass at all (an infinite logit): the greedy token
    }
    if (threadIdx.x == 0) {
        if (a.out) a.out[row] = int32_t(token);
        if (a.keys) a.keys[row] = argmax_key(0.f, token);
    }
}

__global__ void __launch_bounds__(kThreads) logit_stats_kernel(const float *logits, uint32_t V, size_t stride,
                                                               float *out) {
    __shared__ double dred[32];
    __shared__ unsigned long long kred[32];
    grid_dependency_wait();
    grid_dependents_launch();
    const float *l = logits + size_t(blockIdx.x) * stride;
    double ss = 0.0;
    unsigned long long best = 0ull;
    for (uint32_t i = threadIdx.x; i < V; i += blockDim.x) {
        ss += double(l[i]) * double(l[i]);
        const unsigned long long k = argmax_key(l[i], i);
        best = k > best ? k : best;
    }
    ss = block_sum(ss, dred);
    best = block_max_key(best, kred);
    const float mx = argmax_key_value(best);
    double se = 0.0;
    for (uint32_t i = threadIdx.x; i < V; i += blockDim.x) se += exp(double(l[i] - mx));
    se = block_sum(se, dred);
    double ent = 0.0;
    if (se > 0.0) {
        const double inv = 1.0 / se;
        for (uint32_t i = threadIdx.x; i < V; i += blockDim.x) {
            const double p = exp(double(l[i] - mx)) * inv;
            if (p > 0.0) ent -= p * log(p);
        }
    }
    ent = block_sum(ent, dred);
    if (threadIdx.x == 0) {
        float *o = out + size_t(blockIdx.x) * 4;
        o[0] = mx;
        o[1] = float(sqrt(ss));
        o[2] = float(ent);
        o[3] = float(double(mx) + log(se));
    }
}

}  // namespace
}  // namespace opure

using namespace opure;

extern "C" opure_status opure_sample_filtered(opure_ctx *ctx, const opure_sample_args *a) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!a || !a->logits || !a->vocab || a->stride < a->vocab || (!a->out && !a->keys)) return OPURE_ERR_INVALID_ARG;
    if (a->vocab > kMaxVocab) return OPURE_ERR_UNSUPPORTED;
    if (!(a->top_p > 0.f) || a->top_p > 1.f || !(a->rep_penalty > 0.f)) return OPURE_ERR_INVALID_ARG;
    if (a->temperature > 0.f && a->top_k != 1 && !a->u) return OPURE_ERR_INVALID_ARG;
    if (a->rep_penalty != 1.f && a->hist && (!a->hist_len || a->max_len == 0)) return OPURE_ERR_INVALID_ARG;
    if (a->rows == 0) return OPURE_OK;
    static_assert(sizeof(SampleShared) <= 200 * 1024, "shared memory of the sampling CTA");
    const cudaError_t e = cudaFuncSetAttribute(sample_filtered_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               int(sizeof(SampleShared)));
    if (e != cudaSuccess) return cuda_status(e);
    return launch(ctx, sample_filtered_kernel, dim3(a->rows), dim3(kThreads), sizeof(SampleShared), true, *a);
}

extern "C" opure_status opure_logit_stats(opure_ctx *ctx, const float *logits, uint32_t vocab, uint32_t rows,
                                          size_t stride, float *out) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!logits || !out || !vocab || stride < vocab) return OPURE_ERR_INVALID_ARG;
    if (rows == 0) return OPURE_OK;
    return launch(ctx, logit_stats_kernel, dim3(rows), dim3(kThreads), 0, true, logits, vocab, stride, out);
}
