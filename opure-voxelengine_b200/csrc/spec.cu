// spec.cu -- speculative-decode accept/reject and softmax sampling.
//
// The reference has no accept logic: its SpeculativeVerify pipelines
// (shaders/Opure_SpeculativeDecode.usf:60-189) are a copy of decode attention that is
// never dispatched, and MetricsSnapshot.speculativeAcceptance is hard-wired to -1
// (src/engine/Opure_VoxelEngine.cpp:666). These kernels implement the standard rules:
//  - greedy: accept the longest prefix of draft tokens equal to the target's argmax,
//    then emit the target's argmax at the first mismatch (or after the last draft);
//  - rejection sampling at temperature 1 (Leviathan, Kalman & Matias 2023; Chen et al.
//    2023): accept draft d_i when u_i * q_i(d_i) <= p_i(d_i); at the first rejection
//    draw the replacement from max(0, p_i - q_i) renormalised, and if every draft is
//    accepted draw a bonus token from p_k. Draws are inverse-CDF in index order.
// Softmax quantities are computed in double, one CTA per sequence.
#include "ctx.cuh"

namespace opure {
namespace {

constexpr int kThreads = 1024;

__device__ unsigned long long block_max_u64(unsigned long long v, unsigned long long *red) {
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
    return red[0];
}

__device__ double block_sum_d(double v, double *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    return red[0];
}

__device__ uint32_t block_argmax(const float *x, uint32_t n, unsigned long long *red) {
    unsigned long long best = 0ull;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const unsigned long long k = argmax_key(x[i], i);
        best = k > best ? k : best;
    }
    best = block_max_u64(best, red);
    return best ? argmax_key_index(best) : 0u;
}

// Max logit of a row as a double (NaN ignored).
__device__ double block_max_logit(const float *x, uint32_t n, unsigned long long *red) {
    unsigned long long best = 0ull;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const unsigned long long k = argmax_key(x[i], i);
        best = k > best ? k : best;
    }
    best = block_max_u64(best, red);
    return double(argmax_key_value(best));
}

// Inverse-CDF draw over non-negative weights w(x) produced by `wf`, in index order:
// the smallest x with sum_{y<=x} w(y) > u * sum(w). Each thread owns a contiguous
// segment; segment sums are scanned in order, then the owning thread walks its segment.
template <class WF>
__device__ uint32_t block_inverse_cdf(uint32_t n, double u, WF wf, double *dred, uint32_t *pick) {
    const uint32_t seg = (n + blockDim.x - 1) / blockDim.x;
    const uint32_t b = threadIdx.x * seg, e = min(n, b + seg);
    double local = 0.0;
    for (uint32_t i = b; i < e; ++i) local += wf(i);
    // Exclusive scan of segment sums (serial over warps' totals, fine for 1024 threads).
    __shared__ double seg_sum[kThreads];
    seg_sum[threadIdx.x] = local;
    __syncthreads();
    if (threadIdx.x == 0) {
        double run = 0.0;
        for (uint32_t t = 0; t < blockDim.x; ++t) {
            const double s = seg_sum[t];
            seg_sum[t] = run;
            run += s;
        }
        dred[0] = run;
        *pick = 0xffffffffu;
    }
    __syncthreads();
    const double total = dred[0];
    const double thr = u * total;
    double c = seg_sum[threadIdx.x];
    if (c <= thr && c + local > thr) {
        for (uint32_t i = b; i < e; ++i) {
            c += wf(i);
            if (c > thr) {
                atomicMin(pick, i);
                break;
            }
        }
    }
    __syncthreads();
    uint32_t r = *pick;
    if (r == 0xffffffffu) {
        // u * total at the very top (rounding): the last index with non-zero weight.
        __syncthreads();
        if (threadIdx.x == 0) {
            uint32_t last = 0;
            for (uint32_t i = n; i-- > 0;)
                if (wf(i) > 0.0) { last = i; break; }
            *pick = last;
        }
        __syncthreads();
        r = *pick;
    }
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(kThreads) spec_kernel(opure_spec_args a) {
    __shared__ unsigned long long red[32];
    __shared__ double dred[32];
    __shared__ uint32_t pick;
    const uint32_t s = blockIdx.x, k = a.k, V = a.vocab;
    const float *tl = a.target_logits + size_t(s) * (k + 1) * V;
    const int32_t *draft = a.draft + size_t(s) * k;
    int32_t *out = a.out_tokens + size_t(s) * (k + 1);

    grid_dependency_wait();
    grid_dependents_launch();
    if (a.mode == OPURE_SPEC_GREEDY) {
        uint32_t acc = 0;
        for (; acc < k; ++acc) {
            const uint32_t t = block_argmax(tl + size_t(acc) * V, V, red);
            if (int32_t(t) != draft[acc]) break;
            if (threadIdx.x == 0) out[acc] = draft[acc];
        }
        const uint32_t t = block_argmax(tl + size_t(acc) * V, V, red);
        if (threadIdx.x == 0) {
            out[acc] = int32_t(t);
            a.out_accepted[s] = int32_t(acc);
        }
        return;
    }
    const float *dl = a.draft_logits + size_t(s) * k * V;
    const float *ua = a.u_accept + size_t(s) * k;
    const double uf = double(a.u_final[s]);
    for (uint32_t i = 0; i < k; ++i) {
        const float *p = tl + size_t(i) * V, *q = dl + size_t(i) * V;
        const double pm = block_max_logit(p, V, red), qm = block_max_logit(q, V, red);
        double zp = 0.0, zq = 0.0;
        for (uint32_t x = threadIdx.x; x < V; x += blockDim.x) {
            zp += exp(double(p[x]) - pm);
            zq += exp(double(q[x]) - qm);
        }
        zp = block_sum_d(zp, dred);
        zq = block_sum_d(zq, dred);
        const int32_t d = draft[i];
        const bool in_range = d >= 0 && uint32_t(d) < V;
        const double pd = in_range ? exp(double(p[d]) - pm) / zp : 0.0;
        const double qd = in_range ? exp(double(q[d]) - qm) / zq : 0.0;
        if (in_range && double(ua[i]) * qd <= pd) {
            if (threadIdx.x == 0) out[i] = d;
            continue;
        }
        // Residual max(0, p - q); from p itself if the residual is all zero.
        auto resid = [&](uint32_t x) {
            const double r = exp(double(p[x]) - pm) / zp - exp(double(q[x]) - qm) / zq;
            return r > 0.0 ? r : 0.0;
        };
        double zr = 0.0;
        for (uint32_t x = threadIdx.x; x < V; x += blockDim.x) zr += resid(x);
        zr = block_sum_d(zr, dred);
        uint32_t t;
        if (zr > 0.0) {
            t = block_inverse_cdf(V, uf, resid, dred, &pick);
        } else {
            t = block_inverse_cdf(V, uf, [&](uint32_t x) { return exp(double(p[x]) - pm) / zp; }, dred, &pick);
        }
        if (threadIdx.x == 0) {
            out[i] = int32_t(t);
            a.out_accepted[s] = int32_t(i);
        }
        return;
    }
    const float *p = tl + size_t(k) * V;
    const double pm = block_max_logit(p, V, red);
    double zp = 0.0;
    for (uint32_t x = threadIdx.x; x < V; x += blockDim.x) zp += exp(double(p[x]) - pm);
    zp = block_sum_d(zp, dred);
    const uint32_t t = block_inverse_cdf(V, uf, [&](uint32_t x) { return exp(double(p[x]) - pm) / zp; }, dred, &pick);
    if (threadIdx.x == 0) {
        out[k] = int32_t(t);
        a.out_accepted[s] = int32_t(k);
    }
}

// One row per CTA: inverse-CDF draw from softmax(logits[row]) with u[row]. The token
// goes to out[row] and/or, as an argmax key, to keys[row] (where a self-driving decode
// step picks up its next input); `save` receives a copy of the row when given.
__global__ void __launch_bounds__(kThreads) sample_kernel(const float *logits, uint32_t V, const float *u,
                                                          int32_t *out, unsigned long long *keys, float *save,
                                                          size_t save_stride) {
    __shared__ unsigned long long red[32];
    __shared__ double dred[32];
    __shared__ uint32_t pick;
    grid_dependency_wait();
    grid_dependents_launch();
    const float *p = logits + size_t(blockIdx.x) * V;
    if (save)
        for (uint32_t x = threadIdx.x; x < V; x += blockDim.x) save[size_t(blockIdx.x) * save_stride + x] = p[x];
    const double pm = block_max_logit(p, V, red);
    double z = 0.0;
    for (uint32_t x = threadIdx.x; x < V; x += blockDim.x) z += exp(double(p[x]) - pm);
    z = block_sum_d(z, dred);
    const uint32_t t = block_inverse_cdf(V, double(u[blockIdx.x]), [&](uint32_t x) { return exp(double(p[x]) - pm) / z; }, dred, &pick);
    if (threadIdx.x == 0) {
        if (out) out[blockIdx.x] = int32_t(t);
        if (keys) keys[blockIdx.x] = argmax_key(0.f, t);
    }
}

// Per sequence s (one thread each): the draft's proposals d_1..d_k for the round that
// starts at position base[s] are hist[s][base+1 .. base+k-1] (inputs of the draft's
// later steps) and the last step's key (d_k). Writes the target's k+1 verify inputs
// (hist[s][base], d_1..d_k) and the k drafts.
__global__ void gather_kernel(const int32_t *hist, uint32_t max_len, const unsigned long long *keys,
                              const int32_t *base, uint32_t n_seq, uint32_t k, int32_t *verify, int32_t *draft,
                              DeviceStatus *st) {
    grid_dependency_wait();
    grid_dependents_launch();
    const uint32_t s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= n_seq) return;
    const int32_t b = base[s];
    if (b < 0 || uint32_t(b) + k > max_len) {
        report(st, OPURE_ERR_DEVICE_BOUNDS, 70, uint32_t(b));
        return;
    }
    const int32_t *h = hist + size_t(s) * max_len;
    verify[size_t(s) * (k + 1)] = h[b];
    for (uint32_t j = 1; j <= k; ++j) {
        const int32_t d = j < k ? h[b + j] : int32_t(argmax_key_index(keys[s]));
        verify[size_t(s) * (k + 1) + j] = d;
        draft[size_t(s) * k + j - 1] = d;
    }
}

}  // namespace
}  // namespace opure

using namespace opure;

extern "C" opure_status opure_spec_accept(opure_ctx *ctx, const opure_spec_args *a) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!a || !a->target_logits || !a->draft || !a->out_tokens || !a->out_accepted || !a->vocab)
        return OPURE_ERR_INVALID_ARG;
    if (a->mode == OPURE_SPEC_REJECTION && (!a->draft_logits || !a->u_accept || !a->u_final))
        return OPURE_ERR_INVALID_ARG;
    if (a->mode > OPURE_SPEC_REJECTION) return OPURE_ERR_INVALID_ARG;
    if (a->n_seq == 0) return OPURE_OK;
    return launch(ctx, spec_kernel, dim3(a->n_seq), dim3(kThreads), 0, true, *a);
}

extern "C" opure_status opure_sample_softmax(opure_ctx *ctx, const float *logits, uint32_t vocab,
                                             uint32_t rows, const float *u, int32_t *out) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!logits || !u || !out || !vocab) return OPURE_ERR_INVALID_ARG;
    if (rows == 0) return OPURE_OK;
    return launch(ctx, sample_kernel, dim3(rows), dim3(kThreads), 0, true, logits, vocab, u, out,
                  static_cast<unsigned long long *>(nullptr), static_cast<float *>(nullptr), size_t(0));
}

extern "C" opure_status opure_sample_keys(opure_ctx *ctx, const float *logits, uint32_t vocab, uint32_t rows,
                                          const float *u, unsigned long long *keys, float *save,
                                          size_t save_stride) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!logits || !u || !keys || !vocab || (save && save_stride < vocab)) return OPURE_ERR_INVALID_ARG;
    if (rows == 0) return OPURE_OK;
    return launch(ctx, sample_kernel, dim3(rows), dim3(kThreads), 0, true, logits, vocab, u,
                  static_cast<int32_t *>(nullptr), keys, save, save_stride);
}

extern "C" opure_status opure_spec_gather(opure_ctx *ctx, const int32_t *hist, uint32_t max_len,
                                          const unsigned long long *keys, const int32_t *base, uint32_t n_seq,
                                          uint32_t k, int32_t *verify_tokens, int32_t *draft) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!hist || !keys || !base || !verify_tokens || !draft || k == 0 || max_len == 0) return OPURE_ERR_INVALID_ARG;
    if (n_seq == 0) return OPURE_OK;
    return launch(ctx, gather_kernel, dim3(ceil_div(n_seq, 128)), dim3(128), 0, true, hist, max_len, keys, base,
                  n_seq, k, verify_tokens, draft, ctx->status);
}
