// elementwise.cu -- stand-alone kernels that mirror one reference shader each:
// embedding gather, RMSNorm, SwiGLU, residual add, ArgMax, RoPE + KV append.
// The decode path fuses all of them into GEMV prologues/epilogues (decode.cu); these
// entry points keep each reference operation callable and testable on its own.
#include "ctx.cuh"

namespace opure {
namespace {

// EmbeddingMain, shaders/Opure_Embedding.usf:21-35 (row gather, fp16 widened to fp32).
__global__ void embedding_kernel(const __half *embed, uint32_t vocab, const int32_t *tokens,
                                 uint32_t d, float *out, DeviceStatus *st) {
    const uint32_t t = blockIdx.y;
    const int32_t tok = tokens[t];
    if (tok < 0 || uint32_t(tok) >= vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0) report(st, OPURE_ERR_DEVICE_BOUNDS, 1, uint32_t(tok));
        return;
    }
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < d; i += gridDim.x * blockDim.x)
        out[size_t(t) * d + i] = __half2float(embed[size_t(tok) * d + i]);
}

// RMSNormMain, shaders/Opure_RMSNorm.usf:31-79: one CTA per row; sum of squares in
// fp32 with warp shuffles, the inverse root in double as the CPU path computes it.
__global__ void rmsnorm_kernel(const float *x, const __half *g, float *y, uint32_t d, float eps) {
    const float *xr = x + size_t(blockIdx.x) * d;
    float *yr = y + size_t(blockIdx.x) * d;
    float ss = 0.f;
    for (uint32_t i = threadIdx.x; i < d; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
    __shared__ float part[32];
    __shared__ float inv_s;
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (uint32_t w = 0; w < (blockDim.x + 31) / 32; ++w) t += part[w];
        inv_s = float(1.0 / sqrt(double(t) / double(d) + double(eps)));
    }
    __syncthreads();
    const float inv = inv_s;
    for (uint32_t i = threadIdx.x; i < d; i += blockDim.x)
        yr[i] = xr[i] * inv * (g ? __half2float(g[i]) : 1.0f);
}

// SwiGLUMain, shaders/Opure_SwiGLU.usf:19-40; silu(g) = g / (1 + exp(-g)) with the
// float exp of the CPU path (Opure_CpuReference.cpp:195).
__global__ void swiglu_kernel(const float *g, const float *u, float *h, uint32_t n) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const float gv = g[i];
        const float s = 1.0f / (1.0f + expf(-gv));
        h[i] = (gv * s) * u[i];
    }
}

// AddResMain / AddMain, shaders/Opure_AddRes.usf:29-43, Opure_Add.usf:14-27.
__global__ void add_kernel(const float *a, const float *b, float *dst, uint32_t n) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = a[i] + b[i];
}

// ArgMaxMain, shaders/Opure_ArgMax.usf:33-85, one CTA per row, with the lowest-index
// tie rule carried by the packed keys.
__global__ void argmax_kernel(const float *logits, uint32_t n, uint32_t *out_idx, float *out_val) {
    const float *row = logits + size_t(blockIdx.x) * n;
    unsigned long long best = 0ull;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const unsigned long long k = argmax_key(row[i], i);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    __shared__ unsigned long long part[32];
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (uint32_t w = 1; w < (blockDim.x + 31) / 32; ++w) best = part[w] > best ? part[w] : best;
        out_idx[blockIdx.x] = best ? argmax_key_index(best) : 0u;
        if (out_val) out_val[blockIdx.x] = argmax_key_value(best);
    }
}

__global__ void argmax_decode_kernel(const unsigned long long *keys, uint32_t n, uint32_t *idx,
                                     float *val) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const unsigned long long k = keys[i];
        if (idx) idx[i] = k ? argmax_key_index(k) : 0u;
        if (val) val[i] = argmax_key_value(k);
    }
}

// RoPEMain, shaders/Opure_RoPE.usf:33-115: interleaved pairs, frequency
// theta^(-2*pair/hd) (:56); the angle, sin/cos and rotation are computed in double as
// the CPU path does (Opure_CpuReference.cpp:171-189). K (rotated) and V (raw) are
// appended as fp16 into the paged cache; one thread per (q or k) pair.
__global__ void rope_kv_kernel(const float *qkv, uint32_t stride, float *q_out, const int32_t *seq,
                               const int32_t *pos, uint32_t n_heads, double theta,
                               opure_kv_layout kv, DeviceStatus *st) {
    grid_dependency_wait();
    grid_dependents_launch();
    const uint32_t i = blockIdx.y;
    const uint32_t hd = kv.head_dim, half = hd / 2;
    const uint32_t nq = n_heads * half, nk = kv.n_kv * half;
    const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= nq + nk) return;
    const int32_t p = pos[i], s = seq[i];
    const bool is_q = idx < nq;
    const uint32_t local = is_q ? idx : idx - nq;
    const uint32_t head = local / half, pair = local % half;
    const double freq = pow(theta, -2.0 * double(pair) / double(hd));
    double sn, cs;
    sincos(double(p) * freq, &sn, &cs);
    const float *row = qkv + size_t(i) * stride;
    const float *src = is_q ? row + size_t(head) * hd : row + size_t(n_heads + head) * hd;
    const double e0 = src[2 * pair], e1 = src[2 * pair + 1];
    const float r0 = float(e0 * cs - e1 * sn), r1 = float(e0 * sn + e1 * cs);
    if (is_q) {
        float *qd = q_out + (size_t(i) * n_heads + head) * hd;
        qd[2 * pair] = r0;
        qd[2 * pair + 1] = r1;
        return;
    }
    const uint32_t lp = ring_slot(uint32_t(p) / kv.page_size, kv.ring), slot = uint32_t(p) % kv.page_size;
    if (p < 0 || s < 0 || lp >= kv.max_pages) {
        report(st, OPURE_ERR_DEVICE_BOUNDS, 2, uint32_t(p));
        return;
    }
    const int32_t page = kv.page_table[size_t(s) * kv.max_pages + lp];
    if (page < 0 || uint32_t(page) >= kv.n_pages) {
        report(st, OPURE_ERR_DEVICE_BOUNDS, 3, uint32_t(page));
        return;
    }
    const size_t blk = size_t(kv.page_size) * hd;
    __half *kd = reinterpret_cast<__half *>(kv.pool) + (size_t(page) * 2 * kv.n_kv + head) * blk + size_t(slot) * hd;
    __half *vd = kd + size_t(kv.n_kv) * blk;
    const float *vs = row + size_t(n_heads + kv.n_kv + head) * hd;
    kd[2 * pair] = __float2half_rn(r0);
    kd[2 * pair + 1] = __float2half_rn(r1);
    vd[2 * pair] = __float2half_rn(vs[2 * pair]);
    vd[2 * pair + 1] = __float2half_rn(vs[2 * pair + 1]);
}

}  // namespace
}  // namespace opure

using namespace opure;

extern "C" {

opure_status opure_embedding(opure_ctx *ctx, const uint16_t *embed, uint32_t vocab,
                             const int32_t *tokens, uint32_t n, uint32_t d, float *out) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!embed || !tokens || !out || d == 0) return OPURE_ERR_INVALID_ARG;
    if (n == 0) return OPURE_OK;
    return launch(ctx, embedding_kernel, dim3(ceil_div(d, 256), n), dim3(256), 0, false,
                  reinterpret_cast<const __half *>(embed), vocab, tokens, d, out, ctx->status);
}

opure_status opure_rmsnorm(opure_ctx *ctx, const float *x, const uint16_t *g, float *y,
                           uint32_t d, uint32_t rows, float eps) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!x || !y || d == 0) return OPURE_ERR_INVALID_ARG;
    if (rows == 0) return OPURE_OK;
    return launch(ctx, rmsnorm_kernel, dim3(rows), dim3(256), 0, false, x,
                  reinterpret_cast<const __half *>(g), y, d, eps);
}

opure_status opure_swiglu(opure_ctx *ctx, const float *g, const float *u, float *h, uint32_t n) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!g || !u || !h) return OPURE_ERR_INVALID_ARG;
    if (n == 0) return OPURE_OK;
    return launch(ctx, swiglu_kernel, dim3(ceil_div(n, 256)), dim3(256), 0, false, g, u, h, n);
}

opure_status opure_add(opure_ctx *ctx, const float *a, const float *b, float *dst, uint32_t n) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!a || !b || !dst) return OPURE_ERR_INVALID_ARG;
    if (n == 0) return OPURE_OK;
    return launch(ctx, add_kernel, dim3(ceil_div(n, 256)), dim3(256), 0, false, a, b, dst, n);
}

opure_status opure_argmax(opure_ctx *ctx, const float *logits, uint32_t n, uint32_t rows,
                          uint32_t *out_idx, float *out_val) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!logits || !out_idx || n == 0) return OPURE_ERR_INVALID_ARG;
    if (rows == 0) return OPURE_OK;
    return launch(ctx, argmax_kernel, dim3(rows), dim3(1024), 0, false, logits, n, out_idx, out_val);
}

opure_status opure_argmax_decode(opure_ctx *ctx, const unsigned long long *keys, uint32_t n,
                                 uint32_t *idx, float *val) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!keys || (!idx && !val)) return OPURE_ERR_INVALID_ARG;
    if (n == 0) return OPURE_OK;
    return launch(ctx, argmax_decode_kernel, dim3(ceil_div(n, 128)), dim3(128), 0, false, keys,
                  n, idx, val);
}

opure_status opure_rope_kv_append(opure_ctx *ctx, const float *qkv, uint32_t stride, float *q_out,
                                  const int32_t *seq, const int32_t *pos, uint32_t n,
                                  uint32_t n_heads, double theta, const opure_kv_layout *kv) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!qkv || !q_out || !seq || !pos || !kv || !kv->pool || !kv->page_table)
        return OPURE_ERR_INVALID_ARG;
    if (kv->head_dim == 0 || kv->head_dim % 2 || kv->n_kv == 0 || n_heads % kv->n_kv ||
        kv->page_size == 0)
        return OPURE_ERR_INVALID_ARG;
    if (stride < (n_heads + 2 * kv->n_kv) * kv->head_dim) return OPURE_ERR_INVALID_ARG;
    if (n == 0) return OPURE_OK;
    const uint32_t pairs = (n_heads + kv->n_kv) * (kv->head_dim / 2);
    return launch(ctx, rope_kv_kernel, dim3(ceil_div(pairs, 128), n), dim3(128), 0, true, qkv, stride,
                  q_out, seq, pos, n_heads, theta, *kv, ctx->status);
}

}  // extern "C"
