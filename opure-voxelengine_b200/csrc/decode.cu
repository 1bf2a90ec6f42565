// decode.cu -- opure_decode_fused: the latency path of one decode step (1..8 token
// vectors) as three fused kernels per layer plus the lm_head. See opure_cuda.h for the
// phase split. Replaces the per-layer dispatch sequence of VoxelEngine::RecordForward
// (src/engine/Opure_VoxelEngine.cpp:300-491): RMSNorm, GEMV q/k/v, RoPE, Attention,
// GEMV o, AddRes, RMSNorm, GEMV gate/up, SwiGLU, GEMV down, AddRes.
#include <algorithm>

#include "attn_core.cuh"
#include "ctx.cuh"
#include "gemv.cuh"
#include "tma.cuh"

namespace opure {
namespace {


struct KvParams {
    uint16_t *pool;
    const int32_t *page_table;
    uint32_t n_pages, max_pages, page_size;
    uint32_t ring;  // sliding window (opure_kv_layout.ring)
};

// x[v] = base[v] + delta[v] * 2^-32 (rounded to fp32 once, as the reference rounds its fp32
// residual after every add), staged into xs and RMS-normalised with `gain` in place. The
// designated CTA also writes the un-normalised x to base_out and zeroes delta_zero.
// The fp16 norm gain a thread will need, fetched before the kernel waits on its
// predecessor (gains are weights, never written by the previous kernel). Group g covers
// elements 4g..4g+3 of the NV*h staged values.
constexpr int kGainRegs = 4;
struct GainPrefetch {
    uint2 g[kGainRegs];
};

template <int NV>
__device__ __forceinline__ void prefetch_gain(const __half *gain, uint32_t h, GainPrefetch &p) {
    const uint32_t groups = NV * h / 4;
#pragma unroll
    for (int k = 0; k < kGainRegs; ++k) {
        const uint32_t g = threadIdx.x + k * blockDim.x;
        p.g[k] = g < groups ? __ldg(reinterpret_cast<const uint2 *>(gain + (4 * g) % h)) : make_uint2(0, 0);
    }
}

// All of a thread's loads are issued before any is used (16-byte vectors, unrolled), so
// staging costs one memory round trip rather than one per loop iteration. Requires
// NV * h to be a multiple of 4 (h % 8 == 0 is checked at the ABI).
template <int NV>
__device__ __forceinline__ void stage_residual(const float *base, const long long *delta, uint32_t h,
                                               const GainPrefetch &gpre, const __half *gain, float eps,
                                               float *xs, float *red, float *base_out, long long *delta_zero,
                                               bool designated) {
    constexpr int kLoads = 4;  // float4 groups per thread issued together
    const uint32_t groups = NV * h / 4, step = blockDim.x;
    for (uint32_t g0 = threadIdx.x; g0 < groups; g0 += kLoads * step) {
        float4 b[kLoads];
        longlong2 d[kLoads][2];
#pragma unroll
        for (int k = 0; k < kLoads; ++k) {
            const uint32_t g = g0 + k * step;
            if (g < groups) {
                b[k] = __ldcg(reinterpret_cast<const float4 *>(base) + g);
                if (delta) {
                    d[k][0] = __ldcg(reinterpret_cast<const longlong2 *>(delta) + 2 * g);
                    d[k][1] = __ldcg(reinterpret_cast<const longlong2 *>(delta) + 2 * g + 1);
                }
            }
        }
#pragma unroll
        for (int k = 0; k < kLoads; ++k) {
            const uint32_t g = g0 + k * step;
            if (g >= groups) continue;
            float4 x = b[k];
            if (delta) {
                x.x = float(double(x.x) + double(d[k][0].x) * kFixInv);
                x.y = float(double(x.y) + double(d[k][0].y) * kFixInv);
                x.z = float(double(x.z) + double(d[k][1].x) * kFixInv);
                x.w = float(double(x.w) + double(d[k][1].y) * kFixInv);
            }
            reinterpret_cast<float4 *>(xs)[g] = x;
            if (designated) {
                if (base_out) reinterpret_cast<float4 *>(base_out)[g] = x;
                if (delta_zero) {
                    reinterpret_cast<longlong2 *>(delta_zero)[2 * g] = make_longlong2(0, 0);
                    reinterpret_cast<longlong2 *>(delta_zero)[2 * g + 1] = make_longlong2(0, 0);
                }
            }
        }
    }
    __syncthreads();
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, nw = blockDim.x >> 5;
    for (uint32_t v = 0; v < NV; ++v) {
        float ss = 0.f;
        for (uint32_t i = threadIdx.x; i < h; i += blockDim.x) ss = fmaf(xs[v * h + i], xs[v * h + i], ss);
        ss = warp_sum(ss);
        if (lane == 0) red[v * 32 + warp] = ss;
    }
    __syncthreads();
    if (threadIdx.x < NV) {
        float t = 0.f;
        for (uint32_t w = 0; w < nw; ++w) t += red[threadIdx.x * 32 + w];
        red[32 * NV + threadIdx.x] = float(1.0 / sqrt(double(t) / double(h) + double(eps)));
    }
    __syncthreads();
    auto scale = [&](uint32_t g, uint2 gw) {
        const float2 g01 = h2f2(gw.x), g23 = h2f2(gw.y);
        const float inv = red[32 * NV + (4 * g) / h];
        float4 x = reinterpret_cast<float4 *>(xs)[g];
        x.x = x.x * inv * g01.x;
        x.y = x.y * inv * g01.y;
        x.z = x.z * inv * g23.x;
        x.w = x.w * inv * g23.y;
        reinterpret_cast<float4 *>(xs)[g] = x;
    };
#pragma unroll
    for (int k = 0; k < kGainRegs; ++k) {
        const uint32_t g = threadIdx.x + k * step;
        if (g < groups) scale(g, gpre.g[k]);
    }
    for (uint32_t g = threadIdx.x + kGainRegs * step; g < groups; g += step)
        scale(g, __ldg(reinterpret_cast<const uint2 *>(gain + (4 * g) % h)));
    __syncthreads();
}

// stage_residual in one pass: each thread keeps the groups it loaded in registers, sums
// their squares per vector, and after a single block reduction scales and stores them:
// two barriers and no second trip through shared memory. A thread holds NV float4 groups,
// so it needs NV*h/4 <= NV * blockDim.x, i.e. h <= 4 * blockDim.x (stage_residual_fits).
template <int NV>
__device__ __forceinline__ bool stage_residual_fits(uint32_t h) {
    return h <= 4 * blockDim.x;
}

template <int NV>
__device__ __forceinline__ void stage_residual_fast(const float *base, const long long *delta, uint32_t h,
                                                    const GainPrefetch &gpre, const __half *gain, float eps,
                                                    float *xs, float *red, float *base_out, long long *delta_zero,
                                                    bool designated) {
    constexpr int kFastSlots = NV;
    const uint32_t groups = NV * h / 4, step = blockDim.x;
    float4 xv[kFastSlots];
    longlong2 d[kFastSlots][2];
#pragma unroll
    for (int k = 0; k < kFastSlots; ++k) {
        const uint32_t g = threadIdx.x + k * step;
        if (g < groups) {
            xv[k] = __ldcg(reinterpret_cast<const float4 *>(base) + g);
            if (delta) {
                d[k][0] = __ldcg(reinterpret_cast<const longlong2 *>(delta) + 2 * g);
                d[k][1] = __ldcg(reinterpret_cast<const longlong2 *>(delta) + 2 * g + 1);
            }
        }
    }
    float ss[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) ss[v] = 0.f;
#pragma unroll
    for (int k = 0; k < kFastSlots; ++k) {
        const uint32_t g = threadIdx.x + k * step;
        if (g >= groups) continue;
        float4 x = xv[k];
        if (delta) {
            x.x = float(double(x.x) + double(d[k][0].x) * kFixInv);
            x.y = float(double(x.y) + double(d[k][0].y) * kFixInv);
            x.z = float(double(x.z) + double(d[k][1].x) * kFixInv);
            x.w = float(double(x.w) + double(d[k][1].y) * kFixInv);
        }
        xv[k] = x;
        if (designated) {
            if (base_out) reinterpret_cast<float4 *>(base_out)[g] = x;
            if (delta_zero) {
                reinterpret_cast<longlong2 *>(delta_zero)[2 * g] = make_longlong2(0, 0);
                reinterpret_cast<longlong2 *>(delta_zero)[2 * g + 1] = make_longlong2(0, 0);
            }
        }
        const float s2 = fmaf(x.w, x.w, fmaf(x.z, x.z, fmaf(x.y, x.y, x.x * x.x)));
        const uint32_t v = (4 * g) / h;
#pragma unroll
        for (int vv = 0; vv < NV; ++vv)
            if (vv == int(v)) ss[vv] += s2;
    }
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, nw = blockDim.x >> 5;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
        const float t = warp_sum(ss[v]);
        if (lane == 0) red[v * 32 + warp] = t;
    }
    __syncthreads();
    float inv[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
        float t = 0.f;
        for (uint32_t w = 0; w < nw; ++w) t += red[v * 32 + w];
        inv[v] = float(1.0 / sqrt(double(t) / double(h) + double(eps)));
    }
#pragma unroll
    for (int k = 0; k < kFastSlots; ++k) {
        const uint32_t g = threadIdx.x + k * step;
        if (g >= groups) continue;
        const uint32_t v = (4 * g) / h;
        float iv = inv[0];
#pragma unroll
        for (int vv = 1; vv < NV; ++vv)
            if (vv == int(v)) iv = inv[vv];
        const uint2 gw = k < kGainRegs ? gpre.g[k] : __ldg(reinterpret_cast<const uint2 *>(gain + (4 * g) % h));
        const float2 g01 = h2f2(gw.x), g23 = h2f2(gw.y);
        float4 x = xv[k];
        x.x = x.x * iv * g01.x;
        x.y = x.y * iv * g01.y;
        x.z = x.z * iv * g23.x;
        x.w = x.w * iv * g23.y;
        reinterpret_cast<float4 *>(xs)[g] = x;
    }
    __syncthreads();
}

// One 16-byte chunk of a weight row as fp32: 8 fp16, or (Q8) 16 int8 in the reference's
// little-endian packing (Opure_GEMV_Quant.usf:52-93), unscaled.
template <bool Q8>
struct RowChunk {
    static constexpr int E = Q8 ? 16 : 8;
    __device__ __forceinline__ static void unpack(const uint4 &w, float *f) {
        if constexpr (Q8)
            unpack16_i8(w, f);
        else
            unpack8(w, f);
    }
};

// Dot products of R rows held in shared memory (row r at rows[r]; rows >= nrows skipped)
// with NV vectors xs[v * h + i]; lanes stride the rows' 16-byte chunks (nchunks of them).
// Every lane gets the sums. Q8 rows are int8: the caller applies the tensor's scale.
template <int NV, int R, bool Q8 = false>
__device__ __forceinline__ void smem_dot_ptrs(const uint8_t *const (&rows)[R], uint32_t nrows, uint32_t nchunks,
                                              const float *xs, uint32_t h, float (&acc)[R][NV]) {
    constexpr int E = RowChunk<Q8>::E;
    const uint32_t lane = threadIdx.x & 31u;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int v = 0; v < NV; ++v) acc[r][v] = 0.f;
    for (uint32_t c = lane; c < nchunks; c += 32) {
        float xf[NV][E];
#pragma unroll
        for (int v = 0; v < NV; ++v)
#pragma unroll
            for (int q = 0; q < E / 4; ++q) {
                const float4 a = lds_f4(xs + v * h + c * E + 4 * q);
                xf[v][4 * q] = a.x; xf[v][4 * q + 1] = a.y; xf[v][4 * q + 2] = a.z; xf[v][4 * q + 3] = a.w;
            }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            if (r >= int(nrows)) break;
            float wf[E];
            RowChunk<Q8>::unpack(lds128(rows[r] + c * 16), wf);
#pragma unroll
            for (int v = 0; v < NV; ++v)
#pragma unroll
                for (int e = 0; e < E; ++e) acc[r][v] = fmaf(wf[e], xf[v][e], acc[r][v]);
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
        if (r >= int(nrows)) break;
#pragma unroll
        for (int v = 0; v < NV; ++v) acc[r][v] = warp_sum(acc[r][v]);
    }
}

// smem_dot_ptrs over R consecutive rows, row r at w + r * pitch bytes.
template <int NV, int R, bool Q8 = false>
__device__ __forceinline__ void smem_dot(const uint8_t *w, uint32_t pitch, uint32_t nrows, uint32_t nchunks,
                                         const float *xs, uint32_t h, float (&acc)[R][NV]) {
    const uint8_t *rows[R];
#pragma unroll
    for (int r = 0; r < R; ++r) rows[r] = w + size_t(r) * pitch;
    smem_dot_ptrs<NV, R, Q8>(rows, nrows, nchunks, xs, h, acc);
}

// Eight fp16 rows (row r at w + r * pitch; rows >= nrows, 1 <= nrows, are not read) with
// one vector xs, for the lm_head. The loads carry no per-row branch (a missing row reads
// row nrows - 1 again) and the eight sums are reduced together: every level of the xor
// butterfly halves the rows a lane keeps, so 4 + 2 + 1 + 1 + 1 shuffles replace 8 x 5.
// Lane l returns the sum of row (l >> 2) & 7. Each level adds the same pairs of partial
// sums as warp_sum, so every row's sum is bit-identical to smem_dot's.
__device__ __forceinline__ float lm_dot8(const uint8_t *w, uint32_t pitch, uint32_t nrows, uint32_t nchunks,
                                         const float *xs) {
    const uint32_t lane = threadIdx.x & 31u;
    const uint8_t *rows[8];
    float acc[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        rows[r] = w + size_t(min(uint32_t(r), nrows - 1)) * pitch;
        acc[r] = 0.f;
    }
    auto pass = [&](uint32_t c) {
        uint4 raw[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) raw[r] = lds128(rows[r] + c * 16);
        const float4 x0 = lds_f4(xs + c * 8), x1 = lds_f4(xs + c * 8 + 4);
        const float xf[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            float wf[8];
            unpack8(raw[r], wf);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[r] = fmaf(wf[e], xf[e], acc[r]);
        }
    };
    if (nchunks <= 96) {
#pragma unroll
        for (int i = 0; i < 3; ++i)
            if (lane + 32u * i < nchunks) pass(lane + 32u * i);
    } else {
        for (uint32_t c = lane; c < nchunks; c += 32) pass(c);
    }
    // xor 16: keep rows 4 b4 + (0..3); xor 8: rows + 2 b3; xor 4: row + b2; then xor 2, 1.
    const bool b4 = lane & 16u, b3 = lane & 8u, b2 = lane & 4u;
    float u[4], t[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float send = b4 ? acc[i] : acc[i + 4];
        u[i] = (b4 ? acc[i + 4] : acc[i]) + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float send = b3 ? u[i] : u[i + 2];
        t[i] = (b3 ? u[i + 2] : u[i]) + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    float x = (b2 ? t[1] : t[0]) + __shfl_xor_sync(0xffffffffu, b2 ? t[0] : t[1], 4);
    x += __shfl_xor_sync(0xffffffffu, x, 2);
    x += __shfl_xor_sync(0xffffffffu, x, 1);
    return x;
}

// Element offset of (seq, pos, K|V, kv head) row inside a layer's pool, or -1 (reported).
__device__ __forceinline__ long long kv_offset(const KvParams &kv, uint32_t n_kv, uint32_t hd, int32_t seq,
                                               int32_t pos, uint32_t sel, uint32_t head, DeviceStatus *st) {
    const uint32_t lp = ring_slot(uint32_t(pos) / kv.page_size, kv.ring);
    if (seq < 0 || pos < 0 || lp >= kv.max_pages) {
        report(st, OPURE_ERR_DEVICE_BOUNDS, 30, uint32_t(pos));
        return -1;
    }
    const int32_t page = kv.page_table[size_t(seq) * kv.max_pages + lp];
    if (page < 0 || uint32_t(page) >= kv.n_pages) {
        report(st, OPURE_ERR_DEVICE_BOUNDS, 31, uint32_t(page));
        return -1;
    }
    const size_t blk = size_t(kv.page_size) * hd;
    return (long long)(((size_t(page) * 2 + sel) * n_kv + head) * blk + size_t(uint32_t(pos) % kv.page_size) * hd);
}

__device__ __forceinline__ __half *kv_slot(const KvParams &kv, uint32_t n_kv, uint32_t hd, int32_t seq,
                                           int32_t pos, uint32_t sel, uint32_t head, DeviceStatus *st) {
    const long long off = kv_offset(kv, n_kv, hd, seq, pos, sel, head, st);
    return off < 0 ? nullptr : reinterpret_cast<__half *>(kv.pool) + off;
}

// ---------------------------------------------------------------------------------------
// A: RMSNorm + q;k;v GEMV + RoPE + paged KV append.
constexpr uint32_t kARows = 8;      // rows per CTA: 4 warps x one RoPE pair
constexpr uint32_t kAThreads = 128;

struct QkvArgs {
    const __half *w;
    uint32_t rows, h, n_heads, n_kv, hd;
    const __half *gain;
    float eps;
    double theta;
    const float *base_in;
    const long long *delta_in;   // NULL for layer 0 (x is the embedding)
    float *base_out;
    long long *delta_zero;
    float *q_out;
    KvParams kv;
    const int32_t *seq, *pos;
    DeviceStatus *st;
};

template <int NV>
__global__ void __launch_bounds__(kAThreads) qkv_fused_kernel(QkvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bar;
    const uint32_t pitch = a.h * 2;
    const uint32_t row0 = blockIdx.x * kARows;
    const uint32_t nrows = min(kARows, a.rows - row0);
    uint8_t *wsm = smem;
    float *xs = reinterpret_cast<float *>(smem + ((kARows * pitch + 127) & ~127u));
    float *red = xs + NV * a.h;

    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_expect_tx(&bar, nrows * pitch);
        bulk_load(wsm, reinterpret_cast<const uint8_t *>(a.w) + size_t(row0) * pitch, nrows * pitch, &bar);
    }
    GainPrefetch gpre;
    prefetch_gain<NV>(a.gain, a.h, gpre);

    // Everything the epilogue needs besides the dot products depends only on the step's
    // positions and the page table, which the previous kernel does not write: lane v of
    // each warp resolves vector v's position, RoPE angle and KV slot before the wait.
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t r = row0 + 2 * warp;  // this warp's RoPE pair (r, r + 1)
    const uint32_t qrows = a.n_heads * a.hd, krows = a.n_kv * a.hd;
    const bool epi = 2 * warp < nrows && lane < NV;
    double sn = 0.0, cs = 1.0;
    __half *slot = nullptr;
    if (epi) {
        const int32_t p = a.pos[lane], s = a.seq[lane];
        if (r < qrows + krows) {
            // RoPE, interleaved pairs, theta^(-2*pair/hd) (Opure_RoPE.usf:56), in double.
            const uint32_t pair = (r % a.hd) / 2;
            sincos(double(p) * pow(a.theta, -2.0 * double(pair) / double(a.hd)), &sn, &cs);
        }
        if (r >= qrows) {
            const bool is_k = r < qrows + krows;
            const uint32_t rr = is_k ? r - qrows : r - qrows - krows;
            slot = kv_slot(a.kv, a.n_kv, a.hd, s, p, is_k ? 0 : 1, rr / a.hd, a.st);
            if (slot) slot += rr % a.hd;
        }
    }

    grid_dependency_wait();
    grid_dependents_launch();
    stage_residual<NV>(a.base_in, a.delta_in, a.h, gpre, a.gain, a.eps, xs, red, a.base_out, a.delta_zero,
                       blockIdx.x == 0);
    if (!cta_wait_copy(&bar, a.st, 40)) return;

    if (2 * warp >= nrows) return;
    float acc[2][NV];
    smem_dot<NV, 2>(wsm + size_t(2 * warp) * pitch, pitch, min(2u, nrows - 2 * warp), pitch / 16, xs, a.h, acc);
    if (!epi) return;
    const uint32_t v = lane;
    float e0 = 0.f, e1 = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k)
        if (k == int(v)) { e0 = acc[0][k]; e1 = acc[1][k]; }
    if (r < qrows + krows) {
        const float r0 = float(double(e0) * cs - double(e1) * sn);
        const float r1 = float(double(e0) * sn + double(e1) * cs);
        if (r < qrows) {
            a.q_out[size_t(v) * qrows + r] = r0;
            a.q_out[size_t(v) * qrows + r + 1] = r1;
        } else if (slot) {
            slot[0] = __float2half_rn(r0);
            slot[1] = __float2half_rn(r1);
        }
    } else if (slot) {
        slot[0] = __float2half_rn(e0);
        slot[1] = __float2half_rn(e1);
    }
}

// ---------------------------------------------------------------------------------------
// B: attention for one kv head + o_proj partial over that head's input columns.
constexpr uint32_t kBThreads = 256;
constexpr int kBWarps = kBThreads / 32;

struct AttnOArgs {
    const __half *w_o_blk;
    uint32_t h, n_heads, n_kv, rows_per_cta;
    const float *q;
    float scale_log2;
    KvParams kv;
    const int32_t *seq, *pos;
    long long *delta_out;   // residual delta the partial sums are added to
    long long *delta_zero;  // zeroed by the designated CTA for the next kernel
    DeviceStatus *st;
};

template <int NV, int HD, int G>
__global__ void __launch_bounds__(kBThreads) attn_oproj_kernel(AttnOArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ WarpStates<HD, G, kBWarps> ws;
    __shared__ __align__(16) float attn[NV][G * HD];
    constexpr uint32_t cols = G * HD, pitch = cols * 2;
    const uint32_t g = blockIdx.x, rb = blockIdx.y;
    const uint32_t row0 = rb * a.rows_per_cta;
    const uint32_t nrows = min(a.rows_per_cta, a.h - row0);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    uint8_t *wsm = smem;

    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_expect_tx(&bar, nrows * pitch);
        bulk_load(wsm, reinterpret_cast<const uint8_t *>(a.w_o_blk) + (size_t(g) * a.h + row0) * pitch,
                  nrows * pitch, &bar);
    }
    // Positions, sequence slots and their page-table rows are not written by the previous
    // kernel: stage them before waiting on it (page tables of up to kPtStage entries).
    constexpr uint32_t kPtStage = 256;
    __shared__ int32_t s_seq[NV], s_pos[NV];
    __shared__ int32_t s_pt[NV][kPtStage];
    const bool stage_pt = a.kv.max_pages <= kPtStage;
    if (threadIdx.x < NV) {
        s_seq[threadIdx.x] = a.seq[threadIdx.x];
        s_pos[threadIdx.x] = a.pos[threadIdx.x];
    }
    __syncthreads();
    if (stage_pt)
        for (uint32_t i = threadIdx.x; i < NV * a.kv.max_pages; i += blockDim.x) {
            const int32_t s = s_seq[i / a.kv.max_pages];
            s_pt[i / a.kv.max_pages][i % a.kv.max_pages] =
                s >= 0 ? a.kv.page_table[size_t(s) * a.kv.max_pages + i % a.kv.max_pages] : -1;
        }
    grid_dependency_wait();
    grid_dependents_launch();
    if (g == 0 && rb == 0)
        for (uint32_t i = threadIdx.x; i < NV * a.h; i += blockDim.x) a.delta_zero[i] = 0;
    __syncthreads();

    for (int v = 0; v < NV; ++v) {
        float qv[G][AttnShape<HD>::E];
        load_q_slice<HD, G>(a.q + size_t(v) * a.n_heads * HD, g, a.scale_log2, qv);
        AttnState<HD, G> st;
        st.init();
        const int32_t s = s_seq[v];
        KvView kv{reinterpret_cast<const __half *>(a.kv.pool),
                  stage_pt ? s_pt[v] : a.kv.page_table + size_t(max(s, 0)) * a.kv.max_pages,
                  a.kv.max_pages, a.kv.n_pages, a.kv.page_size, a.n_kv, g, s >= 0, a.kv.ring};
        attend_range<HD, G, false, true>(st, qv, kv, window_begin(s_pos[v], a.kv.page_size, a.kv.ring),
                                         uint32_t(max(s_pos[v] + 1, 0)), warp, kBWarps, a.st);
        merge_lane_groups<HD, G>(st);
        store_warp_state<HD, G, kBWarps>(st, ws, warp);
        __syncthreads();
        for (uint32_t idx = threadIdx.x; idx < cols; idx += blockDim.x) {
            float acc, m, l;
            merge_warps<HD, G, kBWarps>(ws, idx / HD, idx % HD, acc, m, l);
            attn[v][idx] = acc / fmaxf(l, 1e-30f);
        }
        __syncthreads();
    }
    if (!cta_wait_copy(&bar, a.st, 41)) return;
    // o_proj partial: rows of this CTA x this kv head's G*HD input columns.
    constexpr uint32_t nch = pitch / 16;
    for (uint32_t rr = warp; rr < nrows; rr += kBWarps) {
        float acc[NV];
#pragma unroll
        for (int v = 0; v < NV; ++v) acc[v] = 0.f;
        for (uint32_t c = lane; c < nch; c += 32) {
            float wf[8];
            unpack8(*reinterpret_cast<const uint4 *>(wsm + size_t(rr) * pitch + c * 16), wf);
#pragma unroll
            for (int v = 0; v < NV; ++v)
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[v] = fmaf(wf[e], attn[v][c * 8 + e], acc[v]);
        }
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            const float t = warp_sum(acc[v]);
            if (lane == uint32_t(v))
                atomicAdd(reinterpret_cast<unsigned long long *>(a.delta_out + size_t(v) * a.h + row0 + rr),
                          static_cast<unsigned long long>(to_fix(t)));
        }
    }
}

// ---------------------------------------------------------------------------------------
// C: RMSNorm + gate;up GEMV + SwiGLU + down_proj partial over a block of F rows of the
// intermediate dimension.
constexpr uint32_t kCThreads = 128;

struct MlpArgs {
    const __half *w_gu, *w_down_t;
    uint32_t h, ff, F;
    const __half *gain;
    float eps;
    const float *base_in;
    const long long *delta_in;
    float *base_out;
    long long *delta_out;
    DeviceStatus *st;
};

template <int NV>
__global__ void __launch_bounds__(kCThreads) mlp_fused_kernel(MlpArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bar;
    const uint32_t pitch = a.h * 2;
    const uint32_t f0 = blockIdx.x * a.F;
    const uint32_t nf = min(a.F, a.ff - f0);
    const uint32_t blk = a.F * pitch;
    uint8_t *wg = smem, *wu = smem + blk, *wd = smem + 2 * blk;
    float *xs = reinterpret_cast<float *>(smem + 3 * blk);
    float *red = xs + NV * a.h;
    float *hs = red + 33 * NV;  // [F][NV]

    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_expect_tx(&bar, 3 * nf * pitch);
        const uint8_t *w = reinterpret_cast<const uint8_t *>(a.w_gu);
        bulk_load(wg, w + size_t(f0) * pitch, nf * pitch, &bar);
        bulk_load(wu, w + (size_t(a.ff) + f0) * pitch, nf * pitch, &bar);
        bulk_load(wd, reinterpret_cast<const uint8_t *>(a.w_down_t) + size_t(f0) * pitch, nf * pitch, &bar);
    }
    GainPrefetch gpre;
    prefetch_gain<NV>(a.gain, a.h, gpre);
    grid_dependency_wait();
    grid_dependents_launch();
    stage_residual<NV>(a.base_in, a.delta_in, a.h, gpre, a.gain, a.eps, xs, red, a.base_out, nullptr,
                       blockIdx.x == 0);
    if (!cta_wait_copy(&bar, a.st, 42)) return;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, nw = kCThreads / 32;
    for (uint32_t f = warp; f < nf; f += nw) {
        float acc[1][NV], accu[1][NV];
        smem_dot<NV, 1>(wg + size_t(f) * pitch, pitch, 1, pitch / 16, xs, a.h, acc);
        smem_dot<NV, 1>(wu + size_t(f) * pitch, pitch, 1, pitch / 16, xs, a.h, accu);
        if (lane == 0) {
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                const float gv = acc[0][v], uv = accu[0][v];
                const float sg = 1.0f / (1.0f + expf(-gv));  // Opure_CpuReference.cpp:195
                hs[f * NV + v] = (gv * sg) * uv;
            }
        }
    }
    __syncthreads();
    // down_proj partial: out[o] = sum_f Wd^T[f][o] * h[f], every o of this block's f rows.
    const __half *wdh = reinterpret_cast<const __half *>(wd);
    for (uint32_t o = threadIdx.x; o < a.h; o += blockDim.x) {
        float acc[NV];
#pragma unroll
        for (int v = 0; v < NV; ++v) acc[v] = 0.f;
        for (uint32_t f = 0; f < nf; ++f) {
            const float wv = __half2float(wdh[size_t(f) * a.h + o]);
#pragma unroll
            for (int v = 0; v < NV; ++v) acc[v] = fmaf(wv, hs[f * NV + v], acc[v]);
        }
#pragma unroll
        for (int v = 0; v < NV; ++v)
            atomicAdd(reinterpret_cast<unsigned long long *>(a.delta_out + size_t(v) * a.h + o),
                      static_cast<unsigned long long>(to_fix(acc[v])));
    }
}

// ---------------------------------------------------------------------------------------
// L: final RMSNorm + lm_head GEMV + argmax keys (+ logits).
constexpr int kLRows = 4;
constexpr uint32_t kLThreads = 128;

struct LmArgs {
    const uint8_t *w;
    uint32_t vocab, h;
    const __half *gain;
    float eps;
    const float *base_in;
    const long long *delta_in;
    float *logits;
    unsigned long long *keys;
};

template <int NV>
__global__ void __launch_bounds__(kLThreads) lm_head_kernel(LmArgs a) {
    extern __shared__ __align__(16) float lsm[];
    float *xs = lsm;
    float *red = lsm + NV * a.h;
    __shared__ unsigned long long cta_best[kLThreads / 32][NV];
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t nwarps = gridDim.x * (kLThreads / 32);
    const uint32_t groups = (a.vocab + kLRows - 1) / kLRows;
    const uint32_t g0 = blockIdx.x * (kLThreads / 32) + warp;
    const size_t pitch = size_t(a.h) * 2;
    const uint32_t nchunks = uint32_t(pitch / 16);
    RowPrefetch<kLRows> pre;
    if (g0 < groups) prefetch_rows(pre, a.w, pitch, g0 * kLRows, min(uint32_t(kLRows), a.vocab - g0 * kLRows), nchunks);
    GainPrefetch gpre;
    prefetch_gain<NV>(a.gain, a.h, gpre);
    grid_dependency_wait();
    grid_dependents_launch();
    stage_residual<NV>(a.base_in, a.delta_in, a.h, gpre, a.gain, a.eps, xs, red, nullptr, nullptr, false);
    unsigned long long best[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) best[v] = 0ull;
    for (uint32_t g = g0; g < groups; g += nwarps) {
        const uint32_t row0 = g * kLRows;
        const uint32_t valid = min(uint32_t(kLRows), a.vocab - row0);
        float acc[kLRows][NV];
        dot_rows<OPURE_W_F16, NV, kLRows>(a.w, pitch, row0, valid, nchunks, xs, a.h, acc, pre, g == g0);
#pragma unroll
        for (int r = 0; r < kLRows; ++r)
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                if (r >= int(valid)) continue;
                const unsigned long long k = argmax_key(acc[r][v], row0 + r);
                best[v] = k > best[v] ? k : best[v];
                if (a.logits && lane == uint32_t((r * NV + v) & 31))
                    a.logits[size_t(v) * a.vocab + row0 + r] = acc[r][v];
            }
    }
    if (lane == 0)
#pragma unroll
        for (int v = 0; v < NV; ++v) cta_best[warp][v] = best[v];
    __syncthreads();
    if (threadIdx.x < NV) {
        unsigned long long b = 0ull;
        for (uint32_t w = 0; w < kLThreads / 32; ++w) b = cta_best[w][threadIdx.x] > b ? cta_best[w][threadIdx.x] : b;
        if (b) atomicMax(a.keys + threadIdx.x, b);
    }
}

// ---------------------------------------------------------------------------------------
// P: the whole step as ONE persistent cooperative kernel, one CTA per SM. Each layer runs
// the A, B and C phases above in turn, separated by grid-wide counters instead of kernel
// boundaries; every CTA's weight slices of layer L+2 are copied (TMA bulk, double-buffered
// per layer) while layers L+1 runs, and the lm_head follows the last layer. Data produced
// inside the kernel by other CTAs (q, the appended KV rows, residual sums) is read through
// L2 (ld.cg / atomics), never through the non-coherent path. Every wait is bounded (1 s):
// a CTA that gives up records DEVICE_TIMEOUT, raises the grid's abort flag (so the others
// leave their waits at once), waits for its own copies in flight and returns.
constexpr uint32_t kPThreads = 256;
constexpr int kPWarps = kPThreads / 32;
constexpr uint32_t kPMaxLayers = 48;
constexpr uint32_t kPtStageP = 256;
constexpr uint32_t kLmBufs = 16;
constexpr uint32_t kKvStageTokens = 256;

struct PLayer {
    const uint8_t *w_qkv, *w_o_blk, *w_gu, *w_down_t;
    const __half *in_norm, *post_norm;
    uint16_t *kv_pool;
    float s_q, s_k, s_v, s_o, s_gate, s_up, s_down;  // int8 tensor scales (1 for fp16)
};

struct PersistArgs {
    PLayer layers[kPMaxLayers];
    uint32_t n_layers, h, inter, n_heads, n_kv, hd, vocab;
    float eps, scale_log2;
    double theta;
    const __half *final_norm;
    const uint8_t *lm_head;
    const int32_t *page_table;
    uint32_t n_pages, max_pages, page_size, kv_ring;
    const int32_t *seq, *pos;
    float *base0, *base1;
    long long *delta0, *delta1;
    float *q, *logits;
    unsigned long long *keys;
    uint32_t *sync;   // [3 n_layers] barrier counters, then the abort flag; zero at launch
    DeviceStatus *st;
    uint32_t qkv_rows, a_ctas;  // A: kARows q;k;v rows per CTA
    uint32_t rows_b, rbs;       // B: CTA b < n_kv * rbs takes kv head b / rbs, o_proj row block b % rbs
    uint32_t F, c_ctas;         // C: F intermediate rows per CTA
    uint32_t slot_bytes, off_b, off_c;
    uint32_t lm_rows, lm_chunk, lm_nbuf;  // lm_head: rows per CTA, rows per TMA chunk, chunk buffers
    uint32_t lm_extra0;                   // first chunk buffer past the slots and KV stage (lm_nbuf: none)
    uint32_t lm_fixed;                    // bytes of the two layer slots + the KV stage
    uint32_t region_bytes;                // layer slots, KV stage / chunk buffers; the scratch follows
    uint32_t kv_cap, kv_off;              // KV stage: tokens per vector, byte offset (kv_cap 0: none)
    unsigned long long *trace;  // optional [grid][3 n_layers + 2][2] %globaltimer stamps, or NULL
};

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid-wide barrier k: every CTA arrives once; thread 0 waits (bounded) for all of them.
// Thread 0 runs `after_arrive` between its arrival and its wait: every thread of the CTA
// has finished the phase by then, so copies into shared memory read in that phase may start.
template <typename Hook>
__device__ bool grid_barrier(const PersistArgs &p, uint32_t k, int *s_ok, Hook &&after_arrive) {
    __syncthreads();
    // Phase trace: [k][0] = this CTA's arrival at barrier k, [k][1] = its release.
    unsigned long long *tr = p.trace ? p.trace + (size_t(blockIdx.x) * (3 * p.n_layers + 2) + k) * 2 : nullptr;
    if (threadIdx.x == 0 && tr) tr[0] = global_ns();
    if (threadIdx.x == 0) {
        uint32_t *ctr = p.sync + k;
        const uint32_t *abort_flag = p.sync + 3 * p.n_layers;
        // Release arrival: the CTA's writes (ordered before thread 0 by the barrier above)
        // are visible to every CTA that acquires the count; cheaper than a full fence.
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
        after_arrive();
        int ok = 1;
        const uint64_t t0 = global_ns();
        for (uint32_t i = 0;; ++i) {
            if (ld_acquire_gpu(ctr) >= gridDim.x) break;
            if ((i & 31u) == 31u) {
                if (ld_acquire_gpu(abort_flag)) {
                    ok = 0;
                    break;
                }
                if (global_ns() - t0 > 1000000000ull) {
                    report(p.st, OPURE_ERR_DEVICE_TIMEOUT, 50, k);
                    atomicExch(p.sync + 3 * p.n_layers, 1u);
                    ok = 0;
                    break;
                }
            }
        }
        *s_ok = ok;
        if (tr) tr[1] = global_ns();
    }
    __syncthreads();
    return *s_ok != 0;
}

__device__ __forceinline__ bool grid_barrier(const PersistArgs &p, uint32_t k, int *s_ok) {
    return grid_barrier(p, k, s_ok, [] {});
}

// This CTA's share of each phase (the same for every layer).
struct PShare {
    uint32_t na, a_row0;               // A rows
    uint32_t nb, g, b_row0;            // B: kv head, o_proj rows
    uint32_t nc, f0;                   // C intermediate rows
};

template <int HD, int G>
__device__ __forceinline__ PShare p_share(const PersistArgs &p) {
    PShare s{};
    const uint32_t b = blockIdx.x;
    if (b < p.a_ctas) {
        s.a_row0 = b * kARows;
        s.na = min(kARows, p.qkv_rows - s.a_row0);
    }
    if (b < p.n_kv * p.rbs) {
        s.g = b / p.rbs;
        s.b_row0 = (b % p.rbs) * p.rows_b;
        s.nb = s.b_row0 < p.h ? min(p.rows_b, p.h - s.b_row0) : 0;
    }
    if (b < p.c_ctas) {
        s.f0 = b * p.F;
        s.nc = s.f0 < p.inter ? min(p.F, p.inter - s.f0) : 0;
    }
    return s;
}

// EB: bytes per weight element (2 fp16, 1 int8).
template <int HD, int G, uint32_t EB>
__device__ __forceinline__ uint32_t p_bytes(const PersistArgs &p, const PShare &s) {
    return (s.na * p.h + s.nb * G * HD + 3 * s.nc * p.h) * EB;
}

// Thread 0: copy layer L's slices of this CTA into `slot`, completing on `bar`.
template <int HD, int G, uint32_t EB>
__device__ void p_issue(const PersistArgs &p, const PShare &s, uint32_t L, uint8_t *slot, uint64_t *bar) {
    const uint32_t bytes = p_bytes<HD, G, EB>(p, s);
    if (!bytes) return;
    const PLayer &ly = p.layers[L];
    const uint32_t pitch = p.h * EB, bpitch = G * HD * EB;
    // The slot was last read through the generic proxy; order that before the async writes.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_expect_tx(bar, bytes);
    if (s.na) bulk_load(slot, ly.w_qkv + size_t(s.a_row0) * pitch, s.na * pitch, bar);
    if (s.nb)
        bulk_load(slot + p.off_b, ly.w_o_blk + (size_t(s.g) * p.h + s.b_row0) * bpitch, s.nb * bpitch, bar);
    if (s.nc) {
        uint8_t *c = slot + p.off_c;
        bulk_load(c, ly.w_gu + size_t(s.f0) * pitch, s.nc * pitch, bar);
        bulk_load(c + p.F * pitch, ly.w_gu + (size_t(p.inter) + s.f0) * pitch, s.nc * pitch, bar);
        bulk_load(c + 2 * p.F * pitch, ly.w_down_t + size_t(s.f0) * pitch, s.nc * pitch, bar);
    }
}

// A position in the lm_head chunk order: q counts positions, m is q's index within its
// round k of lm_nbuf positions (kept incrementally: no divisions in the loop).
struct LmCursor {
    uint32_t q, m, k;
    __device__ __forceinline__ uint32_t buf(uint32_t rot, uint32_t nbuf) const {
        const uint32_t j = m + rot;
        return j >= nbuf ? j - nbuf : j;
    }
    __device__ __forceinline__ void next(uint32_t nbuf) {
        ++q;
        if (++m == nbuf) {
            m = 0;
            ++k;
        }
    }
};

// lm_head rows per warp and pass (chunk = kPWarps of them): eight for one vector (more
// independent dot products per pass; measured 20.8 -> 18.3 us for the config-0 lm_head),
// four for two, two for more (registers).
template <int NV>
constexpr uint32_t kLmRowsPerWarp = NV == 1 ? 8 : (NV <= 2 ? 4 : 2);

// Whole-CTA bounded wait on `bar` reaching the end of phase `parity`.
__device__ bool p_wait_slot(uint64_t *bar, uint32_t parity, const PersistArgs &p, int *s_ok) {
    if (threadIdx.x == 0) {
        *s_ok = 1;
        if (!mbar_wait(bar, parity)) {
            report(p.st, OPURE_ERR_DEVICE_TIMEOUT, 51, blockIdx.x);
            atomicExch(p.sync + 3 * p.n_layers, 1u);  // the others leave their barrier waits
            *s_ok = 0;
        }
    }
    __syncthreads();
    const bool ok = *s_ok != 0;
    if (ok) mbar_wait(bar, parity);  // every thread observes the completed phase
    return ok;
}

// Exact two-pass attention of one query vector over keys [0, T) of kv head g, for contexts
// that fit the shared-memory KV stage (T <= its capacity; hd 64). Rows [0, n_old) are
// already staged (copied a layer ahead); rows [n_old, T) were written by phase A of this
// layer and are fetched here first, in the same memory round trip as the query. Then the
// whole CTA computes every score (8 lanes per key), each head's max and exp sums (one warp
// per head), and the probability-weighted values (one thread per head and dimension pair,
// the keys split in halves): no running rescale and no merging of per-lane or per-warp
// states, which at decode lengths cost more than the arithmetic. Softmax in log2 units
// (q pre-scaled by scale * log2 e), fp32, as attend_range. Writes out[h * 64 + d] =
// sum_t p_t V[t][d] / max(sum_t p_t, 1e-30). sp: shared scratch of kTwoPassScratch floats.
constexpr uint32_t kTwoPassKeys = kKvStageTokens;
template <int G>
constexpr uint32_t kTwoPassScratch = G * kTwoPassKeys + 4 + G * 64;

template <int G>
__device__ __forceinline__ void attend_two_pass(const float *q, float scale_log2, __half *sk, __half *sv,
                                                uint32_t n_old, uint32_t T, const uint16_t *pool,
                                                const int32_t *pt_row, uint32_t page_size, uint32_t n_kv,
                                                uint32_t g, float *sp, float *out) {
    constexpr uint32_t HD = 64;
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const uint32_t sub = lane & 7u, grp = lane >> 3;
    // (1) Loads first: the q slice of this lane, then this step's K/V rows.
    float4 q4[G][2];
#pragma unroll
    for (int h = 0; h < G; ++h) {
        q4[h][0] = __ldcg(reinterpret_cast<const float4 *>(q + h * HD + sub * 8));
        q4[h][1] = __ldcg(reinterpret_cast<const float4 *>(q + h * HD + sub * 8 + 4));
    }
    const uint32_t items = (T - n_old) * 16;  // (row, K|V, 16-byte chunk)
    const size_t blk = size_t(page_size) * HD;
    for (uint32_t i0 = 0; i0 < items; i0 += kPThreads) {
        const uint32_t i = i0 + tid;
        if (i < items) {
            const uint32_t t = n_old + i / 16, sel = (i / 8) & 1u, c = i % 8;
            const int32_t page = pt_row[t / page_size];
            const uint4 val = ldcg_v4(pool + ((size_t(page) * 2 + sel) * n_kv + g) * blk + size_t(t % page_size) * HD + c * 8);
            *reinterpret_cast<uint4 *>((sel ? sv : sk) + size_t(t) * HD + c * 8) = val;
        }
    }
    float qf[G][8];
#pragma unroll
    for (int h = 0; h < G; ++h) {
        qf[h][0] = q4[h][0].x * scale_log2; qf[h][1] = q4[h][0].y * scale_log2;
        qf[h][2] = q4[h][0].z * scale_log2; qf[h][3] = q4[h][0].w * scale_log2;
        qf[h][4] = q4[h][1].x * scale_log2; qf[h][5] = q4[h][1].y * scale_log2;
        qf[h][6] = q4[h][1].z * scale_log2; qf[h][7] = q4[h][1].w * scale_log2;
    }
    __syncthreads();
    // (2) Scores: key t = (r * 8 + warp) * 4 + grp.
    float *S = sp;  // [G][kTwoPassKeys]
    for (uint32_t t0 = warp * 4; t0 < T; t0 += 32) {
        const uint32_t t = t0 + grp;
        const bool ok = t < T;
        float kf[8];
        unpack8(ok ? lds128(sk + size_t(t) * HD + sub * 8) : make_uint4(0, 0, 0, 0), kf);
#pragma unroll
        for (int h = 0; h < G; ++h) {
            float2 d2 = make_float2(0.f, 0.f);
#pragma unroll
            for (int e = 0; e < 8; e += 2)
                d2 = __ffma2_rn(make_float2(qf[h][e], qf[h][e + 1]), make_float2(kf[e], kf[e + 1]), d2);
            float d = d2.x + d2.y;
            d += __shfl_xor_sync(0xffffffffu, d, 4);
            d += __shfl_xor_sync(0xffffffffu, d, 2);
            d += __shfl_xor_sync(0xffffffffu, d, 1);
            if (sub == 0 && ok) S[h * kTwoPassKeys + t] = d;
        }
    }
    __syncthreads();
    // (3) Per head: max, probabilities in place, their sum.
    if (warp < uint32_t(G)) {
        float *Sh = S + warp * kTwoPassKeys;
        float m = -INFINITY;
        for (uint32_t t = lane; t < T; t += 32) m = fmaxf(m, Sh[t]);
        m = warp_max(m);
        float l = 0.f;
        for (uint32_t t = lane; t < T; t += 32) {
            const float pr = fast_exp2(Sh[t] - m);
            Sh[t] = pr;
            l += pr;
        }
        l = warp_sum(l);
        if (lane == 0) sp[G * kTwoPassKeys + warp] = l;
    }
    __syncthreads();
    // (4) Values: thread (half, head, dimension pair); each warp serves one head.
    const uint32_t n_items = G * 32, half = tid / n_items, item = tid % n_items;
    const uint32_t h = item / 32, dp = item % 32;
    float2 acc = make_float2(0.f, 0.f);
    if (half < 2) {
        const float *P = S + h * kTwoPassKeys;
        const uint32_t ta = half ? T / 2 : 0, tb = half ? T : T / 2;
        float2 a1 = make_float2(0.f, 0.f);
        uint32_t t = ta;
        for (; t + 1 < tb; t += 2) {
            const float p0 = P[t], p1 = P[t + 1];
            const float2 v0 = h2f2(*reinterpret_cast<const uint32_t *>(sv + size_t(t) * HD + 2 * dp));
            const float2 v1 = h2f2(*reinterpret_cast<const uint32_t *>(sv + size_t(t + 1) * HD + 2 * dp));
            acc.x = fmaf(p0, v0.x, acc.x);
            acc.y = fmaf(p0, v0.y, acc.y);
            a1.x = fmaf(p1, v1.x, a1.x);
            a1.y = fmaf(p1, v1.y, a1.y);
        }
        if (t < tb) {
            const float p0 = P[t];
            const float2 v0 = h2f2(*reinterpret_cast<const uint32_t *>(sv + size_t(t) * HD + 2 * dp));
            acc.x = fmaf(p0, v0.x, acc.x);
            acc.y = fmaf(p0, v0.y, acc.y);
        }
        acc.x += a1.x;
        acc.y += a1.y;
    }
    float *part = sp + G * kTwoPassKeys + 4;  // [G * 32][2]: the second halves
    if (half == 1) {
        part[2 * item] = acc.x;
        part[2 * item + 1] = acc.y;
    }
    __syncthreads();
    if (half == 0) {
        const float inv = 1.0f / fmaxf(sp[G * kTwoPassKeys + h], 1e-30f);
        out[h * HD + 2 * dp] = (acc.x + part[2 * item]) * inv;
        out[h * HD + 2 * dp + 1] = (acc.y + part[2 * item + 1]) * inv;
    }
    __syncthreads();
}

// Q8: the layer matrices are per-tensor int8 (GEMV_Quant, Opure_GEMV_Quant.usf:38-94): half
// the bytes per slice, each dot product scaled by its tensor's scale; the embedding, norms
// and lm_head stay fp16.
template <int NV, int HD, int G, bool Q8 = false>
__global__ void __launch_bounds__(kPThreads, 1) persistent_step_kernel(const __grid_constant__ PersistArgs p) {
    constexpr uint32_t EB = Q8 ? 1u : 2u;  // bytes per layer-weight element
    extern __shared__ __align__(1024) uint8_t psm[];
    __shared__ __align__(8) uint64_t full[2];
    __shared__ __align__(8) uint64_t lbar[kLmBufs];
    __shared__ __align__(8) uint64_t kvbar;
    __shared__ uint32_t s_nst[NV];
    __shared__ bool s_two[NV];  // this vector's attention runs attend_two_pass
    __shared__ int s_ok;
    __shared__ WarpStates<HD, G, kPWarps> ws;  // also attend_two_pass's scratch
    static_assert(sizeof(ws) >= kTwoPassScratch<G> * sizeof(float), "two-pass scratch does not fit");
    __shared__ int32_t s_seq[NV], s_pos[NV];
    __shared__ int32_t s_pt[NV][kPtStageP];
    __shared__ unsigned long long cta_best[kPWarps][NV];
    constexpr uint32_t cols_b = G * HD, bpitch = cols_b * EB;
    const uint32_t pitch = p.h * 2;      // lm_head rows (fp16)
    const uint32_t wpitch = p.h * EB;    // layer-weight rows of h elements
    uint8_t *slots[2] = {psm, psm + p.slot_bytes};
    float *xs = reinterpret_cast<float *>(psm + p.region_bytes);
    float *red = xs + NV * p.h;
    float *hs = red + ((33 * NV + 3) & ~3u);  // [F][NV], 16-byte aligned like every buffer here
    float *attn = hs + ((p.F * NV + 3) & ~3u);  // [NV][G*HD], 16-byte aligned
    float *gu = attn + NV * G * HD;             // [2F][NV] gate then up sums
    const uint32_t b = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const PShare sh = p_share<HD, G>(p);
    const bool has_bytes = p_bytes<HD, G, EB>(p, sh) != 0;
    const bool stage_pt = p.max_pages <= kPtStageP;
    const uint32_t qrows = p.n_heads * HD, krows = p.n_kv * HD;

    if (threadIdx.x == 0) {
        mbar_init(&full[0], 1);
        mbar_init(&full[1], 1);
        for (uint32_t j = 0; j < kLmBufs; ++j) mbar_init(&lbar[j], 1);
        mbar_init(&kvbar, 1);
    }
    // Sequences, positions and page tables are fixed for the step: stage them once.
    if (threadIdx.x < NV) {
        s_seq[threadIdx.x] = p.seq[threadIdx.x];
        s_pos[threadIdx.x] = p.pos[threadIdx.x];
    }
    __syncthreads();
    if (stage_pt)
        for (uint32_t i = threadIdx.x; i < NV * p.max_pages; i += blockDim.x) {
            const int32_t s = s_seq[i / p.max_pages];
            s_pt[i / p.max_pages][i % p.max_pages] =
                s >= 0 ? p.page_table[size_t(s) * p.max_pages + i % p.max_pages] : -1;
        }
    __syncthreads();
    // KV stage: the attention CTAs copy keys/values [0, s_nst[v]) of their kv head into
    // shared memory one layer ahead. Only rows written before this step qualify (below the
    // first position any vector of the sequence computes now), on pages that are valid.
    if (threadIdx.x < NV) {
        const int32_t sq = s_seq[threadIdx.x];
        int32_t first = s_pos[threadIdx.x];
        for (int u = 0; u < NV; ++u)
            if (s_seq[u] == sq) first = min(first, s_pos[u]);
        // (Not with a sliding window: the staged rows would start at the window.)
        uint32_t n = (sq >= 0 && stage_pt && sh.nb && first > 0 && !p.kv_ring) ? min(uint32_t(first), p.kv_cap) : 0u;
        for (uint32_t i = 0; i * p.page_size < n; ++i) {
            const int32_t pg = i < p.max_pages ? s_pt[threadIdx.x][i] : -1;
            if (pg < 0 || uint32_t(pg) >= p.n_pages) {
                n = i * p.page_size;  // the pool path reports the bad page
                break;
            }
        }
        s_nst[threadIdx.x] = n;
        // Two-pass attention when every key of the vector fits the stage on valid pages.
        const uint32_t T = uint32_t(max(s_pos[threadIdx.x] + 1, 0));
        bool two = HD == 64 && sq >= 0 && stage_pt && sh.nb && !p.kv_ring && T >= 1 && T <= p.kv_cap &&
                   T <= kTwoPassKeys && uint32_t(first) >= n && uint32_t(first) <= T;
        for (uint32_t i = 0; two && i * p.page_size < T; ++i) {
            const int32_t pg = i < p.max_pages ? s_pt[threadIdx.x][i] : -1;
            two = pg >= 0 && uint32_t(pg) < p.n_pages;
        }
        s_two[threadIdx.x] = two;
    }
    __syncthreads();
    uint32_t kv_total = 0;  // bytes per layer
#pragma unroll
    for (int v = 0; v < NV; ++v) kv_total += 2 * s_nst[v] * HD * 2;
    const bool kv_on = kv_total != 0;
    uint8_t *kvs = psm + p.kv_off;
    const uint32_t kv_vbytes = p.kv_cap * HD * 2;  // one vector's K (then V) rows
    auto kv_issue = [&](uint32_t L) {  // thread 0
        const uint16_t *pool = p.layers[L].kv_pool;
        const size_t blk = size_t(p.page_size) * HD;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect_tx(&kvbar, kv_total);
        for (int v = 0; v < NV; ++v)
            for (uint32_t t0 = 0; t0 < s_nst[v]; t0 += p.page_size) {
                const uint32_t nr = min(p.page_size, s_nst[v] - t0);
                const size_t kofs = (size_t(s_pt[v][t0 / p.page_size]) * 2 * p.n_kv + sh.g) * blk;
                uint8_t *dk = kvs + size_t(v) * 2 * kv_vbytes + size_t(t0) * HD * 2;
                bulk_load_keep(dk, pool + kofs, nr * HD * 2, &kvbar);
                bulk_load_keep(dk + kv_vbytes, pool + kofs + size_t(p.n_kv) * blk, nr * HD * 2, &kvbar);
            }
    };
    uint32_t kv_issued = 0, kv_waited = 0;  // layers
    if (kv_on && p.n_layers) {
        if (threadIdx.x == 0) kv_issue(0);
        kv_issued = 1;
    }
    uint32_t issued = 0, waited = 0;
    // Trace rows 3 n_layers (kernel start, in [1]) and 3 n_layers + 1 (end, in [0]).
    unsigned long long *trow = p.trace ? p.trace + size_t(blockIdx.x) * (3 * p.n_layers + 2) * 2 : nullptr;
    if (threadIdx.x == 0 && trow) trow[3 * p.n_layers * 2 + 1] = global_ns();
    if (threadIdx.x == 0) {
        for (uint32_t L = 0; L < 2 && L < p.n_layers; ++L) p_issue<HD, G, EB>(p, sh, L, slots[L], &full[L]);
    }
    issued = min(2u, p.n_layers);
    __syncthreads();

    // RoPE angles and KV-row offsets depend only on the step's positions: resolved once
    // for all layers (lane v < NV of each A warp owns vector v of its row pair).
    const bool fast_stage = stage_residual_fits<NV>(p.h);
    const uint32_t a_r = sh.a_row0 + 2 * warp;
    const bool a_epi = sh.na && 2 * warp < sh.na && lane < NV;
    double a_sn = 0.0, a_cs = 1.0;
    long long a_kv = -1;  // element offset of this lane's K or V pair inside a layer pool
    if (a_epi) {
        const int32_t ps = s_pos[lane], sq = s_seq[lane];
        if (a_r < qrows + krows)
            sincos(double(ps) * pow(p.theta, -2.0 * double((a_r % HD) / 2) / double(HD)), &a_sn, &a_cs);
        if (a_r >= qrows) {
            const bool is_k = a_r < qrows + krows;
            const uint32_t rr = is_k ? a_r - qrows : a_r - qrows - krows;
            const KvParams k0{nullptr, p.page_table, p.n_pages, p.max_pages, p.page_size, p.kv_ring};
            const long long off = kv_offset(k0, p.n_kv, HD, sq, ps, is_k ? 0 : 1, rr / HD, p.st);
            if (off >= 0) a_kv = off + rr % HD;
        }
    }

    // lm_head: this CTA's contiguous rows, streamed by TMA in chunks of lm_chunk rows
    // through lm_nbuf buffers. Buffers lm_extra0.. lie past the two layer slots and the KV
    // stage and are filled at kernel start; the others overlay those and are filled once
    // they are free. Chunks are issued and consumed in one order of positions q: buffer
    // (q + lm_extra0) % lm_nbuf in round q / lm_nbuf (the early buffers come first), holding
    // chunk buffer + round * lm_nbuf when that exists.
    const uint32_t lm_r0 = min(p.vocab, b * p.lm_rows), lm_r1 = min(p.vocab, lm_r0 + p.lm_rows);
    const uint32_t lm_nchunks = (lm_r1 - lm_r0 + p.lm_chunk - 1) / p.lm_chunk;
    const uint32_t lm_cbytes = p.lm_chunk * pitch;
    const uint32_t lm_rot = p.lm_extra0 % p.lm_nbuf;
    const uint32_t lm_npos = (lm_nchunks + p.lm_nbuf - 1) / p.lm_nbuf * p.lm_nbuf;
    LmCursor lm_iss{}, lm_dn{};  // next position to issue / to consume
    auto lm_issue = [&](uint32_t j, uint32_t c) {  // thread 0: chunk c into buffer j
        const uint32_t r0 = lm_r0 + c * p.lm_chunk, nr = min(p.lm_chunk, lm_r1 - r0);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect_tx(&lbar[j], nr * pitch);
        bulk_load(psm + size_t(j) * lm_cbytes, p.lm_head + size_t(r0) * pitch, nr * pitch, &lbar[j]);
    };
    // May buffer j be filled now? stage 0: kernel start (past the slots and KV stage only);
    // 1: last layer (also the slot of layer n_layers - 2); 2: after the last layer (any).
    auto lm_free = [&](uint32_t j, int stage) {
        const size_t lo = size_t(j) * lm_cbytes, hi = lo + lm_cbytes;
        if (stage == 2 || lo >= p.lm_fixed) return true;
        const uint32_t fs = p.n_layers & 1u;
        return stage == 1 && p.n_layers >= 2 && lo >= size_t(fs) * p.slot_bytes && hi <= size_t(fs + 1) * p.slot_bytes;
    };
    // Issues the next positions in order while each one's buffer is free: its previous
    // position consumed and the stage allowing it. Every thread keeps the same counters.
    auto lm_fill = [&](int stage) {
        while (lm_iss.q < lm_npos && lm_iss.q < lm_dn.q + p.lm_nbuf) {
            const uint32_t j = lm_iss.buf(lm_rot, p.lm_nbuf), c = j + lm_iss.k * p.lm_nbuf;
            if (!lm_free(j, stage)) break;
            if (threadIdx.x == 0 && c < lm_nchunks) lm_issue(j, c);
            lm_iss.next(p.lm_nbuf);
        }
    };
    lm_fill(0);

    for (uint32_t L = 0; L < p.n_layers; ++L) {
        const PLayer &ly = p.layers[L];
        uint8_t *sl = slots[L & 1];
        if (has_bytes && !p_wait_slot(&full[L & 1], (L >> 1) & 1u, p, &s_ok)) goto abort;
        ++waited;
        if (L + 1 == p.n_layers) lm_fill(1);  // the other slot is free for the rest of the step
        const KvParams kvp{ly.kv_pool, p.page_table, p.n_pages, p.max_pages, p.page_size, p.kv_ring};

        // ---- A: RMSNorm + q;k;v + RoPE + KV append ----------------------------------
        if (sh.na) {
            GainPrefetch gpre;
            prefetch_gain<NV>(ly.in_norm, p.h, gpre);
            if (fast_stage)
                stage_residual_fast<NV>(p.base0, L == 0 ? nullptr : p.delta1, p.h, gpre, ly.in_norm, p.eps, xs, red,
                                        b == 0 ? p.base1 : nullptr, b == 0 ? p.delta0 : nullptr, b == 0);
            else
                stage_residual<NV>(p.base0, L == 0 ? nullptr : p.delta1, p.h, gpre, ly.in_norm, p.eps, xs, red,
                                   b == 0 ? p.base1 : nullptr, b == 0 ? p.delta0 : nullptr, b == 0);
            if (2 * warp < sh.na) {
                float acc[2][NV];
                smem_dot<NV, 2, Q8>(sl + size_t(2 * warp) * wpitch, wpitch, min(2u, sh.na - 2 * warp), wpitch / 16,
                                    xs, p.h, acc);
                if (a_epi) {
                    const uint32_t v = lane, r = a_r;
                    // A RoPE pair never straddles the q | k | v boundaries (multiples of HD).
                    const float sc = !Q8 ? 1.0f : (r < qrows ? ly.s_q : (r < qrows + krows ? ly.s_k : ly.s_v));
                    float e0 = 0.f, e1 = 0.f;
#pragma unroll
                    for (int k = 0; k < NV; ++k)
                        if (k == int(v)) {
                            e0 = acc[0][k] * sc;
                            e1 = acc[1][k] * sc;
                        }
                    __half *slot = a_kv >= 0 ? reinterpret_cast<__half *>(ly.kv_pool) + a_kv : nullptr;
                    if (r < qrows + krows) {
                        // RoPE, interleaved pairs, theta^(-2*pair/hd) (Opure_RoPE.usf:56), in double.
                        const float r0 = float(double(e0) * a_cs - double(e1) * a_sn);
                        const float r1 = float(double(e0) * a_sn + double(e1) * a_cs);
                        if (r < qrows) {
                            p.q[size_t(v) * qrows + r] = r0;
                            p.q[size_t(v) * qrows + r + 1] = r1;
                        } else if (slot) {
                            slot[0] = __float2half_rn(r0);
                            slot[1] = __float2half_rn(r1);
                        }
                    } else if (slot) {
                        slot[0] = __float2half_rn(e0);
                        slot[1] = __float2half_rn(e1);
                    }
                }
            }
        }
        if (!grid_barrier(p, 3 * L, &s_ok)) goto abort;

        // ---- B: attention of kv head g + o_proj partial sums ------------------------
        if (b == 0)
            for (uint32_t i = threadIdx.x; i < NV * p.h; i += blockDim.x) p.delta1[i] = 0;
        if (sh.nb) {
            if (kv_on) {
                if (!p_wait_slot(&kvbar, L & 1u, p, &s_ok)) goto abort;
                ++kv_waited;
            }
            for (int v = 0; v < NV; ++v) {
                if constexpr (HD == 64) {
                    if (s_two[v]) {
                        attend_two_pass<G>(p.q + size_t(v) * qrows + size_t(sh.g) * G * HD, p.scale_log2,
                                           reinterpret_cast<__half *>(kvs + size_t(v) * 2 * kv_vbytes),
                                           reinterpret_cast<__half *>(kvs + size_t(v) * 2 * kv_vbytes + kv_vbytes),
                                           s_nst[v], uint32_t(s_pos[v] + 1), ly.kv_pool, s_pt[v], p.page_size, p.n_kv,
                                           sh.g, reinterpret_cast<float *>(&ws), attn + v * cols_b);
                        continue;
                    }
                }
                using S = AttnShape<HD>;
                float qv[G][S::E];
                const uint32_t sub = lane % S::LPT;
#pragma unroll
                for (int hh = 0; hh < G; ++hh) {
                    const float4 *qr = reinterpret_cast<const float4 *>(
                        p.q + size_t(v) * qrows + (size_t(sh.g) * G + hh) * HD + sub * S::E);
#pragma unroll
                    for (int e = 0; e < S::E / 4; ++e) {
                        const float4 t = __ldcg(qr + e);
                        qv[hh][4 * e] = t.x * p.scale_log2;
                        qv[hh][4 * e + 1] = t.y * p.scale_log2;
                        qv[hh][4 * e + 2] = t.z * p.scale_log2;
                        qv[hh][4 * e + 3] = t.w * p.scale_log2;
                    }
                }
                AttnState<HD, G> st;
                st.init();
                const int32_t s = s_seq[v];
                KvView kv{reinterpret_cast<const __half *>(ly.kv_pool),
                          stage_pt ? s_pt[v] : p.page_table + size_t(max(s, 0)) * p.max_pages,
                          p.max_pages, p.n_pages, p.page_size, p.n_kv, sh.g, s >= 0, p.kv_ring};
                const KvStage stg{reinterpret_cast<const __half *>(kvs + size_t(v) * 2 * kv_vbytes),
                                  reinterpret_cast<const __half *>(kvs + size_t(v) * 2 * kv_vbytes + kv_vbytes),
                                  s_nst[v]};
                // Two rounds per softmax block: the keys come from shared memory (short
                // latency), and fewer K/V rows in flight keep the kernel's registers from spilling.
                attend_range<HD, G, true, true, true, 2>(st, qv, kv, window_begin(s_pos[v], p.page_size, p.kv_ring),
                                                      uint32_t(max(s_pos[v] + 1, 0)), warp, kPWarps, p.st, stg);
                merge_lane_groups<HD, G>(st);
                store_warp_state<HD, G, kPWarps>(st, ws, warp);
                __syncthreads();
                for (uint32_t idx = threadIdx.x; idx < cols_b; idx += blockDim.x) {
                    float acc, m, l;
                    merge_warps<HD, G, kPWarps>(ws, idx / HD, idx % HD, acc, m, l);
                    attn[v * cols_b + idx] = acc / fmaxf(l, 1e-30f);
                }
                __syncthreads();
            }
            const uint8_t *wsm = sl + p.off_b;
            constexpr uint32_t nch = bpitch / 16;
            // Rows rr and rr + kPWarps of a warp in one pass (the attention chunk is read once).
            for (uint32_t rr = warp; rr < sh.nb; rr += 2 * kPWarps) {
                const bool two = rr + kPWarps < sh.nb;
                float acc[2][NV];
#pragma unroll
                for (int v = 0; v < NV; ++v) acc[0][v] = acc[1][v] = 0.f;
                constexpr int E = RowChunk<Q8>::E;
                for (uint32_t c = lane; c < nch; c += 32) {
                    float wf[2][E];
                    RowChunk<Q8>::unpack(lds128(wsm + size_t(rr) * bpitch + c * 16), wf[0]);
                    if (two) RowChunk<Q8>::unpack(lds128(wsm + size_t(rr + kPWarps) * bpitch + c * 16), wf[1]);
#pragma unroll
                    for (int v = 0; v < NV; ++v) {
                        float av[E];
#pragma unroll
                        for (int q = 0; q < E / 4; ++q) {
                            const float4 a = lds_f4(attn + v * cols_b + c * E + 4 * q);
                            av[4 * q] = a.x; av[4 * q + 1] = a.y; av[4 * q + 2] = a.z; av[4 * q + 3] = a.w;
                        }
#pragma unroll
                        for (int e = 0; e < E; ++e) acc[0][v] = fmaf(wf[0][e], av[e], acc[0][v]);
                        if (two)
#pragma unroll
                            for (int e = 0; e < E; ++e) acc[1][v] = fmaf(wf[1][e], av[e], acc[1][v]);
                    }
                }
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    if (r == 1 && !two) break;
#pragma unroll
                    for (int v = 0; v < NV; ++v) {
                        const float t = warp_sum(acc[r][v]) * (Q8 ? ly.s_o : 1.0f);
                        if (lane == uint32_t(v))
                            atomicAdd(reinterpret_cast<unsigned long long *>(p.delta0 + size_t(v) * p.h + sh.b_row0 +
                                                                             rr + r * kPWarps),
                                      static_cast<unsigned long long>(to_fix(t)));
                    }
                }
            }
        }
        {
            // Arrived: this CTA's KV stage is read; thread 0 starts the next layer's copy.
            const bool next_kv = kv_on && L + 1 < p.n_layers;
            const bool ok = grid_barrier(p, 3 * L + 1, &s_ok, [&] {
                if (next_kv) kv_issue(L + 1);
            });
            kv_issued += next_kv ? 1u : 0u;
            if (!ok) goto abort;
        }

        // ---- C: RMSNorm + gate;up + SwiGLU + down partial sums ----------------------
        if (sh.nc) {
            GainPrefetch gpre;
            prefetch_gain<NV>(ly.post_norm, p.h, gpre);
            if (fast_stage)
                stage_residual_fast<NV>(p.base1, p.delta0, p.h, gpre, ly.post_norm, p.eps, xs, red,
                                        b == 0 ? p.base0 : nullptr, nullptr, b == 0);
            else
                stage_residual<NV>(p.base1, p.delta0, p.h, gpre, ly.post_norm, p.eps, xs, red,
                                   b == 0 ? p.base0 : nullptr, nullptr, b == 0);
            const uint8_t *wg = sl + p.off_c, *wd = wg + 2 * p.F * wpitch;
            // The 2 nc dot products (gate rows f, then up rows f), three rows per warp and
            // pass; SwiGLU once every warp's sums are in shared memory.
            const uint32_t ngu = 2 * sh.nc;
            for (uint32_t j0 = warp; j0 < ngu; j0 += 3 * kPWarps) {
                const uint8_t *rows[3];
                uint32_t nr = 0;
#pragma unroll
                for (int i = 0; i < 3; ++i) {
                    const uint32_t j = j0 + i * kPWarps;
                    rows[i] = wg + size_t(j < sh.nc ? j : p.F + (j - sh.nc)) * wpitch;
                    if (j < ngu) nr = i + 1;
                }
                float acc[3][NV];
                smem_dot_ptrs<NV, 3, Q8>(rows, nr, wpitch / 16, xs, p.h, acc);
                if (lane == 0)
#pragma unroll
                    for (int i = 0; i < 3; ++i)
                        if (i < int(nr)) {
                            const uint32_t j = j0 + i * kPWarps;
                            const float sc = !Q8 ? 1.0f : (j < sh.nc ? ly.s_gate : ly.s_up);
#pragma unroll
                            for (int v = 0; v < NV; ++v) gu[j * NV + v] = acc[i][v] * sc;
                        }
            }
            __syncthreads();
            for (uint32_t i = threadIdx.x; i < sh.nc * NV; i += blockDim.x) {
                const uint32_t f = i / NV, v = i % NV;
                const float gv = gu[f * NV + v], uv = gu[(sh.nc + f) * NV + v];
                const float sg = 1.0f / (1.0f + expf(-gv));  // Opure_CpuReference.cpp:195
                hs[f * NV + v] = (gv * sg) * uv;
            }
            __syncthreads();
            const __half *wdh = reinterpret_cast<const __half *>(wd);
            for (uint32_t o = threadIdx.x; o < p.h; o += blockDim.x) {
                float acc[NV];
#pragma unroll
                for (int v = 0; v < NV; ++v) acc[v] = 0.f;
                for (uint32_t f = 0; f < sh.nc; ++f) {
                    const float wv = Q8 ? lds_s8(wd + size_t(f) * p.h + o) : lds_h(wdh + size_t(f) * p.h + o);
#pragma unroll
                    for (int v = 0; v < NV; ++v) acc[v] = fmaf(wv, lds_f32(hs + f * NV + v), acc[v]);
                }
#pragma unroll
                for (int v = 0; v < NV; ++v)
                    atomicAdd(reinterpret_cast<unsigned long long *>(p.delta1 + size_t(v) * p.h + o),
                              static_cast<unsigned long long>(to_fix(acc[v] * (Q8 ? ly.s_down : 1.0f))));
            }
        }
        if (L + 1 == p.n_layers) {
            __syncthreads();
            lm_fill(2);  // both slots are free now
        }
        {
            // Arrived: this slot's layer is done; thread 0 starts copying layer L+2 into it.
            const bool refill = L + 2 < p.n_layers;
            const bool ok = grid_barrier(p, 3 * L + 2, &s_ok, [&] {
                if (refill) p_issue<HD, G, EB>(p, sh, L + 2, sl, &full[L & 1]);
            });
            issued += refill ? 1u : 0u;
            if (!ok) goto abort;
        }
    }

    {
        // ---- L: final RMSNorm + lm_head + argmax keys (+ logits) ---------------------
        GainPrefetch gpre;
        prefetch_gain<NV>(p.final_norm, p.h, gpre);
        if (fast_stage)
            stage_residual_fast<NV>(p.base0, p.delta1, p.h, gpre, p.final_norm, p.eps, xs, red, nullptr, nullptr,
                                    false);
        else
            stage_residual<NV>(p.base0, p.delta1, p.h, gpre, p.final_norm, p.eps, xs, red, nullptr, nullptr, false);
        unsigned long long best[NV];
#pragma unroll
        for (int v = 0; v < NV; ++v) best[v] = 0ull;
        constexpr uint32_t RW = kLmRowsPerWarp<NV>;
        while (lm_dn.q < lm_npos) {
            const uint32_t j = lm_dn.buf(lm_rot, p.lm_nbuf), c = j + lm_dn.k * p.lm_nbuf;
            if (c < lm_nchunks) {
                if (!p_wait_slot(&lbar[j], lm_dn.k & 1u, p, &s_ok)) goto abort;
                const uint32_t r0 = lm_r0 + c * p.lm_chunk, nr = min(p.lm_chunk, lm_r1 - r0);
                const uint8_t *buf = psm + size_t(j) * lm_cbytes;
                if constexpr (NV == 1) {
                    static_assert(RW == 8, "lm_dot8 takes eight rows per warp");
                    const uint32_t row = (lane >> 2) & 7u;
                    for (uint32_t rr = RW * warp; rr < nr; rr += RW * kPWarps) {
                        const float sum = lm_dot8(buf + size_t(rr) * pitch, pitch, min(RW, nr - rr), pitch / 16, xs);
                        if (rr + row < nr) {
                            const unsigned long long k = argmax_key(sum, r0 + rr + row);
                            best[0] = k > best[0] ? k : best[0];
                            if (p.logits && (lane & 3u) == 0) p.logits[r0 + rr + row] = sum;
                        }
                    }
                } else {
                    for (uint32_t rr = RW * warp; rr < nr; rr += RW * kPWarps) {
                        float acc[RW][NV];
                        smem_dot<NV, RW>(buf + size_t(rr) * pitch, pitch, min(RW, nr - rr), pitch / 16, xs, p.h, acc);
#pragma unroll
                        for (int r = 0; r < int(RW); ++r)
#pragma unroll
                            for (int v = 0; v < NV; ++v) {
                                if (rr + r >= nr) continue;
                                const unsigned long long k = argmax_key(acc[r][v], r0 + rr + r);
                                best[v] = k > best[v] ? k : best[v];
                                if (p.logits && lane == uint32_t((r * NV + v) & 31))
                                    p.logits[size_t(v) * p.vocab + r0 + rr + r] = acc[r][v];
                            }
                    }
                }
                __syncthreads();  // buffer j read by every warp: refill it
            }
            lm_dn.next(p.lm_nbuf);
            lm_fill(2);
        }
        if constexpr (NV == 1)  // lm_dot8 leaves each lane the keys of its own rows
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long k = __shfl_xor_sync(0xffffffffu, best[0], o);
                best[0] = k > best[0] ? k : best[0];
            }
        if (lane == 0)
#pragma unroll
            for (int v = 0; v < NV; ++v) cta_best[warp][v] = best[v];
        __syncthreads();
        if (threadIdx.x < NV) {
            unsigned long long bb = 0ull;
            for (uint32_t w = 0; w < kPWarps; ++w) bb = cta_best[w][threadIdx.x] > bb ? cta_best[w][threadIdx.x] : bb;
            if (bb) atomicMax(p.keys + threadIdx.x, bb);
        }
        if (threadIdx.x == 0 && trow) trow[(3 * p.n_layers + 1) * 2] = global_ns();
    }
    return;

abort:
    // Leave no copy in flight into this CTA's shared memory (bounded waits).
    if (threadIdx.x == 0) {
        if (has_bytes)
            for (uint32_t L = waited; L < issued; ++L) mbar_wait(&full[L & 1], (L >> 1) & 1u);
        for (uint32_t l = kv_waited; l < kv_issued; ++l) mbar_wait(&kvbar, l & 1u);
        for (LmCursor c = lm_dn; c.q < lm_iss.q; c.next(p.lm_nbuf)) {
            const uint32_t j = c.buf(lm_rot, p.lm_nbuf);
            if (j + c.k * p.lm_nbuf < lm_nchunks) mbar_wait(&lbar[j], c.k & 1u);
        }
    }
}

// ---------------------------------------------------------------------------------------
template <typename K>
opure_status allow_smem(K k, size_t bytes) {
    if (bytes <= 48 * 1024) return OPURE_OK;
    const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
    return e == cudaSuccess ? OPURE_OK : cuda_status(e);
}

template <int NV, int HD, int G>
opure_status run_step(opure_ctx *ctx, const opure_fused_step &s) {
    const uint32_t h = s.hidden, hd = s.head_dim;
    const uint32_t qkv_rows = (s.n_heads + 2 * s.n_kv) * hd;
    const KvParams kvp0{nullptr, s.page_table, s.n_pages, s.max_pages, s.page_size, s.kv_ring};
    const size_t a_smem = ((kARows * h * 2 + 127) & ~size_t(127)) + (NV * h + 33 * NV) * 4;
    // B: about one CTA per SM over (kv head, o_proj row block).
    const uint32_t rb_target = std::max<uint32_t>(1, uint32_t(ctx->sm_count) / s.n_kv);
    const uint32_t rows_b = std::max<uint32_t>(1, (h + rb_target - 1) / rb_target);
    const uint32_t rb = (h + rows_b - 1) / rows_b;
    const size_t b_smem = size_t(rows_b) * G * HD * 2;
    // C: blocks of F intermediate rows, F chosen so the three weight slices fit.
    uint32_t F = 16;
    while (F > 1 && 3ull * F * h * 2 > 160 * 1024) F /= 2;
    const size_t c_smem = 3ull * F * h * 2 + (NV * h + 33 * NV + F * NV) * 4;
    const size_t l_smem = (NV * h + 33 * NV) * 4;
    opure_status st;
    if ((st = allow_smem(qkv_fused_kernel<NV>, a_smem))) return st;
    if ((st = allow_smem(attn_oproj_kernel<NV, HD, G>, b_smem))) return st;
    if ((st = allow_smem(mlp_fused_kernel<NV>, c_smem))) return st;
    if ((st = allow_smem(lm_head_kernel<NV>, l_smem))) return st;

    float *base[2] = {s.x, s.base1};
    long long *delta[2] = {s.delta0, s.delta1};
    for (uint32_t L = 0; L < s.n_layers; ++L) {
        const opure_fused_layer &ly = s.layers[L];
        KvParams kvp = kvp0;
        kvp.pool = ly.kv_pool;
        // A: x = base0 + delta1 (layer 0: the embedding in base0) -> base1; zero delta0.
        QkvArgs qa{reinterpret_cast<const __half *>(ly.w_qkv), qkv_rows, h, s.n_heads, s.n_kv, hd,
                   reinterpret_cast<const __half *>(ly.in_norm), s.eps, s.theta, base[0],
                   L == 0 ? nullptr : delta[1], base[1], delta[0], s.q, kvp, s.seq, s.pos, ctx->status};
        if ((st = launch(ctx, qkv_fused_kernel<NV>, dim3((qkv_rows + kARows - 1) / kARows), dim3(kAThreads),
                         a_smem, true, qa)))
            return st;
        // B: attention + o_proj partials into delta0; zero delta1.
        AttnOArgs ba{reinterpret_cast<const __half *>(ly.w_o_blk), h, s.n_heads, s.n_kv, rows_b, s.q,
                     s.attn_scale * 1.4426950408889634f, kvp, s.seq, s.pos, delta[0], delta[1], ctx->status};
        if ((st = launch(ctx, attn_oproj_kernel<NV, HD, G>, dim3(s.n_kv, rb), dim3(kBThreads), b_smem, true, ba)))
            return st;
        // C: x = base1 + delta0 -> base0; MLP partials into delta1.
        MlpArgs ca{reinterpret_cast<const __half *>(ly.w_gate_up), reinterpret_cast<const __half *>(ly.w_down_t),
                   h, s.inter, F, reinterpret_cast<const __half *>(ly.post_norm), s.eps, base[1], delta[0],
                   base[0], delta[1], ctx->status};
        if ((st = launch(ctx, mlp_fused_kernel<NV>, dim3((s.inter + F - 1) / F), dim3(kCThreads), c_smem, true, ca)))
            return st;
    }
    // L: x = base0 + delta1.
    LmArgs la{reinterpret_cast<const uint8_t *>(s.lm_head), s.vocab, h,
              reinterpret_cast<const __half *>(s.final_norm), s.eps, base[0], delta[1], s.logits, s.keys};
    const uint32_t groups = (s.vocab + kLRows - 1) / kLRows;
    const uint32_t ctas = std::min<uint32_t>((groups + 3) / 4, uint32_t(ctx->sm_count) * 8);
    return launch(ctx, lm_head_kernel<NV>, dim3(ctas), dim3(kLThreads), l_smem, true, la);
}

// The persistent kernel when this model and batch fit it: every phase's work in one wave
// of CTAs (one per SM) and a layer's slices of one CTA, double-buffered, in shared memory.
// Sets *ran; returns an error only for a failed launch.
template <int NV, int HD, int G, bool Q8>
opure_status run_persistent(opure_ctx *ctx, const opure_fused_step &s, bool *ran) {
    *ran = false;
    if (!s.sync || s.n_layers > kPMaxLayers || s.head_dim != HD) return OPURE_OK;
    const uint32_t grid = uint32_t(ctx->sm_count);
    const uint32_t h = s.hidden;
    PersistArgs p{};
    p.qkv_rows = (s.n_heads + 2 * s.n_kv) * HD;
    p.a_ctas = (p.qkv_rows + kARows - 1) / kARows;
    const uint32_t rb_target = std::max<uint32_t>(1, grid / s.n_kv);
    p.rows_b = (h + rb_target - 1) / rb_target;
    p.rbs = (h + p.rows_b - 1) / p.rows_b;
    p.F = (s.inter + grid - 1) / grid;
    p.c_ctas = (s.inter + p.F - 1) / p.F;
    if (p.a_ctas > grid || s.n_kv * p.rbs > grid || p.c_ctas > grid) return OPURE_OK;
    const uint32_t pitch = h * 2;                 // lm_head rows (fp16)
    const uint32_t eb = Q8 ? 1u : 2u, wpitch = h * eb;  // layer-weight rows
    p.off_b = (kARows * wpitch + 127) & ~127u;
    p.off_c = (p.off_b + p.rows_b * G * HD * eb + 127) & ~127u;
    p.slot_bytes = (p.off_c + 3 * p.F * wpitch + 1023) & ~1023u;
    const size_t scratch =
        (size_t(NV) * h + ((33 * NV + 3) & ~3u) + ((p.F * NV + 3) & ~3u) + size_t(NV) * G * HD + 2 * size_t(p.F) * NV) *
        4;
    auto kern = persistent_step_kernel<NV, HD, G, Q8>;
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) return OPURE_ERR_CUDA;
    // Shared memory left for the slots / lm_head chunk buffers beside the scratch.
    const size_t fixed = scratch + fa.sharedSizeBytes + 1024;
    if (fixed + 2 * size_t(p.slot_bytes) > ctx->smem_optin) return OPURE_OK;
    const size_t region_max = (ctx->smem_optin - fixed) & ~size_t(127);
    // KV stage: up to kKvStageTokens keys and values per vector, as far as they fit.
    const size_t kv_tok = size_t(NV) * 2 * HD * 2;
    p.kv_off = 2 * p.slot_bytes;
    p.kv_cap = uint32_t(std::min<size_t>(kKvStageTokens, (region_max - 2 * size_t(p.slot_bytes)) / kv_tok)) & ~15u;
    p.lm_fixed = uint32_t((2 * size_t(p.slot_bytes) + p.kv_cap * kv_tok + 127) & ~size_t(127));
    p.lm_rows = (s.vocab + grid - 1) / grid;
    p.lm_chunk = kLmRowsPerWarp<NV> * kPWarps;
    const uint32_t cbytes = p.lm_chunk * pitch;
    p.lm_nbuf = uint32_t(std::min<size_t>(kLmBufs, region_max / cbytes));
    if (p.lm_nbuf < 2) return OPURE_OK;
    p.lm_extra0 = std::min<uint32_t>(p.lm_nbuf, (p.lm_fixed + cbytes - 1) / cbytes);
    p.region_bytes = uint32_t(std::max<size_t>(p.lm_fixed, (size_t(p.lm_nbuf) * cbytes + 127) & ~size_t(127)));
    const size_t smem = p.region_bytes + scratch;
    if (smem + fa.sharedSizeBytes + 1024 > ctx->smem_optin) return OPURE_OK;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
        return OPURE_ERR_CUDA;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kPThreads, smem) != cudaSuccess || per_sm < 1)
        return OPURE_OK;

    p.n_layers = s.n_layers;
    p.h = h;
    p.inter = s.inter;
    p.n_heads = s.n_heads;
    p.n_kv = s.n_kv;
    p.hd = HD;
    p.vocab = s.vocab;
    p.eps = s.eps;
    p.scale_log2 = s.attn_scale * 1.4426950408889634f;
    p.theta = s.theta;
    p.final_norm = reinterpret_cast<const __half *>(s.final_norm);
    p.lm_head = reinterpret_cast<const uint8_t *>(s.lm_head);
    p.page_table = s.page_table;
    p.n_pages = s.n_pages;
    p.max_pages = s.max_pages;
    p.page_size = s.page_size;
    p.kv_ring = s.kv_ring;
    p.seq = s.seq;
    p.pos = s.pos;
    p.base0 = s.x;
    p.base1 = s.base1;
    p.delta0 = s.delta0;
    p.delta1 = s.delta1;
    p.q = s.q;
    p.logits = s.logits;
    p.keys = s.keys;
    p.sync = s.sync;
    p.st = ctx->status;
    p.trace = s.trace;
    for (uint32_t L = 0; L < s.n_layers; ++L) {
        const opure_fused_layer &l = s.layers[L];
        p.layers[L] = PLayer{reinterpret_cast<const uint8_t *>(l.w_qkv), reinterpret_cast<const uint8_t *>(l.w_o_blk),
                             reinterpret_cast<const uint8_t *>(l.w_gate_up),
                             reinterpret_cast<const uint8_t *>(l.w_down_t),
                             reinterpret_cast<const __half *>(l.in_norm), reinterpret_cast<const __half *>(l.post_norm),
                             l.kv_pool, l.s_q, l.s_k, l.s_v, l.s_o, l.s_gate, l.s_up, l.s_down};
    }
    // Barrier counters and the abort flag start at zero (a memset node under capture).
    if (cudaMemsetAsync(s.sync, 0, (3 * size_t(s.n_layers) + 1) * 4, ctx->stream) != cudaSuccess)
        return OPURE_ERR_CUDA;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident, or the launch fails
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess) return cuda_status(e);
    *ran = true;
    return OPURE_OK;
}

template <int NV, int HD>
opure_status pick_g(opure_ctx *ctx, const opure_fused_step &s, uint32_t G) {
    if constexpr (HD == 64) {
        bool ran = false;
        opure_status st = OPURE_OK;
        if (s.w_dtype == OPURE_W_Q8) {
            // int8 layer weights run on the persistent kernel only.
            if (s.mode != OPURE_FUSED_AUTO) return OPURE_ERR_UNSUPPORTED;
            switch (G) {
                case 1: st = run_persistent<NV, HD, 1, true>(ctx, s, &ran); break;
                case 2: st = run_persistent<NV, HD, 2, true>(ctx, s, &ran); break;
                case 3: st = run_persistent<NV, HD, 3, true>(ctx, s, &ran); break;
                case 4: st = run_persistent<NV, HD, 4, true>(ctx, s, &ran); break;
            }
            return st ? st : (ran ? OPURE_OK : OPURE_ERR_UNSUPPORTED);
        }
        if (s.mode == OPURE_FUSED_AUTO) {
            switch (G) {
                case 1: st = run_persistent<NV, HD, 1, false>(ctx, s, &ran); break;
                case 2: st = run_persistent<NV, HD, 2, false>(ctx, s, &ran); break;
                case 3: st = run_persistent<NV, HD, 3, false>(ctx, s, &ran); break;
                case 4: st = run_persistent<NV, HD, 4, false>(ctx, s, &ran); break;
            }
            if (st || ran) return st;
        }
    } else {
        if (s.w_dtype == OPURE_W_Q8) return OPURE_ERR_UNSUPPORTED;
    }
    switch (G) {
        case 1: return run_step<NV, HD, 1>(ctx, s);
        case 2: return run_step<NV, HD, 2>(ctx, s);
        case 3: return run_step<NV, HD, 3>(ctx, s);
        case 4: return run_step<NV, HD, 4>(ctx, s);
    }
    return OPURE_ERR_UNSUPPORTED;
}

template <int NV>
opure_status pick_hd(opure_ctx *ctx, const opure_fused_step &s, uint32_t G) {
    if (s.head_dim == 64) return pick_g<NV, 64>(ctx, s, G);
    if (s.head_dim == 128) return pick_g<NV, 128>(ctx, s, G);
    return OPURE_ERR_UNSUPPORTED;
}

}  // namespace
}  // namespace opure

using namespace opure;

extern "C" opure_status opure_decode_fused(opure_ctx *ctx, const opure_fused_step *s) {
    opure_status st = enter(ctx);
    if (st) return st;
    if (!s || !s->layers || !s->final_norm || !s->lm_head || !s->page_table || !s->seq || !s->pos || !s->x ||
        !s->base1 || !s->delta0 || !s->delta1 || !s->q || !s->keys || !s->n_kv || !s->n_layers)
        return OPURE_ERR_INVALID_ARG;
    if (s->n_heads % s->n_kv || s->hidden % 8 || s->inter == 0 || s->kv_ring > s->max_pages)
        return OPURE_ERR_INVALID_ARG;
    if (s->w_dtype != OPURE_W_F16 && s->w_dtype != OPURE_W_Q8) return OPURE_ERR_INVALID_ARG;
    if (s->w_dtype == OPURE_W_Q8 && (s->hidden % 16 || (s->n_heads / s->n_kv * s->head_dim) % 16))
        return OPURE_ERR_UNSUPPORTED;  // whole 16-byte chunks of int8 per row
    if (s->nvec == 0) return OPURE_OK;
    const uint32_t G = s->n_heads / s->n_kv;
    for (uint32_t L = 0; L < s->n_layers; ++L) {
        const opure_fused_layer &l = s->layers[L];
        if (!l.in_norm || !l.post_norm || !l.w_qkv || !l.w_o_blk || !l.w_gate_up || !l.w_down_t || !l.kv_pool)
            return OPURE_ERR_INVALID_ARG;
        for (const void *p : {static_cast<const void *>(l.w_qkv), static_cast<const void *>(l.w_o_blk),
                              static_cast<const void *>(l.w_gate_up), static_cast<const void *>(l.w_down_t)})
            if (reinterpret_cast<uintptr_t>(p) % 16) return OPURE_ERR_UNSUPPORTED;
    }
    switch (s->nvec) {
        case 1: return pick_hd<1>(ctx, *s, G);
        case 2: return pick_hd<2>(ctx, *s, G);
        case 4: return pick_hd<4>(ctx, *s, G);
        case 8: return pick_hd<8>(ctx, *s, G);
    }
    return OPURE_ERR_UNSUPPORTED;
}
