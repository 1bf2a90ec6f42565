// gemv.cuh -- the weight-streaming dot-product core shared by the GEMV kernels
// (gemv.cu) and the fused decode kernels (decode.cu).
//
// A warp owns a group of R consecutive weight rows. Each lane streams 16-byte chunks of
// those rows with L1-bypassing loads (lanes of a warp touch consecutive chunks, so every
// load instruction covers 512 contiguous bytes of one row) and multiplies them against
// the input vectors held in shared memory as fp32. Accumulation is fp32 per lane, then a
// butterfly warp reduction leaves every row's dot product in every lane.
#pragma once

#include "common.cuh"

namespace opure {

template <int WT>
struct WTraits;
template <>
struct WTraits<OPURE_W_F16> {
    static constexpr int kElems = 8;  // fp16 per 16-byte chunk
};
template <>
struct WTraits<OPURE_W_Q8> {
    static constexpr int kElems = 16;  // int8 per 16-byte chunk
};

// Plain (non-volatile) streaming load so the compiler may hoist it ahead of the FMAs of
// the previous chunk batch; weights are evict-first in L2.
__device__ __forceinline__ uint4 ldg_nc(const void *p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p), "l"(l2_evict_first()));
    return r;
}

template <int WT>
__device__ __forceinline__ void unpack_chunk(const uint4 &w, float *f) {
    if constexpr (WT == OPURE_W_F16) {
        unpack8(w, f);
    } else {
        unpack16_i8(w, f);
    }
}

constexpr int kBatch = 2;  // 16-byte chunks per lane and row loaded ahead of their FMAs

// The first chunk batch of R rows, loaded into registers ahead of use: a kernel issues it
// before waiting on its predecessor (weights never depend on the previous kernel), so the
// DRAM latency overlaps the predecessor's tail.
template <int R>
struct RowPrefetch {
    uint4 w[kBatch][R];
};

template <int R>
__device__ __forceinline__ void prefetch_rows(RowPrefetch<R> &pf, const uint8_t *__restrict__ W,
                                              size_t pitch, uint32_t row0, uint32_t rows_valid,
                                              uint32_t nchunks) {
    const uint32_t lane = threadIdx.x & 31u;
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
        const uint32_t c = lane + 32u * b;
#pragma unroll
        for (int r = 0; r < R; ++r)
            pf.w[b][r] = (c < nchunks && r < int(rows_valid)) ? ldg_nc(W + size_t(row0 + r) * pitch + size_t(c) * 16)
                                                              : make_uint4(0, 0, 0, 0);
    }
}

// Chunk-batched dot products of R rows (row0 .. row0+R-1, rows >= rows_valid are
// skipped) against NV vectors in shared memory: xs[v * xs_stride + i], or with IL the
// chunk-interleaved layout of stage_vectors_il (xs_stride ignored).
// Row r starts at W + (row0 + r) * pitch (bytes); a row has nchunks 16-byte chunks.
// With use_pre, the first batch comes from `pre` (prefetch_rows of the same rows).
// On return every lane holds the full sums in acc.
template <int WT, int NV, int R, bool IL = false>
__device__ __forceinline__ void dot_rows(const uint8_t *__restrict__ W, size_t pitch,
                                         uint32_t row0, uint32_t rows_valid, uint32_t nchunks,
                                         const float *__restrict__ xs, uint32_t xs_stride,
                                         float (&acc)[R][NV], const RowPrefetch<R> &pre,
                                         bool use_pre) {
    constexpr int E = WTraits<WT>::kElems;
    constexpr int BATCH = kBatch;
    const uint32_t lane = threadIdx.x & 31u;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int v = 0; v < NV; ++v) acc[r][v] = 0.f;

    const uint8_t *rowp[R];
#pragma unroll
    for (int r = 0; r < R; ++r) rowp[r] = W + size_t(row0 + (r < int(rows_valid) ? r : 0)) * pitch;

    for (uint32_t c0 = lane; c0 < nchunks; c0 += 32u * BATCH) {
        uint4 w[BATCH][R];
        const bool first = use_pre && c0 == lane;
#pragma unroll
        for (int b = 0; b < BATCH; ++b) {
            const uint32_t c = c0 + 32u * b;
#pragma unroll
            for (int r = 0; r < R; ++r)
                w[b][r] = first ? pre.w[b][r]
                                : ((c < nchunks && r < int(rows_valid)) ? ldg_nc(rowp[r] + size_t(c) * 16)
                                                                        : make_uint4(0, 0, 0, 0));
        }
#pragma unroll
        for (int b = 0; b < BATCH; ++b) {
            const uint32_t c = c0 + 32u * b;
            if (c >= nchunks) break;
            float wf[R][E];
#pragma unroll
            for (int r = 0; r < R; ++r) unpack_chunk<WT>(w[b][r], wf[r]);
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                float xf[E];
                if constexpr (IL) {
                    // Lanes read consecutive float4s: no shared-memory bank conflicts.
                    const float4 *xp = reinterpret_cast<const float4 *>(xs) + size_t(v) * (E / 4) * nchunks + c;
#pragma unroll
                    for (int q = 0; q < E / 4; ++q) {
                        const float4 t = xp[size_t(q) * nchunks];
                        xf[4 * q] = t.x; xf[4 * q + 1] = t.y; xf[4 * q + 2] = t.z; xf[4 * q + 3] = t.w;
                    }
                } else {
                    const float4 *xp = reinterpret_cast<const float4 *>(xs + size_t(v) * xs_stride + size_t(c) * E);
#pragma unroll
                    for (int q = 0; q < E / 4; ++q) {
                        const float4 t = xp[q];
                        xf[4 * q] = t.x; xf[4 * q + 1] = t.y; xf[4 * q + 2] = t.z; xf[4 * q + 3] = t.w;
                    }
                }
#pragma unroll
                for (int r = 0; r < R; ++r)
#pragma unroll
                    for (int e = 0; e < E; ++e) acc[r][v] = fmaf(wf[r][e], xf[e], acc[r][v]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int v = 0; v < NV; ++v) acc[r][v] = warp_sum(acc[r][v]);
}

// Copies NV input vectors into shared memory, optionally RMS-normalised with an fp16
// gain (shaders/Opure_RMSNorm.usf semantics: x * rsqrt(mean(x^2) + eps) * g, the inverse
// root taken in double as Opure_CpuReference.cpp:163-169 does). Whole CTA participates.
template <int NV>
__device__ __forceinline__ void stage_vectors(const float *__restrict__ x, uint32_t x_stride,
                                              uint32_t cols, bool rmsnorm,
                                              const __half *__restrict__ gain, float eps,
                                              float *xs, float *red /* >= 32*NV floats */) {
    for (uint32_t v = 0; v < NV; ++v)
        for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x)
            xs[v * cols + i] = x[size_t(v) * x_stride + i];
    if (!rmsnorm) {
        __syncthreads();
        return;
    }
    __syncthreads();
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, nw = blockDim.x >> 5;
    for (uint32_t v = 0; v < NV; ++v) {
        float ss = 0.f;
        for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) ss = fmaf(xs[v * cols + i], xs[v * cols + i], ss);
        ss = warp_sum(ss);
        if (lane == 0) red[v * 32 + warp] = ss;
    }
    __syncthreads();
    if (threadIdx.x < NV) {
        float t = 0.f;
        for (uint32_t w = 0; w < nw; ++w) t += red[threadIdx.x * 32 + w];
        red[32 * NV + threadIdx.x] = float(1.0 / sqrt(double(t) / double(cols) + double(eps)));
    }
    __syncthreads();
    for (uint32_t v = 0; v < NV; ++v) {
        const float inv = red[32 * NV + v];
        for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x)
            xs[v * cols + i] = xs[v * cols + i] * inv * __half2float(gain[i]);
    }
    __syncthreads();
}

// stage_vectors with a chunk-interleaved layout for dot_rows<..., IL = true>: element i
// of vector v (chunk c = i / E of E elements per 16-byte weight chunk, quarter q = i % E / 4)
// sits at float index ((v * E / 4 + q) * nchunks + c) * 4 + i % 4, so the lanes of a warp,
// which work on consecutive chunks, read consecutive float4s. cols must be a multiple of E.
// Same arithmetic as stage_vectors.
template <int NV, int E>
__device__ __forceinline__ void stage_vectors_il(const float *__restrict__ x, uint32_t x_stride,
                                                 uint32_t cols, bool rmsnorm,
                                                 const __half *__restrict__ gain, float eps,
                                                 float *xs, float *red /* >= 33*NV floats */) {
    const uint32_t nchunks = cols / E;
    if (rmsnorm) {
        const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, nw = blockDim.x >> 5;
        for (uint32_t v = 0; v < NV; ++v) {
            float ss = 0.f;
            for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) {
                const float t = x[size_t(v) * x_stride + i];
                ss = fmaf(t, t, ss);
            }
            ss = warp_sum(ss);
            if (lane == 0) red[v * 32 + warp] = ss;
        }
        __syncthreads();
        if (threadIdx.x < NV) {
            float t = 0.f;
            for (uint32_t w = 0; w < nw; ++w) t += red[threadIdx.x * 32 + w];
            red[32 * NV + threadIdx.x] = float(1.0 / sqrt(double(t) / double(cols) + double(eps)));
        }
        __syncthreads();
    }
    for (uint32_t v = 0; v < NV; ++v) {
        const float inv = rmsnorm ? red[32 * NV + v] : 1.f;
        for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) {
            float t = x[size_t(v) * x_stride + i];
            if (rmsnorm) t = t * inv * __half2float(gain[i]);
            const uint32_t c = i / E, q = (i % E) / 4;
            xs[((size_t(v) * (E / 4) + q) * nchunks + c) * 4 + i % 4] = t;
        }
    }
    __syncthreads();
}

}  // namespace opure
