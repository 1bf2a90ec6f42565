// gemv.cu -- opure_gemv: fp16 / int8 weight-streaming GEMV with fused prologue and
// epilogue. Replaces GEMVMain (shaders/Opure_GEMV.usf:40-88) and GEMVQuantMain
// (shaders/Opure_GEMV_Quant.usf:38-94), which run one 256-thread group per output row
// with 4-byte loads; here a warp streams four rows with 16-byte loads and the vector is
// shared by every row of the CTA from shared memory.
#include "ctx.cuh"
#include "gemm_tc.cuh"
#include "gemv.cuh"

namespace opure {
namespace {

constexpr int kRows = 4;          // rows per warp task
constexpr int kThreads = 128;     // 4 warps per CTA
constexpr int kMaxNv = 9;

struct GemvParams {
    const uint8_t *w;
    size_t pitch;                 // bytes per weight row
    uint32_t rows, cols, nchunks;
    float scale;                  // scale_w * scale_x for int8, 1 for fp16
    float scale2;                 // scale of the up half (SwiGLU), same convention
    const float *x;
    uint32_t x_stride;
    float *y;
    uint32_t y_stride;
    const __half *gain;
    float eps;
    const float *residual;
    unsigned long long *keys;
};

template <int WT, int NV, int PRO, int EPI>
__global__ void __launch_bounds__(kThreads) gemv_kernel(GemvParams p) {
    extern __shared__ __align__(16) float smem[];
    float *xs = smem;
    float *red = smem + NV * p.cols;
    __shared__ unsigned long long cta_best[kThreads / 32][NV];

    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t nwarps = gridDim.x * (kThreads / 32);
    const uint32_t groups = (p.rows + kRows - 1) / kRows;
    const uint32_t g0 = blockIdx.x * (kThreads / 32) + warp;

    // Weights do not depend on the previous kernel: start this warp's first row group
    // before waiting on it.
    RowPrefetch<kRows> pre, pre_up;
    if (g0 < groups) {
        const uint32_t valid0 = min(uint32_t(kRows), p.rows - g0 * kRows);
        prefetch_rows(pre, p.w, p.pitch, g0 * kRows, valid0, p.nchunks);
        if constexpr (EPI == OPURE_EPI_SWIGLU)
            prefetch_rows(pre_up, p.w + size_t(p.rows) * p.pitch, p.pitch, g0 * kRows, valid0, p.nchunks);
    }

    grid_dependency_wait();
    grid_dependents_launch();
    // int8 chunks span 16 elements: their vectors are staged chunk-interleaved (no bank
    // conflicts on the 64-byte-per-lane reads); fp16 keeps the plain layout, measured faster.
    constexpr bool kIL = WT == OPURE_W_Q8;
    if constexpr (kIL)
        stage_vectors_il<NV, WTraits<WT>::kElems>(p.x, p.x_stride, p.cols, PRO == OPURE_PRO_RMSNORM, p.gain, p.eps,
                                                  xs, red);
    else
        stage_vectors<NV>(p.x, p.x_stride, p.cols, PRO == OPURE_PRO_RMSNORM, p.gain, p.eps, xs, red);

    unsigned long long best[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) best[v] = 0ull;

    for (uint32_t g = g0; g < groups; g += nwarps) {
        const uint32_t row0 = g * kRows;
        const uint32_t valid = min(uint32_t(kRows), p.rows - row0);
        float acc[kRows][NV];
        dot_rows<WT, NV, kRows, kIL>(p.w, p.pitch, row0, valid, p.nchunks, xs, p.cols, acc, pre, g == g0);
        float acc_up[kRows][NV];
        if constexpr (EPI == OPURE_EPI_SWIGLU)
            dot_rows<WT, NV, kRows, kIL>(p.w + size_t(p.rows) * p.pitch, p.pitch, row0, valid, p.nchunks,
                                          xs, p.cols, acc_up, pre_up, g == g0);
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                if (r >= int(valid)) continue;
                const float val = acc[r][v] * p.scale;
                const size_t o = size_t(v) * p.y_stride + row0 + r;
                if constexpr (EPI == OPURE_EPI_ARGMAX) {
                    const unsigned long long k = argmax_key(val, row0 + r);
                    best[v] = k > best[v] ? k : best[v];
                }
                if (lane != uint32_t((r * NV + v) & 31)) continue;
                if constexpr (EPI == OPURE_EPI_STORE) {
                    p.y[o] = val;
                } else if constexpr (EPI == OPURE_EPI_ADD) {
                    p.y[o] = p.residual[o] + val;
                } else if constexpr (EPI == OPURE_EPI_SWIGLU) {
                    const float u = acc_up[r][v] * p.scale2;
                    const float s = 1.0f / (1.0f + expf(-val));
                    p.y[o] = (val * s) * u;
                } else {
                    if (p.y) p.y[o] = val;
                }
            }
        }
    }
    if constexpr (EPI == OPURE_EPI_ARGMAX) {
        if (lane == 0)
#pragma unroll
            for (int v = 0; v < NV; ++v) cta_best[warp][v] = best[v];
        __syncthreads();
        if (threadIdx.x < NV) {
            unsigned long long b = 0ull;
            for (int w = 0; w < kThreads / 32; ++w) b = cta_best[w][threadIdx.x] > b ? cta_best[w][threadIdx.x] : b;
            if (b) atomicMax(p.keys + threadIdx.x, b);
        }
    }
}

template <int WT, int NV, int PRO, int EPI>
opure_status run(opure_ctx *ctx, const GemvParams &p) {
    auto kern = gemv_kernel<WT, NV, PRO, EPI>;
    const size_t smem = (size_t(NV) * p.cols + 33 * NV) * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e != cudaSuccess) return cuda_status(e);
    }
    const uint32_t groups = ceil_div(p.rows, kRows);
    const uint32_t ctas = std::min<uint32_t>(ceil_div(groups, kThreads / 32), uint32_t(ctx->sm_count) * 8);
    return launch(ctx, kern, dim3(ctas), dim3(kThreads), smem, true, p);
}

template <int WT, int NV, int PRO>
opure_status pick_epi(opure_ctx *ctx, uint32_t epi, const GemvParams &p) {
    switch (epi) {
        case OPURE_EPI_STORE: return run<WT, NV, PRO, OPURE_EPI_STORE>(ctx, p);
        case OPURE_EPI_ADD: return run<WT, NV, PRO, OPURE_EPI_ADD>(ctx, p);
        case OPURE_EPI_SWIGLU: return run<WT, NV, PRO, OPURE_EPI_SWIGLU>(ctx, p);
        case OPURE_EPI_ARGMAX: return run<WT, NV, PRO, OPURE_EPI_ARGMAX>(ctx, p);
    }
    return OPURE_ERR_INVALID_ARG;
}

template <int WT, int NV>
opure_status pick_pro(opure_ctx *ctx, uint32_t pro, uint32_t epi, const GemvParams &p) {
    return pro == OPURE_PRO_RMSNORM ? pick_epi<WT, NV, OPURE_PRO_RMSNORM>(ctx, epi, p)
                                    : pick_epi<WT, NV, OPURE_PRO_NONE>(ctx, epi, p);
}

template <int WT>
opure_status pick_nv(opure_ctx *ctx, uint32_t nv, uint32_t pro, uint32_t epi, const GemvParams &p) {
    switch (nv) {
        case 1: return pick_pro<WT, 1>(ctx, pro, epi, p);
        case 2: return pick_pro<WT, 2>(ctx, pro, epi, p);
        case 3: return pick_pro<WT, 3>(ctx, pro, epi, p);
        case 4: return pick_pro<WT, 4>(ctx, pro, epi, p);
        case 5: return pick_pro<WT, 5>(ctx, pro, epi, p);
        case 6: return pick_pro<WT, 6>(ctx, pro, epi, p);
        case 7: return pick_pro<WT, 7>(ctx, pro, epi, p);
        case 8: return pick_pro<WT, 8>(ctx, pro, epi, p);
        case 9: return pick_pro<WT, 9>(ctx, pro, epi, p);
    }
    return OPURE_ERR_INVALID_ARG;
}

}  // namespace
}  // namespace opure

using namespace opure;

extern "C" opure_status opure_gemv(opure_ctx *ctx, const opure_gemv_args *a) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!a || !a->w || (!a->x && !a->x_packed) || a->rows == 0 || a->cols == 0) return OPURE_ERR_INVALID_ARG;
    if (a->nvec == 0) return OPURE_OK;
    if (a->w_dtype != OPURE_W_F16 && a->w_dtype != OPURE_W_Q8) return OPURE_ERR_INVALID_ARG;
    if (a->prologue > OPURE_PRO_RMSNORM || a->epilogue > OPURE_EPI_ARGMAX) return OPURE_ERR_INVALID_ARG;
    if (a->prologue == OPURE_PRO_RMSNORM && !a->norm_gain && !a->x_packed) return OPURE_ERR_INVALID_ARG;
    if (a->epilogue != OPURE_EPI_ARGMAX && !a->y) return OPURE_ERR_INVALID_ARG;
    if (a->epilogue == OPURE_EPI_ADD && !a->residual) return OPURE_ERR_INVALID_ARG;
    if (a->epilogue == OPURE_EPI_ARGMAX && !a->argmax_keys) return OPURE_ERR_INVALID_ARG;
    const uint32_t eb = a->w_dtype == OPURE_W_F16 ? 2u : 1u;
    // 16-byte chunks: each row must be a whole number of them and start aligned.
    if ((uint64_t(a->cols) * eb) % 16 || reinterpret_cast<uintptr_t>(a->w) % 16) return OPURE_ERR_UNSUPPORTED;
    if (a->y && a->y_stride < a->rows) return OPURE_ERR_INVALID_ARG;
    if (!a->x_packed) {
        if (a->x_stride < a->cols) return OPURE_ERR_INVALID_ARG;
        if (a->x_stride % 4 || reinterpret_cast<uintptr_t>(a->x) % 16) return OPURE_ERR_UNSUPPORTED;
    }
    if (a->x_packed || a->y_packed || a->y_sumsq) {
        // Chained operands exist only on the tensor-core path.
        if (!gemv_tc_eligible(ctx, a)) return OPURE_ERR_UNSUPPORTED;
        return gemv_tc(ctx, a);
    }
    // Many vectors sharing the weights: a dense contraction for the tensor cores.
    if (gemv_tc_eligible(ctx, a)) return gemv_tc(ctx, a);

    GemvParams p{};
    p.w = static_cast<const uint8_t *>(a->w);
    p.pitch = size_t(a->cols) * eb;
    p.rows = a->rows;
    p.cols = a->cols;
    p.nchunks = uint32_t(p.pitch / 16);
    p.scale = a->w_dtype == OPURE_W_Q8 ? a->scale_w * a->scale_x : 1.0f;
    p.scale2 = a->w_dtype == OPURE_W_Q8 ? (a->scale_w2 != 0.f ? a->scale_w2 : a->scale_w) * a->scale_x : 1.0f;
    p.x_stride = a->x_stride;
    p.y_stride = a->y_stride;
    p.gain = reinterpret_cast<const __half *>(a->norm_gain);
    p.eps = a->eps;
    // Input vectors are staged in shared memory: pass as many as fit at once.
    const size_t budget = std::min<size_t>(ctx->smem_optin, 200 * 1024);
    uint32_t per_pass = uint32_t(std::min<size_t>(kMaxNv, budget / (size_t(a->cols) * 4 + 33 * 4)));
    if (per_pass == 0) return OPURE_ERR_UNSUPPORTED;
    for (uint32_t v0 = 0; v0 < a->nvec; v0 += per_pass) {
        const uint32_t nv = std::min(per_pass, a->nvec - v0);
        p.x = a->x + size_t(v0) * a->x_stride;
        p.y = a->y ? a->y + size_t(v0) * a->y_stride : nullptr;
        p.residual = a->residual ? a->residual + size_t(v0) * a->y_stride : nullptr;
        p.keys = a->argmax_keys ? a->argmax_keys + v0 : nullptr;
        s = a->w_dtype == OPURE_W_F16 ? pick_nv<OPURE_W_F16>(ctx, nv, a->prologue, a->epilogue, p)
                                      : pick_nv<OPURE_W_Q8>(ctx, nv, a->prologue, a->epilogue, p);
        if (s) return s;
    }
    return OPURE_OK;
}

extern "C" size_t opure_packed_bytes(uint32_t nvec, uint32_t len) { return packed_bytes(nvec, len); }
