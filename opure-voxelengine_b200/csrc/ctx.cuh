// ctx.cuh -- the opure_ctx object and kernel-launch helpers shared by the ABI files.
#pragma once

#include "common.cuh"

namespace opure {
// Tensor-core GEMV workspace: up to 256 vectors x 16384 columns packed as fp16 pairs
// (16 MiB), their scales and split-K tickets, and 32 MiB of split-K partial sums.
constexpr size_t kTcWorkspaceBytes = size_t(48) << 20;
}  // namespace opure

struct opure_ctx {
    int device = -1;
    cudaStream_t stream = nullptr;
    opure::DeviceStatus *status = nullptr;  // device memory
    int sm_count = 0;
    size_t smem_optin = 0;
    // Host-side fault injection (opure_debug_inject_failure).
    uint32_t inject_after = 0;
    uint32_t inject_count = 0;
    // Programmatic dependent launch for kernels enqueued by this ctx.
    bool pdl = true;
    // Device workspace of the tensor-core GEMV path (packed vectors, split-K partial sums
    // and their tickets), allocated and zeroed once by opure_init so kernel calls allocate
    // nothing; calls on one ctx are stream-ordered, so they share it safely.
    void *ws = nullptr;
    size_t ws_bytes = 0;
};

namespace opure {

// Common prologue of every ABI entry that touches the GPU: validates the ctx,
// applies fault injection and makes the ctx's device current.
inline opure_status enter(opure_ctx *ctx) {
    if (!ctx || !ctx->stream) return OPURE_ERR_INVALID_ARG;
    if (ctx->inject_count) {
        if (ctx->inject_after) {
            --ctx->inject_after;
        } else {
            --ctx->inject_count;
            return OPURE_ERR_INJECTED;
        }
    }
    if (cudaSetDevice(ctx->device) != cudaSuccess) return OPURE_ERR_CUDA;
    return OPURE_OK;
}

// Launches `kernel` on the ctx stream; with `pdl` the launch may overlap the tail
// of the previous kernel on the stream (the kernel must grid_dependency_wait()).
template <typename... KArgs, typename... Args>
opure_status launch(opure_ctx *ctx, void (*kernel)(KArgs...), dim3 grid, dim3 block,
                    size_t smem, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (pdl && ctx->pdl) ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
    return e == cudaSuccess ? OPURE_OK : cuda_status(e);
}

inline uint32_t ceil_div(uint64_t a, uint64_t b) { return uint32_t((a + b - 1) / b); }

}  // namespace opure
