// context.cu -- lifetime, memory, synchronisation, graphs and timing of the C ABI.
// Replaces the reference's D3D12 device layer (src/core/Opure_Dx12.{h,cpp}).
#include <chrono>
#include <cstdio>
#include <cstring>
#include <new>
#include <thread>

#include "ctx.cuh"

struct opure_graph {
    int device = -1;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
};

struct opure_event {
    int device = -1;
    cudaEvent_t ev = nullptr;
};

using opure::enter;

extern "C" {

const char *opure_strerror(opure_status s) {
    switch (s) {
        case OPURE_OK: return "ok";
        case OPURE_ERR_INVALID_ARG: return "invalid argument";
        case OPURE_ERR_NO_DEVICE: return "no usable CUDA device (sm_100 required)";
        case OPURE_ERR_CUDA: return "CUDA runtime error";
        case OPURE_ERR_OUT_OF_MEMORY: return "out of device memory";
        case OPURE_ERR_TIMEOUT: return "timed out waiting for the device";
        case OPURE_ERR_DEVICE_TIMEOUT: return "a device-side wait gave up";
        case OPURE_ERR_UNSUPPORTED: return "unsupported shape or option";
        case OPURE_ERR_INJECTED: return "injected failure";
        case OPURE_ERR_DEVICE_BOUNDS: return "a kernel refused an out-of-range index";
    }
    return "unknown status";
}

opure_status opure_init(int device, opure_ctx **out) {
    if (!out) return OPURE_ERR_INVALID_ARG;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return OPURE_ERR_NO_DEVICE;
    if (device < 0 || device >= n) return OPURE_ERR_INVALID_ARG;
    cudaDeviceProp prop;
    OPURE_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    // The kernels are built for sm_100a only.
    if (prop.major != 10) return OPURE_ERR_NO_DEVICE;
    OPURE_CUDA_TRY(cudaSetDevice(device));
    auto *ctx = new (std::nothrow) opure_ctx;
    if (!ctx) return OPURE_ERR_OUT_OF_MEMORY;
    ctx->device = device;
    ctx->sm_count = prop.multiProcessorCount;
    ctx->smem_optin = prop.sharedMemPerBlockOptin;
    cudaError_t e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&ctx->status, sizeof(opure::DeviceStatus));
    if (e == cudaSuccess) e = cudaMemset(ctx->status, 0, sizeof(opure::DeviceStatus));
    if (e == cudaSuccess) e = cudaMalloc(&ctx->ws, opure::kTcWorkspaceBytes);
    if (e == cudaSuccess) e = cudaMemset(ctx->ws, 0, opure::kTcWorkspaceBytes);
    if (e == cudaSuccess) ctx->ws_bytes = opure::kTcWorkspaceBytes;
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        if (ctx->ws) cudaFree(ctx->ws);
        if (ctx->status) cudaFree(ctx->status);
        if (ctx->stream) cudaStreamDestroy(ctx->stream);
        delete ctx;
        return opure::cuda_status(e);
    }
    *out = ctx;
    return OPURE_OK;
}

opure_status opure_shutdown(opure_ctx *ctx) {
    if (!ctx) return OPURE_ERR_INVALID_ARG;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    if (ctx->ws) cudaFree(ctx->ws);
    if (ctx->status) cudaFree(ctx->status);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
    return OPURE_OK;
}

opure_status opure_get_device_info(opure_ctx *ctx, opure_device_info *info) {
    if (!ctx || !info) return OPURE_ERR_INVALID_ARG;
    cudaDeviceProp prop;
    OPURE_CUDA_TRY(cudaGetDeviceProperties(&prop, ctx->device));
    std::memset(info, 0, sizeof(*info));
    info->device = ctx->device;
    info->sm_count = prop.multiProcessorCount;
    info->cc_major = prop.major;
    info->cc_minor = prop.minor;
    info->hbm_bytes = prop.totalGlobalMem;
    info->l2_bytes = uint64_t(prop.l2CacheSize);
    info->smem_per_block_optin = uint32_t(prop.sharedMemPerBlockOptin);
    int clk = 0;
    cudaDeviceGetAttribute(&clk, cudaDevAttrClockRate, ctx->device);
    info->clock_mhz_max = uint32_t(clk / 1000);
    std::snprintf(info->name, sizeof(info->name), "%.95s", prop.name);
    return OPURE_OK;
}

void *opure_stream(opure_ctx *ctx) { return ctx ? static_cast<void *>(ctx->stream) : nullptr; }

opure_status opure_last_error_detail(opure_ctx *ctx, uint32_t *where, uint32_t *detail) {
    opure_status s = enter(ctx);
    if (s) return s;
    OPURE_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    opure::DeviceStatus st;
    OPURE_CUDA_TRY(cudaMemcpy(&st, ctx->status, sizeof(st), cudaMemcpyDeviceToHost));
    if (st.code) OPURE_CUDA_TRY(cudaMemset(ctx->status, 0, sizeof(st)));
    if (where) *where = st.code ? st.where : 0;
    if (detail) *detail = st.code ? st.detail : 0;
    return static_cast<opure_status>(st.code);
}

opure_status opure_last_error(opure_ctx *ctx) { return opure_last_error_detail(ctx, nullptr, nullptr); }

// ---- memory ---------------------------------------------------------------
opure_status opure_alloc(opure_ctx *ctx, size_t bytes, void **dptr) {
    if (!dptr) return OPURE_ERR_INVALID_ARG;
    *dptr = nullptr;
    opure_status s = enter(ctx);
    if (s) return s;
    if (bytes == 0) return OPURE_OK;
    OPURE_CUDA_TRY(cudaMalloc(dptr, bytes));  // 256-byte aligned
    return OPURE_OK;
}

opure_status opure_free(opure_ctx *ctx, void *dptr) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (dptr) OPURE_CUDA_TRY(cudaFree(dptr));
    return OPURE_OK;
}

opure_status opure_alloc_host(opure_ctx *ctx, size_t bytes, void **hptr) {
    if (!hptr) return OPURE_ERR_INVALID_ARG;
    *hptr = nullptr;
    opure_status s = enter(ctx);
    if (s) return s;
    if (bytes == 0) return OPURE_OK;
    OPURE_CUDA_TRY(cudaMallocHost(hptr, bytes));
    return OPURE_OK;
}

opure_status opure_free_host(opure_ctx *ctx, void *hptr) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (hptr) OPURE_CUDA_TRY(cudaFreeHost(hptr));
    return OPURE_OK;
}

static opure_status copy(opure_ctx *ctx, void *dst, const void *src, size_t n, cudaMemcpyKind k) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (n == 0) return OPURE_OK;
    if (!dst || !src) return OPURE_ERR_INVALID_ARG;
    OPURE_CUDA_TRY(cudaMemcpyAsync(dst, src, n, k, ctx->stream));
    return OPURE_OK;
}

opure_status opure_h2d(opure_ctx *ctx, void *dst, const void *src, size_t n) {
    return copy(ctx, dst, src, n, cudaMemcpyHostToDevice);
}
opure_status opure_d2h(opure_ctx *ctx, void *dst, const void *src, size_t n) {
    return copy(ctx, dst, src, n, cudaMemcpyDeviceToHost);
}
opure_status opure_d2d(opure_ctx *ctx, void *dst, const void *src, size_t n) {
    return copy(ctx, dst, src, n, cudaMemcpyDeviceToDevice);
}

opure_status opure_fill(opure_ctx *ctx, void *dst, uint8_t byte, size_t n) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (n == 0) return OPURE_OK;
    if (!dst) return OPURE_ERR_INVALID_ARG;
    OPURE_CUDA_TRY(cudaMemsetAsync(dst, byte, n, ctx->stream));
    return OPURE_OK;
}

opure_status opure_sync(opure_ctx *ctx, uint32_t timeout_ms) {
    opure_status s = enter(ctx);
    if (s) return s;
    // Poll instead of blocking so a wedged stream surfaces as a timeout. The first 2 ms
    // poll without sleeping (a decode step is ~0.5 ms, and a sleep of a few microseconds
    // wakes tens of microseconds late under the kernel's timer slack); longer waits sleep.
    const auto t0 = std::chrono::steady_clock::now();
    const auto deadline = t0 + std::chrono::milliseconds(timeout_ms);
    const auto spin_until = t0 + std::chrono::milliseconds(2);
    for (;;) {
        cudaError_t e = cudaStreamQuery(ctx->stream);
        if (e == cudaSuccess) return OPURE_OK;
        if (e != cudaErrorNotReady) return opure::cuda_status(e);
        const auto now = std::chrono::steady_clock::now();
        if (now >= deadline) return OPURE_ERR_TIMEOUT;
        if (now < spin_until)
            std::this_thread::yield();
        else
            std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

// ---- graphs ----------------------------------------------------------------
opure_status opure_graph_begin(opure_ctx *ctx) {
    opure_status s = enter(ctx);
    if (s) return s;
    OPURE_CUDA_TRY(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
    return OPURE_OK;
}

opure_status opure_graph_end(opure_ctx *ctx, opure_graph **out) {
    if (!out) return OPURE_ERR_INVALID_ARG;
    *out = nullptr;
    opure_status s = enter(ctx);
    if (s) return s;
    cudaGraph_t g = nullptr;
    OPURE_CUDA_TRY(cudaStreamEndCapture(ctx->stream, &g));
    cudaGraphExec_t ex = nullptr;
    cudaError_t e = cudaGraphInstantiate(&ex, g, 0);
    if (e != cudaSuccess) {
        cudaGraphDestroy(g);
        return opure::cuda_status(e);
    }
    auto *G = new (std::nothrow) opure_graph;
    if (!G) {
        cudaGraphExecDestroy(ex);
        cudaGraphDestroy(g);
        return OPURE_ERR_OUT_OF_MEMORY;
    }
    G->device = ctx->device;
    G->graph = g;
    G->exec = ex;
    *out = G;
    return OPURE_OK;
}

opure_status opure_graph_launch(opure_ctx *ctx, opure_graph *g) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!g || g->device != ctx->device) return OPURE_ERR_INVALID_ARG;
    OPURE_CUDA_TRY(cudaGraphLaunch(g->exec, ctx->stream));
    return OPURE_OK;
}

opure_status opure_graph_free(opure_graph *g) {
    if (!g) return OPURE_ERR_INVALID_ARG;
    cudaSetDevice(g->device);
    if (g->exec) cudaGraphExecDestroy(g->exec);
    if (g->graph) cudaGraphDestroy(g->graph);
    delete g;
    return OPURE_OK;
}

// ---- events -----------------------------------------------------------------
opure_status opure_event_create(opure_ctx *ctx, opure_event **out) {
    if (!out) return OPURE_ERR_INVALID_ARG;
    *out = nullptr;
    opure_status s = enter(ctx);
    if (s) return s;
    auto *e = new (std::nothrow) opure_event;
    if (!e) return OPURE_ERR_OUT_OF_MEMORY;
    e->device = ctx->device;
    cudaError_t r = cudaEventCreate(&e->ev);
    if (r != cudaSuccess) {
        delete e;
        return opure::cuda_status(r);
    }
    *out = e;
    return OPURE_OK;
}

opure_status opure_event_record(opure_ctx *ctx, opure_event *e) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!e) return OPURE_ERR_INVALID_ARG;
    OPURE_CUDA_TRY(cudaEventRecord(e->ev, ctx->stream));
    return OPURE_OK;
}

opure_status opure_event_elapsed_ms(opure_event *a, opure_event *b, float *ms) {
    if (!a || !b || !ms) return OPURE_ERR_INVALID_ARG;
    cudaSetDevice(a->device);
    OPURE_CUDA_TRY(cudaEventSynchronize(b->ev));
    OPURE_CUDA_TRY(cudaEventElapsedTime(ms, a->ev, b->ev));
    return OPURE_OK;
}

opure_status opure_event_free(opure_event *e) {
    if (!e) return OPURE_ERR_INVALID_ARG;
    cudaSetDevice(e->device);
    cudaEventDestroy(e->ev);
    delete e;
    return OPURE_OK;
}

opure_status opure_debug_inject_failure(opure_ctx *ctx, uint32_t after_calls, uint32_t count) {
    if (!ctx) return OPURE_ERR_INVALID_ARG;
    ctx->inject_after = after_calls;
    ctx->inject_count = count;
    return OPURE_OK;
}

}  // extern "C"
