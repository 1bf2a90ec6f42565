// comm.cu -- NCCL communicators for the tensor-parallel large-model decode (8 GPUs over
// NVLink/NVSwitch), plus the small kernel that turns a vocabulary shard's argmax keys
// into global ones. NCCL is loaded at run time (libnccl.so.2): only callers of these
// entry points need it. Communicators are created non-blocking and polled against a
// host deadline, so a rank that never joins ends in OPURE_ERR_TIMEOUT rather than a hang.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <new>
#include <thread>
#include <type_traits>

#include "ctx.cuh"

struct opure_comm {
    ncclComm_t comm = nullptr;
    uint32_t n_ranks = 0, rank = 0;
    uint32_t timeout_ms = 0;
};

namespace opure {
namespace {

struct NcclApi {
    ncclResult_t (*getUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*initRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
    ncclResult_t (*getAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*allReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*commAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*commFinalize)(ncclComm_t) = nullptr;
    bool ok = false;
};

const NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        auto sym = [&](auto &fn, const char *name) { fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name)); };
        sym(api.getUniqueId, "ncclGetUniqueId");
        sym(api.initRankConfig, "ncclCommInitRankConfig");
        sym(api.getAsyncError, "ncclCommGetAsyncError");
        sym(api.allReduce, "ncclAllReduce");
        sym(api.commAbort, "ncclCommAbort");
        sym(api.commDestroy, "ncclCommDestroy");
        sym(api.commFinalize, "ncclCommFinalize");
        api.ok = api.getUniqueId && api.initRankConfig && api.getAsyncError && api.allReduce && api.commAbort &&
                 api.commDestroy && api.commFinalize;
    });
    return api;
}

// Polls a non-blocking communicator until its pending operation settles or the deadline.
opure_status settle(ncclComm_t comm, uint32_t timeout_ms) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        if (nccl().getAsyncError(comm, &st) != ncclSuccess) return OPURE_ERR_CUDA;
        if (st == ncclSuccess) return OPURE_OK;
        if (st != ncclInProgress) return OPURE_ERR_CUDA;
        if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) return OPURE_ERR_TIMEOUT;
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

opure_status allreduce(opure_ctx *ctx, opure_comm *c, void *buf, size_t n, ncclDataType_t dt, ncclRedOp_t op) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!c || !c->comm || !buf) return OPURE_ERR_INVALID_ARG;
    if (n == 0) return OPURE_OK;
    const ncclResult_t r = nccl().allReduce(buf, buf, n, dt, op, c->comm, ctx->stream);
    if (r == ncclInProgress) return settle(c->comm, c->timeout_ms);
    return r == ncclSuccess ? OPURE_OK : OPURE_ERR_CUDA;
}

// keys[i] of a vocabulary shard starting at row `offset`: same value bits, global index.
__global__ void key_offset_kernel(unsigned long long *keys, uint32_t n, uint32_t offset) {
    grid_dependency_wait();
    grid_dependents_launch();
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const unsigned long long k = keys[i];
    if (!k) return;
    const uint32_t idx = argmax_key_index(k) + offset;
    keys[i] = (k & 0xffffffff00000000ull) | (0xffffffffu - idx);
}

}  // namespace
}  // namespace opure

using namespace opure;

extern "C" {

opure_status opure_comm_unique_id(uint8_t *id) {
    if (!id) return OPURE_ERR_INVALID_ARG;
    if (!nccl().ok) return OPURE_ERR_UNSUPPORTED;
    ncclUniqueId u;
    if (nccl().getUniqueId(&u) != ncclSuccess) return OPURE_ERR_CUDA;
    std::memcpy(id, u.internal, NCCL_UNIQUE_ID_BYTES);
    return OPURE_OK;
}

opure_status opure_comm_init(opure_ctx *ctx, uint32_t n_ranks, uint32_t rank, const uint8_t *id,
                             uint32_t timeout_ms, opure_comm **out) {
    if (!out || !id || n_ranks == 0 || rank >= n_ranks) return OPURE_ERR_INVALID_ARG;
    *out = nullptr;
    opure_status s = enter(ctx);
    if (s) return s;
    if (!nccl().ok) return OPURE_ERR_UNSUPPORTED;
    auto *c = new (std::nothrow) opure_comm;
    if (!c) return OPURE_ERR_OUT_OF_MEMORY;
    c->n_ranks = n_ranks;
    c->rank = rank;
    c->timeout_ms = timeout_ms ? timeout_ms : 60000;
    ncclUniqueId u;
    std::memcpy(u.internal, id, NCCL_UNIQUE_ID_BYTES);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    const ncclResult_t r = nccl().initRankConfig(&c->comm, int(n_ranks), u, int(rank), &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        delete c;
        return OPURE_ERR_CUDA;
    }
    s = settle(c->comm, c->timeout_ms);
    if (s) {
        if (c->comm) nccl().commAbort(c->comm);
        delete c;
        return s;
    }
    *out = c;
    return OPURE_OK;
}

opure_status opure_comm_destroy(opure_comm *c) {
    if (!c) return OPURE_ERR_INVALID_ARG;
    opure_status s = OPURE_OK;
    if (c->comm) {
        // Flush outstanding work (bounded), then free; abort if it does not settle.
        const ncclResult_t f = nccl().commFinalize(c->comm);
        s = (f == ncclSuccess || f == ncclInProgress) ? settle(c->comm, c->timeout_ms) : OPURE_ERR_CUDA;
        if (s == OPURE_OK)
            nccl().commDestroy(c->comm);
        else
            nccl().commAbort(c->comm);
    }
    delete c;
    return s;
}

opure_status opure_comm_info(const opure_comm *c, uint32_t *n_ranks, uint32_t *rank) {
    if (!c) return OPURE_ERR_INVALID_ARG;
    if (n_ranks) *n_ranks = c->n_ranks;
    if (rank) *rank = c->rank;
    return OPURE_OK;
}

opure_status opure_allreduce_sum_f32(opure_ctx *ctx, opure_comm *c, float *buf, size_t n) {
    return allreduce(ctx, c, buf, n, ncclFloat32, ncclSum);
}

opure_status opure_allreduce_max_u64(opure_ctx *ctx, opure_comm *c, unsigned long long *buf, size_t n) {
    return allreduce(ctx, c, buf, n, ncclUint64, ncclMax);
}

opure_status opure_argmax_key_offset(opure_ctx *ctx, unsigned long long *keys, uint32_t n, uint32_t offset) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!keys) return OPURE_ERR_INVALID_ARG;
    if (n == 0) return OPURE_OK;
    return launch(ctx, key_offset_kernel, dim3(ceil_div(n, 128)), dim3(128), 0, true, keys, n, offset);
}

}  // extern "C"
