// peer.cu -- tensor-parallel all-reduce over NVLink peer memory, fused into the kernels that
// produce the values being reduced.
//
// The tensor-parallel decode step sums, twice per layer, every rank's partial o_proj and
// down_proj outputs (one fp32 vector of hidden size per token) and adds the sum to the
// replicated residual stream; at the end it takes the largest argmax key over the vocabulary
// shards. Through NCCL each of those is a separate collective launch of ~26 us for 8 KB.
// Here each is ONE kernel on each rank:
//
//  * Every rank owns a mailbox allocation that every other rank maps with CUDA IPC (one
//    process per GPU, all GPUs on one NVSwitch). Layout (byte offsets):
//      [kFlagsOff] u32 flags[src rank][CTA]     -- argmax exchange: written by the sender
//      [kCtlOff]   u32 seq, ticket, exchange    -- local only
//      [kKeysOff]  u64 keys[parity][src][vec]   -- argmax keys
//      [kRowsOff]  u64 rows[parity][src][vec][max_rows] -- (tag << 32) | fp32 bits
//  * The GEMV CTA c computes its rows of this rank's partial and stores each value, with
//    the collective's tag (seq + 1) in the upper half of the same 8-byte word, straight into
//    slot `rank` of every rank's mailbox (relaxed system-scope 64-bit stores over NVLink).
//    An aligned 64-bit access is single-copy atomic, so a reader that sees the tag also sees
//    the value: no flag, no fence, one NVLink write latency per collective. The CTA then
//    loads the n words of each of its rows from its own mailbox until every tag matches
//    (bounded by a deadline) and sums the values in rank order 0..n-1 -- the same order on
//    every rank, so the replicated residual stays bit-identical everywhere -- into y
//    (optionally residual + sum). Every rank runs the same grid over the same rows, so CTA
//    c only ever waits for the CTAs c of the other GPUs; the grid is at most one CTA per
//    SM, so all of it is resident at once.
//  * The argmax exchange (one CTA, 8-byte keys with no room for a tag) publishes per-rank
//    flags with a system-scope release store after a CTA barrier, and waits on its own
//    flags with acquire loads.
//  * `seq` counts the collectives this rank has run. Every kernel reads it after its
//    predecessor completes; the last CTA out (ticket) advances it. Data slots alternate by
//    seq parity: a rank can be at most one collective ahead of any other (collective k+1 on
//    rank A needs rank B's collective-(k+1) pushes, which B makes only after its kernel k
//    completed), so the slot of k+2 is never written while k's is still being read.
//
// Waits give up after the peer group's timeout (or at once when the ctx status word already
// holds a failure), record OPURE_ERR_DEVICE_TIMEOUT with the waiting rank index, and return.
// No TMA, no multicast: peers' memory is only touched by plain stores and flag stores.
#include <cstring>
#include <new>
#include <vector>

#include "ctx.cuh"
#include "gemv.cuh"
#include "tma.cuh"

struct opure_peer {
    int device = -1;
    uint32_t n_ranks = 0, rank = 0, max_rows = 0;
    uint64_t timeout_ns = 0;
    size_t bytes = 0;
    uint8_t *local = nullptr;
    uint8_t *peer[OPURE_PEER_MAX_RANKS] = {};
};

namespace opure {
namespace {

constexpr uint32_t kMaxRanks = OPURE_PEER_MAX_RANKS;
constexpr uint32_t kMaxCtas = 256;                 // flag slots per source rank
constexpr uint32_t kPassVec = 9;                   // vectors per collective pass
constexpr uint32_t kMaxKeys = OPURE_PEER_MAX_KEYS; // argmax keys per collective
constexpr size_t kFlagsOff = 0;
constexpr size_t kCtlOff = kFlagsOff + size_t(kMaxRanks) * kMaxCtas * 4;   // 8 KB
constexpr size_t kXchgOff = kCtlOff + 256;                                 // host exchange words
constexpr size_t kKeysOff = kCtlOff + 2048;
constexpr size_t kRowsOff = kKeysOff + size_t(2) * kMaxRanks * kMaxKeys * 8;
static_assert(kRowsOff % 256 == 0, "row slots 256-byte aligned");
constexpr uint32_t kXchgWords = 10;                // per rank: 8 handle words, device, ok

constexpr int kRows = 4;       // rows per warp task (as opure_gemv)
constexpr int kThreads = 128;  // 4 warps per CTA

struct PeerView {
    uint8_t *peer[kMaxRanks];  // mailbox base of every rank (peer[rank] is this rank's own)
    uint32_t n_ranks, rank, max_rows;
    uint64_t timeout_ns;
};

__device__ __forceinline__ uint32_t *flag_at(uint8_t *base, uint32_t src, uint32_t cta) {
    return reinterpret_cast<uint32_t *>(base + kFlagsOff) + size_t(src) * kMaxCtas + cta;
}
__device__ __forceinline__ uint32_t *ctl_at(uint8_t *base) { return reinterpret_cast<uint32_t *>(base + kCtlOff); }
__device__ __forceinline__ unsigned long long *row_slot(uint8_t *base, uint32_t par, uint32_t src, uint32_t v,
                                                        uint32_t max_rows) {
    return reinterpret_cast<unsigned long long *>(base + kRowsOff) +
           ((size_t(par) * kMaxRanks + src) * kPassVec + v) * max_rows;
}
__device__ __forceinline__ unsigned long long *key_slot(uint8_t *base, uint32_t par, uint32_t src) {
    return reinterpret_cast<unsigned long long *>(base + kKeysOff) + (size_t(par) * kMaxRanks + src) * kMaxKeys;
}

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long tagged(float v, uint32_t tag) {
    return (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
}

// Publishes this CTA's pushes to every rank and waits until the CTA of the same index on
// every rank has published collective `want`. Whole CTA; the barrier at entry makes every
// thread's pushes precede (in causality order) the release stores that thread 0..n-1 make at
// system scope, the one at exit orders the acquire loads before any thread reads the
// mailbox. Returns false after a timeout (recorded in the status word).
__device__ bool exchange(const PeerView &pv, uint32_t want, DeviceStatus *st, uint32_t where) {
    __shared__ int failed;
    if (threadIdx.x == 0) failed = 0;
    __syncthreads();
    if (threadIdx.x < pv.n_ranks) {
        st_release_sys(flag_at(pv.peer[threadIdx.x], pv.rank, blockIdx.x), want);
        const uint32_t *f = flag_at(pv.peer[pv.rank], threadIdx.x, blockIdx.x);
        if (int32_t(ld_acquire_sys(f) - want) < 0) {
            const uint64_t t0 = global_ns();
            for (uint32_t i = 1;; ++i) {
                if (int32_t(ld_acquire_sys(f) - want) >= 0) break;
                if ((i & 63u) == 0 &&
                    (global_ns() - t0 > pv.timeout_ns || *reinterpret_cast<volatile uint32_t *>(&st->code))) {
                    failed = 1;
                    report(st, OPURE_ERR_DEVICE_TIMEOUT, where, threadIdx.x);
                    break;
                }
            }
        }
    }
    __syncthreads();
    return !failed;
}

struct ArParams {
    const uint8_t *w;
    size_t pitch;
    uint32_t rows, cols, nchunks;
    float scale;
    const float *x;
    uint32_t x_stride;
    float *y;
    uint32_t y_stride;
    const float *residual;
    const __half *gain;
    float eps;
    DeviceStatus *st;
};

// y[v][row] = (residual[v][row] +) sum over ranks of scale * W_rank[row,:] . x_rank[v,:].
template <int WT, int NV, int PRO, bool ADD>
__global__ void __launch_bounds__(kThreads) gemv_allreduce_kernel(ArParams p, PeerView pv) {
    extern __shared__ __align__(16) float smem[];
    float *xs = smem;
    float *red = smem + NV * p.cols;
    __shared__ uint32_t s_seq;

    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t nwarps = gridDim.x * (kThreads / 32);
    const uint32_t groups = (p.rows + kRows - 1) / kRows;
    const uint32_t g0 = blockIdx.x * (kThreads / 32) + warp;

    RowPrefetch<kRows> pre;
    if (g0 < groups) prefetch_rows(pre, p.w, p.pitch, g0 * kRows, min(uint32_t(kRows), p.rows - g0 * kRows), p.nchunks);

    grid_dependency_wait();
    grid_dependents_launch();
    uint8_t *const local = pv.peer[pv.rank];
    if (threadIdx.x == 0) s_seq = *reinterpret_cast<volatile uint32_t *>(ctl_at(local));
    // int8 chunks span 16 elements: their vectors are staged chunk-interleaved (no bank
    // conflicts on the 64-byte-per-lane reads); fp16 keeps the plain layout, measured faster.
    constexpr bool kIL = WT == OPURE_W_Q8;
    if constexpr (kIL)
        stage_vectors_il<NV, WTraits<WT>::kElems>(p.x, p.x_stride, p.cols, PRO == OPURE_PRO_RMSNORM, p.gain, p.eps,
                                                  xs, red);
    else
        stage_vectors<NV>(p.x, p.x_stride, p.cols, PRO == OPURE_PRO_RMSNORM, p.gain, p.eps, xs, red);
    const uint32_t seq = s_seq, par = seq & 1u, want = seq + 1u;

    // This rank's partial rows, pushed into slot `rank` of every mailbox.
    for (uint32_t g = g0; g < groups; g += nwarps) {
        const uint32_t row0 = g * kRows;
        const uint32_t valid = min(uint32_t(kRows), p.rows - row0);
        float acc[kRows][NV];
        dot_rows<WT, NV, kRows, kIL>(p.w, p.pitch, row0, valid, p.nchunks, xs, p.cols, acc, pre, g == g0);
#pragma unroll
        for (int r = 0; r < kRows; ++r)
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                if (r >= int(valid) || lane != uint32_t((r * NV + v) & 31)) continue;
                const unsigned long long word = tagged(acc[r][v] * p.scale, want);
                for (uint32_t q = 0; q < pv.n_ranks; ++q)
                    st_relaxed_sys_u64(row_slot(pv.peer[q], par, pv.rank, v, pv.max_rows) + row0 + r, word);
            }
    }

    // Sum the ranks' words of this CTA's rows in rank order, once every tag is this
    // collective's. All n loads of a row are issued before any is checked.
    for (uint32_t g = g0; g < groups; g += nwarps) {
        const uint32_t row0 = g * kRows;
        const uint32_t valid = min(uint32_t(kRows), p.rows - row0);
#pragma unroll
        for (int r = 0; r < kRows; ++r)
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                if (r >= int(valid) || lane != uint32_t((r * NV + v) & 31)) continue;
                unsigned long long w[kMaxRanks];
                uint32_t missing = 0;
#pragma unroll
                for (uint32_t q = 0; q < kMaxRanks; ++q)
                    if (q < pv.n_ranks) {
                        w[q] = ld_relaxed_sys_u64(row_slot(local, par, q, v, pv.max_rows) + row0 + r);
                        if (uint32_t(w[q] >> 32) != want) missing |= 1u << q;
                    }
                if (missing) {
                    const uint64_t t0 = global_ns();
                    for (uint32_t i = 1; missing; ++i) {
#pragma unroll
                        for (uint32_t q = 0; q < kMaxRanks; ++q)
                            if (missing & (1u << q)) {
                                w[q] = ld_relaxed_sys_u64(row_slot(local, par, q, v, pv.max_rows) + row0 + r);
                                if (uint32_t(w[q] >> 32) == want) missing &= ~(1u << q);
                            }
                        if (missing && (i & 63u) == 0 &&
                            (global_ns() - t0 > pv.timeout_ns || *reinterpret_cast<volatile uint32_t *>(&p.st->code))) {
                            report(p.st, OPURE_ERR_DEVICE_TIMEOUT, 90, __ffs(missing) - 1);
                            break;
                        }
                    }
                }
                if (missing) continue;  // timed out: y keeps its old value, the status word says why
                float s = 0.f;
#pragma unroll
                for (uint32_t q = 0; q < kMaxRanks; ++q)
                    if (q < pv.n_ranks) s += __uint_as_float(uint32_t(w[q]));
                const size_t o = size_t(v) * p.y_stride + row0 + r;
                p.y[o] = ADD ? p.residual[o] + s : s;
            }
    }
    __syncthreads();

    // The last CTA out advances the collective sequence (every CTA read it before its ticket).
    if (threadIdx.x == 0) {
        uint32_t *ctl = ctl_at(local);
        if (atomicAdd(ctl + 1, 1u) == gridDim.x - 1) {
            atomicExch(ctl + 1, 0u);
            atomicAdd(ctl, 1u);
        }
    }
}

// keys[v] <- the largest argmax key over every rank's keys[v], after rewriting this rank's
// keys to global vocabulary indices (this shard's first row is `offset`). One CTA.
__global__ void __launch_bounds__(256) peer_argmax_kernel(unsigned long long *keys, uint32_t n, uint32_t offset,
                                                          PeerView pv, DeviceStatus *st) {
    grid_dependency_wait();
    grid_dependents_launch();
    __shared__ uint32_t s_seq;
    uint8_t *const local = pv.peer[pv.rank];
    if (threadIdx.x == 0) s_seq = *reinterpret_cast<volatile uint32_t *>(ctl_at(local));
    __syncthreads();
    const uint32_t seq = s_seq, par = seq & 1u;
    for (uint32_t v = threadIdx.x; v < n; v += blockDim.x) {
        unsigned long long k = keys[v];
        if (k) {
            const uint32_t idx = argmax_key_index(k) + offset;
            k = (k & 0xffffffff00000000ull) | (0xffffffffu - idx);
        }
        for (uint32_t q = 0; q < pv.n_ranks; ++q) key_slot(pv.peer[q], par, pv.rank)[v] = k;
    }
    exchange(pv, seq + 1u, st, 91);
    for (uint32_t v = threadIdx.x; v < n; v += blockDim.x) {
        unsigned long long best = 0ull;
        for (uint32_t q = 0; q < pv.n_ranks; ++q) {
            const unsigned long long k = __ldcg(key_slot(local, par, q) + v);
            best = k > best ? k : best;
        }
        keys[v] = best;
    }
    __syncthreads();
    if (threadIdx.x == 0) atomicAdd(ctl_at(local), 1u);
}

PeerView view(const opure_peer *pr) {
    PeerView pv{};
    for (uint32_t q = 0; q < pr->n_ranks; ++q) pv.peer[q] = pr->peer[q];
    pv.n_ranks = pr->n_ranks;
    pv.rank = pr->rank;
    pv.max_rows = pr->max_rows;
    pv.timeout_ns = pr->timeout_ns;
    return pv;
}

template <int WT, int NV, int PRO, bool ADD>
opure_status run_ar(opure_ctx *ctx, const ArParams &p, const PeerView &pv) {
    auto kern = gemv_allreduce_kernel<WT, NV, PRO, ADD>;
    const size_t smem = (size_t(NV) * p.cols + 33 * NV) * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e != cudaSuccess) return cuda_status(e);
    }
    // At most one CTA per SM and per flag slot: the whole grid is resident at once, and the
    // grid (hence each CTA's rows) is the same on every rank.
    const uint32_t groups = ceil_div(p.rows, kRows);
    const uint32_t cap = std::min<uint32_t>(uint32_t(ctx->sm_count), kMaxCtas);
    const uint32_t ctas = std::min<uint32_t>(ceil_div(groups, kThreads / 32), cap);
    return launch(ctx, kern, dim3(ctas), dim3(kThreads), smem, true, p, pv);
}

template <int WT, int NV>
opure_status pick_ar(opure_ctx *ctx, uint32_t pro, bool add, const ArParams &p, const PeerView &pv) {
    if (pro == OPURE_PRO_RMSNORM)
        return add ? run_ar<WT, NV, OPURE_PRO_RMSNORM, true>(ctx, p, pv) : run_ar<WT, NV, OPURE_PRO_RMSNORM, false>(ctx, p, pv);
    return add ? run_ar<WT, NV, OPURE_PRO_NONE, true>(ctx, p, pv) : run_ar<WT, NV, OPURE_PRO_NONE, false>(ctx, p, pv);
}

template <int WT>
opure_status pick_ar_nv(opure_ctx *ctx, uint32_t nv, uint32_t pro, bool add, const ArParams &p, const PeerView &pv) {
    switch (nv) {
        case 1: return pick_ar<WT, 1>(ctx, pro, add, p, pv);
        case 2: return pick_ar<WT, 2>(ctx, pro, add, p, pv);
        case 3: return pick_ar<WT, 3>(ctx, pro, add, p, pv);
        case 4: return pick_ar<WT, 4>(ctx, pro, add, p, pv);
        case 5: return pick_ar<WT, 5>(ctx, pro, add, p, pv);
        case 6: return pick_ar<WT, 6>(ctx, pro, add, p, pv);
        case 7: return pick_ar<WT, 7>(ctx, pro, add, p, pv);
        case 8: return pick_ar<WT, 8>(ctx, pro, add, p, pv);
        case 9: return pick_ar<WT, 9>(ctx, pro, add, p, pv);
    }
    return OPURE_ERR_INVALID_ARG;
}

// All-gather of kXchgWords u64 per rank through the communicator (each rank fills its own
// row, the others are zero, and a max all-reduce leaves every row everywhere).
opure_status gather_words(opure_ctx *ctx, opure_comm *comm, uint64_t *dev, std::vector<uint64_t> &tab,
                          uint32_t timeout_ms) {
    OPURE_CUDA_TRY(cudaMemcpyAsync(dev, tab.data(), tab.size() * 8, cudaMemcpyHostToDevice, ctx->stream));
    opure_status s = opure_allreduce_max_u64(ctx, comm, reinterpret_cast<unsigned long long *>(dev), tab.size());
    if (!s) s = opure_sync(ctx, timeout_ms);  // bounded: a rank that never joins ends here
    if (s) return s;
    OPURE_CUDA_TRY(cudaMemcpy(tab.data(), dev, tab.size() * 8, cudaMemcpyDeviceToHost));
    return OPURE_OK;
}

// Every rank learns whether any rank failed (a max all-reduce of one word).
opure_status agree(opure_ctx *ctx, opure_comm *comm, uint64_t *dev, uint32_t n_ranks, uint32_t rank, bool failed,
                   uint32_t timeout_ms, bool *any_failed) {
    std::vector<uint64_t> tab(size_t(n_ranks) * kXchgWords, 0);
    tab[size_t(rank) * kXchgWords] = failed ? 1 : 0;
    opure_status s = gather_words(ctx, comm, dev, tab, timeout_ms);
    if (s) return s;
    *any_failed = false;
    for (uint32_t q = 0; q < n_ranks; ++q) *any_failed |= tab[size_t(q) * kXchgWords] != 0;
    return OPURE_OK;
}

void release(opure_peer *pr) {
    for (uint32_t q = 0; q < pr->n_ranks; ++q)
        if (pr->peer[q] && pr->peer[q] != pr->local) cudaIpcCloseMemHandle(pr->peer[q]);
    if (pr->local) cudaFree(pr->local);
    cudaGetLastError();
    delete pr;
}

}  // namespace
}  // namespace opure

using namespace opure;

extern "C" {

opure_status opure_peer_create(opure_ctx *ctx, opure_comm *comm, uint32_t max_rows, uint32_t timeout_ms,
                               opure_peer **out) {
    if (!out) return OPURE_ERR_INVALID_ARG;
    *out = nullptr;
    opure_status s = enter(ctx);
    if (s) return s;
    uint32_t n = 0, rank = 0;
    if (!comm || max_rows == 0 || opure_comm_info(comm, &n, &rank) != OPURE_OK) return OPURE_ERR_INVALID_ARG;
    if (n > kMaxRanks) return OPURE_ERR_UNSUPPORTED;
    const uint32_t host_ms = 60000;  // bound of the set-up collectives
    auto *pr = new (std::nothrow) opure_peer;
    if (!pr) return OPURE_ERR_OUT_OF_MEMORY;
    pr->device = ctx->device;
    pr->n_ranks = n;
    pr->rank = rank;
    pr->max_rows = max_rows;
    pr->timeout_ns = uint64_t(timeout_ms ? timeout_ms : 2000) * 1000000ull;
    pr->bytes = (kRowsOff + size_t(2) * kMaxRanks * kPassVec * max_rows * 8 + 255) & ~size_t(255);
    void *mem = nullptr;
    cudaError_t e = cudaMalloc(&mem, pr->bytes);
    pr->local = e == cudaSuccess ? static_cast<uint8_t *>(mem) : nullptr;
    if (e == cudaSuccess) e = cudaMemsetAsync(pr->local, 0, pr->bytes, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        release(pr);
        return cuda_status(e);
    }
    pr->peer[rank] = pr->local;
    uint64_t *xchg = reinterpret_cast<uint64_t *>(pr->local + kXchgOff);
    static_assert(kXchgOff + size_t(kMaxRanks) * kXchgWords * 8 <= kKeysOff, "exchange words fit the control area");

    // Exchange (IPC handle, device ordinal, usable) with every rank.
    std::vector<uint64_t> tab(size_t(n) * kXchgWords, 0);
    cudaIpcMemHandle_t h{};
    const bool exported = cudaIpcGetMemHandle(&h, pr->local) == cudaSuccess;
    cudaGetLastError();
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle is 64 bytes");
    std::memcpy(&tab[size_t(rank) * kXchgWords], &h, 64);
    tab[size_t(rank) * kXchgWords + 8] = uint64_t(ctx->device) + 1;
    tab[size_t(rank) * kXchgWords + 9] = exported ? 1 : 0;
    s = gather_words(ctx, comm, xchg, tab, host_ms);
    if (s) {
        release(pr);
        return s;
    }
    // Map every other rank's mailbox. Two ranks on one GPU, a GPU pair without peer access or
    // a failed mapping on any rank makes every rank refuse (the caller keeps NCCL).
    bool failed = false;
    for (uint32_t q = 0; q < n && !failed; ++q) {
        if (q == rank) continue;
        const uint64_t *row = &tab[size_t(q) * kXchgWords];
        const int dev = int(row[8]) - 1;
        int can = 0;
        if (!row[9] || dev < 0 || dev == ctx->device || cudaDeviceCanAccessPeer(&can, ctx->device, dev) != cudaSuccess ||
            !can) {
            failed = true;
            break;
        }
        cudaIpcMemHandle_t hq;
        std::memcpy(&hq, row, 64);
        void *p = nullptr;
        if (cudaIpcOpenMemHandle(&p, hq, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            failed = true;
            break;
        }
        pr->peer[q] = static_cast<uint8_t *>(p);
    }
    cudaGetLastError();
    bool any = false;
    s = agree(ctx, comm, xchg, n, rank, failed, host_ms, &any);
    if (s || any) {
        release(pr);
        return s ? s : OPURE_ERR_UNSUPPORTED;
    }
    // Every mailbox was zeroed before the first exchange, so a rank may push as soon as it
    // returns from here; the exchange words are never read by the kernels.
    *out = pr;
    return OPURE_OK;
}

opure_status opure_peer_destroy(opure_ctx *ctx, opure_comm *comm, opure_peer *pr) {
    if (!pr) return OPURE_ERR_INVALID_ARG;
    opure_status s = enter(ctx);
    if (s) return s;
    if (ctx->device != pr->device) return OPURE_ERR_INVALID_ARG;
    s = opure_sync(ctx, 60000);
    // Every rank's kernels are done with every mailbox before any mapping is closed, and
    // every mapping of this rank's mailbox is closed before it is freed.
    bool any = false;
    uint64_t *xchg = reinterpret_cast<uint64_t *>(pr->local + kXchgOff);
    if (comm && !s) s = agree(ctx, comm, xchg, pr->n_ranks, pr->rank, false, 60000, &any);
    for (uint32_t q = 0; q < pr->n_ranks; ++q)
        if (pr->peer[q] && pr->peer[q] != pr->local) {
            cudaIpcCloseMemHandle(pr->peer[q]);
            pr->peer[q] = nullptr;
        }
    if (comm && !s) s = agree(ctx, comm, xchg, pr->n_ranks, pr->rank, false, 60000, &any);
    release(pr);
    return s;
}

opure_status opure_peer_info(const opure_peer *pr, uint32_t *n_ranks, uint32_t *rank, uint32_t *max_rows) {
    if (!pr) return OPURE_ERR_INVALID_ARG;
    if (n_ranks) *n_ranks = pr->n_ranks;
    if (rank) *rank = pr->rank;
    if (max_rows) *max_rows = pr->max_rows;
    return OPURE_OK;
}

opure_status opure_gemv_allreduce(opure_ctx *ctx, opure_peer *pr, const opure_gemv_args *a) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!pr || !a || !a->w || !a->x || !a->y || a->rows == 0 || a->cols == 0) return OPURE_ERR_INVALID_ARG;
    if (a->x_packed || a->y_packed || a->y_sumsq) return OPURE_ERR_UNSUPPORTED;
    if (ctx->device != pr->device) return OPURE_ERR_INVALID_ARG;
    if (a->nvec == 0) return OPURE_OK;
    if (a->w_dtype != OPURE_W_F16 && a->w_dtype != OPURE_W_Q8) return OPURE_ERR_INVALID_ARG;
    if (a->prologue > OPURE_PRO_RMSNORM) return OPURE_ERR_INVALID_ARG;
    if (a->epilogue != OPURE_EPI_STORE && a->epilogue != OPURE_EPI_ADD) return OPURE_ERR_INVALID_ARG;
    if (a->prologue == OPURE_PRO_RMSNORM && !a->norm_gain) return OPURE_ERR_INVALID_ARG;
    if (a->epilogue == OPURE_EPI_ADD && !a->residual) return OPURE_ERR_INVALID_ARG;
    if (a->rows > pr->max_rows) return OPURE_ERR_UNSUPPORTED;
    const uint32_t eb = a->w_dtype == OPURE_W_F16 ? 2u : 1u;
    if ((uint64_t(a->cols) * eb) % 16 || reinterpret_cast<uintptr_t>(a->w) % 16) return OPURE_ERR_UNSUPPORTED;
    if (a->x_stride < a->cols || a->y_stride < a->rows) return OPURE_ERR_INVALID_ARG;
    if (a->x_stride % 4 || reinterpret_cast<uintptr_t>(a->x) % 16) return OPURE_ERR_UNSUPPORTED;

    ArParams p{};
    p.w = static_cast<const uint8_t *>(a->w);
    p.pitch = size_t(a->cols) * eb;
    p.rows = a->rows;
    p.cols = a->cols;
    p.nchunks = uint32_t(p.pitch / 16);
    p.scale = a->w_dtype == OPURE_W_Q8 ? a->scale_w * a->scale_x : 1.0f;
    p.x_stride = a->x_stride;
    p.y_stride = a->y_stride;
    p.gain = reinterpret_cast<const __half *>(a->norm_gain);
    p.eps = a->eps;
    p.st = ctx->status;
    const PeerView pv = view(pr);
    const size_t budget = std::min<size_t>(ctx->smem_optin, 200 * 1024);
    const uint32_t per_pass = uint32_t(std::min<size_t>(kPassVec, budget / (size_t(a->cols) * 4 + 33 * 4)));
    if (per_pass == 0) return OPURE_ERR_UNSUPPORTED;
    const bool add = a->epilogue == OPURE_EPI_ADD;
    // One collective per pass of up to nine vectors; every rank makes the same passes.
    for (uint32_t v0 = 0; v0 < a->nvec; v0 += per_pass) {
        const uint32_t nv = std::min(per_pass, a->nvec - v0);
        p.x = a->x + size_t(v0) * a->x_stride;
        p.y = a->y + size_t(v0) * a->y_stride;
        p.residual = add ? a->residual + size_t(v0) * a->y_stride : nullptr;
        s = a->w_dtype == OPURE_W_F16 ? pick_ar_nv<OPURE_W_F16>(ctx, nv, a->prologue, add, p, pv)
                                      : pick_ar_nv<OPURE_W_Q8>(ctx, nv, a->prologue, add, p, pv);
        if (s) return s;
    }
    return OPURE_OK;
}

opure_status opure_peer_argmax(opure_ctx *ctx, opure_peer *pr, unsigned long long *keys, uint32_t n,
                               uint32_t offset) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!pr || !keys || ctx->device != pr->device) return OPURE_ERR_INVALID_ARG;
    if (n > kMaxKeys) return OPURE_ERR_UNSUPPORTED;
    if (n == 0) return OPURE_OK;
    return launch(ctx, peer_argmax_kernel, dim3(1), dim3(256), 0, true, keys, n, offset, view(pr), ctx->status);
}

}  // extern "C"
