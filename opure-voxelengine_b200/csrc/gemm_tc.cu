// gemm_tc.cu -- opure_gemv for 16..256 token vectors per pass on the tcgen05 tensor cores.
//
// With many vectors (batched decode, the k+1-position speculative verify pass) the GEMV
// Y[v][row] = sum_k W[row][k] x[v][k] is a dense contraction: weights are streamed once
// for all vectors and the products run on the 5th-generation tensor cores.
//
//   pack   one CTA per vector: optional RMSNorm (the GEMV prologue), then the vector is
//          scaled by a power of two s_v and split into two fp16 halves
//          x / s_v = hi + lo  (hi = fp16(x / s_v), lo = fp16(x / s_v - hi)),
//          which keeps ~22 significant bits: W.x = s_v (W.hi + W.lo) with fp16 x fp16
//          products accumulated in fp32, the accuracy of the fp32 CUDA-core GEMV.
//   gemm   one CTA per (128-row tile, K split, vector slice of nt). Thread 0 streams
//          128x64 weight tiles and the matching 64-column slices of the packed vectors with
//          TMA (128-byte swizzle) into a ring of shared-memory stages, the slice's hi rows
//          and lo rows side by side; thread 32 issues one tcgen05.mma per K=16 step with
//          M=128 and N=2 nt (hi and lo vectors together, fp16 in, fp32 out), so each weight
//          tile is read once for both halves, into a TMEM accumulator whose first nt
//          columns hold W.hi and next nt W.lo (a second one for the SwiGLU up half), and
//          frees each stage with tcgen05.commit. The eight warps then read the accumulator
//          rows with tcgen05.ld (warps w and w + 4 share TMEM lanes 32 (w % 4) .. = tile
//          rows, each taking half of every 16-column chunk) and apply the epilogue: store,
//          residual add, SwiGLU, or argmax keys (+ logits). With a K split every
//          CTA adds its sums into a 64-bit fixed-point accumulator with integer atomics
//          and the last CTA of the tile (ticket counter) converts them and runs the
//          epilogue, so results do not depend on the order the splits finish in.
//   chained  consecutive GEMVs of a decode layer skip the pack kernel: the producer (a
//          GEMM epilogue, or the attention kernel) writes its output vectors as scale-free
//          fp16 pairs hi = fp16(v), lo = fp16((v - hi) 2^11) (store_packed), and the
//          consumer accumulates W.hi and W.lo in two TMEM accumulators and adds them as
//          D_hi + 2^-11 D_lo. The RMSNorm of a chained input moves into the consumer's
//          epilogue: the producer multiplies the packed values by the norm gain and writes,
//          per 128-row tile, the sum of squares of each vector (deterministic: one writer per
//          tile and vector); the consumer adds the tiles' sums in tile order and scales its
//          results by 1/rms. W.(g x / rms) = (W.(g x)) / rms.
// All waits are bounded (1 s); a timeout is reported in the ctx status word and the CTA
// still releases its TMEM. No TMA multicast is used.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "gemm_tc.cuh"
#include "tma.cuh"

namespace opure {
namespace {

constexpr uint32_t kTileM = 128;   // weight rows per tile = TMEM lanes
constexpr uint32_t kTileK = 64;    // 64 fp16 = one 128-byte swizzle row
constexpr uint32_t kThreads = 256;  // 8 warps: warp w reads TMEM lanes 32 (w % 4) .., columns half w / 4
constexpr uint32_t kHalfCols = 8;   // epilogue columns per thread per 16-column chunk
constexpr uint32_t kMaxN = 256;    // vectors per pass (MMA N limit)
constexpr uint32_t kMaxStages = 8;
constexpr uint32_t kMaxTickets = 4096;
// Workspace layout (ctx->ws).
constexpr size_t kPackOff = 0;
constexpr size_t kPackBytes = size_t(2) * kMaxN * kTcMaxCols * 2;
constexpr size_t kScaleOff = kPackOff + kPackBytes;
constexpr size_t kTicketOff = kScaleOff + kMaxN * 4;
constexpr size_t kPartialOff = (kTicketOff + kMaxTickets * 4 + 255) & ~size_t(255);
static_assert(kPartialOff < kTcWorkspaceBytes, "workspace layout");

// ---- PTX wrappers -------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint32_t x, uint32_t y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor of a K-major tile stored as 128-byte swizzled rows
// (the layout TMA writes with CU_TENSOR_MAP_SWIZZLE_128B): 8-row groups 1024 bytes
// apart, descriptor version 1, layout type 2 (128-byte swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    return uint64_t((addr & 0x3FFFFu) >> 4) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
           (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (fp16 inputs, fp32 accumulate).
__device__ __forceinline__ void mma_f16(uint32_t tmem, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem),
        "l"(da), "l"(db), "r"(idesc), "r"(acc)
        : "memory");
}

// Arrives on `bar` once every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

// Issues the load of 8 consecutive fp32 accumulator columns of this thread's TMEM lane
// into r (valid after tmem_wait_ld).
__device__ __forceinline__ void tmem_ld8_issue(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xffffffffu, v, o);
        v = t > v ? t : v;
    }
    return v;
}

// ---- pack ---------------------------------------------------------------------------
constexpr uint32_t kPackThreads = 256;

struct PackParams {
    const float *x;
    uint32_t x_stride, K, npad;
    uint32_t rmsnorm;
    const __half *gain;
    float eps;
    __half *xp;      // [2 npad][K]: hi rows 0..npad-1, lo rows npad..2 npad-1
    float *xscale;   // [npad]
};

__device__ float block_reduce(float v, bool is_max, float *red) {
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float t = __shfl_xor_sync(0xffffffffu, v, o);
        v = is_max ? fmaxf(v, t) : v + t;
    }
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float r = is_max ? 0.f : 0.f;
    for (uint32_t w = 0; w < nw; ++w) r = is_max ? fmaxf(r, red[w]) : r + red[w];
    return r;
}

__global__ void __launch_bounds__(kPackThreads) pack_kernel(PackParams p) {
    extern __shared__ float row[];  // [K]
    __shared__ float red[32];
    grid_dependency_wait();
    grid_dependents_launch();
    const uint32_t v = blockIdx.x;
    const float *x = p.x + size_t(v) * p.x_stride;
    float ss = 0.f;
    for (uint32_t i = threadIdx.x; i < p.K; i += blockDim.x) {
        const float t = x[i];
        row[i] = t;
        ss = fmaf(t, t, ss);
    }
    float inv = 1.f;
    if (p.rmsnorm) {
        const float tot = block_reduce(ss, false, red);
        // The GEMV prologue's RMSNorm (RMSNormMain, Opure_RMSNorm.usf:31-79).
        inv = float(1.0 / sqrt(double(tot) / double(p.K) + double(p.eps)));
    }
    float amax = 0.f;
    for (uint32_t i = threadIdx.x; i < p.K; i += blockDim.x) {
        float t = row[i];
        if (p.rmsnorm) t = t * inv * __half2float(p.gain[i]);
        row[i] = t;
        amax = fmaxf(amax, fabsf(t));
    }
    amax = block_reduce(amax, true, red);
    // s = 2^(e - 14) with amax < 2^e, so |x / s| < 2^14 stays inside fp16's range.
    int e = 0;
    if (amax > 0.f && amax <= 3.0e38f) frexpf(amax, &e);
    const float s = ldexpf(1.f, e - 14), rs = ldexpf(1.f, 14 - e);
    if (threadIdx.x == 0) p.xscale[v] = s;
    __half *hi = p.xp + size_t(v) * p.K;
    __half *lo = p.xp + size_t(p.npad + v) * p.K;
    for (uint32_t i = threadIdx.x; i < p.K; i += blockDim.x) {
        const float t = row[i] * rs;
        const __half h = __float2half_rn(t);
        hi[i] = h;
        lo[i] = __float2half_rn(t - __half2float(h));
    }
    // The GEMM reads these rows through TMA (the async proxy).
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---- GEMM ---------------------------------------------------------------------------
struct TcParams {
    uint32_t rows, n, npad, ktiles, kt_per_split, splits, stages;
    uint32_t nt;        // vectors per CTA (blockIdx.z selects vectors [z nt, z nt + nt))
    float *y;
    uint32_t y_stride;
    const float *residual;
    unsigned long long *keys;
    const float *xscale;
    long long *accum;   // [tiles][npad / nt][accumulators * nt][128] fixed-point split-K sums
    uint32_t *tickets;  // [tiles][npad / nt]
    DeviceStatus *st;
    // Chained operands (see the file comment).
    uint32_t chained;       // the B operand is a scale-free packed operand
    uint32_t K;
    const float *x_sumsq;   // chained RMSNorm: [ceil(K / 128)][n] partial sums of squares
    float eps;
    __half *y_packed;       // [2][npad][rows] or null
    const __half *y_gain;   // [rows] or null
    float *y_sumsq;         // [tiles][n] or null
};

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap, TcParams p) {
    constexpr bool kSwiglu = EPI == OPURE_EPI_SWIGLU;
    constexpr uint32_t kAcc = kSwiglu ? 2 : 1;
    extern __shared__ uint8_t dsm[];
    __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages], done;
    __shared__ uint32_t tmem_base;
    __shared__ int fail, last;
    __shared__ uint32_t issued_s, consumed_s;
    __shared__ float s_scale[kMaxN];
    __shared__ float s_red[4][16];
    __shared__ __align__(16) __half s_pk[2][16][kTileM];  // packed output chunk, transposed

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t tile = blockIdx.x, split = blockIdx.y;
    const uint32_t m0 = tile * kTileM;
    const uint32_t nt = p.nt, n0 = blockIdx.z * nt;        // this CTA's vectors
    const uint32_t slice = tile * gridDim.z + blockIdx.z;  // (tile, vector slice) index
    const uint32_t kt0 = split * p.kt_per_split;
    const uint32_t nk = min(p.ktiles, kt0 + p.kt_per_split) - kt0;
    const uint32_t a_bytes = kTileM * 128, b_bytes = nt * 128;
    const uint32_t stage_bytes = kAcc * a_bytes + 2 * b_bytes;
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
    auto a_tile = [&](uint32_t s, uint32_t j) { return base + size_t(s) * stage_bytes + j * a_bytes; };
    auto b_tile = [&](uint32_t s, uint32_t j) { return base + size_t(s) * stage_bytes + kAcc * a_bytes + j * b_bytes; };
    // Accumulator a (gate / up) spans columns [2 nt a, 2 nt a + 2 nt): W.hi, then W.lo.
    const float lo_scale = p.chained ? 1.0f / 2048.0f : 1.0f;
    uint32_t ncols = 32;
    while (ncols < kAcc * 2 * nt) ncols <<= 1;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < p.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&done, 1);
        fail = 0;
        last = 0;
        issued_s = 0;
        consumed_s = 0;
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&wmap)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
    }
    if (warp == 2) tmem_alloc(&tmem_base, ncols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;

    // The next norm's gain of this thread's epilogue row is a weight too: requested now,
    // converted only in the epilogue.
    const uint32_t erow = m0 + (warp & 3u) * 32 + lane;
    __half gain_h = __float2half_rn(1.f);
    if (p.y_packed && p.y_gain && erow < p.rows) gain_h = p.y_gain[erow];
    // Producer (warp 0, one lane). Weight tiles do not depend on earlier kernels: the
    // first stages are requested before waiting on them; the packed vectors only after.
    const uint32_t pre = min(p.stages, nk);
    if (warp == 0 && lane == 0)
        for (uint32_t i = 0; i < pre; ++i) {
            mbar_expect_tx(&full[i], stage_bytes);
            tma_load_2d(a_tile(i, 0), &wmap, (kt0 + i) * kTileK, m0, &full[i]);
            if (kSwiglu) tma_load_2d(a_tile(i, 1), &wmap, (kt0 + i) * kTileK, p.rows + m0, &full[i]);
        }
    grid_dependency_wait();
    grid_dependents_launch();
    if (warp == 0) {
        if (lane == 0) {
            for (uint32_t i = 0; i < pre; ++i) {
                tma_load_2d(b_tile(i, 0), &xmap, (kt0 + i) * kTileK, n0, &full[i]);
                tma_load_2d(b_tile(i, 1), &xmap, (kt0 + i) * kTileK, p.npad + n0, &full[i]);
            }
            uint32_t i = pre;
            for (; i < nk; ++i) {
                const uint32_t s = i % p.stages;
                if (!mbar_wait(&empty[s], ((i / p.stages) & 1u) ^ 1u)) {
                    report(p.st, OPURE_ERR_DEVICE_TIMEOUT, 60, blockIdx.x);
                    fail = 1;
                    break;
                }
                mbar_expect_tx(&full[s], stage_bytes);
                tma_load_2d(a_tile(s, 0), &wmap, (kt0 + i) * kTileK, m0, &full[s]);
                if (kSwiglu) tma_load_2d(a_tile(s, 1), &wmap, (kt0 + i) * kTileK, p.rows + m0, &full[s]);
                tma_load_2d(b_tile(s, 0), &xmap, (kt0 + i) * kTileK, n0, &full[s]);
                tma_load_2d(b_tile(s, 1), &xmap, (kt0 + i) * kTileK, p.npad + n0, &full[s]);
            }
            issued_s = i;
        }
        // The other lanes park here rather than spinning beside the issuing lane.
        __syncwarp();
    } else if (warp >= 2) {
        // Per-vector scales written by the pack kernel, or for a chained input 1 / rms from
        // the producer's per-tile sums of squares; used only by the epilogue.
        for (uint32_t v = threadIdx.x - 64; v < p.npad; v += blockDim.x - 64) {
            float sc = 0.f;
            if (v < p.n) {
                if (!p.chained) {
                    sc = p.xscale[v];
                } else if (p.x_sumsq) {
                    double ss = 0.0;
                    for (uint32_t t = 0; t < (p.K + kTileM - 1) / kTileM; ++t)
                        ss += double(__ldcg(p.x_sumsq + size_t(t) * p.n + v));
                    // The GEMV prologue's RMSNorm (RMSNormMain, Opure_RMSNorm.usf:31-79).
                    sc = float(1.0 / sqrt(ss / double(p.K) + double(p.eps)));
                } else {
                    sc = 1.f;
                }
            }
            s_scale[v] = sc;
        }
    }
    if (warp == 1) {
        if (lane == 0) {
            // MMA issuer: per 64-wide K tile, four K=16 steps (32 bytes along the swizzled
            // rows) of hi and lo products.
            const uint32_t idesc = (1u << 4) | (((2 * nt) >> 3) << 17) | ((kTileM >> 4) << 24);
            uint32_t i = 0;
            for (; i < nk; ++i) {
                const uint32_t s = i % p.stages;
                if (!mbar_wait(&full[s], (i / p.stages) & 1u)) {
                    report(p.st, OPURE_ERR_DEVICE_TIMEOUT, 61, blockIdx.x);
                    fail = 1;
                    break;
                }
                tc_fence_after();
                // b_tile(s, 1) follows b_tile(s, 0) directly: one K-major operand of 2 nt rows.
                const uint32_t a0 = smem_addr(a_tile(s, 0)), bh = smem_addr(b_tile(s, 0));
#pragma unroll
                for (uint32_t k = 0; k < kTileK / 16; ++k) {
                    const uint64_t db = smem_desc(bh + 32 * k);
                    const uint64_t da = smem_desc(a0 + 32 * k);
                    const uint32_t accum = (i | k) != 0;
                    mma_f16(tmem, da, db, idesc, accum);
                    if (kSwiglu) {
                        const uint64_t du = smem_desc(smem_addr(a_tile(s, 1)) + 32 * k);
                        mma_f16(tmem + 2 * nt, du, db, idesc, accum);
                    }
                }
                mma_commit(&empty[s]);
            }
            consumed_s = i;
            mma_commit(&done);
        }
        __syncwarp();
    }

    // Epilogue: every thread owns one tile row (TMEM lane).
    if (!mbar_wait(&done, 0)) report(p.st, OPURE_ERR_DEVICE_TIMEOUT, 62, blockIdx.x);
    tc_fence_after();
    __syncthreads();
    __syncwarp();
    if (fail) {
        // Leave no copy in flight into this CTA's shared memory.
        if (threadIdx.x == 0)
            for (uint32_t i = consumed_s; i < issued_s; ++i) mbar_wait(&full[i % p.stages], (i / p.stages) & 1u);
    } else {
        // Warps w and w + 4 share TMEM lanes 32 (w % 4) .. (tile rows); in each 16-column
        // chunk warp w takes columns 0..7 and warp w + 4 columns 8..15.
        const uint32_t quarter = warp & 3u, half = warp >> 2;
        const uint32_t lrow = quarter * 32 + lane;
        const uint32_t row = m0 + lrow;
        const uint32_t taddr = tmem + ((quarter * 32) << 16);
        const uint32_t acc_cols = kAcc * nt;
        // Result columns c .. c+7 (accumulator c / nt) of this thread's row: W.hi plus W.lo
        // (scaled by 2^-11 for a chained operand).
        auto tm_col = [&](uint32_t c, float (&r)[kHalfCols]) {
            const uint32_t col = (c / nt) * 2 * nt + c % nt;
            uint32_t h[kHalfCols], l[kHalfCols];
            tmem_ld8_issue(taddr + col, h);
            tmem_ld8_issue(taddr + col + nt, l);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < int(kHalfCols); ++j) r[j] = fmaf(__uint_as_float(l[j]), lo_scale, __uint_as_float(h[j]));
        };
        bool run_epi = true;
        long long *acc64 = nullptr;
        if (p.splits > 1) {
            // K split: add this split's sums into the tile's 64-bit fixed-point (2^-32)
            // accumulator; integer adds are associative, so the total does not depend on
            // the order the splits arrive in. Column-major: a warp's adds are contiguous.
            acc64 = p.accum + size_t(slice) * acc_cols * kTileM;
            for (uint32_t c0 = half * kHalfCols; c0 < acc_cols; c0 += 16) {
                float r[kHalfCols];
                tm_col(c0, r);
#pragma unroll
                for (int j = 0; j < int(kHalfCols); ++j)
                    atomicAdd(reinterpret_cast<unsigned long long *>(acc64 + size_t(c0 + j) * kTileM + lrow),
                              static_cast<unsigned long long>(to_fix(r[j])));
            }
            __threadfence();
            __syncthreads();
            if (threadIdx.x == 0) {
                const uint32_t t = atomicAdd(&p.tickets[slice], 1u);
                last = t == p.splits - 1;
                if (last) p.tickets[slice] = 0;  // ready for the next call
            }
            __syncthreads();
            run_epi = last;
            __threadfence();
        }
        if (run_epi) {
            // Full sums of this thread's 8 columns from c (the last split also clears the
            // accumulator for the next call).
            auto column = [&](uint32_t c, float (&r)[kHalfCols]) {
                if (p.splits == 1) {
                    tm_col(c, r);
                } else {
                    long long a[kHalfCols];
#pragma unroll
                    for (int j = 0; j < int(kHalfCols); ++j) a[j] = __ldcg(acc64 + size_t(c + j) * kTileM + lrow);
#pragma unroll
                    for (int j = 0; j < int(kHalfCols); ++j) {
                        acc64[size_t(c + j) * kTileM + lrow] = 0;
                        r[j] = float(double(a[j]) * kFixInv);
                    }
                }
            };
            // Per chunk: every global load (the residual) is issued before any store, and the
            // vector scales come from shared memory, so a thread pays one memory round trip
            // per chunk rather than one per column.
            const bool in = row < p.rows;
            const float ygain = __half2float(gain_h);
            for (uint32_t c16 = 0; c16 < nt; c16 += 16) {
                const uint32_t c0 = c16 + half * kHalfCols;  // this thread's first column
                float outv[kHalfCols];
                float g[kHalfCols], u[kHalfCols], res[kHalfCols];
                column(c0, g);
                if (kSwiglu) column(nt + c0, u);
#pragma unroll
                for (int j = 0; j < int(kHalfCols); ++j) {
                    res[j] = 0.f;
                    if constexpr (EPI == OPURE_EPI_ADD)
                        if (in && n0 + c0 + j < p.n) res[j] = __ldcg(p.residual + size_t(n0 + c0 + j) * p.y_stride + row);
                }
#pragma unroll
                for (int j = 0; j < int(kHalfCols); ++j) {
                    const uint32_t v = n0 + c0 + j;
                    const bool ok = in && v < p.n;
                    const float val = g[j] * s_scale[v];
                    const size_t o = size_t(v) * p.y_stride + row;
                    outv[j] = 0.f;
                    if constexpr (EPI == OPURE_EPI_STORE) {
                        outv[j] = val;
                        if (ok) p.y[o] = val;
                    } else if constexpr (EPI == OPURE_EPI_ADD) {
                        outv[j] = res[j] + val;
                        if (ok) p.y[o] = outv[j];
                    } else if constexpr (EPI == OPURE_EPI_SWIGLU) {
                        const float uv = u[j] * s_scale[v];
                        const float sg = 1.0f / (1.0f + expf(-val));
                        outv[j] = (val * sg) * uv;
                        if (ok) p.y[o] = outv[j];
                    } else {
                        if (ok && p.y) p.y[o] = val;
                        const unsigned long long k = warp_max_u64(ok ? argmax_key(val, row) : 0ull);
                        if (lane == 0 && k) atomicMax(p.keys + v, k);
                    }
                }
                if constexpr (EPI != OPURE_EPI_ARGMAX) {
                    // The next GEMV's packed operand: each thread's hi/lo halves go to shared
                    // memory by vector, then every vector's 128-row slice leaves as 16-byte
                    // stores (rows is a multiple of 8).
                    if (p.y_packed) {
#pragma unroll
                        for (int j = 0; j < int(kHalfCols); ++j) {
                            float v = outv[j] * ygain;
                            if (!(fabsf(v) < 65504.f)) {
                                if (in && n0 + c0 + j < p.n) report(p.st, OPURE_ERR_DEVICE_BOUNDS, 63, row);
                                v = 0.f;
                            }
                            const __half hi = __float2half_rn(v);
                            s_pk[0][half * kHalfCols + j][lrow] = hi;
                            s_pk[1][half * kHalfCols + j][lrow] = __float2half_rn((v - __half2float(hi)) * 2048.f);
                        }
                        __syncthreads();
                        for (uint32_t idx = threadIdx.x; idx < 2 * 16 * (kTileM / 8); idx += blockDim.x) {
                            const uint32_t r = idx / (kTileM / 8), c = idx % (kTileM / 8);
                            const uint32_t h = r / 16, j = r % 16, v = n0 + c16 + j;
                            if (v < p.n && m0 + c * 8 < p.rows)
                                *reinterpret_cast<uint4 *>(p.y_packed + (size_t(h) * p.npad + v) * p.rows + m0 + c * 8) =
                                    *reinterpret_cast<const uint4 *>(&s_pk[h][j][c * 8]);
                        }
                        __syncthreads();
                    }
                    if (p.y_sumsq) {
#pragma unroll
                        for (int j = 0; j < int(kHalfCols); ++j) {
                            const float sq = warp_sum((in && n0 + c0 + j < p.n) ? outv[j] * outv[j] : 0.f);
                            if (lane == 0) s_red[quarter][half * kHalfCols + j] = sq;
                        }
                        __syncthreads();
                        if (threadIdx.x < 16 && n0 + c16 + threadIdx.x < p.n) {
                            float t = 0.f;
                            for (uint32_t q = 0; q < 4; ++q) t += s_red[q][threadIdx.x];
                            p.y_sumsq[size_t(tile) * p.n + n0 + c16 + threadIdx.x] = t;
                        }
                        __syncthreads();
                    }
                }
            }
            // A packed output is read by the next kernel's TMA (the async proxy).
            if (p.y_packed) asm volatile("fence.proxy.async.global;" ::: "memory");
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) tmem_dealloc(tmem, ncols);
}

// ---- host ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// Row-major fp16 [rows][K] matrix, boxes of 64 columns x box_rows rows, 128-byte swizzle.
bool make_map(CUtensorMap *m, const void *ptr, uint32_t K, uint32_t rows, uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {K, rows};
    const cuuint64_t strides[1] = {cuuint64_t(K) * 2};
    const cuuint32_t box[2] = {kTileK, box_rows};
    const cuuint32_t es[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int EPI>
opure_status launch_gemm(opure_ctx *ctx, const CUtensorMap &wm, const CUtensorMap &xm, const TcParams &p,
                         uint32_t tiles, size_t smem) {
    static_assert(EPI >= 0, "");
    const cudaError_t e =
        cudaFuncSetAttribute(gemm_tc_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return cuda_status(e);
    return launch(ctx, gemm_tc_kernel<EPI>, dim3(tiles, p.splits, p.npad / p.nt), dim3(kThreads), smem, true, wm, xm, p);
}

}  // namespace

bool gemv_tc_eligible(const opure_ctx *ctx, const opure_gemv_args *a) {
    return ctx->ws && ctx->ws_bytes >= kTcWorkspaceBytes && a->w_dtype == OPURE_W_F16 && a->nvec >= kTcMinVec &&
           a->cols % kTileK == 0 && a->cols <= kTcMaxCols && encode_fn() != nullptr;
}

size_t packed_bytes(uint32_t nvec, uint32_t len) {
    return size_t(2) * ((nvec + 15) & ~15u) * len * 2;
}

opure_status gemv_tc(opure_ctx *ctx, const opure_gemv_args *a) {
    const uint32_t K = a->cols, rows = a->rows;
    const uint32_t epi = a->epilogue;
    const uint32_t acc = epi == OPURE_EPI_SWIGLU ? 2 : 1;
    const bool chained_in = a->x_packed != nullptr;
    const bool chained = chained_in || a->y_packed || a->y_sumsq;
    if (chained) {
        // One pass; the packed buffers hold all vectors.
        if (a->nvec > kMaxN || epi == OPURE_EPI_ARGMAX && (a->y_packed || a->y_sumsq)) return OPURE_ERR_UNSUPPORTED;
        if (chained_in && a->prologue == OPURE_PRO_RMSNORM && !a->x_sumsq) return OPURE_ERR_INVALID_ARG;
        if (chained_in && reinterpret_cast<uintptr_t>(a->x_packed) % 16) return OPURE_ERR_UNSUPPORTED;
        if (a->y_packed && (rows % 8 || reinterpret_cast<uintptr_t>(a->y_packed) % 16)) return OPURE_ERR_UNSUPPORTED;
    }
    uint8_t *ws = static_cast<uint8_t *>(ctx->ws);
    __half *xp = reinterpret_cast<__half *>(ws + kPackOff);
    float *xscale = reinterpret_cast<float *>(ws + kScaleOff);
    uint32_t *tickets = reinterpret_cast<uint32_t *>(ws + kTicketOff);
    long long *accum = reinterpret_cast<long long *>(ws + kPartialOff);
    const size_t accum_cap = (ctx->ws_bytes - kPartialOff) / 8;

    CUtensorMap wm;
    if (!make_map(&wm, a->w, K, acc * rows, kTileM)) return OPURE_ERR_UNSUPPORTED;
    const size_t pack_smem = size_t(K) * 4;
    if (pack_smem > 48 * 1024) {
        const cudaError_t e =
            cudaFuncSetAttribute(pack_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(pack_smem));
        if (e != cudaSuccess) return cuda_status(e);
    }
    const uint32_t tiles = ceil_div(rows, kTileM);
    const uint32_t ktiles = K / kTileK;
    for (uint32_t v0 = 0; v0 < a->nvec; v0 += kMaxN) {
        const uint32_t n = std::min(kMaxN, a->nvec - v0);
        const uint32_t npad = (n + 15) & ~15u;
        opure_status s = OPURE_OK;
        if (!chained_in) {
            PackParams pp{a->x + size_t(v0) * a->x_stride, a->x_stride, K, npad, a->prologue == OPURE_PRO_RMSNORM,
                          reinterpret_cast<const __half *>(a->norm_gain), a->eps, xp, xscale};
            s = launch(ctx, pack_kernel, dim3(n), dim3(kPackThreads), pack_smem, true, pp);
            if (s) return s;
        }
        // Work split, latency first. Vector slices (blockIdx.z) need no reduction: as many
        // as fit one wave. A K split adds a fixed-point atomic reduction and a ticket, so it
        // is used only for long K (more than 12 tiles of 64), about one CTA per SM at most.
        const uint32_t sms = uint32_t(ctx->sm_count);
        // The MMA's N is 2 nt (hi and lo rows) <= 256, and the accumulators take
        // acc * 2 nt of the SM's 512 TMEM columns.
        uint32_t nz = 1;
        for (uint32_t c = 1; c <= npad / 16; ++c)
            if ((npad / 16) % c == 0 && tiles * c <= sms) nz = c;
        while (npad / nz > 128 || acc * 2 * (npad / nz) > 512) {
            uint32_t c = nz + 1;
            while ((npad / 16) % c) ++c;
            nz = c;
        }
        const uint32_t nt = npad / nz;
        uint32_t splits = 1;
        if (ktiles > 12 && tiles * nz < sms && size_t(tiles) * nz <= kMaxTickets &&
            size_t(tiles) * acc * npad * kTileM <= accum_cap)
            splits = std::max<uint32_t>(1, std::min<uint32_t>(ceil_div(ktiles, 12), sms / (tiles * nz)));
        const uint32_t kt_per = ceil_div(ktiles, splits);
        splits = ceil_div(ktiles, kt_per);
        CUtensorMap xm;
        if (!make_map(&xm, chained_in ? static_cast<const void *>(a->x_packed) : xp, K, 2 * npad, nt))
            return OPURE_ERR_UNSUPPORTED;

        const uint32_t stage_bytes = acc * kTileM * 128 + 2 * nt * 128;
        // Dynamic shared memory left after the kernel's static arrays and the 1 KB used to
        // align the stages.
        cudaFuncAttributes fa{};
        if (cudaFuncGetAttributes(&fa, gemm_tc_kernel<OPURE_EPI_SWIGLU>) != cudaSuccess) return OPURE_ERR_CUDA;
        const size_t budget = std::min<size_t>(ctx->smem_optin, 227 * 1024) - fa.sharedSizeBytes - 1024 - 256;
        const uint32_t stages = std::min<uint32_t>({kMaxStages, uint32_t(budget / stage_bytes), kt_per});
        if (stages < 1 || (stages < 2 && kt_per > 1)) return OPURE_ERR_UNSUPPORTED;

        TcParams p{};
        p.rows = rows;
        p.n = n;
        p.npad = npad;
        p.nt = nt;
        p.ktiles = ktiles;
        p.kt_per_split = kt_per;
        p.splits = splits;
        p.stages = stages;
        p.y = a->y ? a->y + size_t(v0) * a->y_stride : nullptr;
        p.y_stride = a->y_stride;
        p.residual = a->residual ? a->residual + size_t(v0) * a->y_stride : nullptr;
        p.keys = a->argmax_keys ? a->argmax_keys + v0 : nullptr;
        p.xscale = xscale;
        p.accum = accum;
        p.tickets = tickets;
        p.st = ctx->status;
        p.chained = chained_in;
        p.K = K;
        p.x_sumsq = chained_in && a->prologue == OPURE_PRO_RMSNORM ? a->x_sumsq : nullptr;
        p.eps = a->eps;
        p.y_packed = reinterpret_cast<__half *>(a->y_packed);
        p.y_gain = reinterpret_cast<const __half *>(a->y_pack_gain);
        p.y_sumsq = a->y_sumsq;
        // Request enough shared memory that no more CTAs fit on an SM than its 512 TMEM
        // columns can serve, so tcgen05.alloc never waits on a co-resident CTA.
        uint32_t ncols = 32;
        while (ncols < acc * 2 * nt) ncols <<= 1;
        const size_t per_sm = ctx->smem_optin + 1024;
        const size_t smem = std::max<size_t>(size_t(stages) * stage_bytes + 1024, per_sm / (512 / ncols + 1) + 1);
        if (smem + fa.sharedSizeBytes > ctx->smem_optin) return OPURE_ERR_UNSUPPORTED;
        switch (epi) {
            case OPURE_EPI_STORE: s = launch_gemm<OPURE_EPI_STORE>(ctx, wm, xm, p, tiles, smem); break;
            case OPURE_EPI_ADD: s = launch_gemm<OPURE_EPI_ADD>(ctx, wm, xm, p, tiles, smem); break;
            case OPURE_EPI_SWIGLU: s = launch_gemm<OPURE_EPI_SWIGLU>(ctx, wm, xm, p, tiles, smem); break;
            default: s = launch_gemm<OPURE_EPI_ARGMAX>(ctx, wm, xm, p, tiles, smem); break;
        }
        if (s) return s;
    }
    return OPURE_OK;
}

}  // namespace opure
