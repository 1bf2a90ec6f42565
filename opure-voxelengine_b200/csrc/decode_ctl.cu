// decode_ctl.cu -- opure_step_begin / opure_step_end: per-step token bookkeeping on the
// device, so a captured decode-step graph needs no host round trip between tokens.
#include "ctx.cuh"

namespace opure {
namespace {

__global__ void step_begin_kernel(opure_step_io io, DeviceStatus *st) {
    const uint32_t v = blockIdx.x;
    __shared__ int32_t tok_s;
    grid_dependency_wait();
    grid_dependents_launch();
    if (threadIdx.x == 0) {
        const int32_t s = io.seq[v], p = io.pos[v];
        int32_t tok = -1;
        if (s < 0 || p < 0 || uint32_t(p) >= io.max_len) {
            report(st, OPURE_ERR_DEVICE_BOUNDS, 20, uint32_t(p));
        } else {
            int32_t *hist = io.tokens + size_t(s) * io.max_len;
            if ((io.flags[v] & OPURE_VEC_AUTO) && p >= io.known[v]) {
                // Past the known tokens: the previous step's argmax is this step's input.
                const unsigned long long k = io.keys[v];
                tok = k ? int32_t(argmax_key_index(k)) : 0;
                hist[p] = tok;
                io.known[v] = p + 1;
            } else if (!(io.flags[v] & OPURE_VEC_AUTO) && io.in_tokens) {
                tok = io.in_tokens[v];
                hist[p] = tok;
            } else {
                tok = hist[p];
            }
            io.keys[v] = 0ull;
            io.seq_len[v] = p + 1;
            if (tok < 0 || uint32_t(tok) >= io.vocab) {
                report(st, OPURE_ERR_DEVICE_BOUNDS, 21, uint32_t(tok));
                tok = -1;
            }
        }
        tok_s = tok;
    }
    __syncthreads();
    const int32_t tok = tok_s;
    float *x = io.x + size_t(v) * io.hidden;
    const __half *row = reinterpret_cast<const __half *>(io.embed) + size_t(tok < 0 ? 0 : tok) * io.hidden;
    for (uint32_t i = threadIdx.x; i < io.hidden; i += blockDim.x)
        x[i] = tok < 0 ? 0.f : __half2float(row[i]);
}

__global__ void step_end_kernel(opure_step_io io) {
    grid_dependency_wait();
    grid_dependents_launch();
    const uint32_t v = blockIdx.x * blockDim.x + threadIdx.x;
    if (v < io.nvec && (io.flags[v] & OPURE_VEC_AUTO)) io.pos[v] += 1;
}

bool valid(const opure_step_io *io) {
    return io && io->seq && io->pos && io->seq_len && io->known && io->flags && io->tokens &&
           io->keys && io->embed && io->x && io->max_len && io->vocab && io->hidden;
}

}  // namespace
}  // namespace opure

using namespace opure;

extern "C" opure_status opure_step_begin(opure_ctx *ctx, const opure_step_io *io) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!valid(io)) return OPURE_ERR_INVALID_ARG;
    if (io->nvec == 0) return OPURE_OK;
    return launch(ctx, step_begin_kernel, dim3(io->nvec), dim3(256), 0, true, *io, ctx->status);
}

extern "C" opure_status opure_step_end(opure_ctx *ctx, const opure_step_io *io) {
    opure_status s = enter(ctx);
    if (s) return s;
    if (!valid(io)) return OPURE_ERR_INVALID_ARG;
    if (io->nvec == 0) return OPURE_OK;
    return launch(ctx, step_end_kernel, dim3(ceil_div(io->nvec, 128)), dim3(128), 0, true, *io);
}
