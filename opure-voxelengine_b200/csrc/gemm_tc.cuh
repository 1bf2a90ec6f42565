// gemm_tc.cuh -- internal entry of the tensor-core GEMV path (gemm_tc.cu), used by
// opure_gemv when many token vectors share one weight matrix.
#pragma once

#include "ctx.cuh"

namespace opure {

// Smallest vector count routed to the tensor cores, and the shape limits of that path.
constexpr uint32_t kTcMinVec = 16;
constexpr uint32_t kTcMaxCols = 16384;

// True when `a` (already validated by opure_gemv) can run on the tensor-core path.
bool gemv_tc_eligible(const opure_ctx *ctx, const opure_gemv_args *a);

// Enqueues the GEMV as pack + tcgen05 GEMM launches (passes of up to 256 vectors); with a
// chained input (x_packed) the pack launch is skipped.
opure_status gemv_tc(opure_ctx *ctx, const opure_gemv_args *a);

// Bytes of a packed operand of nvec vectors of length len.
size_t packed_bytes(uint32_t nvec, uint32_t len);

}  // namespace opure
