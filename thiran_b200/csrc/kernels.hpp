// Ahead-of-time compiled sm_100a kernels (reductions, row-wise softmax) and
// their launchers. Every launcher validates its sizes on the host and returns
// the launch status; nothing here allocates.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace thb::kernels {

// y[r, :] = softmax(x[r, :]) for a row-major [rows, cols] f32 matrix:
// m = max_j x, e_j = exp(x_j - m), y_j = e_j / sum_j e_j, with the row sum
// accumulated in f32 over a fixed tree. Rows up to kMaxSmemRowCols columns are
// staged whole into shared memory with the bulk-copy (TMA) engine.
cudaError_t softmaxRowsF32(const float* x, float* y, std::uint64_t rows, std::uint64_t cols, int smCount,
                           cudaStream_t stream, std::uint32_t* status);
// y[r] = max_j x[r, j].
cudaError_t maxRowsF32(const float* x, float* y, std::uint64_t rows, std::uint64_t cols, int smCount,
                       cudaStream_t stream, std::uint32_t* status);
// y[r] = sum_j x[r, j], accumulated in f64, rounded once to f32.
cudaError_t sumRowsF32(const float* x, float* y, std::uint64_t rows, std::uint64_t cols, int smCount,
                       cudaStream_t stream, std::uint32_t* status);
// y[c] = sum_r x[r, c], accumulated in f64, rounded once to f32.
cudaError_t sumColsF32(const float* x, float* y, std::uint64_t rows, std::uint64_t cols, int smCount,
                       cudaStream_t stream);

// Full-tensor sum in two deterministic passes: pass 1 writes one f64 partial
// per block of a fixed grid into `partials`, pass 2 adds them in block order.
// `out64` (optional) receives the f64 total, `out32` (optional) its f32
// rounding. `partials` must hold sumAllPartialCount(n, smCount) doubles.
// Large aligned inputs stream through 48 KiB bulk-copy tiles with one
// partial per SM; `status` (optional) gets bit 4 if a bounded wait runs out,
// and the sum is then NaN.
std::uint32_t sumAllPartialCount(std::uint64_t n, int smCount);
cudaError_t sumAllF32(const float* x, std::uint64_t n, double* partials, std::uint32_t partialCount, double* out64,
                      float* out32, int smCount, cudaStream_t stream, std::uint32_t* status = nullptr);

// y[c, r] = x[r, c] for a row-major [rows, cols] matrix of 4- or 8-byte
// elements (32x32 shared-memory tiles, coalesced on both sides).
cudaError_t transpose(const void* x, void* y, std::uint64_t rows, std::uint64_t cols, std::size_t elementBytes,
                      int smCount, cudaStream_t stream);
// y[r, c] = axis == 0 ? src[c] : src[r] over a row-major [rows, cols] target
// (BroadcastToShape: the source is the target with `axis` removed).
cudaError_t broadcastF32(const float* src, float* y, std::uint64_t rows, std::uint64_t cols, int axis, int smCount,
                         cudaStream_t stream);
// y[i] = *deviceScalar (when not null) else value, for i < n.
cudaError_t fillF32(const float* deviceScalar, float value, float* y, std::uint64_t n, int smCount,
                    cudaStream_t stream);

// C = A B for row-major A [m, k], B [k, n], C [m, n] on the CUDA cores, in
// the reference Evaluator's order (src/semantic/v0/Evaluator.cpp:125-154):
// every element sums its products for k = 0, 1, ... with separately rounded
// f32 operations (bit-exact), or with checked i64 arithmetic, raising bit 0
// (value 1) of `status` when any product or partial sum overflows.
cudaError_t matmulExactF32(const float* a, const float* b, float* c, std::uint64_t m, std::uint64_t k,
                           std::uint64_t n, cudaStream_t stream);
cudaError_t matmulCheckedI64(const std::int64_t* a, const std::int64_t* b, std::int64_t* c, std::uint64_t m,
                             std::uint64_t k, std::uint64_t n, std::uint32_t* status, cudaStream_t stream);
// i64 sums with the reference's checked-add semantics
// (src/semantic/v0/Evaluator.cpp:237-250): exact totals; bit 0 (value 1) of
// `status` when any prefix sum in the reference's order leaves the i64
// range. Rows: sum over the last axis; columns: over the leading axis; all:
// every element of a vector, two passes over sumAllI64ScratchBytes() of
// scratch.
cudaError_t sumRowsI64(const std::int64_t* x, std::int64_t* y, std::uint64_t rows, std::uint64_t cols, int smCount,
                       cudaStream_t stream, std::uint32_t* status);
cudaError_t sumColsI64(const std::int64_t* x, std::int64_t* y, std::uint64_t rows, std::uint64_t cols,
                       cudaStream_t stream, std::uint32_t* status);
std::uint32_t sumAllI64Blocks(std::uint64_t n, int smCount);
std::size_t sumAllI64ScratchBytes(std::uint64_t n, int smCount);
cudaError_t sumAllI64(const std::int64_t* x, std::uint64_t n, void* scratch, std::int64_t* out, int smCount,
                      cudaStream_t stream, std::uint32_t* status);
// y [rowsPad, ldPad] bf16 = bf16(x [rows, cols] f32), zero outside x.
cudaError_t castPadBf16(const float* x, void* y, std::uint64_t rows, std::uint64_t cols, std::uint64_t rowsPad,
                        std::uint64_t ldPad, int smCount, cudaStream_t stream);

// Largest row length the shared-memory staged softmax handles (longer rows
// take the streaming two-pass kernel).
constexpr std::uint64_t kMaxSmemRowCols = 8192;

} // namespace thb::kernels
