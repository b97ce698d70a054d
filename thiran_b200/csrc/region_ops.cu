// Layout kernels of the reverse-AD region operations: Transpose
// (src/semantic/v0/Evaluator.cpp:200-213) and BroadcastToShape (:278-309).
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.hpp"

namespace thb::kernels {
namespace {

constexpr unsigned kTile = 32;
constexpr unsigned kRowsPerPass = 8;

// One 32x32 tile per CTA (32x8 threads); reads rows of x, writes rows of y,
// both coalesced; the +1 column avoids shared-memory bank conflicts.
template <class T>
__global__ void __launch_bounds__(kTile * kRowsPerPass) transposeKernel(const T* __restrict__ x, T* __restrict__ y,
                                                                        std::uint64_t rows, std::uint64_t cols) {
    __shared__ T tile[kTile][kTile + 1];
    const std::uint64_t c0 = static_cast<std::uint64_t>(blockIdx.x) * kTile;
    const std::uint64_t r0 = static_cast<std::uint64_t>(blockIdx.y) * kTile;
    for (unsigned j = threadIdx.y; j < kTile; j += kRowsPerPass) {
        const std::uint64_t r = r0 + j, c = c0 + threadIdx.x;
        if (r < rows && c < cols) tile[j][threadIdx.x] = x[r * cols + c];
    }
    __syncthreads();
    for (unsigned j = threadIdx.y; j < kTile; j += kRowsPerPass) {
        const std::uint64_t r = c0 + j, c = r0 + threadIdx.x;  // y is [cols, rows]
        if (r < cols && c < rows) y[r * rows + c] = tile[threadIdx.x][j];
    }
}

__global__ void __launch_bounds__(256) broadcastKernel(const float* __restrict__ src, float* __restrict__ y,
                                                       std::uint64_t rows, std::uint64_t cols, int axis) {
    const std::uint64_t n = rows * cols;
    const std::uint64_t stride = static_cast<std::uint64_t>(gridDim.x) * blockDim.x;
    for (std::uint64_t i = static_cast<std::uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
        y[i] = axis == 0 ? src[i % cols] : src[i / cols];
}

__global__ void __launch_bounds__(256) fillKernel(const float* __restrict__ scalar, float value, float* __restrict__ y,
                                                  std::uint64_t n) {
    const float v = scalar ? *scalar : value;
    const std::uint64_t stride = static_cast<std::uint64_t>(gridDim.x) * blockDim.x;
    for (std::uint64_t i = static_cast<std::uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) y[i] = v;
}

} // namespace

cudaError_t fillF32(const float* deviceScalar, float value, float* y, std::uint64_t n, int smCount,
                    cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    const std::uint64_t blocks = (n + 255) / 256, cap = static_cast<std::uint64_t>(smCount) * 8;
    fillKernel<<<static_cast<unsigned>(blocks < cap ? blocks : cap), 256, 0, stream>>>(deviceScalar, value, y, n);
    return cudaGetLastError();
}

cudaError_t transpose(const void* x, void* y, std::uint64_t rows, std::uint64_t cols, std::size_t elementBytes,
                      int, cudaStream_t stream) {
    if (rows == 0 || cols == 0) return cudaSuccess;
    const std::uint64_t gx = (cols + kTile - 1) / kTile, gy = (rows + kTile - 1) / kTile;
    if (gx > 0x7fffffffu || gy > 65535u) return cudaErrorInvalidValue;
    const dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy)), block(kTile, kRowsPerPass);
    if (elementBytes == 4)
        transposeKernel<float><<<grid, block, 0, stream>>>(static_cast<const float*>(x), static_cast<float*>(y), rows, cols);
    else if (elementBytes == 8)
        transposeKernel<long long><<<grid, block, 0, stream>>>(static_cast<const long long*>(x),
                                                               static_cast<long long*>(y), rows, cols);
    else
        return cudaErrorInvalidValue;
    return cudaGetLastError();
}

cudaError_t broadcastF32(const float* src, float* y, std::uint64_t rows, std::uint64_t cols, int axis, int smCount,
                         cudaStream_t stream) {
    const std::uint64_t n = rows * cols;
    if (n == 0) return cudaSuccess;
    const std::uint64_t blocks = (n + 255) / 256, cap = static_cast<std::uint64_t>(smCount) * 8;
    broadcastKernel<<<static_cast<unsigned>(blocks < cap ? blocks : cap), 256, 0, stream>>>(src, y, rows, cols, axis);
    return cudaGetLastError();
}

} // namespace thb::kernels
