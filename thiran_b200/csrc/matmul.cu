// MatMul region nodes that the tensor cores cannot serve exactly.
//
// The reference's matmul (src/semantic/v0/Evaluator.cpp:125-154) computes
// every C[i,j] as acc = 0; acc = acc + A[i,k] * B[k,j] for k = 0, 1, ... in
// order, each product and each sum rounded separately (f32), or with checked
// i64 multiply and add (TH-SPEC-I64-OVERFLOW on any overflow). The tensor
// cores sum in their own order and take bf16 or 8-bit operands, so:
//  - matmulExactF32 reproduces the f32 rule bit for bit on the CUDA cores
//    (__fmul_rn / __fadd_rn, never contracted into an FMA);
//  - matmulCheckedI64 is the i64 rule (no tensor-core form exists for i64
//    on B200); any overflowing product or partial sum raises bit 0 (value 1)
//    of the caller's status word, which the host reports as
//    TH-SPEC-I64-OVERFLOW. The reference stops at the first overflow; the
//    failure id is the same whichever element overflows first.
// Both tile C in 64 x 64 blocks per 256-thread CTA (4 x 4 outputs per
// thread, rows ty + 16 i and columns tx + 16 j so that shared-memory reads
// are broadcasts or consecutive words), staging 16-deep K slices of A
// (transposed) and B in shared memory. Each thread walks k in increasing
// order, which is the reference's order for every element.
//
// castPadBf16 feeds the tensor-core path of f32 MatMul nodes whose K or N is
// not a multiple of 8 (the GEMM's operands need 16-byte row strides): it
// writes the bf16 rounding of a row-major [rows, cols] f32 matrix into a
// [rowsPad, ldPad] buffer whose extra rows and columns are zero, so the
// padding adds exact zeros to every dot product.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.hpp"

namespace thb::kernels {
namespace {

constexpr unsigned kMmTile = 64;
constexpr unsigned kMmDepth = 16;
constexpr unsigned kMmThreads = 256;

__device__ __forceinline__ float mmStep(float acc, float a, float b, std::uint32_t&) {
    return __fadd_rn(acc, __fmul_rn(a, b));
}

// Two's-complement overflow tests (the reference's checked '*' and '+',
// src/semantic/v0/Evaluator.cpp:143-153): the product overflows when its high
// word is not the sign extension of the low word; the sum when both operands
// have the sign opposite to the result's.
__device__ __forceinline__ long long mmStep(long long acc, long long a, long long b, std::uint32_t& flag) {
    const long long lo = static_cast<long long>(static_cast<unsigned long long>(a) * static_cast<unsigned long long>(b));
    const long long hi = __mul64hi(a, b);
    flag |= static_cast<std::uint32_t>(hi != (lo >> 63));
    const long long r = static_cast<long long>(static_cast<unsigned long long>(acc) + static_cast<unsigned long long>(lo));
    flag |= static_cast<std::uint32_t>(((r ^ acc) & (r ^ lo)) < 0);
    return r;
}

template <class T>
__global__ void __launch_bounds__(kMmThreads) matmulTiled(const T* __restrict__ a, const T* __restrict__ b,
                                                          T* __restrict__ c, std::uint64_t m, std::uint64_t k,
                                                          std::uint64_t n, std::uint32_t* __restrict__ status) {
    __shared__ T as[kMmDepth][kMmTile];  // A slice, transposed: as[kk][row]
    __shared__ T bs[kMmDepth][kMmTile];  // B slice: bs[kk][col]
    const unsigned tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const std::uint64_t row0 = static_cast<std::uint64_t>(blockIdx.y) * kMmTile;
    const std::uint64_t col0 = static_cast<std::uint64_t>(blockIdx.x) * kMmTile;
    T acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = T(0);
    std::uint32_t flag = 0;
    for (std::uint64_t k0 = 0; k0 < k; k0 += kMmDepth) {
        // A: 64 rows x 16 k; thread t loads (row t / 4 + 64 q / 4 ..., k t % 16)
        // so that 16 consecutive threads read 16 consecutive k of one row.
#pragma unroll
        for (unsigned q = 0; q < kMmTile * kMmDepth / kMmThreads; ++q) {
            const unsigned e = threadIdx.x + q * kMmThreads;
            const unsigned r = e / kMmDepth, kk = e % kMmDepth;
            const std::uint64_t gr = row0 + r, gk = k0 + kk;
            as[kk][r] = (gr < m && gk < k) ? a[gr * k + gk] : T(0);
        }
        // B: 16 k x 64 columns, consecutive threads on consecutive columns.
#pragma unroll
        for (unsigned q = 0; q < kMmTile * kMmDepth / kMmThreads; ++q) {
            const unsigned e = threadIdx.x + q * kMmThreads;
            const unsigned kk = e / kMmTile, cc = e % kMmTile;
            const std::uint64_t gk = k0 + kk, gc = col0 + cc;
            bs[kk][cc] = (gk < k && gc < n) ? b[gk * n + gc] : T(0);
        }
        __syncthreads();
        const unsigned depth = static_cast<unsigned>(k - k0 < kMmDepth ? k - k0 : kMmDepth);
        for (unsigned kk = 0; kk < depth; ++kk) {
            T av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) av[i] = as[kk][ty + 16 * i];
#pragma unroll
            for (int j = 0; j < 4; ++j) bv[j] = bs[kk][tx + 16 * j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = mmStep(acc[i][j], av[i], bv[j], flag);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const std::uint64_t gr = row0 + ty + 16 * i;
        if (gr >= m) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const std::uint64_t gc = col0 + tx + 16 * j;
            if (gc < n) c[gr * n + gc] = acc[i][j];
        }
    }
    // Only outputs inside C can overflow: the zero fill adds nothing.
    if (flag && status) atomicOr(status, 1u);
}

__global__ void __launch_bounds__(256) castPadKernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                                     std::uint64_t rows, std::uint64_t cols, std::uint64_t rowsPad,
                                                     std::uint64_t ldPad) {
    const std::uint64_t total = rowsPad * ldPad;
    const std::uint64_t stride = static_cast<std::uint64_t>(gridDim.x) * blockDim.x;
    for (std::uint64_t i = static_cast<std::uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        const std::uint64_t r = i / ldPad, cc = i % ldPad;
        y[i] = __float2bfloat16_rn(r < rows && cc < cols ? x[r * cols + cc] : 0.0f);
    }
}

template <class T>
cudaError_t launchMatmul(const T* a, const T* b, T* c, std::uint64_t m, std::uint64_t k, std::uint64_t n,
                         std::uint32_t* status, cudaStream_t stream) {
    if (m == 0 || n == 0) return cudaSuccess;
    const std::uint64_t gx = (n + kMmTile - 1) / kMmTile, gy = (m + kMmTile - 1) / kMmTile;
    if (gx > 0x7fffffffu || gy > 65535u) return cudaErrorInvalidValue;
    matmulTiled<T><<<dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy)), kMmThreads, 0, stream>>>(a, b, c, m, k,
                                                                                                          n, status);
    return cudaGetLastError();
}

} // namespace

cudaError_t matmulExactF32(const float* a, const float* b, float* c, std::uint64_t m, std::uint64_t k,
                           std::uint64_t n, cudaStream_t stream) {
    return launchMatmul<float>(a, b, c, m, k, n, nullptr, stream);
}

cudaError_t matmulCheckedI64(const std::int64_t* a, const std::int64_t* b, std::int64_t* c, std::uint64_t m,
                             std::uint64_t k, std::uint64_t n, std::uint32_t* status, cudaStream_t stream) {
    return launchMatmul<long long>(reinterpret_cast<const long long*>(a), reinterpret_cast<const long long*>(b),
                                   reinterpret_cast<long long*>(c), m, k, n, status, stream);
}

cudaError_t castPadBf16(const float* x, void* y, std::uint64_t rows, std::uint64_t cols, std::uint64_t rowsPad,
                        std::uint64_t ldPad, int smCount, cudaStream_t stream) {
    const std::uint64_t total = rowsPad * ldPad;
    if (total == 0) return cudaSuccess;
    if (rowsPad < rows || ldPad < cols) return cudaErrorInvalidValue;
    const std::uint64_t blocks = (total + 255) / 256, cap = static_cast<std::uint64_t>(smCount) * 8;
    castPadKernel<<<static_cast<unsigned>(blocks < cap ? blocks : cap), 256, 0, stream>>>(
        x, static_cast<__nv_bfloat16*>(y), rows, cols, rowsPad, ldPad);
    return cudaGetLastError();
}

} // namespace thb::kernels
