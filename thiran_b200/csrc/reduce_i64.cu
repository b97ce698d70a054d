// i64 sums of the Sum region node, exact and checked.
//
// The reference sums i64 tensors sequentially with a checked add
// (src/semantic/v0/Evaluator.cpp:237-250): acc = 0; acc = checked(acc + v)
// for every v in order, failing with TH-SPEC-I64-OVERFLOW when a partial sum
// leaves the i64 range. The result is the exact total whenever no prefix sum
// overflows, so a parallel sum must decide overflow from the prefix sums,
// not from its own (reordered) partial sums. Each piece of the input is
// therefore summarised exactly in 128-bit integers as
//   (total, lowest prefix sum, highest prefix sum)
// and pieces combine in order: A then B has total A.s + B.s, lowest
// min(A.lo, A.s + B.lo) and highest max(A.hi, A.s + B.hi). The sum overflows
// exactly when the lowest prefix is below INT64_MIN or the highest above
// INT64_MAX; the status word then gets bit 0 (value 1), which the host
// reports as TH-SPEC-I64-OVERFLOW.
//
//  - rows (sum over the last axis): one warp per row; lane j summarises a
//    contiguous stretch of the row, and lane 0 combines the 32 summaries in
//    lane order;
//  - columns (sum over the leading axis): one thread per column walking the
//    rows in order with the checked add itself (coalesced across threads);
//  - all elements: pass 1 summarises one contiguous segment per block (the
//    block's threads take contiguous stretches, combined in thread order),
//    pass 2 combines the block summaries in order.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.hpp"

namespace thb::kernels {
namespace {

constexpr unsigned kThreads = 256;

struct Summary {
    __int128 s, lo, hi;
    bool empty;
};

__device__ __forceinline__ Summary emptySummary() { return {0, 0, 0, true}; }

__device__ __forceinline__ Summary combine(const Summary& a, const Summary& b) {
    if (a.empty) return b;
    if (b.empty) return a;
    Summary r;
    r.s = a.s + b.s;
    r.lo = a.lo < a.s + b.lo ? a.lo : a.s + b.lo;
    r.hi = a.hi > a.s + b.hi ? a.hi : a.s + b.hi;
    r.empty = false;
    return r;
}

// Summary of x[begin, end) walked in order.
__device__ __forceinline__ Summary summarise(const long long* __restrict__ x, std::uint64_t begin, std::uint64_t end) {
    Summary r = emptySummary();
    for (std::uint64_t i = begin; i < end; ++i) {
        const __int128 p = (r.empty ? 0 : r.s) + static_cast<__int128>(x[i]);
        if (r.empty) {
            r.lo = r.hi = p;
            r.empty = false;
        } else {
            if (p < r.lo) r.lo = p;
            if (p > r.hi) r.hi = p;
        }
        r.s = p;
    }
    return r;
}

__device__ __forceinline__ bool overflows(const Summary& r) {
    const __int128 lo = static_cast<__int128>(static_cast<long long>(0x8000000000000000ULL));
    const __int128 hi = static_cast<__int128>(static_cast<long long>(0x7fffffffffffffffULL));
    return !r.empty && (r.lo < lo || r.hi > hi);
}

__device__ __forceinline__ Summary shuffleSummary(const Summary& v, unsigned src) {
    Summary r;
    const unsigned long long sLo = static_cast<unsigned long long>(v.s), sHi = static_cast<unsigned long long>(v.s >> 64);
    const unsigned long long lLo = static_cast<unsigned long long>(v.lo), lHi = static_cast<unsigned long long>(v.lo >> 64);
    const unsigned long long hLo = static_cast<unsigned long long>(v.hi), hHi = static_cast<unsigned long long>(v.hi >> 64);
    auto join = [](unsigned long long lo, unsigned long long hi) {
        return static_cast<__int128>((static_cast<unsigned __int128>(hi) << 64) | lo);
    };
    r.s = join(__shfl_sync(0xffffffffu, sLo, src), __shfl_sync(0xffffffffu, sHi, src));
    r.lo = join(__shfl_sync(0xffffffffu, lLo, src), __shfl_sync(0xffffffffu, lHi, src));
    r.hi = join(__shfl_sync(0xffffffffu, hLo, src), __shfl_sync(0xffffffffu, hHi, src));
    r.empty = __shfl_sync(0xffffffffu, v.empty ? 1 : 0, src) != 0;
    return r;
}

__global__ void __launch_bounds__(kThreads) sumRowsI64Kernel(const long long* __restrict__ x, long long* __restrict__ y,
                                                             std::uint64_t rows, std::uint64_t cols,
                                                             std::uint32_t* __restrict__ status) {
    const unsigned lane = threadIdx.x % 32;
    const std::uint64_t warps = static_cast<std::uint64_t>(gridDim.x) * (kThreads / 32);
    const std::uint64_t stretch = (cols + 31) / 32;
    std::uint32_t flag = 0;
    for (std::uint64_t r = static_cast<std::uint64_t>(blockIdx.x) * (kThreads / 32) + threadIdx.x / 32; r < rows;
         r += warps) {
        const std::uint64_t begin = lane * stretch < cols ? lane * stretch : cols;
        const std::uint64_t end = begin + stretch < cols ? begin + stretch : cols;
        const Summary mine = summarise(x + r * cols, begin, end);
        Summary total = emptySummary();
        for (unsigned j = 0; j < 32; ++j) total = combine(total, shuffleSummary(mine, j));
        if (lane == 0) {
            y[r] = static_cast<long long>(total.empty ? 0 : total.s);
            flag |= overflows(total) ? 1u : 0u;
        }
    }
    if (flag) atomicOr(status, flag);
}

__global__ void __launch_bounds__(kThreads) sumColsI64Kernel(const long long* __restrict__ x, long long* __restrict__ y,
                                                             std::uint64_t rows, std::uint64_t cols,
                                                             std::uint32_t* __restrict__ status) {
    const std::uint64_t c = static_cast<std::uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (c >= cols) return;
    long long acc = 0;
    std::uint32_t flag = 0;
    for (std::uint64_t r = 0; r < rows; ++r) {
        const long long v = x[r * cols + c];
        const long long s = static_cast<long long>(static_cast<unsigned long long>(acc) + static_cast<unsigned long long>(v));
        flag |= static_cast<std::uint32_t>(((s ^ acc) & (s ^ v)) < 0);
        acc = s;
    }
    y[c] = acc;
    if (flag) atomicOr(status, 1u);
}

// One contiguous segment per block: thread t summarises its stretch of the
// segment, thread 0 combines the block's summaries in thread order.
__global__ void __launch_bounds__(kThreads) sumAllI64Pass1(const long long* __restrict__ x, std::uint64_t n,
                                                           std::uint64_t segment, Summary* __restrict__ partials) {
    __shared__ Summary parts[kThreads];
    const std::uint64_t begin = static_cast<std::uint64_t>(blockIdx.x) * segment;
    const std::uint64_t end = begin + segment < n ? begin + segment : n;
    const std::uint64_t stretch = (segment + kThreads - 1) / kThreads;
    const std::uint64_t b = begin + threadIdx.x * stretch < end ? begin + threadIdx.x * stretch : end;
    const std::uint64_t e = b + stretch < end ? b + stretch : end;
    parts[threadIdx.x] = summarise(x, b, e);
    __syncthreads();
    if (threadIdx.x == 0) {
        Summary total = emptySummary();
        for (unsigned t = 0; t < kThreads; ++t) total = combine(total, parts[t]);
        partials[blockIdx.x] = total;
    }
}

__global__ void sumAllI64Pass2(const Summary* __restrict__ partials, unsigned count, long long* __restrict__ out,
                               std::uint32_t* __restrict__ status) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    Summary total = emptySummary();
    for (unsigned k = 0; k < count; ++k) total = combine(total, partials[k]);
    *out = static_cast<long long>(total.empty ? 0 : total.s);
    if (overflows(total)) atomicOr(status, 1u);
}

} // namespace

std::size_t sumAllI64ScratchBytes(std::uint64_t n, int smCount) {
    const std::uint64_t blocks = sumAllI64Blocks(n, smCount);
    return static_cast<std::size_t>(blocks) * sizeof(Summary);
}

std::uint32_t sumAllI64Blocks(std::uint64_t n, int smCount) {
    const std::uint64_t byWork = (n + kThreads * 64 - 1) / (kThreads * 64);  // >= 64 elements per thread
    const std::uint64_t cap = static_cast<std::uint64_t>(smCount > 0 ? smCount : 1) * 2;
    return static_cast<std::uint32_t>(byWork < 1 ? 1 : (byWork < cap ? byWork : cap));
}

cudaError_t sumRowsI64(const std::int64_t* x, std::int64_t* y, std::uint64_t rows, std::uint64_t cols, int smCount,
                       cudaStream_t stream, std::uint32_t* status) {
    if (rows == 0) return cudaSuccess;
    const std::uint64_t blocks = (rows + kThreads / 32 - 1) / (kThreads / 32);
    const std::uint64_t cap = static_cast<std::uint64_t>(smCount > 0 ? smCount : 1) * 8;
    sumRowsI64Kernel<<<static_cast<unsigned>(blocks < cap ? blocks : cap), kThreads, 0, stream>>>(
        reinterpret_cast<const long long*>(x), reinterpret_cast<long long*>(y), rows, cols, status);
    return cudaGetLastError();
}

cudaError_t sumColsI64(const std::int64_t* x, std::int64_t* y, std::uint64_t rows, std::uint64_t cols,
                       cudaStream_t stream, std::uint32_t* status) {
    if (cols == 0) return cudaSuccess;
    const std::uint64_t blocks = (cols + kThreads - 1) / kThreads;
    if (blocks > 0x7fffffffu) return cudaErrorInvalidValue;
    sumColsI64Kernel<<<static_cast<unsigned>(blocks), kThreads, 0, stream>>>(
        reinterpret_cast<const long long*>(x), reinterpret_cast<long long*>(y), rows, cols, status);
    return cudaGetLastError();
}

cudaError_t sumAllI64(const std::int64_t* x, std::uint64_t n, void* scratch, std::int64_t* out, int smCount,
                      cudaStream_t stream, std::uint32_t* status) {
    const std::uint32_t blocks = sumAllI64Blocks(n, smCount);
    const std::uint64_t segment = (n + blocks - 1) / blocks;
    Summary* partials = static_cast<Summary*>(scratch);
    sumAllI64Pass1<<<blocks, kThreads, 0, stream>>>(reinterpret_cast<const long long*>(x), n, segment ? segment : 1,
                                                    partials);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    sumAllI64Pass2<<<1, 32, 0, stream>>>(partials, blocks, reinterpret_cast<long long*>(out), status);
    return cudaGetLastError();
}

} // namespace thb::kernels
