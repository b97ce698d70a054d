// Row-wise and full-tensor reductions for sm_100a.
//
// Row kernels (softmax / max / sum over the last axis) are persistent and
// read every element from HBM once (softmax writes it once):
//  - rows up to 4096 columns: one warp per row with the row in registers
//    (rowWarp); reductions are warp shuffles, with no shared memory and no
//    CTA barrier. On B200 softmax over 65536 x 4096 ran at 0.97 of the
//    measured copy peak this way, against 0.86 for the staged kernel;
//  - rows up to 8192 columns: each CTA walks rows blockIdx.x,
//    blockIdx.x + gridDim.x, ... and stages whole rows in shared memory with
//    the bulk-copy engine (cp.async.bulk global->shared, completion on an
//    mbarrier), keeping two rows in flight while it computes a third. Softmax
//    writes its result back into the staged row and the bulk-copy engine
//    stores it (shared->global). Every mbarrier wait is bounded; on expiry
//    the kernel raises bit 4 of its status word, drains its own copies and
//    returns.
// The full-tensor sum streams 48 KiB tiles through the bulk-copy engine
// (0.99 of the copy peak against 0.97 for 128-bit loads).
// THB_ROWS=staged keeps the staged kernels (and the 128-bit full-sum pass).
//
// The reference has no native reduction (src/backend/v0/TensorRegion.cpp:425
// "Sum lowering deferred"); its Evaluator sums sequentially in f32
// (src/semantic/v0/Evaluator.cpp:214-251) and the legacy stack lowers softmax
// to torch.softmax(dim=-1) (src/region/RegionPythonEmitter.cpp:293-294).
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>

#include "kernels.hpp"

namespace thb::kernels {
namespace {

constexpr unsigned kRowThreads = 256;
constexpr unsigned kRowWarps = kRowThreads / 32;
constexpr unsigned kStages = 4;
constexpr unsigned kWaitStatus = 16u;            // status bit raised on a wait timeout
constexpr unsigned kDrainStatus = 32u;           // ... and when the copies in flight could not be drained
constexpr std::uint64_t kSpinLimit = 1ull << 22; // bounded mbarrier polling (~seconds at most)
constexpr std::uint64_t kDrainLimit = kSpinLimit << 4;

enum class RowOp { Softmax, Max, Sum };

__device__ __forceinline__ std::uint32_t smemAddress(const void* p) {
    return static_cast<std::uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbarInit(std::uint64_t* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smemAddress(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbarExpect(std::uint64_t* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smemAddress(bar)), "r"(bytes)
                 : "memory");
}

// Polls the barrier phase `parity`; false when the poll budget (`limit`
// polls) ran out. After a timeout the drain of the copies still in flight
// polls 16 times longer (kDrainLimit) before it gives up.
__device__ __forceinline__ bool mbarWait(std::uint64_t* bar, unsigned parity, std::uint64_t limit = kSpinLimit) {
    const std::uint32_t addr = smemAddress(bar);
    for (std::uint64_t spin = 0; spin < limit; ++spin) {
        std::uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

__device__ __forceinline__ void bulkLoad(void* dst, const void* src, unsigned bytes, std::uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smemAddress(dst)),
                 "l"(src), "r"(bytes), "r"(smemAddress(bar))
                 : "memory");
}

__device__ __forceinline__ void bulkStore(void* dst, const void* src, unsigned bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smemAddress(src)),
                 "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void bulkWaitRead() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void bulkWaitAll() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ float warpMax(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

template <class T>
__device__ __forceinline__ T warpSum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Combines one value per warp in warp order; every thread gets the same result.
template <class T, class F>
__device__ __forceinline__ T blockCombine(T mine, T* scratch, F op) {
    const unsigned warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (lane == 0) scratch[warp] = mine;
    __syncthreads();
    T r = scratch[0];
#pragma unroll
    for (unsigned w = 1; w < kRowWarps; ++w) r = op(r, scratch[w]);
    return r;
}

// VPT = float4 packets per thread (cols <= VPT * 4 * kRowThreads).
template <RowOp OP, int VPT>
__global__ void __launch_bounds__(kRowThreads) rowStaged(const float* __restrict__ x, float* __restrict__ y,
                                                         std::uint64_t rows, unsigned cols,
                                                         std::uint32_t* __restrict__ status) {
    extern __shared__ __align__(128) float stage[];
    __shared__ __align__(8) std::uint64_t full[kStages];
    __shared__ float redA[kRowWarps];
    __shared__ float redB[kRowWarps];
    __shared__ double redD[kRowWarps];
    __shared__ int abortFlag;

    const unsigned packets = cols / 4;
    const unsigned rowBytes = cols * 4u;
    const std::uint64_t first = blockIdx.x;
    const std::uint64_t step = gridDim.x;
    const std::uint64_t mine = first < rows ? (rows - first + step - 1) / step : 0;  // rows of this CTA
    auto rowOf = [&](std::uint64_t it) { return first + it * step; };
    auto buffer = [&](unsigned s) { return stage + static_cast<std::size_t>(s) * cols; };

    if (threadIdx.x == 0) {
        abortFlag = 0;
        for (unsigned s = 0; s < kStages; ++s) mbarInit(&full[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (std::uint64_t it = 0; it < 2 && it < mine; ++it) {
            mbarExpect(&full[it], rowBytes);
            bulkLoad(buffer(static_cast<unsigned>(it)), x + rowOf(it) * cols, rowBytes, &full[it]);
        }
    }
    __syncthreads();

    std::uint64_t it = 0;
    for (; it < mine; ++it) {
        const unsigned s = static_cast<unsigned>(it % kStages);
        if (threadIdx.x == 0 && it + 2 < mine) {
            // Stage (it+2)%4 last held row it-2, whose store must have finished
            // reading shared memory; at most the store of row it-1 may remain.
            bulkWaitRead<1>();
            const unsigned ns = static_cast<unsigned>((it + 2) % kStages);
            mbarExpect(&full[ns], rowBytes);
            bulkLoad(buffer(ns), x + rowOf(it + 2) * cols, rowBytes, &full[ns]);
        }
        if (!mbarWait(&full[s], static_cast<unsigned>((it / kStages) & 1u))) abortFlag = 1;
        __syncthreads();
        if (abortFlag) break;

        float* row = buffer(s);
        float4 v[VPT];
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const unsigned p = threadIdx.x + k * kRowThreads;
            if (p < packets) v[k] = reinterpret_cast<const float4*>(row)[p];
            else v[k] = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        }
        const std::uint64_t r = rowOf(it);
        if constexpr (OP == RowOp::Sum) {
            double acc = 0.0;
#pragma unroll
            for (int k = 0; k < VPT; ++k)
                if (threadIdx.x + k * kRowThreads < packets)
                    acc += (double)v[k].x + (double)v[k].y + (double)v[k].z + (double)v[k].w;
            acc = warpSum(acc);
            const double total = blockCombine(acc, redD, [](double a, double b) { return a + b; });
            if (threadIdx.x == 0) y[r] = static_cast<float>(total);
            __syncthreads();
        } else {
            float m = -INFINITY;
#pragma unroll
            for (int k = 0; k < VPT; ++k) m = fmaxf(m, fmaxf(fmaxf(v[k].x, v[k].y), fmaxf(v[k].z, v[k].w)));
            m = warpMax(m);
            const float rowMax = blockCombine(m, redA, [](float a, float b) { return fmaxf(a, b); });
            if constexpr (OP == RowOp::Max) {
                if (threadIdx.x == 0) y[r] = rowMax;
                __syncthreads();
            } else {
                float sum = 0.0f;
#pragma unroll
                for (int k = 0; k < VPT; ++k) {
                    // The fast intrinsic: x - max <= 0, so the result is in
                    // (0, 1] with ~2 ulp error, inside the 1e-5 relative bar.
                    v[k].x = __expf(v[k].x - rowMax);
                    v[k].y = __expf(v[k].y - rowMax);
                    v[k].z = __expf(v[k].z - rowMax);
                    v[k].w = __expf(v[k].w - rowMax);
                    if (threadIdx.x + k * kRowThreads < packets) sum += (v[k].x + v[k].y) + (v[k].z + v[k].w);
                }
                sum = warpSum(sum);
                const float total = blockCombine(sum, redB, [](float a, float b) { return a + b; });
                const float inv = 1.0f / total;
#pragma unroll
                for (int k = 0; k < VPT; ++k) {
                    const unsigned p = threadIdx.x + k * kRowThreads;
                    if (p < packets) {
                        float4 o;
                        o.x = v[k].x * inv;
                        o.y = v[k].y * inv;
                        o.z = v[k].z * inv;
                        o.w = v[k].w * inv;
                        reinterpret_cast<float4*>(row)[p] = o;
                    }
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncthreads();
                if (threadIdx.x == 0) bulkStore(y + r * cols, row, rowBytes);
            }
        }
    }
    if (threadIdx.x == 0) {
        if (abortFlag) {
            // Drain loads still in flight (rows it, it+1, it+2 may have been
            // issued) for rows this CTA will not process. A copy that still
            // has not landed may write into shared memory after this CTA
            // exits: bit 5 tells the host to trust nothing of this device.
            bool drained = true;
            for (std::uint64_t k = it; k < it + 3 && k < mine; ++k)
                drained &= mbarWait(&full[k % kStages], static_cast<unsigned>((k / kStages) & 1u), kDrainLimit);
            atomicOr(status, kWaitStatus | (drained ? 0u : kDrainStatus));
        }
        bulkWaitAll();
    }
}

// Rows up to 128 * VPT columns with one warp per row and the row in
// registers: VPT independent 16-byte streaming loads per lane, max and sums
// by warp shuffles (row sums in f64), and for softmax one streaming store
// pass. No shared memory and no CTA barrier, so each of the SM's warps keeps
// a whole row in flight.
constexpr unsigned kWarpRowThreads = 128;

template <RowOp OP, int VPT>
__global__ void __launch_bounds__(kWarpRowThreads) rowWarp(const float* __restrict__ x, float* __restrict__ y,
                                                            std::uint64_t rows, unsigned cols) {
    const unsigned lane = threadIdx.x % 32;
    const unsigned packets = cols / 4;
    const std::uint64_t warps = static_cast<std::uint64_t>(gridDim.x) * (kWarpRowThreads / 32);
    for (std::uint64_t r = static_cast<std::uint64_t>(blockIdx.x) * (kWarpRowThreads / 32) + threadIdx.x / 32;
         r < rows; r += warps) {
        const float4* src = reinterpret_cast<const float4*>(x + r * cols);
        float4 v[VPT];
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const unsigned p = lane + 32u * k;
            v[k] = p < packets ? __ldcs(src + p) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        }
        if constexpr (OP == RowOp::Sum) {
            double acc = 0.0;
#pragma unroll
            for (int k = 0; k < VPT; ++k)
                if (lane + 32u * k < packets) acc += (double)v[k].x + (double)v[k].y + (double)v[k].z + (double)v[k].w;
            acc = warpSum(acc);
            if (lane == 0) y[r] = static_cast<float>(acc);
            continue;
        }
        float m = -INFINITY;
#pragma unroll
        for (int k = 0; k < VPT; ++k) m = fmaxf(m, fmaxf(fmaxf(v[k].x, v[k].y), fmaxf(v[k].z, v[k].w)));
        m = warpMax(m);
        if constexpr (OP == RowOp::Max) {
            if (lane == 0) y[r] = m;
            continue;
        }
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            // The fast intrinsic: x - max <= 0, so the result is in (0, 1]
            // with ~2 ulp error, inside the 1e-5 relative bar.
            v[k].x = __expf(v[k].x - m);
            v[k].y = __expf(v[k].y - m);
            v[k].z = __expf(v[k].z - m);
            v[k].w = __expf(v[k].w - m);
            if (lane + 32u * k < packets) sum += (v[k].x + v[k].y) + (v[k].z + v[k].w);
        }
        const float inv = 1.0f / warpSum(sum);
        float4* dst = reinterpret_cast<float4*>(y + r * cols);
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const unsigned p = lane + 32u * k;
            if (p < packets) __stcs(dst + p, make_float4(v[k].x * inv, v[k].y * inv, v[k].z * inv, v[k].w * inv));
        }
    }
}

// Streaming fallback for rows that are not bulk-copy aligned or too long for
// shared memory: one CTA per row, three read passes for softmax.
template <RowOp OP>
__global__ void __launch_bounds__(kRowThreads) rowStreaming(const float* __restrict__ x, float* __restrict__ y,
                                                            std::uint64_t rows, std::uint64_t cols) {
    __shared__ float redA[kRowWarps];
    __shared__ float redB[kRowWarps];
    __shared__ double redD[kRowWarps];
    for (std::uint64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const float* in = x + r * cols;
        if constexpr (OP == RowOp::Sum) {
            double acc = 0.0;
            for (std::uint64_t j = threadIdx.x; j < cols; j += kRowThreads) acc += in[j];
            acc = warpSum(acc);
            const double total = blockCombine(acc, redD, [](double a, double b) { return a + b; });
            if (threadIdx.x == 0) y[r] = static_cast<float>(total);
        } else {
            float m = -INFINITY;
            for (std::uint64_t j = threadIdx.x; j < cols; j += kRowThreads) m = fmaxf(m, in[j]);
            m = warpMax(m);
            const float rowMax = blockCombine(m, redA, [](float a, float b) { return fmaxf(a, b); });
            if constexpr (OP == RowOp::Max) {
                if (threadIdx.x == 0) y[r] = rowMax;
            } else {
                float sum = 0.0f;
                for (std::uint64_t j = threadIdx.x; j < cols; j += kRowThreads) sum += expf(in[j] - rowMax);
                sum = warpSum(sum);
                const float total = blockCombine(sum, redB, [](float a, float b) { return a + b; });
                const float inv = 1.0f / total;
                for (std::uint64_t j = threadIdx.x; j < cols; j += kRowThreads) y[r * cols + j] = expf(in[j] - rowMax) * inv;
            }
        }
        __syncthreads();
    }
}

template <RowOp OP>
cudaError_t launchRows(const float* x, float* y, std::uint64_t rows, std::uint64_t cols, int smCount,
                       cudaStream_t stream, std::uint32_t* status) {
    if (rows == 0 || cols == 0) return cudaSuccess;
    const bool aligned = (reinterpret_cast<std::uintptr_t>(x) % 16 == 0) &&
                         (OP != RowOp::Softmax || reinterpret_cast<std::uintptr_t>(y) % 16 == 0) && cols % 4 == 0;
    static const bool warpRows = [] {
        const char* e = std::getenv("THB_ROWS");
        return !(e && std::strcmp(e, "staged") == 0);
    }();
    if (aligned && warpRows && cols <= 128u * 32u) {
        auto kernel = cols <= 128u * 8u ? rowWarp<OP, 8> : cols <= 128u * 16u ? rowWarp<OP, 16> : rowWarp<OP, 32>;
        int perSm = 0;
        cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&perSm, kernel, kWarpRowThreads, 0);
        if (e != cudaSuccess) return e;
        if (perSm < 1) perSm = 1;
        const std::uint64_t warpsPerCta = kWarpRowThreads / 32;
        const std::uint64_t grid = std::min<std::uint64_t>((rows + warpsPerCta - 1) / warpsPerCta,
                                                           static_cast<std::uint64_t>(smCount) * perSm);
        kernel<<<static_cast<unsigned>(grid), kWarpRowThreads, 0, stream>>>(x, y, rows, static_cast<unsigned>(cols));
        return cudaGetLastError();
    }
    if (aligned && cols <= kMaxSmemRowCols) {
        const unsigned c = static_cast<unsigned>(cols);
        const std::size_t smem = static_cast<std::size_t>(kStages) * c * sizeof(float);
        auto kernel = cols <= 4 * kRowThreads * 4 ? rowStaged<OP, 4> : rowStaged<OP, 8>;
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        int perSm = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&perSm, kernel, kRowThreads, smem);
        if (e != cudaSuccess) return e;
        if (perSm < 1) perSm = 1;
        const std::uint64_t grid = std::min<std::uint64_t>(rows, static_cast<std::uint64_t>(smCount) * perSm);
        kernel<<<static_cast<unsigned>(grid), kRowThreads, smem, stream>>>(x, y, rows, c, status);
        return cudaGetLastError();
    }
    const std::uint64_t grid = std::min<std::uint64_t>(rows, static_cast<std::uint64_t>(smCount) * 8);
    rowStreaming<OP><<<static_cast<unsigned>(grid), kRowThreads, 0, stream>>>(x, y, rows, cols);
    return cudaGetLastError();
}

// ---- full-tensor and column sums -----------------------------------------------

constexpr unsigned kSumThreads = 256;

template <bool VEC>
__global__ void __launch_bounds__(kSumThreads) sumAllPass1(const float* __restrict__ x, std::uint64_t n,
                                                           double* __restrict__ partials) {
    __shared__ double red[kSumThreads / 32];
    double acc = 0.0;
    const std::uint64_t stride = static_cast<std::uint64_t>(gridDim.x) * kSumThreads;
    std::uint64_t i = static_cast<std::uint64_t>(blockIdx.x) * kSumThreads + threadIdx.x;
    if constexpr (VEC) {
        const float4* p = reinterpret_cast<const float4*>(x);
        const std::uint64_t packets = n / 4;
        for (; i + 3 * stride < packets; i += 4 * stride) {
            float4 a[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) a[u] = __ldcs(p + i + u * stride);
#pragma unroll
            for (int u = 0; u < 4; ++u) acc += ((double)a[u].x + (double)a[u].y) + ((double)a[u].z + (double)a[u].w);
        }
        for (; i < packets; i += stride) {
            const float4 a = __ldcs(p + i);
            acc += ((double)a.x + (double)a.y) + ((double)a.z + (double)a.w);
        }
        if (blockIdx.x == 0 && threadIdx.x < n % 4) acc += x[packets * 4 + threadIdx.x];
    } else {
        for (; i < n; i += stride) acc += x[i];
    }
    acc = warpSum(acc);
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = red[0];
        for (unsigned w = 1; w < kSumThreads / 32; ++w) t += red[w];
        partials[blockIdx.x] = t;
    }
}

// Pass 1 over whole 48 KiB tiles with the bulk-copy engine: one persistent
// CTA per SM takes tiles blockIdx.x, blockIdx.x + gridDim.x, ...; thread 0
// keeps a 3-stage ring of them in shared memory full (cp.async.bulk,
// mbarrier completion) and all threads add their part of each tile in f64.
// The elements past the last whole tile take plain loads. A wait that runs
// out raises the status bit (when given) and poisons the partial with NaN.
// Callers that pass no status word see only the NaN.
constexpr unsigned kSumStages = 3;
constexpr unsigned kSumTileFloats = 12288;  // 48 KiB
constexpr std::size_t kSumBulkSmem = static_cast<std::size_t>(kSumStages) * kSumTileFloats * sizeof(float);

__global__ void __launch_bounds__(kSumThreads) sumAllBulk(const float* __restrict__ x, std::uint64_t n,
                                                          double* __restrict__ partials,
                                                          std::uint32_t* __restrict__ status) {
    extern __shared__ __align__(128) float tileSmem[];
    __shared__ __align__(8) std::uint64_t full[kSumStages];
    __shared__ double red[kSumThreads / 32];
    __shared__ int abortFlag;
    const std::uint64_t tiles = n / kSumTileFloats;
    const std::uint64_t first = blockIdx.x, step = gridDim.x;
    constexpr unsigned kTileBytes = kSumTileFloats * sizeof(float);
    auto issue = [&](std::uint64_t t, unsigned s) {
        if (t >= tiles) return;
        mbarExpect(&full[s], kTileBytes);
        bulkLoad(tileSmem + static_cast<std::size_t>(s) * kSumTileFloats, x + t * kSumTileFloats, kTileBytes, &full[s]);
    };
    if (threadIdx.x == 0) {
        abortFlag = 0;
        for (unsigned s = 0; s < kSumStages; ++s) mbarInit(&full[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (unsigned s = 0; s < kSumStages; ++s) issue(first + s * step, s);
    }
    __syncthreads();
    double acc = 0.0;
    unsigned st = 0, phase = 0;
    for (std::uint64_t t = first; t < tiles; t += step) {
        if (threadIdx.x == 0 && !mbarWait(&full[st], phase)) {
            // Loads still in flight land before the CTA exits (bounded; bit 5
            // of the status word when they did not).
            abortFlag = 1;
            unsigned s = st, ph = phase;
            for (unsigned q = 0; q < kSumStages; ++q) {
                if (t + q * step < tiles && !mbarWait(&full[s], ph, kDrainLimit)) abortFlag = 2;
                if (++s == kSumStages) { s = 0; ph ^= 1u; }
            }
        }
        __syncthreads();
        if (abortFlag) break;
        const float4* tile = reinterpret_cast<const float4*>(tileSmem + static_cast<std::size_t>(st) * kSumTileFloats);
#pragma unroll 4
        for (unsigned q = threadIdx.x; q < kSumTileFloats / 4; q += kSumThreads) {
            const float4 a = tile[q];
            acc += ((double)a.x + (double)a.y) + ((double)a.z + (double)a.w);
        }
        __syncthreads();  // every thread is done with the stage
        if (threadIdx.x == 0) issue(t + kSumStages * step, st);
        if (++st == kSumStages) { st = 0; phase ^= 1u; }
    }
    if (abortFlag) {
        if (threadIdx.x == 0) {
            if (status) atomicOr(status, kWaitStatus | (abortFlag == 2 ? kDrainStatus : 0u));
            acc = __longlong_as_double(0x7ff8000000000000ll);  // NaN
        }
    } else {
        const std::uint64_t stride = step * kSumThreads;
        for (std::uint64_t i = tiles * kSumTileFloats + first * kSumThreads + threadIdx.x; i < n; i += stride) acc += x[i];
    }
    acc = warpSum(acc);
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = red[0];
        for (unsigned w = 1; w < kSumThreads / 32; ++w) t += red[w];
        partials[blockIdx.x] = t;
    }
}

__global__ void __launch_bounds__(kSumThreads) sumAllPass2(const double* __restrict__ partials, unsigned count,
                                                           double* __restrict__ out64, float* __restrict__ out32) {
    __shared__ double red[kSumThreads / 32];
    double acc = 0.0;
    for (unsigned j = threadIdx.x; j < count; j += kSumThreads) acc += partials[j];
    acc = warpSum(acc);
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = red[0];
        for (unsigned w = 1; w < kSumThreads / 32; ++w) t += red[w];
        if (out64) *out64 = t;
        if (out32) *out32 = static_cast<float>(t);
    }
}

// Column sums: CTA (bx) covers 256 consecutive columns over all rows, one
// column per thread, rows walked in order; every output is one thread's f64
// sequential sum, so the result is deterministic without scratch.
__global__ void __launch_bounds__(kSumThreads) sumCols(const float* __restrict__ x, float* __restrict__ y,
                                                       std::uint64_t rows, std::uint64_t cols) {
    const std::uint64_t c = static_cast<std::uint64_t>(blockIdx.x) * kSumThreads + threadIdx.x;
    if (c >= cols) return;
    double acc = 0.0;
    std::uint64_t r = 0;
    for (; r + 4 <= rows; r += 4) {
        const float a = x[r * cols + c], b = x[(r + 1) * cols + c], d = x[(r + 2) * cols + c], e = x[(r + 3) * cols + c];
        acc += a;
        acc += b;
        acc += d;
        acc += e;
    }
    for (; r < rows; ++r) acc += x[r * cols + c];
    y[c] = static_cast<float>(acc);
}

} // namespace

cudaError_t softmaxRowsF32(const float* x, float* y, std::uint64_t rows, std::uint64_t cols, int smCount,
                           cudaStream_t stream, std::uint32_t* status) {
    return launchRows<RowOp::Softmax>(x, y, rows, cols, smCount, stream, status);
}

cudaError_t maxRowsF32(const float* x, float* y, std::uint64_t rows, std::uint64_t cols, int smCount,
                       cudaStream_t stream, std::uint32_t* status) {
    return launchRows<RowOp::Max>(x, y, rows, cols, smCount, stream, status);
}

cudaError_t sumRowsF32(const float* x, float* y, std::uint64_t rows, std::uint64_t cols, int smCount,
                       cudaStream_t stream, std::uint32_t* status) {
    return launchRows<RowOp::Sum>(x, y, rows, cols, smCount, stream, status);
}

cudaError_t sumColsF32(const float* x, float* y, std::uint64_t rows, std::uint64_t cols, int, cudaStream_t stream) {
    if (cols == 0) return cudaSuccess;
    const std::uint64_t grid = (cols + kSumThreads - 1) / kSumThreads;
    sumCols<<<static_cast<unsigned>(grid), kSumThreads, 0, stream>>>(x, y, rows, cols);
    return cudaGetLastError();
}

std::uint32_t sumAllPartialCount(std::uint64_t n, int smCount) {
    const std::uint64_t byWork = (n / 4 + kSumThreads * 4 - 1) / (kSumThreads * 4);
    const std::uint64_t cap = static_cast<std::uint64_t>(smCount) * 4;
    return static_cast<std::uint32_t>(std::max<std::uint64_t>(1, std::min(cap, byWork)));
}

cudaError_t sumAllF32(const float* x, std::uint64_t n, double* partials, std::uint32_t partialCount, double* out64,
                      float* out32, int smCount, cudaStream_t stream, std::uint32_t* status) {
    if (partialCount == 0) return cudaErrorInvalidValue;
    if (n == 0) {
        sumAllPass2<<<1, kSumThreads, 0, stream>>>(partials, 0, out64, out32);
        return cudaGetLastError();
    }
    const bool aligned = reinterpret_cast<std::uintptr_t>(x) % 16 == 0;
    // Bulk tiles once every SM has one (THB_ROWS=staged keeps the vector
    // pass, for comparison).
    static const bool bulk = [] {
        const char* e = std::getenv("THB_ROWS");
        return !(e && std::strcmp(e, "staged") == 0);
    }();
    const std::uint64_t tiles = n / kSumTileFloats;
    if (aligned && bulk && smCount > 0 && tiles >= static_cast<std::uint64_t>(smCount) &&
        partialCount >= static_cast<std::uint32_t>(smCount)) {
        cudaError_t e = cudaFuncSetAttribute(sumAllBulk, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kSumBulkSmem));
        if (e != cudaSuccess) return e;
        sumAllBulk<<<smCount, kSumThreads, kSumBulkSmem, stream>>>(x, n, partials, status);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        sumAllPass2<<<1, kSumThreads, 0, stream>>>(partials, static_cast<unsigned>(smCount), out64, out32);
        return cudaGetLastError();
    }
    if (aligned)
        sumAllPass1<true><<<partialCount, kSumThreads, 0, stream>>>(x, n, partials);
    else
        sumAllPass1<false><<<partialCount, kSumThreads, 0, stream>>>(x, n, partials);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    sumAllPass2<<<1, kSumThreads, 0, stream>>>(partials, partialCount, out64, out32);
    return cudaGetLastError();
}

} // namespace thb::kernels
