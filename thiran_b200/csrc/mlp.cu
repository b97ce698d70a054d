// Two-layer MLP training step on the tensor cores.
//
// The reference trains only in its Evaluator: trainingStep
// (src/training/v0/Training.cpp:382-432) runs the generated forward, the
// reverse-AD backward (src/autodiff/v0/Autodiff.cpp:72-294; matmul rule
// :216-227) and SGD, optionally with momentum (Training.cpp:366-372). Here
// one step is
//   Xb = bf16(X)
//   H  = relu(Xb W1b + b1)         GEMM, bias + ReLU fused in the epilogue (bf16 out)
//   Y  = H W2b + b2                GEMM, bias fused (f32 out)
//   D  = Y - T; loss += sum D^2; G = D * 2/(B*O); dY = bf16(G);
//   db2 = column sums of G         one fused pass (+ a small partials reduce)
//   dH = (dY W2b^T) * [H > 0]      GEMM, mask and db1 column partials fused
//   dW2 = H^T dY ; dW1 = Xb^T dH   GEMMs with MN-major operands (no transposes)
//   p -= lr * d (d = g, or v = mu v + g) ; Wb = bf16(W)   one fused pass per parameter
// The biases b1 [hidden], b2 [out] broadcast over the rows (the
// examples/mlp.th structure; their gradients are the reference's
// reduceToShape, Evaluator.cpp:258-277) and are optional.
// W1 is stored [in][hidden], W2 [hidden][out] (the reference's X*W1 layout).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "gemm.hpp"
#include "mlp.hpp"
#include "sgd.cuh"

namespace thb::mlp {
namespace {

constexpr unsigned kThreads = 256;

__global__ void __launch_bounds__(kThreads) castKernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                                       std::uint64_t n) {
    const std::uint64_t stride = static_cast<std::uint64_t>(gridDim.x) * kThreads;
    const std::uint64_t packets = n / 4;
    for (std::uint64_t i = static_cast<std::uint64_t>(blockIdx.x) * kThreads + threadIdx.x; i < packets; i += stride) {
        const float4 v = __ldcs(reinterpret_cast<const float4*>(x) + i);
        __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
        uint2 packed;
        packed.x = *reinterpret_cast<std::uint32_t*>(&lo);
        packed.y = *reinterpret_cast<std::uint32_t*>(&hi);
        reinterpret_cast<uint2*>(y)[i] = packed;
    }
    if (blockIdx.x == 0 && threadIdx.x < n % 4) y[packets * 4 + threadIdx.x] = __float2bfloat16_rn(x[packets * 4 + threadIdx.x]);
}

template <class T>
__device__ __forceinline__ T warpSum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// D = Y - T; G = D * scale; dY = bf16(G). Block (x, y) covers columns
// 1024x .. 1024x+1023 of the rows of chunk y, four adjacent columns per
// thread (16-byte loads; a warp reads 512 contiguous bytes of Y and of T per
// row; cols is a multiple of 4 and rows are 16-byte aligned):
// partial[block] = sum D^2 (f64) and, when colSums is given,
// colSums[y][col] = sum over the chunk's rows of G (f32, row order).
__global__ void __launch_bounds__(kThreads) lossGradKernel(const float* __restrict__ y, const float* __restrict__ t,
                                                           __nv_bfloat16* __restrict__ dy, double* __restrict__ partials,
                                                           float* __restrict__ colSums, std::uint64_t rows,
                                                           std::uint64_t cols, std::uint64_t rowsPerChunk, float scale) {
    __shared__ double red[kThreads / 32];
    double acc = 0.0;
    const std::uint64_t col = (static_cast<std::uint64_t>(blockIdx.x) * kThreads + threadIdx.x) * 4;
    const std::uint64_t r0 = static_cast<std::uint64_t>(blockIdx.y) * rowsPerChunk;
    const std::uint64_t r1 = r0 + rowsPerChunk < rows ? r0 + rowsPerChunk : rows;
    if (col < cols) {
        float c[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 4
        for (std::uint64_t r = r0; r < r1; ++r) {
            const std::uint64_t i = r * cols + col;
            const float4 yv = __ldcs(reinterpret_cast<const float4*>(y + i));
            const float4 tv = __ldcs(reinterpret_cast<const float4*>(t + i));
            const float d[4] = {__fsub_rn(yv.x, tv.x), __fsub_rn(yv.y, tv.y), __fsub_rn(yv.z, tv.z),
                                __fsub_rn(yv.w, tv.w)};
            float g[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                acc += static_cast<double>(d[j]) * static_cast<double>(d[j]);
                g[j] = __fmul_rn(d[j], scale);
                c[j] = __fadd_rn(c[j], g[j]);
            }
            const __nv_bfloat162 lo = __floats2bfloat162_rn(g[0], g[1]), hi = __floats2bfloat162_rn(g[2], g[3]);
            uint2 packed;
            packed.x = *reinterpret_cast<const std::uint32_t*>(&lo);
            packed.y = *reinterpret_cast<const std::uint32_t*>(&hi);
            __stcs(reinterpret_cast<uint2*>(dy + i), packed);
        }
        if (colSums)
            *reinterpret_cast<float4*>(colSums + static_cast<std::uint64_t>(blockIdx.y) * cols + col) =
                make_float4(c[0], c[1], c[2], c[3]);
    }
    acc = warpSum(acc);
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = red[0];
        for (unsigned w = 1; w < kThreads / 32; ++w) s += red[w];
        partials[static_cast<std::uint64_t>(blockIdx.y) * gridDim.x + blockIdx.x] = s;
    }
}

// out[col] = sum over r of partials[r][col], f64 in row order, rounded once.
__global__ void __launch_bounds__(kThreads) columnReduceKernel(const float* __restrict__ partials, std::uint64_t rows,
                                                               std::uint64_t cols, float* __restrict__ out) {
    const std::uint64_t col = static_cast<std::uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (col >= cols) return;
    double acc = 0.0;
    for (std::uint64_t r = 0; r < rows; ++r) acc += static_cast<double>(partials[r * cols + col]);
    out[col] = static_cast<float>(acc);
}

__global__ void __launch_bounds__(kThreads) sumPartialsKernel(const double* __restrict__ partials, unsigned count,
                                                              double* __restrict__ out) {
    __shared__ double red[kThreads / 32];
    double acc = 0.0;
    for (unsigned j = threadIdx.x; j < count; j += kThreads) acc += partials[j];
    acc = warpSum(acc);
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = red[0];
        for (unsigned w = 1; w < kThreads / 32; ++w) s += red[w];
        *out = s;
    }
}

__device__ __forceinline__ float updateOne(float p, float g, float* v, float lr, float mu) {
    return sgdStep(p, g, v, lr, mu);
}

// p = update(p, g, v); pb = bf16(p) when pb is given. Vectorised by 4.
__global__ void __launch_bounds__(kThreads) sgdKernel(float* __restrict__ w, const float* __restrict__ g,
                                                      float* __restrict__ vel, __nv_bfloat16* __restrict__ wb,
                                                      std::uint64_t n, float lr, float mu) {
    const std::uint64_t stride = static_cast<std::uint64_t>(gridDim.x) * kThreads;
    const std::uint64_t packets = n / 4;
    for (std::uint64_t i = static_cast<std::uint64_t>(blockIdx.x) * kThreads + threadIdx.x; i < packets; i += stride) {
        float4 p = reinterpret_cast<float4*>(w)[i];
        const float4 d = __ldcs(reinterpret_cast<const float4*>(g) + i);
        if (vel) {
            float4 v = reinterpret_cast<float4*>(vel)[i];
            p.x = updateOne(p.x, d.x, &v.x, lr, mu);
            p.y = updateOne(p.y, d.y, &v.y, lr, mu);
            p.z = updateOne(p.z, d.z, &v.z, lr, mu);
            p.w = updateOne(p.w, d.w, &v.w, lr, mu);
            reinterpret_cast<float4*>(vel)[i] = v;
        } else {
            p.x = updateOne(p.x, d.x, nullptr, lr, mu);
            p.y = updateOne(p.y, d.y, nullptr, lr, mu);
            p.z = updateOne(p.z, d.z, nullptr, lr, mu);
            p.w = updateOne(p.w, d.w, nullptr, lr, mu);
        }
        reinterpret_cast<float4*>(w)[i] = p;
        if (wb) {
            __nv_bfloat162 lo = __floats2bfloat162_rn(p.x, p.y), hi = __floats2bfloat162_rn(p.z, p.w);
            uint2 packed;
            packed.x = *reinterpret_cast<std::uint32_t*>(&lo);
            packed.y = *reinterpret_cast<std::uint32_t*>(&hi);
            reinterpret_cast<uint2*>(wb)[i] = packed;
        }
    }
    if (blockIdx.x == 0 && threadIdx.x < n % 4) {
        const std::uint64_t k = packets * 4 + threadIdx.x;
        w[k] = updateOne(w[k], g[k], vel ? vel + k : nullptr, lr, mu);
        if (wb) wb[k] = __float2bfloat16_rn(w[k]);
    }
}

unsigned gridFor(std::uint64_t work, int smCount) {
    const std::uint64_t blocks = (work + kThreads - 1) / kThreads;
    const std::uint64_t cap = static_cast<std::uint64_t>(smCount) * 8;
    return static_cast<unsigned>(blocks < 1 ? 1 : (blocks < cap ? blocks : cap));
}

} // namespace

// Columns per loss block (four per thread).
constexpr std::uint64_t kLossCols = kThreads * 4;

unsigned lossRowChunks(std::uint64_t rows, std::uint64_t cols, int smCount) {
    const std::uint64_t colBlocks = (cols + kLossCols - 1) / kLossCols;
    std::uint64_t chunks = (static_cast<std::uint64_t>(smCount) * 8 + colBlocks - 1) / colBlocks;
    if (chunks > rows) chunks = rows;
    return static_cast<unsigned>(chunks < 1 ? 1 : chunks);
}

unsigned lossPartialCount(std::uint64_t rows, std::uint64_t cols, int smCount) {
    return static_cast<unsigned>((cols + kLossCols - 1) / kLossCols) * lossRowChunks(rows, cols, smCount);
}

cudaError_t castToBf16(const float* x, void* y, std::uint64_t n, int smCount, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    castKernel<<<gridFor(n / 4 + 1, smCount), kThreads, 0, s>>>(x, static_cast<__nv_bfloat16*>(y), n);
    return cudaGetLastError();
}

// Loss, dY and (when db is given) db = column sums of the f32 gradient G.
cudaError_t lossAndGradient(const float* y, const float* t, void* dy, double* partials, double* lossSum,
                            float* colSums, float* db, std::uint64_t rows, std::uint64_t cols, float scale, int smCount,
                            cudaStream_t s) {
    const unsigned chunks = lossRowChunks(rows, cols, smCount);
    const unsigned colBlocks = static_cast<unsigned>((cols + kLossCols - 1) / kLossCols);
    const std::uint64_t rowsPerChunk = (rows + chunks - 1) / chunks;
    lossGradKernel<<<dim3(colBlocks, chunks), kThreads, 0, s>>>(y, t, static_cast<__nv_bfloat16*>(dy), partials,
                                                                db ? colSums : nullptr, rows, cols, rowsPerChunk, scale);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    sumPartialsKernel<<<1, kThreads, 0, s>>>(partials, colBlocks * chunks, lossSum);
    if ((e = cudaGetLastError()) != cudaSuccess || !db) return e;
    // One thread per column (the loss blocks above take four columns each).
    columnReduceKernel<<<static_cast<unsigned>((cols + kThreads - 1) / kThreads), kThreads, 0, s>>>(colSums, chunks,
                                                                                                 cols, db);
    return cudaGetLastError();
}

cudaError_t columnSums(const float* partials, std::uint64_t rows, std::uint64_t cols, float* out, cudaStream_t s) {
    columnReduceKernel<<<static_cast<unsigned>((cols + kThreads - 1) / kThreads), kThreads, 0, s>>>(partials, rows, cols,
                                                                                                 out);
    return cudaGetLastError();
}

cudaError_t sgdUpdate(float* p, const float* g, float* v, void* pb, std::uint64_t n, float lr, float momentum,
                      int smCount, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    sgdKernel<<<gridFor(n / 4 + 1, smCount), kThreads, 0, s>>>(p, g, v, static_cast<__nv_bfloat16*>(pb), n, lr,
                                                                 momentum);
    return cudaGetLastError();
}

cudaError_t forwardBackward(const Buffers& b, const float* x, const float* t, int smCount, std::uint32_t* status,
                            cudaStream_t s, GemmTimer* timer, const float* fusedLr) {
    GemmTimer none;
    GemmTimer& tm = timer ? *timer : none;
    const bool reduced = b.dw1Reduce.cPeers[0] || b.dw2Reduce.cPeers[0];
    // A data-parallel fused step needs the parameters of every rank bound.
    if (fusedLr && reduced && !(b.dw1Reduce.update.paramPeers[0] && b.dw2Reduce.update.paramPeers[0]))
        return cudaErrorInvalidValue;
    // Weight-gradient GEMM epilogue: store dW, all-reduce it (and, with
    // fusedLr, apply the update in the reduction), or apply the optimizer
    // step to the parameters in place.
    const bool momentum = b.momentum > 0.0f;
    auto weightGradient = [&](gemm::Problem& q, float* dw, float* w, float* vw, void* wb, const gemm::AllReduce& r) {
        if (r.cPeers[0]) {
            q.c = dw;
            q.epilogue = gemm::kEpiAllReduceF32;
            q.reduce = r;
            q.reduce.update.enabled = fusedLr != nullptr;
            if (fusedLr) {
                q.reduce.update.velocity = momentum ? vw : nullptr;
                q.reduce.update.lr = *fusedLr;
                q.reduce.update.momentum = b.momentum;
            }
        } else if (fusedLr) {
            q.c = w;
            q.epilogue = gemm::kEpiSgdF32;
            q.update.velocity = momentum ? vw : nullptr;
            q.update.copy = wb;
            q.update.lr = *fusedLr;
            q.update.momentum = b.momentum;
        } else {
            q.c = dw;
            q.epilogue = gemm::kEpiF32;
        }
    };
    auto runGemm = [&](const gemm::Problem& q) {
        tm.begin(s);
        const cudaError_t r = gemm::run(q, smCount, status, s);
        tm.end(s);
        return r;
    };
    cudaError_t e = castToBf16(x, b.xb, b.batch * b.in, smCount, s);
    if (e != cudaSuccess) return e;
    gemm::Problem q;
    // H = relu(Xb W1b): A = Xb [B][in] K-major, B = W1b [in][hidden] MN-major.
    q = {};
    q.m = b.batch; q.n = b.hidden; q.k = b.in;
    q.a = b.xb; q.lda = b.in;
    q.b = b.w1b; q.bMajorMN = true; q.ldb = b.hidden;
    q.c = b.h; q.ldc = b.hidden; q.epilogue = gemm::kEpiReluBf16;
    q.bias = b.b1;  // relu(acc + b1)
    if ((e = runGemm(q)) != cudaSuccess) return e;
    // Y = H W2b: A = H [B][hidden] K-major, B = W2b [hidden][out] MN-major.
    q = {};
    q.m = b.batch; q.n = b.out; q.k = b.hidden;
    q.a = b.h; q.lda = b.hidden;
    q.b = b.w2b; q.bMajorMN = true; q.ldb = b.out;
    q.c = b.y; q.ldc = b.out; q.epilogue = gemm::kEpiF32;
    q.bias = b.b2;  // acc + b2
    if ((e = runGemm(q)) != cudaSuccess) return e;
    // Loss and dY = 2 (Y - T) / (global batch * out); db2 = column sums of dY.
    const float scale = 2.0f / static_cast<float>(b.globalBatch * b.out);
    if ((e = lossAndGradient(b.y, t, b.dy, b.lossPartials, b.lossSum, b.dyColSums, b.b1 ? b.db2 : nullptr, b.batch,
                             b.out, scale, smCount, s)) != cudaSuccess)
        return e;
    // dH = (dY W2b^T) * [H > 0]: A = dY [B][out] K-major, B = W2b [hidden][out] K-major (N=hidden).
    q = {};
    q.m = b.batch; q.n = b.hidden; q.k = b.out;
    q.a = b.dy; q.lda = b.out;
    q.b = b.w2b; q.ldb = b.out;
    q.c = b.dh; q.ldc = b.hidden; q.epilogue = gemm::kEpiMaskBf16;
    q.aux = b.h; q.ldAux = b.hidden;
    if (b.b1) q.colSums = b.dhColSums;  // db1 = column sums of dH (f32, before rounding)
    if ((e = runGemm(q)) != cudaSuccess) return e;
    if (b.b1 && (e = columnSums(b.dhColSums, gemm::colSumRows(b.batch), b.hidden, b.db1, s)) != cudaSuccess) return e;
    // dW2 = H^T dY: A = H stored [B][hidden] (MN-major), B = dY stored [B][out] (MN-major).
    q = {};
    q.m = b.hidden; q.n = b.out; q.k = b.batch;
    q.a = b.h; q.aMajorMN = true; q.lda = b.hidden;
    q.b = b.dy; q.bMajorMN = true; q.ldb = b.out;
    q.ldc = b.out;
    // (W2's bf16 copy may be rewritten here: the dH GEMM above has read it.)
    weightGradient(q, b.dw2, b.w2, b.vw2, b.w2b, b.dw2Reduce);
    if ((e = runGemm(q)) != cudaSuccess) return e;
    // dW1 = Xb^T dH: A = Xb stored [B][in] (MN-major), B = dH stored [B][hidden] (MN-major).
    q = {};
    q.m = b.in; q.n = b.hidden; q.k = b.batch;
    q.a = b.xb; q.aMajorMN = true; q.lda = b.in;
    q.b = b.dh; q.bMajorMN = true; q.ldb = b.hidden;
    q.ldc = b.hidden;
    weightGradient(q, b.dw1, b.w1, b.vw1, b.w1b, b.dw1Reduce);
    return runGemm(q);
}

cudaError_t applySgd(const Buffers& b, float lr, int smCount, cudaStream_t s, bool weights) {
    const float mu = b.momentum;
    const bool m = mu > 0.0f;
    cudaError_t e = cudaSuccess;
    if (weights) {
        if ((e = sgdUpdate(b.w1, b.dw1, m ? b.vw1 : nullptr, b.w1b, b.in * b.hidden, lr, mu, smCount, s)) !=
            cudaSuccess)
            return e;
        if ((e = sgdUpdate(b.w2, b.dw2, m ? b.vw2 : nullptr, b.w2b, b.hidden * b.out, lr, mu, smCount, s)) !=
            cudaSuccess)
            return e;
    }
    if (!b.b1) return cudaSuccess;
    if ((e = sgdUpdate(b.b1, b.db1, m ? b.vb1 : nullptr, nullptr, b.hidden, lr, mu, smCount, s)) != cudaSuccess) return e;
    return sgdUpdate(b.b2, b.db2, m ? b.vb2 : nullptr, nullptr, b.out, lr, mu, smCount, s);
}

} // namespace thb::mlp
