// Two-layer MLP training step on the tensor cores.
//
// The reference trains only in its Evaluator: trainingStep
// (src/training/v0/Training.cpp:382-432) runs the generated forward, the
// reverse-AD backward (src/autodiff/v0/Autodiff.cpp:72-294; matmul rule
// :216-227) and SGD p <- p - lr*g (Training.cpp:368-371). Here one step is
//   Xb = bf16(X)
//   H  = relu(Xb W1b)              GEMM, ReLU fused in the epilogue (bf16 out)
//   Y  = H W2b                     GEMM (f32 out)
//   D  = Y - T; loss += sum D^2; dY = bf16(D * 2/(B*O))   one fused pass
//   dH = (dY W2b^T) * [H > 0]      GEMM, mask fused in the epilogue
//   dW2 = H^T dY ; dW1 = Xb^T dH   GEMMs with MN-major operands (no transposes)
//   W -= lr dW ; Wb = bf16(W)      one fused pass per weight
// W1 is stored [in][hidden], W2 [hidden][out] (the reference's X*W1 layout).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "gemm.hpp"
#include "mlp.hpp"

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

// D = Y - T; partial[block] = sum D^2 (f64); dY = bf16(D * scale).
__global__ void __launch_bounds__(kThreads) lossGradKernel(const float* __restrict__ y, const float* __restrict__ t,
                                                           __nv_bfloat16* __restrict__ dy, double* __restrict__ partials,
                                                           std::uint64_t n, float scale) {
    __shared__ double red[kThreads / 32];
    double acc = 0.0;
    const std::uint64_t stride = static_cast<std::uint64_t>(gridDim.x) * kThreads;
    for (std::uint64_t i = static_cast<std::uint64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n; i += stride) {
        const float d = __fsub_rn(y[i], t[i]);
        acc += static_cast<double>(d) * static_cast<double>(d);
        dy[i] = __float2bfloat16_rn(__fmul_rn(d, scale));
    }
    acc = warpSum(acc);
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = red[0];
        for (unsigned w = 1; w < kThreads / 32; ++w) s += red[w];
        partials[blockIdx.x] = s;
    }
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

// w = w - lr * g ; wb = bf16(w)   (Training.cpp:368-371 with plain SGD)
__global__ void __launch_bounds__(kThreads) sgdKernel(float* __restrict__ w, const float* __restrict__ g,
                                                      __nv_bfloat16* __restrict__ wb, std::uint64_t n, float lr) {
    const std::uint64_t stride = static_cast<std::uint64_t>(gridDim.x) * kThreads;
    const std::uint64_t packets = n / 4;
    for (std::uint64_t i = static_cast<std::uint64_t>(blockIdx.x) * kThreads + threadIdx.x; i < packets; i += stride) {
        float4 v = reinterpret_cast<float4*>(w)[i];
        const float4 d = __ldcs(reinterpret_cast<const float4*>(g) + i);
        v.x = __fsub_rn(v.x, __fmul_rn(lr, d.x));
        v.y = __fsub_rn(v.y, __fmul_rn(lr, d.y));
        v.z = __fsub_rn(v.z, __fmul_rn(lr, d.z));
        v.w = __fsub_rn(v.w, __fmul_rn(lr, d.w));
        reinterpret_cast<float4*>(w)[i] = v;
        __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
        uint2 packed;
        packed.x = *reinterpret_cast<std::uint32_t*>(&lo);
        packed.y = *reinterpret_cast<std::uint32_t*>(&hi);
        reinterpret_cast<uint2*>(wb)[i] = packed;
    }
    if (blockIdx.x == 0 && threadIdx.x < n % 4) {
        const std::uint64_t k = packets * 4 + threadIdx.x;
        w[k] = __fsub_rn(w[k], __fmul_rn(lr, g[k]));
        wb[k] = __float2bfloat16_rn(w[k]);
    }
}

unsigned gridFor(std::uint64_t work, int smCount) {
    const std::uint64_t blocks = (work + kThreads - 1) / kThreads;
    const std::uint64_t cap = static_cast<std::uint64_t>(smCount) * 8;
    return static_cast<unsigned>(blocks < 1 ? 1 : (blocks < cap ? blocks : cap));
}

} // namespace

unsigned lossPartialCount(int smCount) { return static_cast<unsigned>(smCount) * 4; }

cudaError_t castToBf16(const float* x, void* y, std::uint64_t n, int smCount, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    castKernel<<<gridFor(n / 4 + 1, smCount), kThreads, 0, s>>>(x, static_cast<__nv_bfloat16*>(y), n);
    return cudaGetLastError();
}

cudaError_t lossAndGradient(const float* y, const float* t, void* dy, double* partials, double* lossSum,
                            std::uint64_t n, float scale, int smCount, cudaStream_t s) {
    const unsigned parts = lossPartialCount(smCount);
    lossGradKernel<<<parts, kThreads, 0, s>>>(y, t, static_cast<__nv_bfloat16*>(dy), partials, n, scale);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    sumPartialsKernel<<<1, kThreads, 0, s>>>(partials, parts, lossSum);
    return cudaGetLastError();
}

cudaError_t sgdUpdate(float* w, const float* g, void* wb, std::uint64_t n, float lr, int smCount, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    sgdKernel<<<gridFor(n / 4 + 1, smCount), kThreads, 0, s>>>(w, g, static_cast<__nv_bfloat16*>(wb), n, lr);
    return cudaGetLastError();
}

cudaError_t forwardBackward(const Buffers& b, const float* x, const float* t, int smCount, std::uint32_t* status,
                            cudaStream_t s, GemmTimer* timer) {
    GemmTimer none;
    GemmTimer& tm = timer ? *timer : none;
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
    if ((e = runGemm(q)) != cudaSuccess) return e;
    // Y = H W2b: A = H [B][hidden] K-major, B = W2b [hidden][out] MN-major.
    q = {};
    q.m = b.batch; q.n = b.out; q.k = b.hidden;
    q.a = b.h; q.lda = b.hidden;
    q.b = b.w2b; q.bMajorMN = true; q.ldb = b.out;
    q.c = b.y; q.ldc = b.out; q.epilogue = gemm::kEpiF32;
    if ((e = runGemm(q)) != cudaSuccess) return e;
    // Loss and dY = 2 (Y - T) / (global batch * out).
    const float scale = 2.0f / static_cast<float>(b.globalBatch * b.out);
    if ((e = lossAndGradient(b.y, t, b.dy, b.lossPartials, b.lossSum, b.batch * b.out, scale, smCount, s)) != cudaSuccess)
        return e;
    // dH = (dY W2b^T) * [H > 0]: A = dY [B][out] K-major, B = W2b [hidden][out] K-major (N=hidden).
    q = {};
    q.m = b.batch; q.n = b.hidden; q.k = b.out;
    q.a = b.dy; q.lda = b.out;
    q.b = b.w2b; q.ldb = b.out;
    q.c = b.dh; q.ldc = b.hidden; q.epilogue = gemm::kEpiMaskBf16;
    q.aux = b.h; q.ldAux = b.hidden;
    if ((e = runGemm(q)) != cudaSuccess) return e;
    // dW2 = H^T dY: A = H stored [B][hidden] (MN-major), B = dY stored [B][out] (MN-major).
    q = {};
    q.m = b.hidden; q.n = b.out; q.k = b.batch;
    q.a = b.h; q.aMajorMN = true; q.lda = b.hidden;
    q.b = b.dy; q.bMajorMN = true; q.ldb = b.out;
    q.c = b.dw2; q.ldc = b.out; q.epilogue = gemm::kEpiF32;
    if (b.dw2Reduce.cPeers[0]) { q.epilogue = gemm::kEpiAllReduceF32; q.reduce = b.dw2Reduce; }
    if ((e = runGemm(q)) != cudaSuccess) return e;
    // dW1 = Xb^T dH: A = Xb stored [B][in] (MN-major), B = dH stored [B][hidden] (MN-major).
    q = {};
    q.m = b.in; q.n = b.hidden; q.k = b.batch;
    q.a = b.xb; q.aMajorMN = true; q.lda = b.in;
    q.b = b.dh; q.bMajorMN = true; q.ldb = b.hidden;
    q.c = b.dw1; q.ldc = b.hidden; q.epilogue = gemm::kEpiF32;
    if (b.dw1Reduce.cPeers[0]) { q.epilogue = gemm::kEpiAllReduceF32; q.reduce = b.dw1Reduce; }
    return runGemm(q);
}

cudaError_t applySgd(const Buffers& b, float lr, int smCount, cudaStream_t s) {
    cudaError_t e = sgdUpdate(b.w1, b.dw1, b.w1b, b.in * b.hidden, lr, smCount, s);
    if (e != cudaSuccess) return e;
    return sgdUpdate(b.w2, b.dw2, b.w2b, b.hidden * b.out, lr, smCount, s);
}

} // namespace thb::mlp
