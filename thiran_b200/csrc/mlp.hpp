// Two-layer MLP training step (see mlp.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "gemm.hpp"

namespace thb::mlp {

// Device buffers of one training session (all owned by the session).
struct Buffers {
    std::uint64_t batch = 0, globalBatch = 0, in = 0, hidden = 0, out = 0;
    float* w1 = nullptr;       // f32 [in][hidden]
    float* w2 = nullptr;       // f32 [hidden][out]
    void* w1b = nullptr;       // bf16 copies
    void* w2b = nullptr;
    void* xb = nullptr;        // bf16 [batch][in]
    void* h = nullptr;         // bf16 [batch][hidden]
    float* y = nullptr;        // f32 [batch][out]
    void* dy = nullptr;        // bf16 [batch][out]
    void* dh = nullptr;        // bf16 [batch][hidden]
    float* dw1 = nullptr;      // f32 [in][hidden]
    float* dw2 = nullptr;      // f32 [hidden][out]
    double* lossPartials = nullptr;
    double* lossSum = nullptr; // sum over this rank's batch of (Y - T)^2
    // Broadcast biases (examples/mlp.th structure), enabled by setting b1:
    // H = relu(X W1 + b1), Y = H W2 + b2, gradients = column sums of dH, dY.
    float* b1 = nullptr;       // f32 [hidden]
    float* b2 = nullptr;       // f32 [out]
    float* db1 = nullptr;      // f32 [hidden]
    float* db2 = nullptr;      // f32 [out]
    float* dyColSums = nullptr;  // f32 [lossRowChunks][out] partial column sums of dY
    float* dhColSums = nullptr;  // f32 [colSumRows(batch)][hidden] partial column sums of dH
    // SGD with momentum (Training.cpp:366-372) when momentum > 0: velocities.
    float momentum = 0.0f;
    float* vw1 = nullptr;
    float* vw2 = nullptr;
    float* vb1 = nullptr;
    float* vb2 = nullptr;
    // Data-parallel gradient all-reduce fused into the dW GEMMs (no peers =
    // plain local store). The caller advances `target` every step.
    gemm::AllReduce dw1Reduce;
    gemm::AllReduce dw2Reduce;
    // With the all-reduce, the parameters and their bf16 copies on every rank
    // (paramPeers / copyPeers / multicast of dwNReduce.update), so the owner
    // of each tile can apply the update in the reduction.
};

// Optional CUDA-event timing of the GEMM launches of a step (recorded on the
// launching stream).
struct GemmTimer {
    bool enabled = false;
    std::uint64_t launches = 0;
    cudaEvent_t events[2 * 512] = {};
    unsigned used = 0;  // events recorded since the last read
    void begin(cudaStream_t s) {
        if (enabled && used + 2 <= sizeof(events) / sizeof(events[0])) cudaEventRecord(events[used], s);
    }
    void end(cudaStream_t s) {
        if (enabled && used + 2 <= sizeof(events) / sizeof(events[0])) {
            cudaEventRecord(events[used + 1], s);
            used += 2;
            ++launches;
        }
    }
};

// Loss kernel layout: column blocks of 256 x row chunks; one f64 loss
// partial per block.
unsigned lossRowChunks(std::uint64_t rows, std::uint64_t cols, int smCount);
unsigned lossPartialCount(std::uint64_t rows, std::uint64_t cols, int smCount);
cudaError_t castToBf16(const float* x, void* y, std::uint64_t n, int smCount, cudaStream_t s);
// p -= lr * d with d = g (v null) or d = v * momentum + g, v = d; refreshes
// the bf16 copy pb when given.
cudaError_t sgdUpdate(float* p, const float* g, float* v, void* pb, std::uint64_t n, float lr, float momentum,
                      int smCount, cudaStream_t s);
// Forward, loss and backward: fills h, y, dy, dh, dw1, dw2, the bias
// gradients and lossSum. With `fusedLr` (single device, no all-reduce bound)
// the weight updates run in the dW GEMM epilogues instead (kEpiSgdF32): W1,
// W2, their velocities and bf16 copies are updated and dw1, dw2 are not
// written; applySgd(..., weights = false) then updates the biases.
cudaError_t forwardBackward(const Buffers&, const float* x, const float* t, int smCount, std::uint32_t* status,
                            cudaStream_t s, GemmTimer* timer = nullptr, const float* fusedLr = nullptr);
// p -= lr * g for every parameter (the weights only when `weights`),
// refreshing the bf16 copies.
cudaError_t applySgd(const Buffers&, float lr, int smCount, cudaStream_t s, bool weights = true);

} // namespace thb::mlp
