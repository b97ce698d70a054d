// tcgen05 bf16 GEMM (see gemm.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace thb::gemm {

// Epilogues fused into the accumulator read-out.
enum : int {
    kEpiF32 = 0,       // C (f32) = acc
    kEpiBf16 = 1,      // C (bf16) = acc
    kEpiReluBf16 = 2,  // C (bf16) = max(acc, 0)            (forward ReLU)
    kEpiMaskBf16 = 3,  // C (bf16) = aux > 0 ? acc : 0       (ReLU backward mask, aux bf16 [M][N])
    kEpiRedF32 = 4,    // C (f32) += acc on every GPU: `c` is an NVLink multicast address and the
                       // epilogue issues multimem.red.add, so the switch sums all ranks' tiles
};

struct Problem {
    std::uint64_t m = 0, n = 0, k = 0;
    const void* a = nullptr;  // bf16; K-major [M][K] or MN-major [K][M]
    bool aMajorMN = false;
    std::uint64_t lda = 0;
    const void* b = nullptr;  // bf16; K-major [N][K] or MN-major [K][N]
    bool bMajorMN = false;
    std::uint64_t ldb = 0;
    void* c = nullptr;        // row-major [M][N], f32 or bf16 per epilogue
    std::uint64_t ldc = 0;
    int epilogue = kEpiF32;
    const void* aux = nullptr;  // bf16 [M][N] for kEpiMaskBf16
    std::uint64_t ldAux = 0;
    void* c2 = nullptr;         // optional f32 copy (bf16 epilogues), ld = ldc
};

// Returns an error text for an invalid problem, or nullptr.
const char* validate(const Problem&);
// Launches on `stream`; `status` receives bit 4 when a bounded wait expired.
cudaError_t run(const Problem&, int smCount, std::uint32_t* status, cudaStream_t stream);

} // namespace thb::gemm
