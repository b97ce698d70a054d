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
    kEpiAllReduceF32 = 4,  // C (f32) = sum over ranks of acc, on every rank (see AllReduce)
    kEpiSgdF32 = 5,        // C (f32 parameters) updated in place with gradient acc (see Update)
};

// The optimizer step fused into the read-out of a weight-gradient GEMM
// (kEpiSgdF32): C holds the f32 parameters, g = acc, and per element
// d = g (or d = v*mu + g, v = d when `velocity` is given), C = C - d*lr, each
// operation rounded to f32 as the standalone SGD pass does
// (src/training/v0/Training.cpp:366-372); `copy` (bf16, optional) receives
// the updated parameters. The gradient itself is never stored. velocity and
// copy share C's leading dimension.
struct Update {
    float* velocity = nullptr;
    void* copy = nullptr;
    float lr = 0.0f;
    float momentum = 0.0f;
};

// Cross-GPU all-reduce fused into the epilogue (kEpiAllReduceF32). Every rank
// runs the same GEMM on its own rows of K (its part of the batch); C and the
// signal words are symmetric buffers every rank maps. Each finished tile is
// stored locally and announced by a release add on its owner rank's signal
// word; the owner's reducer warps wait for all ranks' announcements, sum the
// tile and write the total into every rank's C while later tiles compute:
//  - peer mode (cMulticast null): plain NVLink loads of every rank's tile,
//    summed in rank order, and plain stores to every rank. Each GPU moves
//    2(world-1)/world of C each way, as a ring all-reduce does.
//  - switch mode: multimem.ld_reduce sums the tile inside NVSwitch and
//    multimem.st writes the total to all ranks; about (1 + 1/world) of C each
//    way, less than peer mode from 3 ranks up.
constexpr int kMaxRanks = 8;

// Optional optimizer step fused into the all-reduce: instead of writing the
// summed tile to every rank's C, the owner applies the update to the f32
// parameters P (same layout as C; its own copy is every rank's, since all
// ranks hold the same parameters) and writes the new P, and its bf16 copy,
// to every rank. Per element, in the order of the standalone pass
// (src/training/v0/Training.cpp:366-372): d = g (or d = v*mu + g, v = d),
// P = P - d*lr, each operation rounded to f32. The velocity of a tile lives
// on its owner only (ownership is fixed for a given problem and grid).
struct ReduceUpdate {
    bool enabled = false;
    float* paramPeers[kMaxRanks] = {};  // P as mapped on this GPU, for every rank
    void* copyPeers[kMaxRanks] = {};    // bf16 copy of P, for every rank
    float* paramMulticast = nullptr;    // switch mode: multicast addresses of P and of its copy
    void* copyMulticast = nullptr;
    float* velocity = nullptr;          // this rank's velocities (momentum > 0)
    float lr = 0.0f, momentum = 0.0f;
};

// Compact form of the fused update (`compact`, needs update.enabled): each
// rank stores its tile as bf16 (C is then bf16 [M][ldc]); the owner sums the
// ranks' bf16 tiles with f32 accumulation (multimem.ld_reduce ...
// .acc::f32.v4.bf16x2 in switch mode, f32 sums of peer loads in rank order
// in peer mode), applies the update to its own f32 parameters only, and
// writes the bf16 copy to every rank. The f32 parameters are thereby sharded
// by tile owner (every rank's copy of a tile it does not own goes stale;
// gatherOwned assembles them), and each element costs about 2 bytes of
// NVLink traffic per direction instead of 10.
struct AllReduce {
    void* cMulticast = nullptr;                   // switch mode: NVLS multicast address of C
    void* cPeers[kMaxRanks] = {};                 // C as mapped on this GPU, for every rank
    std::uint32_t* flagsPeers[kMaxRanks] = {};    // signal words (4 per tile), for every rank
    std::uint32_t rank = 0, world = 1;
    std::uint32_t target = 0;                     // each signal word's value once this launch's ranks all announced
    bool compact = false;                         // bf16 payload, parameters sharded by tile owner
    ReduceUpdate update;
};

// Tiles of an M x N output (signal words needed: 4 per tile).
std::uint64_t tileCount(std::uint64_t m, std::uint64_t n);

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
    AllReduce reduce;           // kEpiAllReduceF32
    // Optional f32 bias [N] added to every row before the epilogue op (F32,
    // Bf16 and ReluBf16 epilogues): C = op(acc + bias).
    const float* bias = nullptr;
    // Optional column partial sums of the f32 epilogue result (MaskBf16):
    // colSums[(mTile * 4 + q) * N + j] = sum over rows 32q..32q+31 of the
    // M tile of C[row][j], rows past M counting 0. Fixed summation order.
    float* colSums = nullptr;
    Update update;              // kEpiSgdF32
};

// Rows of partial sums `colSums` receives for an M x N problem.
std::uint64_t colSumRows(std::uint64_t m);

// Returns an error text for an invalid problem, or nullptr.
const char* validate(const Problem&);
// Launches on `stream`; `status` receives bit 4 when a bounded wait expired.
cudaError_t run(const Problem&, int smCount, std::uint32_t* status, cudaStream_t stream);

// For a compact fused update (AllReduce::compact): copies every tile this
// rank does not own from its owner's f32 parameters (reduce.update.
// paramPeers[owner], plain peer loads) into this rank's, so that this rank
// holds the full parameters again. The tile-to-owner map is the one `run`
// uses for the same problem on `smCount` SMs.
cudaError_t gatherOwned(const Problem&, int smCount, cudaStream_t stream);

} // namespace thb::gemm
