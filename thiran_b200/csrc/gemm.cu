// bf16 x bf16 -> f32 GEMM on the 5th-generation tensor cores (tcgen05) for sm_100a.
//
// C[M,N] = A[M,K] * B[K,N] with f32 accumulation in tensor memory. Operands
// are read by TMA (no multicast) into 128B-swizzled shared memory; each
// operand may be K-major (A stored [M][K], B stored [N][K]) or MN-major
// (A stored [K][M], B stored [K][N]), so the transposed products of a
// reverse-AD backward pass (dW = X^T dH) need no transpose copies.
//
// One persistent CTA per SM, 192 threads (320 for the epilogues below that
// read global memory or all-reduce):
//   warp 0      TMA producer (one lane): 4-stage ring of {A 128x64, B 256x64}
//   warp 1      TMEM owner (alloc/dealloc 512 columns) and MMA issuer (one
//               lane): 4 x tcgen05.mma (M=128, N=256, K=16) per stage
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time, fused op, stores
//               (warps 2..9, two per TMEM lane quadrant splitting the
//               columns, for the optimizer-step and ReLU-mask epilogues)
//   warps 6..9  (fused all-reduce only) reducers: sum the tiles this rank
//               owns over all ranks and write the totals to every rank
// Two TMEM accumulators (2 x 256 columns) let the epilogue of tile i overlap
// the MMAs of tile i+1. Past one 128-row block the same roles run in CTA
// pairs (clusters of two, tcgen05 cta_group::2) on 256x256 tiles: each CTA
// stages half of A and half of B, the even CTA issues M=256 MMAs over both,
// and each CTA's epilogue drains its own 128 TMEM lanes (the fused
// all-reduce keeps single CTAs: its signal words are per 128-row tile).
// Every wait (mbarrier, tile queue, other ranks' signal words) is bounded:
// on expiry the CTA raises bit 4 of the status word, drains its copies and
// MMAs, frees TMEM and returns.
//
// The reference's only matmul is its Evaluator's sequential f32 triple loop
// (src/semantic/v0/Evaluator.cpp:125-154); reverse-mode rules dA = dZ B^T,
// dB = A^T dZ come from src/autodiff/v0/Autodiff.cpp:216-227.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstdlib>
#include <mutex>

#include "gemm.hpp"
#include "sgd.cuh"

namespace thb::gemm {
namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64, kStages = 4;
// The fused all-reduce adds 4 reducer warps (warps 6..9).
// Epilogue warps: 4 (one per TMEM lane quadrant), or 8 (two per quadrant,
// each taking half of the tile's columns) for the epilogues that also read
// global memory per element (the optimizer step reads the parameters, the
// ReLU mask reads H): twice the loads in flight.
constexpr int epilogueWarps(int epilogue) { return epilogue == kEpiSgdF32 || epilogue == kEpiMaskBf16 ? 8 : 4; }
constexpr int threadsFor(int epilogue) {
    return 64 + 32 * epilogueWarps(epilogue) + (epilogue == kEpiAllReduceF32 ? 128 : 0);
}
constexpr uint32_t kABytes = kBM * kBK * 2;  // 16 KB

// Stage geometry. PAIR = a cluster of two CTAs on one 256x256 tile with
// tcgen05.mma.cta_group::2 (M = 256): each CTA stages its 128 rows of A and
// its 128 columns of B, so a stage is 32 KB and six fit where four single-CTA
// stages (48 KB) did. Operand bytes moved from L2 per FLOP drop by a third.
template <bool PAIR>
struct Geometry {
    static constexpr int stages = PAIR ? 6 : kStages;
    static constexpr uint32_t bRows = PAIR ? kBN / 2 : kBN;  // B rows (N) staged per CTA
    static constexpr uint32_t bBytes = bRows * kBK * 2;
    static constexpr uint32_t stageBytes = kABytes + bBytes;
    static constexpr uint32_t tileM = PAIR ? 2 * kBM : kBM;
    static constexpr uint32_t smemBytes = stages * stageBytes + 1024;
};
static_assert(Geometry<true>::smemBytes <= 232448 && Geometry<false>::smemBytes <= 232448, "shared memory");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kWaitStatus = 16u;
constexpr uint64_t kSpinLimit = 1ull << 24;

__device__ __forceinline__ uint32_t smem(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void mbarInit(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbarExpect(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbarArrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem(b)) : "memory");
}
// True when the phase with parity `parity` has completed; false on timeout,
// or as soon as `abort` (when given) reads non-zero.
__device__ __forceinline__ bool mbarWait(uint64_t* b, uint32_t parity, const volatile int* abort = nullptr) {
    const uint32_t addr = smem(b);
    for (uint64_t spin = 0; spin < kSpinLimit; ++spin) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
        if (abort && (spin & 255u) == 255u && *abort) return false;
    }
    return false;
}

__device__ __forceinline__ void tmaLoad2d(void* dst, const CUtensorMap* map, int32_t x, int32_t y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem(bar))
        : "memory");
}

// UMMA shared-memory descriptor, 128B swizzle, sm_100 version bits.
__device__ __forceinline__ uint64_t ummaDesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;  // descriptor version (sm_100)
    d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
    return d;
}

// Instruction descriptor: bf16 x bf16 -> f32, dense, N=256, M=128 (one CTA)
// or M=256 (a CTA pair).
template <bool A_MN, bool B_MN, bool PAIR>
__device__ __forceinline__ constexpr uint32_t instrDesc() {
    return (1u << 4)                          // D format f32
           | (1u << 7)                        // A bf16
           | (1u << 10)                       // B bf16
           | (static_cast<uint32_t>(A_MN) << 15) | (static_cast<uint32_t>(B_MN) << 16) |
           (static_cast<uint32_t>(kBN >> 3) << 17) | (static_cast<uint32_t>(Geometry<PAIR>::tileM >> 4) << 24);
}

__device__ __forceinline__ void mma(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mmaCommit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem(bar))
                 : "memory");
}

// ---- CTA pairs (cta_group::2) ----
__device__ __forceinline__ uint32_t clusterRank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Shared-memory address of the same object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t pairAddress(const void* p, uint32_t rank) {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem(p)), "r"(rank));
    return a;
}

// All threads of both CTAs.
__device__ __forceinline__ void clusterSync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void mbarArriveCluster(uint32_t clusterAddress) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(clusterAddress) : "memory");
}

// A load into this CTA's shared memory whose completion is counted on an
// mbarrier of either CTA of the pair (.cta_group::2). No multicast: each CTA
// loads only its own half of the operands.
__device__ __forceinline__ void tmaLoad2dPair(void* dst, const CUtensorMap* map, int32_t x, int32_t y,
                                              uint32_t barClusterAddress) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(barClusterAddress)
        : "memory");
}

__device__ __forceinline__ void mmaPair(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives on the barrier at this offset in both CTAs once the pair's MMAs
// issued so far have completed.
__device__ __forceinline__ void mmaCommitPair(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                     smem(bar)),
                 "h"(static_cast<uint16_t>(3))
                 : "memory");
}

__device__ __forceinline__ void fenceAfter() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fenceBefore() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmemLoad32(uint32_t addr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(addr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

struct Params {
    uint32_t m, n, k;
    uint32_t mTiles, nTiles, kBlocks;
    uint32_t group;  // m-blocks per raster group
    void* c;
    uint64_t ldc;
    const __nv_bfloat16* aux;
    uint64_t ldAux;
    void* c2;  // optional f32 copy of the epilogue result
    uint32_t* status;
    uint32_t grid;  // persistent CTAs; CTA g takes tiles g, g + grid, ...
    // kEpiAllReduceF32
    float* cMc;                     // switch mode when non-null
    float* cPeers[kMaxRanks];       // peer mode
    uint32_t* flagsPeers[kMaxRanks];
    uint32_t rank, world, target;
    const float* bias;              // [n] or null
    float* colSums;                 // [mTiles * 4][n] or null (kEpiMaskBf16)
    // kEpiSgdF32, and kEpiAllReduceF32 with the fused update
    float* velocity;                // [m][ldc] or null
    __nv_bfloat16* copy;            // [m][ldc] or null (kEpiSgdF32)
    float lr, mu;
    // kEpiAllReduceF32 with the fused update: parameters and their bf16
    // copies on every rank (peer pointers; multicast in switch mode)
    uint32_t fusedUpdate;
    uint32_t compact;               // bf16 payload, parameters sharded by tile owner (needs fusedUpdate)
    float* pPeers[kMaxRanks];
    __nv_bfloat16* pbPeers[kMaxRanks];
    float* pMc;
    __nv_bfloat16* pbMc;
};

// Lane j ends with the sum over the warp's 32 lanes of s[j] (a butterfly
// transpose-reduce: 31 shuffles, fixed order, so the result is
// reproducible). Destroys s.
__device__ __forceinline__ float columnSum32(float (&s)[32], uint32_t lane) {
#pragma unroll
    for (int width = 16; width >= 1; width >>= 1) {
        const bool upper = (lane & width) != 0;
#pragma unroll
        for (int i = 0; i < width; ++i) {
            const float send = upper ? s[i] : s[i + width];
            const float keep = upper ? s[i + width] : s[i];
            s[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, width));
        }
    }
    return s[0];
}

// Tile order: groups of p.group m-blocks, walked down m within each n-block
// (L2 reuse of the B tiles across the group).
__device__ __forceinline__ void tileCoords(uint32_t tile, const Params& p, uint32_t& mb, uint32_t& nb) {
    const uint32_t perGroup = p.group * p.nTiles;
    const uint32_t group = tile / perGroup;
    const uint32_t first = group * p.group;
    const uint32_t size = min(p.mTiles - first, p.group);
    const uint32_t local = tile % perGroup;
    mb = first + local % size;
    nb = local / size;
}

// Stores 32 consecutive results of a row as bf16 (16-byte vectors when the
// chunk is whole and aligned; `left` = columns left in the row otherwise).
__device__ __forceinline__ void storeBf16x32(__nv_bfloat16* dst, const float (&v)[32], bool full32, uint32_t left) {
    if (full32 && reinterpret_cast<uintptr_t>(dst) % 16 == 0) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint4 packed;
            __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&packed);
#pragma unroll
            for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[q * 8 + 2 * e], v[q * 8 + 2 * e + 1]);
            *reinterpret_cast<uint4*>(dst + q * 8) = packed;
        }
    } else {
        for (uint32_t j = 0; j < 32; ++j)
            if (j < left) dst[j] = __float2bfloat16_rn(v[j]);
    }
}

template <int EPI>
__device__ __forceinline__ float epilogueValue(float acc, float aux) {
    if constexpr (EPI == kEpiReluBf16) return acc > 0.0f ? acc : 0.0f;
    if constexpr (EPI == kEpiMaskBf16) return aux > 0.0f ? acc : 0.0f;
    return acc;
}

// ---- fused all-reduce (kEpiAllReduceF32) ----
constexpr uint32_t kNoTile = 0xffffffffu;
constexpr uint64_t kSignalSpinLimit = 1ull << 21;  // polls of ~0.1-1 us each

// Owned tiles pass from an epilogue warp to the reducer warp of the same TMEM
// quadrant through a small ring in shared memory (lane 0 of each side; the
// slot is written before the head moves).
constexpr uint32_t kQueueDepth = 4;
constexpr uint64_t kQueueSpinLimit = 1ull << 27;  // polls of >= 128 ns: > 15 s
struct TileQueue {
    uint32_t slot[kQueueDepth];
    uint32_t head, tail;
};

__device__ __forceinline__ bool pushTile(TileQueue& q, uint32_t tile, uint32_t lane, const volatile int* abort) {
    uint32_t ok = 0;
    if (lane == 0) {
        volatile uint32_t* head = &q.head;
        volatile uint32_t* tail = &q.tail;
        const uint32_t h = *head;
        for (uint64_t spin = 0; spin < kQueueSpinLimit && !*abort; ++spin) {
            if (h - *tail < kQueueDepth) {
                ok = 1;
                break;
            }
            __nanosleep(128);
        }
        if (ok) {
            reinterpret_cast<volatile uint32_t*>(q.slot)[h % kQueueDepth] = tile;
            __threadfence_block();
            *head = h + 1;
        }
    }
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Next tile of the queue; kNoTile once the epilogue is done. A wait that runs
// out or sees the CTA abort sets `abort` and ends the reducer.
__device__ __forceinline__ uint32_t popTile(TileQueue& q, uint32_t lane, volatile int* abort) {
    uint32_t tile = kNoTile;
    if (lane == 0) {
        volatile uint32_t* head = &q.head;
        volatile uint32_t* tail = &q.tail;
        const uint32_t t = *tail;
        bool got = false;
        for (uint64_t spin = 0; spin < kQueueSpinLimit && !*abort; ++spin) {
            if (*head != t) {
                __threadfence_block();
                tile = reinterpret_cast<volatile uint32_t*>(q.slot)[t % kQueueDepth];
                *tail = t + 1;
                got = true;
                break;
            }
            __nanosleep(128);
        }
        if (!got) *abort = 1;
    }
    return __shfl_sync(0xffffffffu, tile, 0);
}

// Owner rank of a tile: alternates along each CTA's tile sequence and across
// neighbouring CTAs, so every CTA reduces about 1/world of its tiles.
__device__ __forceinline__ uint32_t tileOwner(const Params& p, uint32_t tile) {
    return (tile % p.grid + tile / p.grid) % p.world;
}

// Announces this warp's 32 rows of `tile` to the tile's owner rank. All
// lanes' stores of the rows precede the announcement (warp barrier, then a
// system-scope fence and a release add by lane 0 on the owner's word).
__device__ __forceinline__ void announceRows(const Params& p, uint32_t tile, uint32_t quadrant, uint32_t lane) {
    __syncwarp();
    if (lane == 0) {
        uint32_t* word = p.flagsPeers[tileOwner(p, tile)] + tile * 4u + quadrant;
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(word), "r"(1u) : "memory");
    }
}

// Lane 0 polls this rank's signal word until every rank has announced
// (wrap-safe compare); false after the poll limit or once another warp of
// the CTA has aborted.
__device__ __forceinline__ bool awaitRows(const Params& p, uint32_t tile, uint32_t quadrant, uint32_t lane,
                                          const volatile int* abort) {
    uint32_t ok = 1;
    if (lane == 0) {
        ok = 0;
        const uint32_t* word = p.flagsPeers[p.rank] + tile * 4u + quadrant;
        for (uint64_t spin = 0; spin < kSignalSpinLimit && !*abort; ++spin) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(word) : "memory");
            if (static_cast<int32_t>(v - p.target) >= 0) {
                ok = 1;
                break;
            }
            __nanosleep(128);
        }
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __syncwarp();
    return ok != 0;
}

// The fused update of 4 parameters at element offset `at` (16-byte aligned)
// from their summed gradients g: reads this rank's parameters (and
// velocities), then writes the new parameters and their bf16 copy to every
// rank, through the switch (multimem.st) or by peer stores.
__device__ __forceinline__ void updateVector(const Params& p, uint64_t at, const float4& g, bool multicast) {
    float4 w = __ldcg(reinterpret_cast<const float4*>(p.pPeers[p.rank] + at));
    if (p.velocity) {
        float4 m = *reinterpret_cast<const float4*>(p.velocity + at);
        w.x = sgdStep(w.x, g.x, &m.x, p.lr, p.mu);
        w.y = sgdStep(w.y, g.y, &m.y, p.lr, p.mu);
        w.z = sgdStep(w.z, g.z, &m.z, p.lr, p.mu);
        w.w = sgdStep(w.w, g.w, &m.w, p.lr, p.mu);
        *reinterpret_cast<float4*>(p.velocity + at) = m;
    } else {
        w.x = sgdStep(w.x, g.x, nullptr, p.lr, p.mu);
        w.y = sgdStep(w.y, g.y, nullptr, p.lr, p.mu);
        w.z = sgdStep(w.z, g.z, nullptr, p.lr, p.mu);
        w.w = sgdStep(w.w, g.w, nullptr, p.lr, p.mu);
    }
    const __nv_bfloat162 lo = __floats2bfloat162_rn(w.x, w.y), hi = __floats2bfloat162_rn(w.z, w.w);
    const uint32_t loBits = *reinterpret_cast<const uint32_t*>(&lo), hiBits = *reinterpret_cast<const uint32_t*>(&hi);
    if (multicast) {
        asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p.pMc + at), "f"(w.x),
                     "f"(w.y), "f"(w.z), "f"(w.w)
                     : "memory");
        asm volatile("multimem.st.relaxed.sys.global.v2.bf16x2 [%0], {%1, %2};" ::"l"(p.pbMc + at), "r"(loBits),
                     "r"(hiBits)
                     : "memory");
    } else {
        for (uint32_t k = 0; k < p.world; ++k) {
            __stcg(reinterpret_cast<float4*>(p.pPeers[k] + at), w);
            __stcg(reinterpret_cast<uint2*>(p.pbPeers[k] + at), make_uint2(loBits, hiBits));
        }
    }
}

// The same for one parameter (ragged tile edges), always by peer stores.
__device__ __forceinline__ void updateScalar(const Params& p, uint64_t at, float g) {
    const float w = sgdStep(__ldcg(p.pPeers[p.rank] + at), g, p.velocity ? p.velocity + at : nullptr, p.lr, p.mu);
    const __nv_bfloat16 b = __float2bfloat16_rn(w);
    for (uint32_t k = 0; k < p.world; ++k) {
        __stcg(p.pPeers[k] + at, w);
        p.pbPeers[k][at] = b;
    }
}

// Switch mode, full-width rows: the switch sums 16-byte vectors over all
// ranks (multimem.ld_reduce) and writes the totals to all (multimem.st), or
// the owner applies the fused update. Lane takes vectors lane and lane + 32
// of 8 rows per round: 16 in flight.
__device__ __forceinline__ void switchReduceRows(const Params& p, uint64_t offset, uint32_t rows, uint32_t lane) {
    float* base = p.cMc + offset;
    const uint64_t ldc = p.ldc;
    for (uint32_t r0 = 0; r0 < rows; r0 += 8) {
        float4 v[16];
#pragma unroll
        for (uint32_t i = 0; i < 16; ++i) {
            const uint32_t r = r0 + i / 2;
            if (r < rows) {
                const float* src = base + r * ldc + 4u * (lane + 32u * (i % 2));
                asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                             : "=f"(v[i].x), "=f"(v[i].y), "=f"(v[i].z), "=f"(v[i].w)
                             : "l"(src)
                             : "memory");
            }
        }
#pragma unroll
        for (uint32_t i = 0; i < 16; ++i) {
            const uint32_t r = r0 + i / 2;
            if (r < rows) {
                const uint64_t at = r * ldc + 4u * (lane + 32u * (i % 2));
                if (p.fusedUpdate) {
                    updateVector(p, offset + at, v[i], true);
                } else {
                    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(base + at),
                                 "f"(v[i].x), "f"(v[i].y), "f"(v[i].z), "f"(v[i].w)
                                 : "memory");
                }
            }
        }
    }
}

// Peer mode, full-width rows: every rank's vectors are read over NVLink
// (L2-only loads), summed in rank order (so all ranks get the same bits) and
// stored to every rank. 8 vectors per lane per round.
__device__ __forceinline__ void peerReduceRows(const Params& p, uint64_t offset, uint32_t rows, uint32_t lane) {
    for (uint32_t r0 = 0; r0 < rows; r0 += 4) {
        float4 acc[8];
#pragma unroll
        for (uint32_t i = 0; i < 8; ++i) acc[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (uint32_t k = 0; k < p.world; ++k) {
            const float* src = p.cPeers[k] + offset;
            float4 w[8];
#pragma unroll
            for (uint32_t i = 0; i < 8; ++i) {
                const uint32_t r = r0 + i / 2;
                if (r < rows) w[i] = __ldcg(reinterpret_cast<const float4*>(src + r * p.ldc + 4u * (lane + 32u * (i % 2))));
            }
#pragma unroll
            for (uint32_t i = 0; i < 8; ++i) {
                acc[i].x = __fadd_rn(acc[i].x, w[i].x);
                acc[i].y = __fadd_rn(acc[i].y, w[i].y);
                acc[i].z = __fadd_rn(acc[i].z, w[i].z);
                acc[i].w = __fadd_rn(acc[i].w, w[i].w);
            }
        }
        if (p.fusedUpdate) {
#pragma unroll
            for (uint32_t i = 0; i < 8; ++i) {
                const uint32_t r = r0 + i / 2;
                if (r < rows) updateVector(p, offset + r * p.ldc + 4u * (lane + 32u * (i % 2)), acc[i], false);
            }
            continue;
        }
        for (uint32_t k = 0; k < p.world; ++k) {
            float* dst = p.cPeers[k] + offset;
#pragma unroll
            for (uint32_t i = 0; i < 8; ++i) {
                const uint32_t r = r0 + i / 2;
                if (r < rows) __stcg(reinterpret_cast<float4*>(dst + r * p.ldc + 4u * (lane + 32u * (i % 2))), acc[i]);
            }
        }
    }
}

// ---- compact form: bf16 payload, parameters sharded by tile owner ----

// bf16 pairs in a 32-bit word (element 0 in the low half). Widening to f32
// is exact: the bf16 bits are the f32's upper half.
__device__ __forceinline__ float2 unpackBf16x2(uint32_t bits) {
    return make_float2(__uint_as_float(bits << 16), __uint_as_float(bits & 0xffff0000u));
}

// Round-to-nearest-even of (a, b) to a bf16 pair, a in the low half.
__device__ __forceinline__ uint32_t packBf16x2(float a, float b) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
    return r;
}

// The compact update of 4 parameters at element offset `at` (16-byte
// aligned) from their summed gradients g: the owner's own f32 parameters (and
// velocities) are updated in place; returns their bf16 rounding, packed.
__device__ __forceinline__ uint2 updateCompact4(const Params& p, uint64_t at, float g0, float g1, float g2, float g3) {
    float* own = p.pPeers[p.rank] + at;
    float4 w = __ldcg(reinterpret_cast<const float4*>(own));
    if (p.velocity) {
        float4 m = *reinterpret_cast<const float4*>(p.velocity + at);
        w.x = sgdStep(w.x, g0, &m.x, p.lr, p.mu);
        w.y = sgdStep(w.y, g1, &m.y, p.lr, p.mu);
        w.z = sgdStep(w.z, g2, &m.z, p.lr, p.mu);
        w.w = sgdStep(w.w, g3, &m.w, p.lr, p.mu);
        *reinterpret_cast<float4*>(p.velocity + at) = m;
    } else {
        w.x = sgdStep(w.x, g0, nullptr, p.lr, p.mu);
        w.y = sgdStep(w.y, g1, nullptr, p.lr, p.mu);
        w.z = sgdStep(w.z, g2, nullptr, p.lr, p.mu);
        w.w = sgdStep(w.w, g3, nullptr, p.lr, p.mu);
    }
    *reinterpret_cast<float4*>(own) = w;
    return make_uint2(packBf16x2(w.x, w.y), packBf16x2(w.z, w.w));
}

// The compact update of 8 parameters at `at` (32-byte aligned in P, 16-byte
// in the bf16 copy), gradients as 4 packed bf16 pairs (the switch's sums) or
// as 8 floats: the owner's f32 parameters are updated, the bf16 copy is
// written to every rank.
__device__ __forceinline__ void storeCompactCopy(const Params& p, uint64_t at, const uint2& lo, const uint2& hi,
                                                 bool multicast) {
    if (multicast) {
        asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(p.pbMc + at), "r"(lo.x),
                     "r"(lo.y), "r"(hi.x), "r"(hi.y)
                     : "memory");
    } else {
        const uint4 b = make_uint4(lo.x, lo.y, hi.x, hi.y);
        for (uint32_t k = 0; k < p.world; ++k) __stcg(reinterpret_cast<uint4*>(p.pbPeers[k] + at), b);
    }
}

__device__ __forceinline__ void updateCompact8(const Params& p, uint64_t at, const uint4& sums) {
    float2 a = unpackBf16x2(sums.x), b = unpackBf16x2(sums.y);
    const uint2 lo = updateCompact4(p, at, a.x, a.y, b.x, b.y);
    a = unpackBf16x2(sums.z);
    b = unpackBf16x2(sums.w);
    const uint2 hi = updateCompact4(p, at + 4, a.x, a.y, b.x, b.y);
    storeCompactCopy(p, at, lo, hi, true);
}

__device__ __forceinline__ void updateCompact8(const Params& p, uint64_t at, const float (&g)[8]) {
    const uint2 lo = updateCompact4(p, at, g[0], g[1], g[2], g[3]);
    const uint2 hi = updateCompact4(p, at + 4, g[4], g[5], g[6], g[7]);
    storeCompactCopy(p, at, lo, hi, false);
}

// Full-width rows of an owned tile in compact form: lane takes the 8
// columns 8*lane .. 8*lane+7 of each row (one 16-byte bf16 vector per rank).
// Switch mode keeps kCompactSwitchRows sums in flight per lane and unpacks
// them one row at a time; peer mode sums kCompactPeerRows rows of every rank
// in f32, in rank order. (The row counts keep the reducer inside the
// kernel's register budget.)
constexpr uint32_t kCompactSwitchRows = 4;
constexpr uint32_t kCompactPeerRows = 1;

__device__ __forceinline__ void unpack8(const uint4& v, float (&g)[8]) {
    const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float2 f = unpackBf16x2(words[q]);
        g[2 * q] = f.x;
        g[2 * q + 1] = f.y;
    }
}

__device__ __forceinline__ void compactReduceRows(const Params& p, uint64_t offset, uint32_t rows, uint32_t lane) {
    if (p.cMc) {
        const __nv_bfloat16* mc = reinterpret_cast<const __nv_bfloat16*>(p.cMc) + offset + 8u * lane;
        // The owner's parameters (and velocities) of the rows are pulled into
        // L2 before the first sums return (8 ranks: 1.468 against 1.484 ms per
        // step).
        {
            const float* own = p.pPeers[p.rank] + offset + 8u * lane;
            for (uint32_t r = 0; r < rows; ++r) {
                asm volatile("prefetch.global.L2 [%0];" ::"l"(own + r * p.ldc));
                if (p.velocity) asm volatile("prefetch.global.L2 [%0];" ::"l"(p.velocity + offset + 8u * lane + r * p.ldc));
            }
        }
        for (uint32_t r0 = 0; r0 < rows; r0 += kCompactSwitchRows) {
            uint4 v[kCompactSwitchRows];
#pragma unroll
            for (uint32_t i = 0; i < kCompactSwitchRows; ++i) {
                if (r0 + i < rows)
                    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
                                 : "=r"(v[i].x), "=r"(v[i].y), "=r"(v[i].z), "=r"(v[i].w)
                                 : "l"(mc + (r0 + i) * p.ldc)
                                 : "memory");
            }
#pragma unroll
            for (uint32_t i = 0; i < kCompactSwitchRows; ++i)
                if (r0 + i < rows) updateCompact8(p, offset + (r0 + i) * p.ldc + 8u * lane, v[i]);
        }
        return;
    }
    for (uint32_t r0 = 0; r0 < rows; r0 += kCompactPeerRows) {
        float acc[kCompactPeerRows][8];
#pragma unroll
        for (uint32_t i = 0; i < kCompactPeerRows; ++i)
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[i][e] = 0.0f;
        for (uint32_t k = 0; k < p.world; ++k) {
            const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(p.cPeers[k]) + offset + 8u * lane;
            uint4 v[kCompactPeerRows];
#pragma unroll
            for (uint32_t i = 0; i < kCompactPeerRows; ++i)
                if (r0 + i < rows) v[i] = __ldcg(reinterpret_cast<const uint4*>(src + (r0 + i) * p.ldc));
#pragma unroll
            for (uint32_t i = 0; i < kCompactPeerRows; ++i) {
                float g[8];
                unpack8(v[i], g);
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[i][e] = __fadd_rn(acc[i][e], g[e]);
            }
        }
#pragma unroll
        for (uint32_t i = 0; i < kCompactPeerRows; ++i)
            if (r0 + i < rows) updateCompact8(p, offset + (r0 + i) * p.ldc + 8u * lane, acc[i]);
    }
}

// One element of a ragged tile edge in compact form: the ranks' bf16 values
// summed in f32 in rank order by peer loads, the owner's parameter updated,
// the bf16 copy stored to every rank.
__device__ __forceinline__ void compactReduceScalar(const Params& p, uint64_t at) {
    float x = 0.0f;
    for (uint32_t k = 0; k < p.world; ++k)
        x = __fadd_rn(x, __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.cPeers[k])[at]));
    float* own = p.pPeers[p.rank] + at;
    const float w = sgdStep(__ldcg(own), x, p.velocity ? p.velocity + at : nullptr, p.lr, p.mu);
    *own = w;
    const __nv_bfloat16 b = __float2bfloat16_rn(w);
    for (uint32_t k = 0; k < p.world; ++k) p.pbPeers[k][at] = b;
}

// Sums this warp's 32 rows of an owned tile over all ranks and writes the
// totals to every rank, once all ranks have announced them. Ragged edge
// tiles go element by element.
__device__ __forceinline__ bool reduceRows(const Params& p, uint32_t tile, uint32_t quadrant, uint32_t lane,
                                           const volatile int* abort) {
    if (!awaitRows(p, tile, quadrant, lane, abort)) return false;
    uint32_t mb, nb;
    tileCoords(tile, p, mb, nb);
    const uint64_t row0 = static_cast<uint64_t>(mb) * kBM + quadrant * 32u;
    const uint64_t col0 = static_cast<uint64_t>(nb) * kBN;
    if (row0 >= p.m) return true;
    const uint32_t rows = p.m - row0 < 32 ? static_cast<uint32_t>(p.m - row0) : 32u;
    const uint32_t cols = p.n - col0 < kBN ? static_cast<uint32_t>(p.n - col0) : kBN;
    const uint64_t offset = row0 * p.ldc + col0;
    if (p.compact) {
        if (cols == kBN) {
            compactReduceRows(p, offset, rows, lane);
        } else {
            for (uint32_t r = 0; r < rows; ++r)
                for (uint32_t c = lane; c < cols; c += 32) compactReduceScalar(p, offset + r * p.ldc + c);
        }
        return true;
    }
    if (cols == kBN) {
        if (p.cMc) switchReduceRows(p, offset, rows, lane);
        else peerReduceRows(p, offset, rows, lane);
        return true;
    }
    for (uint32_t r = 0; r < rows; ++r)
        for (uint32_t c = lane; c < cols; c += 32) {
            const uint64_t at = offset + r * p.ldc + c;
            if (p.cMc) {
                float x;
                asm volatile("multimem.ld_reduce.relaxed.sys.global.add.f32 %0, [%1];" : "=f"(x) : "l"(p.cMc + at) : "memory");
                if (p.fusedUpdate) updateScalar(p, at, x);
                else asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(p.cMc + at), "f"(x) : "memory");
            } else {
                float x = 0.0f;
                for (uint32_t k = 0; k < p.world; ++k) x = __fadd_rn(x, __ldcg(p.cPeers[k] + at));
                if (p.fusedUpdate) {
                    updateScalar(p, at, x);
                    continue;
                }
                for (uint32_t k = 0; k < p.world; ++k) __stcg(p.cPeers[k] + at, x);
            }
        }
    return true;
}

// PAIR: launched as clusters of two CTAs. Rank 0 (the leader) issues the
// MMAs of the 256-row tile for both; each CTA stages its own halves, its
// epilogue reads its own 128 TMEM lanes (rows), and both epilogues release an
// accumulator on the leader's tmemEmpty barrier.
template <bool A_MN, bool B_MN, int EPI, bool PAIR>
__global__ void __launch_bounds__(threadsFor(EPI), 1)
    gemmKernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB, const Params p) {
    using G = Geometry<PAIR>;
    extern __shared__ uint8_t dynamicSmem[];
    __shared__ __align__(8) uint64_t full[G::stages], empty[G::stages], tmemFull[2], tmemEmpty[2], mmaDone;
    __shared__ uint32_t tmemSlot;
    __shared__ volatile int abortFlag;
    __shared__ TileQueue queues[4];  // kEpiAllReduceF32: one per TMEM quadrant

    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dynamicSmem) + 1023) & ~uintptr_t(1023));
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t tiles = p.mTiles * p.nTiles;
    const uint32_t rank = PAIR ? clusterRank() : 0u;
    // Tile schedule: pairs (clusters) or single CTAs take tiles g, g + n, ...
    const uint32_t first = PAIR ? blockIdx.x / 2 : blockIdx.x;
    const uint32_t step = PAIR ? gridDim.x / 2 : gridDim.x;

    if (threadIdx.x == 0) {
        abortFlag = 0;
        for (auto& q : queues) q.head = q.tail = 0;
        for (int s = 0; s < G::stages; ++s) {
            mbarInit(&full[s], 1);
            mbarInit(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbarInit(&tmemFull[a], 1);
            mbarInit(&tmemEmpty[a], (PAIR ? 2 : 1) * 32 * epilogueWarps(EPI));
        }
        mbarInit(&mmaDone, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        if constexpr (PAIR) {
            // Collective over the pair: the same columns in both CTAs.
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem(&tmemSlot)),
                         "r"(kTmemCols)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem(&tmemSlot)),
                         "r"(kTmemCols)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        }
    }
    fenceBefore();
    __syncthreads();
    // The peer's barriers are initialised before any remote arrival or load.
    if constexpr (PAIR) clusterSync();
    fenceAfter();
    const uint32_t tmemBase = tmemSlot;

    if (warp == 0 && lane == 0) {
        // ---- TMA producer ----
        uint32_t stage = 0, phase = 0;
        uint32_t issuedParity[G::stages];
        uint32_t issued = 0;  // bitmask of stages with a load issued
        for (uint32_t tile = first; tile < tiles && !abortFlag; tile += step) {
            uint32_t mb, nb;
            tileCoords(tile, p, mb, nb);
            // This CTA's rows of A and columns of B.
            const int32_t row0 = static_cast<int32_t>(mb * G::tileM + rank * kBM);
            const int32_t col0 = static_cast<int32_t>(nb * kBN + rank * G::bRows);
            for (uint32_t kb = 0; kb < p.kBlocks; ++kb) {
                if (!mbarWait(&empty[stage], phase ^ 1u, &abortFlag)) { abortFlag = 1; break; }
                uint8_t* a = base + stage * G::stageBytes;
                uint8_t* b = a + kABytes;
                const int32_t k0 = static_cast<int32_t>(kb * kBK);
                if constexpr (PAIR) {
                    // Both CTAs' loads complete on the leader's barrier, which
                    // expects the bytes of the whole pair.
                    if (rank == 0) mbarExpect(&full[stage], 2 * G::stageBytes);
                    const uint32_t bar = pairAddress(&full[stage], 0);
                    if constexpr (A_MN) {
                        tmaLoad2dPair(a, &mapA, row0, k0, bar);
                        tmaLoad2dPair(a + kABytes / 2, &mapA, row0 + 64, k0, bar);
                    } else {
                        tmaLoad2dPair(a, &mapA, k0, row0, bar);
                    }
                    if constexpr (B_MN) {
#pragma unroll
                        for (int j = 0; j < static_cast<int>(G::bRows / 64); ++j)
                            tmaLoad2dPair(b + j * (G::bBytes / (G::bRows / 64)), &mapB, col0 + 64 * j, k0, bar);
                    } else {
                        tmaLoad2dPair(b, &mapB, k0, col0, bar);
                    }
                } else {
                    mbarExpect(&full[stage], G::stageBytes);
                    if constexpr (A_MN) {
                        tmaLoad2d(a, &mapA, row0, k0, &full[stage]);
                        tmaLoad2d(a + kABytes / 2, &mapA, row0 + 64, k0, &full[stage]);
                    } else {
                        tmaLoad2d(a, &mapA, k0, row0, &full[stage]);
                    }
                    if constexpr (B_MN) {
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            tmaLoad2d(b + j * (G::bBytes / 4), &mapB, col0 + 64 * j, k0, &full[stage]);
                    } else {
                        tmaLoad2d(b, &mapB, k0, col0, &full[stage]);
                    }
                }
                issuedParity[stage] = phase;
                issued |= 1u << stage;
                if (++stage == G::stages) { stage = 0; phase ^= 1u; }
            }
        }
        if (abortFlag) {
            // Let loads already issued land before the CTA can exit. A pair
            // counts them on the leader's barriers, which only the leader can
            // wait on; the peer gives its loads a fixed 200 us instead.
            if (!PAIR || rank == 0) {
                for (int s = 0; s < G::stages; ++s)
                    if (issued & (1u << s)) (void)mbarWait(&full[s], issuedParity[s]);
            } else {
                for (int k = 0; k < 2000; ++k) __nanosleep(100);
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer ----
        // (PAIR: the leader only; its MMAs read both CTAs' stages and write
        // both CTAs' TMEM, and its commits arrive in both CTAs.)
        if (!PAIR || rank == 0) {
            constexpr uint32_t idesc = instrDesc<A_MN, B_MN, PAIR>();
            constexpr uint32_t bAtom = G::bBytes / (G::bRows / 64);  // MN-major B: 64-column atoms
            auto commit = [](uint64_t* bar) {
                if constexpr (PAIR) mmaCommitPair(bar);
                else mmaCommit(bar);
            };
            uint32_t stage = 0, phase = 0, acc = 0, accPhase = 0;
            for (uint32_t tile = first; tile < tiles && !abortFlag; tile += step) {
                if (!mbarWait(&tmemEmpty[acc], accPhase ^ 1u, &abortFlag)) { abortFlag = 1; break; }
                fenceAfter();
                const uint32_t d = tmemBase + acc * kBN;
                bool ok = true;
                for (uint32_t kb = 0; kb < p.kBlocks; ++kb) {
                    if (!mbarWait(&full[stage], phase, &abortFlag)) { abortFlag = 1; ok = false; break; }
                    fenceAfter();
                    const uint32_t a = smem(base + stage * G::stageBytes);
                    const uint32_t b = a + kABytes;
#pragma unroll
                    for (uint32_t ks = 0; ks < kBK / 16; ++ks) {
                        const uint64_t da =
                            A_MN ? ummaDesc(a + ks * 2048u, kABytes / 2, 1024u) : ummaDesc(a + ks * 32u, 16u, 1024u);
                        const uint64_t db = B_MN ? ummaDesc(b + ks * 2048u, bAtom, 1024u) : ummaDesc(b + ks * 32u, 16u, 1024u);
                        if constexpr (PAIR) mmaPair(d, da, db, idesc, (kb | ks) != 0 ? 1u : 0u);
                        else mma(d, da, db, idesc, (kb | ks) != 0 ? 1u : 0u);
                    }
                    commit(&empty[stage]);
                    if (++stage == G::stages) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                commit(&tmemFull[acc]);
                if (++acc == 2) { acc = 0; accPhase ^= 1u; }
            }
            // All MMAs issued by this thread complete before TMEM is released.
            commit(&mmaDone);
            if (!mbarWait(&mmaDone, 0)) abortFlag = 1;
        }
    } else if (warp >= 2 && warp < 2 + epilogueWarps(EPI)) {
        // ---- epilogue ----
        const uint32_t quadrant = warp % 4;  // TMEM lanes 32*quadrant .. +31
        // With 8 epilogue warps the two warps of a quadrant split the tile's
        // 32-column chunks.
        constexpr uint32_t kChunks = kBN / 32, kChunksPerWarp = kChunks * 4 / epilogueWarps(EPI);
        const uint32_t firstChunk = (warp - 2) / 4 * kChunksPerWarp;
        const uint32_t row = quadrant * 32 + lane;
        uint32_t acc = 0, accPhase = 0;
        TileQueue& queue = queues[quadrant];
        (void)queue;
        // This CTA's 128-row block (its TMEM holds those rows of the tile).
        const uint32_t blocksPerTile = G::tileM / kBM;
        const uint32_t releaseAddress = PAIR ? pairAddress(&tmemEmpty[0], 0) : 0u;
        for (uint32_t tile = first; tile < tiles; tile += step) {
            uint32_t mb, nb;
            tileCoords(tile, p, mb, nb);
            const uint32_t rowBlock = mb * blocksPerTile + rank;
            const uint64_t grow = static_cast<uint64_t>(rowBlock) * kBM + row;
            // A pair's second row block can lie wholly past M (no rows, and
            // no column-sum rows either).
            const uint32_t lastChunk = static_cast<uint64_t>(rowBlock) * kBM < p.m ? firstChunk + kChunksPerWarp : 0u;
            // Optimizer-step read-out over whole, aligned tiles: the
            // parameters of a chunk are loaded one chunk ahead, the first
            // chunk's before the accumulator is ready, so their latency
            // overlaps the MMAs and the previous chunk's work.
            bool fastUpdate = false;
            float4 pc[8];
            if constexpr (EPI == kEpiSgdF32) {
                const uint64_t colBase = static_cast<uint64_t>(nb) * kBN;
                fastUpdate = colBase + kBN <= p.n && p.ldc % 4 == 0 &&
                             ((reinterpret_cast<uintptr_t>(p.c) | reinterpret_cast<uintptr_t>(p.velocity)) % 16) == 0 &&
                             reinterpret_cast<uintptr_t>(p.copy) % 8 == 0;
                if (fastUpdate && grow < p.m && firstChunk < lastChunk) {
                    const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(p.c) + grow * p.ldc +
                                                                        colBase + firstChunk * 32u);
#pragma unroll
                    for (int q = 0; q < 8; ++q) pc[q] = src[q];
                }
            }
            if (!mbarWait(&tmemFull[acc], accPhase, &abortFlag)) abortFlag = 1;
            if (abortFlag) break;
            fenceAfter();
            if constexpr (EPI == kEpiSgdF32) {
                if (fastUpdate) {
                    const bool rowValid = grow < p.m;
                    const uint64_t rowOffset = grow * p.ldc + static_cast<uint64_t>(nb) * kBN;
#pragma unroll 1
                    for (uint32_t chunk = firstChunk; chunk < lastChunk; ++chunk) {
                        uint32_t r[32];
                        tmemLoad32(tmemBase + ((quadrant * 32u) << 16) + acc * kBN + chunk * 32u, r);
                        const uint64_t off = rowOffset + chunk * 32u;
                        float4 pn[8];
                        const bool more = chunk + 1 < lastChunk;
                        if (rowValid && more) {
                            const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(p.c) + off + 32u);
#pragma unroll
                            for (int q = 0; q < 8; ++q) pn[q] = src[q];
                        }
                        if (rowValid) {
                            float* dst = static_cast<float*>(p.c) + off;
                            float* vel = p.velocity ? p.velocity + off : nullptr;
                            __nv_bfloat16* cp = p.copy ? p.copy + off : nullptr;
#pragma unroll
                            for (int q = 0; q < 8; ++q) {
                                float4 w = pc[q];
                                const float g0 = __uint_as_float(r[4 * q]), g1 = __uint_as_float(r[4 * q + 1]);
                                const float g2 = __uint_as_float(r[4 * q + 2]), g3 = __uint_as_float(r[4 * q + 3]);
                                if (vel) {
                                    float4 m = *reinterpret_cast<const float4*>(vel + 4 * q);
                                    w.x = sgdStep(w.x, g0, &m.x, p.lr, p.mu);
                                    w.y = sgdStep(w.y, g1, &m.y, p.lr, p.mu);
                                    w.z = sgdStep(w.z, g2, &m.z, p.lr, p.mu);
                                    w.w = sgdStep(w.w, g3, &m.w, p.lr, p.mu);
                                    *reinterpret_cast<float4*>(vel + 4 * q) = m;
                                } else {
                                    w.x = sgdStep(w.x, g0, nullptr, p.lr, p.mu);
                                    w.y = sgdStep(w.y, g1, nullptr, p.lr, p.mu);
                                    w.z = sgdStep(w.z, g2, nullptr, p.lr, p.mu);
                                    w.w = sgdStep(w.w, g3, nullptr, p.lr, p.mu);
                                }
                                *reinterpret_cast<float4*>(dst + 4 * q) = w;
                                if (cp) {
                                    const __nv_bfloat162 lo = __floats2bfloat162_rn(w.x, w.y);
                                    const __nv_bfloat162 hi = __floats2bfloat162_rn(w.z, w.w);
                                    uint2 packed;
                                    packed.x = *reinterpret_cast<const uint32_t*>(&lo);
                                    packed.y = *reinterpret_cast<const uint32_t*>(&hi);
                                    *reinterpret_cast<uint2*>(cp + 4 * q) = packed;
                                }
                            }
                        }
                        if (more) {
#pragma unroll
                            for (int q = 0; q < 8; ++q) pc[q] = pn[q];
                        }
                    }
                }
            }
#pragma unroll 1
            for (uint32_t chunk = firstChunk; chunk < (fastUpdate ? firstChunk : lastChunk); ++chunk) {
                uint32_t r[32];
                tmemLoad32(tmemBase + ((quadrant * 32u) << 16) + acc * kBN + chunk * 32u, r);
                const uint64_t col0 = static_cast<uint64_t>(nb) * kBN + chunk * 32u;
                const bool rowValid = grow < p.m;
                // Column sums need every lane of the warp (rows past M add 0).
                const bool sums = EPI == kEpiMaskBf16 && p.colSums != nullptr;
                if (col0 >= p.n || (!rowValid && !sums)) continue;
                const bool full32 = col0 + 32 <= p.n;
                float aux[32];
                if constexpr (EPI == kEpiMaskBf16) {
                    const __nv_bfloat16* src = p.aux + grow * p.ldAux + col0;
                    if (!rowValid) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) aux[j] = 0.0f;
                    } else if (full32 && (reinterpret_cast<uintptr_t>(src) % 16 == 0)) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const uint4 v = *reinterpret_cast<const uint4*>(src + q * 8);
                            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float2 f = __bfloat1622float2(h[e]);
                                aux[q * 8 + 2 * e] = f.x;
                                aux[q * 8 + 2 * e + 1] = f.y;
                            }
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) aux[j] = col0 + j < p.n ? __bfloat162float(src[j]) : 0.0f;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) aux[j] = 0.0f;
                }
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
                if (p.bias) {
                    const float* bsrc = p.bias + col0;
                    if (full32 && reinterpret_cast<uintptr_t>(bsrc) % 16 == 0) {
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            const float4 bv = __ldg(reinterpret_cast<const float4*>(bsrc) + q);
                            v[4 * q] = __fadd_rn(v[4 * q], bv.x);
                            v[4 * q + 1] = __fadd_rn(v[4 * q + 1], bv.y);
                            v[4 * q + 2] = __fadd_rn(v[4 * q + 2], bv.z);
                            v[4 * q + 3] = __fadd_rn(v[4 * q + 3], bv.w);
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (col0 + j < p.n) v[j] = __fadd_rn(v[j], __ldg(bsrc + j));
                    }
                }
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = epilogueValue<EPI>(v[j], aux[j]);
                if constexpr (EPI == kEpiMaskBf16) {
                    if (sums) {
                        float s[32];
#pragma unroll
                        for (int j = 0; j < 32; ++j) s[j] = rowValid ? v[j] : 0.0f;
                        const float total = columnSum32(s, lane);
                        if (col0 + lane < p.n)
                            p.colSums[(static_cast<uint64_t>(rowBlock) * 4 + quadrant) * p.n + col0 + lane] = total;
                        if (!rowValid) continue;
                    }
                }
                if constexpr (EPI == kEpiSgdF32) {
                    // v[] is the gradient; C holds the parameters.
                    float* dst = static_cast<float*>(p.c) + grow * p.ldc + col0;
                    float* vel = p.velocity ? p.velocity + grow * p.ldc + col0 : nullptr;
                    __nv_bfloat16* cp = p.copy ? p.copy + grow * p.ldc + col0 : nullptr;
                    const uintptr_t bits = reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(vel) |
                                           reinterpret_cast<uintptr_t>(cp);
                    if (full32 && bits % 16 == 0) {
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            float4 w = *reinterpret_cast<const float4*>(dst + 4 * q);
                            if (vel) {
                                float4 m = *reinterpret_cast<const float4*>(vel + 4 * q);
                                w.x = sgdStep(w.x, v[4 * q], &m.x, p.lr, p.mu);
                                w.y = sgdStep(w.y, v[4 * q + 1], &m.y, p.lr, p.mu);
                                w.z = sgdStep(w.z, v[4 * q + 2], &m.z, p.lr, p.mu);
                                w.w = sgdStep(w.w, v[4 * q + 3], &m.w, p.lr, p.mu);
                                *reinterpret_cast<float4*>(vel + 4 * q) = m;
                            } else {
                                w.x = sgdStep(w.x, v[4 * q], nullptr, p.lr, p.mu);
                                w.y = sgdStep(w.y, v[4 * q + 1], nullptr, p.lr, p.mu);
                                w.z = sgdStep(w.z, v[4 * q + 2], nullptr, p.lr, p.mu);
                                w.w = sgdStep(w.w, v[4 * q + 3], nullptr, p.lr, p.mu);
                            }
                            *reinterpret_cast<float4*>(dst + 4 * q) = w;
                            if (cp) {
                                const __nv_bfloat162 lo = __floats2bfloat162_rn(w.x, w.y);
                                const __nv_bfloat162 hi = __floats2bfloat162_rn(w.z, w.w);
                                uint2 packed;
                                packed.x = *reinterpret_cast<const uint32_t*>(&lo);
                                packed.y = *reinterpret_cast<const uint32_t*>(&hi);
                                *reinterpret_cast<uint2*>(cp + 4 * q) = packed;
                            }
                        }
                    } else {
                        for (int j = 0; j < 32; ++j) {
                            if (col0 + j >= p.n) break;
                            const float w = sgdStep(dst[j], v[j], vel ? vel + j : nullptr, p.lr, p.mu);
                            dst[j] = w;
                            if (cp) cp[j] = __float2bfloat16_rn(w);
                        }
                    }
                } else if constexpr (EPI == kEpiF32 || EPI == kEpiAllReduceF32) {
                    if (EPI == kEpiAllReduceF32 && p.compact) {
                        // Compact all-reduce: the rank's tile travels as bf16.
                        storeBf16x32(static_cast<__nv_bfloat16*>(p.c) + grow * p.ldc + col0, v, full32, p.n - col0);
                    } else {
                        float* dst = static_cast<float*>(p.c) + grow * p.ldc + col0;
                        if (full32 && reinterpret_cast<uintptr_t>(dst) % 16 == 0) {
#pragma unroll
                            for (int q = 0; q < 8; ++q)
                                *reinterpret_cast<float4*>(dst + 4 * q) =
                                    make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                        } else {
                            for (int j = 0; j < 32; ++j)
                                if (col0 + j < p.n) dst[j] = v[j];
                        }
                    }
                } else {
                    storeBf16x32(static_cast<__nv_bfloat16*>(p.c) + grow * p.ldc + col0, v, full32, p.n - col0);
                    if (p.c2) {
                        float* dst2 = static_cast<float*>(p.c2) + grow * p.ldc + col0;
                        for (int j = 0; j < 32; ++j)
                            if (col0 + j < p.n) dst2[j] = v[j];
                    }
                }
            }
            fenceBefore();
            // The accumulator is free once both CTAs of a pair have read it;
            // the leader's barrier counts the epilogue threads of both.
            if (PAIR && rank != 0) mbarArriveCluster(releaseAddress + acc * static_cast<uint32_t>(sizeof(uint64_t)));
            else mbarArrive(&tmemEmpty[acc]);
            if (++acc == 2) { acc = 0; accPhase ^= 1u; }
            if constexpr (EPI == kEpiAllReduceF32) {
                // Announce this tile; owned tiles go to this quadrant's reducer warp.
                announceRows(p, tile, quadrant, lane);
                if (tileOwner(p, tile) == p.rank && !pushTile(queue, tile, lane, &abortFlag)) abortFlag = 1;
                if (abortFlag) break;
            }
        }
        if constexpr (EPI == kEpiAllReduceF32) (void)pushTile(queue, kNoTile, lane, &abortFlag);
    } else if (EPI == kEpiAllReduceF32 && warp >= 2 + epilogueWarps(EPI)) {
        // ---- reducers: owned tiles, summed over ranks in the switch ----
        const uint32_t quadrant = warp % 4;
        TileQueue& queue = queues[quadrant];
        for (;;) {
            const uint32_t tile = popTile(queue, lane, &abortFlag);
            if (tile == kNoTile) break;
            if (!reduceRows(p, tile, quadrant, lane, &abortFlag)) {
                abortFlag = 1;
                break;
            }
        }
        asm volatile("fence.acq_rel.sys;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0 && abortFlag) atomicOr(p.status, kWaitStatus);
    // A pair stays resident until both CTAs are done: the leader's MMAs read
    // the peer's shared memory and the peer arrives on the leader's barriers.
    if constexpr (PAIR) clusterSync();
    if (warp == 1) {
        fenceAfter();
        if constexpr (PAIR)
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmemBase), "r"(kTmemCols) : "memory");
        else
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmemBase), "r"(kTmemCols) : "memory");
    }
}

// m-blocks per raster group (THB_GEMM_GROUP overrides the default 16).
uint32_t rasterGroup() {
    static const uint32_t group = [] {
        const char* e = std::getenv("THB_GEMM_GROUP");
        const long g = e ? std::atol(e) : 0;
        return static_cast<uint32_t>(g > 0 && g <= 1024 ? g : 16);
    }();
    return group;
}

PFN_cuTensorMapEncodeTiled_v12000 encodeFn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D bf16 tensor map over a row-major [outer][inner] matrix with leading
// dimension `ld` elements; box = 64 inner elements (one 128 B swizzle row)
// by `boxOuter` rows.
bool makeMap(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t boxOuter) {
    auto fn = encodeFn();
    if (!fn) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {64, boxOuter};
    cuuint32_t elem[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, elem,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// p.grid CTAs; a pair kernel is launched as clusters of two (p.grid even).
template <bool A_MN, bool B_MN, int EPI, bool PAIR>
cudaError_t launchTyped(const CUtensorMap& a, const CUtensorMap& b, const Params& p, cudaStream_t stream) {
    auto kernel = gemmKernel<A_MN, B_MN, EPI, PAIR>;
    constexpr uint32_t smemBytes = Geometry<PAIR>::smemBytes;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smemBytes);
    if (e != cudaSuccess) return e;
    if constexpr (!PAIR) {
        kernel<<<p.grid, threadsFor(EPI), smemBytes, stream>>>(a, b, p);
        return cudaGetLastError();
    } else {
        cudaLaunchConfig_t config{};
        config.gridDim = dim3(p.grid);
        config.blockDim = dim3(threadsFor(EPI));
        config.dynamicSmemBytes = smemBytes;
        config.stream = stream;
        cudaLaunchAttribute attribute{};
        attribute.id = cudaLaunchAttributeClusterDimension;
        attribute.val.clusterDim.x = 2;
        attribute.val.clusterDim.y = 1;
        attribute.val.clusterDim.z = 1;
        config.attrs = &attribute;
        config.numAttrs = 1;
        // Persistent pairs: no more clusters than can be resident at once
        // (SMs left over by the GPC layout cannot host a pair).
        static int resident = -1;
        if (resident < 0) {
            int clusters = 0;
            resident = cudaOccupancyMaxActiveClusters(&clusters, kernel, &config) == cudaSuccess ? clusters : 0;
            (void)cudaGetLastError();
        }
        if (resident > 0 && p.grid > 2u * static_cast<uint32_t>(resident)) config.gridDim = dim3(2u * resident);
        return cudaLaunchKernelEx(&config, kernel, a, b, p);
    }
}

template <bool A_MN, bool B_MN>
cudaError_t launchEpi(int epi, bool pair, const CUtensorMap& a, const CUtensorMap& b, const Params& p, cudaStream_t s) {
    if (pair) {
        switch (epi) {
        case kEpiF32: return launchTyped<A_MN, B_MN, kEpiF32, true>(a, b, p, s);
        case kEpiBf16: return launchTyped<A_MN, B_MN, kEpiBf16, true>(a, b, p, s);
        case kEpiReluBf16: return launchTyped<A_MN, B_MN, kEpiReluBf16, true>(a, b, p, s);
        case kEpiMaskBf16: return launchTyped<A_MN, B_MN, kEpiMaskBf16, true>(a, b, p, s);
        case kEpiSgdF32: return launchTyped<A_MN, B_MN, kEpiSgdF32, true>(a, b, p, s);
        }
        return cudaErrorInvalidValue;
    }
    switch (epi) {
    case kEpiF32: return launchTyped<A_MN, B_MN, kEpiF32, false>(a, b, p, s);
    case kEpiBf16: return launchTyped<A_MN, B_MN, kEpiBf16, false>(a, b, p, s);
    case kEpiReluBf16: return launchTyped<A_MN, B_MN, kEpiReluBf16, false>(a, b, p, s);
    case kEpiMaskBf16: return launchTyped<A_MN, B_MN, kEpiMaskBf16, false>(a, b, p, s);
    case kEpiSgdF32: return launchTyped<A_MN, B_MN, kEpiSgdF32, false>(a, b, p, s);
    case kEpiAllReduceF32: return launchTyped<A_MN, B_MN, kEpiAllReduceF32, false>(a, b, p, s);
    }
    return cudaErrorInvalidValue;
}

// CTA pairs for every epilogue but the cross-GPU all-reduce (whose signal
// words are per 128-row tile), once M spans two row blocks and there are at
// least as many pair tiles as pairs of SMs would want work. THB_GEMM_PAIR=0
// keeps single CTAs.
bool usePairs(const Problem& q) {
    static const bool enabled = [] {
        const char* e = std::getenv("THB_GEMM_PAIR");
        return !(e && e[0] == '0');
    }();
    return enabled && q.epilogue != kEpiAllReduceF32 && q.m > static_cast<uint64_t>(kBM);
}

} // namespace

const char* validate(const Problem& q) {
    if (q.m == 0 || q.n == 0 || q.k == 0) return "GEMM extents must be positive";
    if (q.m > (1u << 30) || q.n > (1u << 30) || q.k > (1u << 30)) return "GEMM extent too large";
    if (!q.a || !q.b || !q.c) return "GEMM operand pointer is null";
    if (q.lda % 8 || q.ldb % 8) return "operand leading dimensions must be multiples of 8 elements (16 bytes)";
    if ((reinterpret_cast<uintptr_t>(q.a) | reinterpret_cast<uintptr_t>(q.b)) % 16) return "operands must be 16-byte aligned";
    if (q.lda < (q.aMajorMN ? q.m : q.k) || q.ldb < (q.bMajorMN ? q.n : q.k)) return "leading dimension too small";
    if (q.ldc < q.n) return "ldc smaller than N";
    if (q.epilogue == kEpiMaskBf16 && (!q.aux || q.ldAux < q.n)) return "mask epilogue needs an auxiliary bf16 matrix";
    if (q.epilogue < kEpiF32 || q.epilogue > kEpiSgdF32) return "unknown epilogue";
    if (q.epilogue == kEpiSgdF32) {
        const Update& u = q.update;
        if (!(u.momentum >= 0.0f && u.momentum < 1.0f)) return "the fused update needs momentum in [0, 1)";
        if (u.momentum > 0.0f && !u.velocity) return "momentum needs the velocity buffer";
    }
    if (q.bias && (q.epilogue == kEpiMaskBf16 || q.epilogue == kEpiAllReduceF32))
        return "a bias applies to the f32, bf16 and ReLU epilogues only";
    if (q.colSums && q.epilogue != kEpiMaskBf16) return "column sums are produced by the mask epilogue only";
    if (q.epilogue == kEpiAllReduceF32) {
        const AllReduce& r = q.reduce;
        if (r.world == 0 || r.world > static_cast<uint32_t>(kMaxRanks) || r.rank >= r.world)
            return "the all-reduce needs 1..8 ranks and a rank inside the world";
        if ((reinterpret_cast<uintptr_t>(q.c) | reinterpret_cast<uintptr_t>(r.cMulticast)) % 16 || q.ldc % 4)
            return "the all-reduce target must be 16-byte aligned with ldc a multiple of 4";
        if (r.cPeers[r.rank] != q.c) return "the all-reduce's own peer entry must be C";
        for (uint32_t k = 0; k < r.world; ++k) {
            if (!r.cPeers[k] || !r.flagsPeers[k]) return "the all-reduce needs every rank's C and signal words";
            if (reinterpret_cast<uintptr_t>(r.cPeers[k]) % 16 || reinterpret_cast<uintptr_t>(r.flagsPeers[k]) % 4)
                return "peer C must be 16-byte and signal words 4-byte aligned";
        }
        const ReduceUpdate& u = r.update;
        if (u.enabled) {
            if (!(u.momentum >= 0.0f && u.momentum < 1.0f)) return "the fused update needs momentum in [0, 1)";
            if (u.momentum > 0.0f && (!u.velocity || reinterpret_cast<uintptr_t>(u.velocity) % 16))
                return "momentum needs a 16-byte aligned velocity buffer";
            for (uint32_t k = 0; k < r.world; ++k)
                if (!u.paramPeers[k] || !u.copyPeers[k] || reinterpret_cast<uintptr_t>(u.paramPeers[k]) % 16 ||
                    reinterpret_cast<uintptr_t>(u.copyPeers[k]) % 8)
                    return "the fused update needs every rank's parameters (16-byte aligned) and bf16 copy (8-byte)";
            if (!r.cMulticast != !u.paramMulticast || !u.paramMulticast != !u.copyMulticast)
                return "switch mode needs multicast addresses of C, the parameters and their copy";
            if ((reinterpret_cast<uintptr_t>(u.paramMulticast) % 16) || (reinterpret_cast<uintptr_t>(u.copyMulticast) % 8))
                return "multicast parameters must be 16-byte and their copy 8-byte aligned";
        }
        if (r.compact) {
            if (!u.enabled) return "the compact all-reduce applies the update in the reduction";
            if (q.ldc % 8) return "the compact all-reduce needs ldc a multiple of 8 (16-byte bf16 rows)";
            for (uint32_t k = 0; k < r.world; ++k)
                if (reinterpret_cast<uintptr_t>(u.copyPeers[k]) % 16)
                    return "the compact all-reduce needs 16-byte aligned bf16 copies";
            if (reinterpret_cast<uintptr_t>(u.copyMulticast) % 16)
                return "the compact all-reduce needs a 16-byte aligned multicast copy";
        }
    }
    return nullptr;
}

std::uint64_t tileCount(std::uint64_t m, std::uint64_t n) { return ((m + kBM - 1) / kBM) * ((n + kBN - 1) / kBN); }

std::uint64_t colSumRows(std::uint64_t m) { return 4 * ((m + kBM - 1) / kBM); }

cudaError_t run(const Problem& q, int smCount, uint32_t* status, cudaStream_t stream) {
    const bool pair = usePairs(q) && smCount >= 2;
    const uint32_t tileM = pair ? Geometry<true>::tileM : Geometry<false>::tileM;
    const uint32_t bRows = pair ? Geometry<true>::bRows : Geometry<false>::bRows;
    CUtensorMap a, b;
    const bool okA = q.aMajorMN ? makeMap(&a, q.a, q.m, q.k, q.lda, 64) : makeMap(&a, q.a, q.k, q.m, q.lda, kBM);
    const bool okB = q.bMajorMN ? makeMap(&b, q.b, q.n, q.k, q.ldb, 64) : makeMap(&b, q.b, q.k, q.n, q.ldb, bRows);
    if (!okA || !okB) return cudaErrorInvalidValue;
    Params p{};
    p.m = static_cast<uint32_t>(q.m);
    p.n = static_cast<uint32_t>(q.n);
    p.k = static_cast<uint32_t>(q.k);
    p.mTiles = static_cast<uint32_t>((q.m + tileM - 1) / tileM);
    p.nTiles = static_cast<uint32_t>((q.n + kBN - 1) / kBN);
    p.kBlocks = static_cast<uint32_t>((q.k + kBK - 1) / kBK);
    // 16 m-blocks per group: on the MLP step it cut the DRAM reads of the
    // two GEMMs with N=16384 by a third against 8 (H = X W1: 614 -> 399 MB
    // per launch), and the step measured best of 2, 4, 8, 16 and 32.
    // THB_GEMM_GROUP overrides.
    p.group = rasterGroup();
    p.c = q.c;
    p.ldc = q.ldc;
    p.aux = static_cast<const __nv_bfloat16*>(q.aux);
    p.ldAux = q.ldAux;
    p.c2 = q.c2;
    p.status = status;
    const uint32_t tiles = p.mTiles * p.nTiles;
    const uint32_t slots = pair ? static_cast<uint32_t>(smCount) / 2 : static_cast<uint32_t>(smCount);
    p.grid = (tiles < slots ? tiles : slots) * (pair ? 2u : 1u);
    p.cMc = static_cast<float*>(q.reduce.cMulticast);
    for (int r = 0; r < kMaxRanks; ++r) {
        p.cPeers[r] = static_cast<float*>(q.reduce.cPeers[r]);
        p.flagsPeers[r] = q.reduce.flagsPeers[r];
    }
    p.rank = q.reduce.rank;
    p.world = q.reduce.world ? q.reduce.world : 1;
    p.target = q.reduce.target;
    p.bias = q.bias;
    p.colSums = q.colSums;
    p.velocity = q.update.momentum > 0.0f ? q.update.velocity : nullptr;
    p.copy = static_cast<__nv_bfloat16*>(q.update.copy);
    p.lr = q.update.lr;
    p.mu = q.update.momentum;
    const ReduceUpdate& u = q.reduce.update;
    p.fusedUpdate = q.epilogue == kEpiAllReduceF32 && u.enabled ? 1u : 0u;
    p.compact = p.fusedUpdate && q.reduce.compact ? 1u : 0u;
    if (p.fusedUpdate) {
        p.velocity = u.momentum > 0.0f ? u.velocity : nullptr;
        p.lr = u.lr;
        p.mu = u.momentum;
        for (int r = 0; r < kMaxRanks; ++r) {
            p.pPeers[r] = u.paramPeers[r];
            p.pbPeers[r] = static_cast<__nv_bfloat16*>(u.copyPeers[r]);
        }
        p.pMc = u.paramMulticast;
        p.pbMc = static_cast<__nv_bfloat16*>(u.copyMulticast);
    }
    if (q.aMajorMN) {
        if (q.bMajorMN) return launchEpi<true, true>(q.epilogue, pair, a, b, p, stream);
        return launchEpi<true, false>(q.epilogue, pair, a, b, p, stream);
    }
    if (q.bMajorMN) return launchEpi<false, true>(q.epilogue, pair, a, b, p, stream);
    return launchEpi<false, false>(q.epilogue, pair, a, b, p, stream);
}

namespace {

// One CTA per tile of P: tiles owned by another rank are copied from the
// owner's parameters (the same tile order and owner map as gemmKernel).
__global__ void __launch_bounds__(256) gatherOwnedKernel(const Params p, float* __restrict__ own) {
    const uint32_t tile = blockIdx.x;
    const uint32_t owner = tileOwner(p, tile);
    if (owner == p.rank) return;
    uint32_t mb, nb;
    tileCoords(tile, p, mb, nb);
    const uint64_t row0 = static_cast<uint64_t>(mb) * kBM, col0 = static_cast<uint64_t>(nb) * kBN;
    const float* src = p.pPeers[owner];
    for (uint32_t e = threadIdx.x; e < kBM * kBN; e += blockDim.x) {
        const uint64_t r = row0 + e / kBN, c = col0 + e % kBN;
        if (r < p.m && c < p.n) own[r * p.ldc + c] = __ldcg(src + r * p.ldc + c);
    }
}

} // namespace

cudaError_t gatherOwned(const Problem& q, int smCount, cudaStream_t stream) {
    const AllReduce& r = q.reduce;
    if (q.epilogue != kEpiAllReduceF32 || !r.update.enabled || r.world == 0 || r.rank >= r.world ||
        !r.update.paramPeers[r.rank])
        return cudaErrorInvalidValue;
    // The fused all-reduce runs on single CTAs (128 x 256 tiles); the map
    // must match gemm::run's for this problem.
    if (usePairs(q)) return cudaErrorInvalidValue;
    Params p{};
    p.m = static_cast<uint32_t>(q.m);
    p.n = static_cast<uint32_t>(q.n);
    p.mTiles = static_cast<uint32_t>((q.m + kBM - 1) / kBM);
    p.nTiles = static_cast<uint32_t>((q.n + kBN - 1) / kBN);
    p.group = rasterGroup();
    p.ldc = q.ldc;
    p.rank = r.rank;
    p.world = r.world;
    const uint32_t tiles = p.mTiles * p.nTiles;
    p.grid = tiles < static_cast<uint32_t>(smCount) ? tiles : static_cast<uint32_t>(smCount);
    for (int k = 0; k < kMaxRanks; ++k) p.pPeers[k] = r.update.paramPeers[k];
    if (tiles == 0) return cudaSuccess;
    gatherOwnedKernel<<<tiles, 256, 0, stream>>>(p, r.update.paramPeers[r.rank]);
    return cudaGetLastError();
}

} // namespace thb::gemm

