// Tile rasterizer of the GPU renderer (see graphics.hpp).
//
// One CTA of 256 threads per 16x16 tile, one thread per pixel. The tile's
// triangle list (submission order) is staged into shared memory 32 triangles
// at a time (6 KB, 16-byte vector loads); each thread then applies, in order,
// the reference rasterizer's per-pixel steps (src/graphics/v0/Graphics.cpp:
// 277-318): bounding box, three f64 edge functions with the top-left rule,
// barycentric weights, interpolated depth with range check and clamp,
// perspective-correct colour, then the strict-less f32 depth test. Every f64
// operation is an explicit round-to-nearest intrinsic, so nothing is fused
// into an FMA and the bits equal the CPU's. Pixel counters are reduced per
// CTA and added to two global u64 counters.
#include <cuda_runtime.h>

#include <cstdint>

#include "graphics.hpp"

namespace thb::graphics {
namespace {

constexpr unsigned kThreads = kTile * kTile;
constexpr unsigned kStage = 32;

__device__ __forceinline__ double edgeAt(double ax, double ay, double bx, double by, double x, double y) {
    const double first = __dmul_rn(__dsub_rn(bx, ax), __dsub_rn(y, ay));
    const double second = __dmul_rn(__dsub_rn(by, ay), __dsub_rn(x, ax));
    return __dsub_rn(first, second);
}

__device__ __forceinline__ bool covered(double v, bool inclusive) { return v > 0.0 || (v == 0.0 && inclusive); }

__device__ __forceinline__ double clamp01(double v) { return v < 0.0 ? 0.0 : (v > 1.0 ? 1.0 : v); }

__global__ void __launch_bounds__(kThreads) rasterKernel(const RasterTriangle* __restrict__ triangles,
                                                         const std::uint32_t* __restrict__ offsets,
                                                         const std::uint32_t* __restrict__ lists, std::uint32_t tilesX,
                                                         std::uint32_t width, std::uint32_t height, float4 clear,
                                                         float* __restrict__ color, float* __restrict__ depth,
                                                         unsigned long long* __restrict__ stats) {
    __shared__ RasterTriangle stage[kStage];
    __shared__ unsigned long long sums[2][kThreads / 32];
    const std::uint32_t tile = blockIdx.x;
    const std::int32_t px = static_cast<std::int32_t>((tile % tilesX) * kTile + threadIdx.x % kTile);
    const std::int32_t py = static_cast<std::int32_t>((tile / tilesX) * kTile + threadIdx.x / kTile);
    const bool inside = static_cast<std::uint32_t>(px) < width && static_cast<std::uint32_t>(py) < height;
    const double cx = static_cast<double>(px) + 0.5, cy = static_cast<double>(py) + 0.5;
    float best = __int_as_float(0x7f800000);  // +inf: the cleared depth
    float4 out = clear;
    std::uint32_t shaded = 0, passes = 0;
    const std::uint32_t begin = offsets[tile], end = offsets[tile + 1];
    for (std::uint32_t base = begin; base < end; base += kStage) {
        const std::uint32_t count = end - base < kStage ? end - base : kStage;
        for (std::uint32_t i = threadIdx.x; i < count * 12; i += kThreads) {
            const std::uint32_t t = i / 12, q = i % 12;
            reinterpret_cast<uint4*>(&stage[t])[q] = __ldg(reinterpret_cast<const uint4*>(&triangles[lists[base + t]]) + q);
        }
        __syncthreads();
        if (inside) {
            for (std::uint32_t k = 0; k < count; ++k) {
                const RasterTriangle& t = stage[k];
                if (px < t.x0 || px > t.x1 || py < t.y0 || py > t.y1) continue;
                const double e0 = edgeAt(t.x[1], t.y[1], t.x[2], t.y[2], cx, cy);
                const double e1 = edgeAt(t.x[2], t.y[2], t.x[0], t.y[0], cx, cy);
                const double e2 = edgeAt(t.x[0], t.y[0], t.x[1], t.y[1], cx, cy);
                if (!covered(e0, t.inclusive & 1u) || !covered(e1, t.inclusive & 2u) || !covered(e2, t.inclusive & 4u))
                    continue;
                const double w0 = __ddiv_rn(e0, t.area), w1 = __ddiv_rn(e1, t.area), w2 = __ddiv_rn(e2, t.area);
                double d = __dadd_rn(__dadd_rn(__dmul_rn(w0, t.depth[0]), __dmul_rn(w1, t.depth[1])),
                                     __dmul_rn(w2, t.depth[2]));
                if (!isfinite(d) || d < -1.0e-6 || d > 1.0 + 1.0e-6) continue;
                d = clamp01(d);
                const double den = __dadd_rn(__dadd_rn(__dmul_rn(w0, t.rw[0]), __dmul_rn(w1, t.rw[1])),
                                             __dmul_rn(w2, t.rw[2]));
                if (!isfinite(den) || den <= 0.0) continue;
                float c[4];
                bool valid = true;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const double a = __dmul_rn(__dmul_rn(w0, static_cast<double>(t.color[0][j])), t.rw[0]);
                    const double b = __dmul_rn(__dmul_rn(w1, static_cast<double>(t.color[1][j])), t.rw[1]);
                    const double e = __dmul_rn(__dmul_rn(w2, static_cast<double>(t.color[2][j])), t.rw[2]);
                    const double value = __ddiv_rn(__dadd_rn(__dadd_rn(a, b), e), den);
                    if (!isfinite(value)) valid = false;
                    c[j] = __double2float_rn(clamp01(value));
                }
                if (!valid) continue;
                ++shaded;
                const float fd = __double2float_rn(d);
                if (!(fd < best)) continue;
                best = fd;
                out = make_float4(c[0], c[1], c[2], c[3]);
                ++passes;
            }
        }
        __syncthreads();
    }
    if (inside) {
        const std::uint64_t pixel = static_cast<std::uint64_t>(py) * width + static_cast<std::uint32_t>(px);
        reinterpret_cast<float4*>(color)[pixel] = out;
        depth[pixel] = best;
    }
    unsigned long long s = shaded, p = passes;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        s += __shfl_xor_sync(0xffffffffu, s, o);
        p += __shfl_xor_sync(0xffffffffu, p, o);
    }
    if (threadIdx.x % 32 == 0) {
        sums[0][threadIdx.x / 32] = s;
        sums[1][threadIdx.x / 32] = p;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long ts = 0, tp = 0;
        for (unsigned w = 0; w < kThreads / 32; ++w) {
            ts += sums[0][w];
            tp += sums[1][w];
        }
        if (ts) atomicAdd(&stats[0], ts);
        if (tp) atomicAdd(&stats[1], tp);
    }
}

} // namespace

cudaError_t rasterize(const RasterTriangle* triangles, const std::uint32_t* tileOffsets, const std::uint32_t* tileLists,
                      std::uint32_t tilesX, std::uint32_t tilesY, std::uint32_t width, std::uint32_t height,
                      const float* clear, float* color, float* depth, unsigned long long* stats, cudaStream_t stream) {
    const std::uint64_t tiles = static_cast<std::uint64_t>(tilesX) * tilesY;
    if (tiles == 0) return cudaSuccess;
    rasterKernel<<<static_cast<unsigned>(tiles), kThreads, 0, stream>>>(
        triangles, tileOffsets, tileLists, tilesX, width, height, make_float4(clear[0], clear[1], clear[2], clear[3]),
        color, depth, stats);
    return cudaGetLastError();
}

} // namespace thb::graphics
