// GPU preparation of the renderer (see graphics.hpp): the f32 vertex
// transform, Sutherland-Hodgman clipping against the six homogeneous planes,
// screen setup and tile binning of prepare() (graphics.cpp), as kernels.
//
// Every f32 and f64 operation is an explicit round-to-nearest intrinsic in
// the order of the host code, so nothing contracts into an FMA and the screen
// triangles carry the bits of the reference's prepareRender /
// prepareScreenTriangle (src/graphics/v0/Graphics.cpp:102-421). Output order
// is submission order: each input triangle's surviving fan triangles go to
// an exclusive prefix sum of the per-triangle counts. Each tile's list keeps
// that order: the screen triangles are cut into contiguous chunks, one warp
// per chunk walks its triangles in order (counting, then filling), and the
// per-(chunk, tile) offsets are tile-major then chunk-major prefix sums, as
// the host binning does with its thread chunks.
#include <cuda_runtime.h>

#include <cstdint>
#include <limits>
#include <memory>
#include <vector>

#include "graphics.hpp"
#include "runtime.hpp"

namespace thb::graphics {
namespace {

constexpr unsigned kThreads = 256;
constexpr std::uint32_t kFlagTransform = 1u, kFlagClip = 2u;

struct ClipVertex {
    float p[4];
    float c[4];
};

struct Matrix {
    float m[16];
};

// Device scalars: flags, post-clip triangles, a prefix-sum total.
struct Meta {
    std::uint32_t flags;
    std::uint32_t pad;
    unsigned long long postClip;
    unsigned long long total;
};

// ---- transform (prepare(): clip[v] = MVP * (p, 1)) ----

__global__ void __launch_bounds__(kThreads) transformKernel(const float* __restrict__ positions,
                                                            const float* __restrict__ colors, std::uint64_t vertices,
                                                            Matrix mvp, ClipVertex* __restrict__ out,
                                                            Meta* __restrict__ meta) {
    const std::uint64_t stride = static_cast<std::uint64_t>(gridDim.x) * kThreads;
    bool bad = false;
    for (std::uint64_t v = static_cast<std::uint64_t>(blockIdx.x) * kThreads + threadIdx.x; v < vertices; v += stride) {
        const float in[4] = {positions[v * 3], positions[v * 3 + 1], positions[v * 3 + 2], 1.0f};
        ClipVertex r;
#pragma unroll
        for (int row = 0; row < 4; ++row) {
            float acc = 0.0f;
#pragma unroll
            for (int col = 0; col < 4; ++col) acc = __fadd_rn(acc, __fmul_rn(mvp.m[row * 4 + col], in[col]));
            if (!isfinite(acc)) bad = true;
            r.p[row] = acc;
        }
        const float4 c = *reinterpret_cast<const float4*>(colors + v * 4);
        r.c[0] = c.x;
        r.c[1] = c.y;
        r.c[2] = c.z;
        r.c[3] = c.w;
        out[v] = r;
    }
    if (bad) atomicOr(&meta->flags, kFlagTransform);
}

// ---- clipping and screen setup (graphics.cpp clipPlane / toScreen / pack) ----

__device__ __forceinline__ float planeDistance(const ClipVertex& v, int k) {
    switch (k) {
    case 0: return __fadd_rn(v.p[0], v.p[3]);
    case 1: return __fadd_rn(v.p[3], -v.p[0]);
    case 2: return __fadd_rn(v.p[1], v.p[3]);
    case 3: return __fadd_rn(v.p[3], -v.p[1]);
    case 4: return v.p[2];
    default: return __fadd_rn(v.p[3], -v.p[2]);
    }
}

__device__ __forceinline__ ClipVertex lerp(const ClipVertex& a, const ClipVertex& b, float t) {
    ClipVertex r;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        r.p[k] = __fadd_rn(a.p[k], __fmul_rn(t, __fadd_rn(b.p[k], -a.p[k])));
        r.c[k] = __fadd_rn(a.c[k], __fmul_rn(t, __fadd_rn(b.c[k], -a.c[k])));
    }
    return r;
}

// One Sutherland-Hodgman pass; -1 on a numeric failure (TH019-CLIP-NUMERIC).
__device__ int clipPlane(const ClipVertex* in, int n, int plane, ClipVertex* out) {
    if (n == 0) return 0;
    int m = 0;
    ClipVertex prev = in[n - 1];
    float prevDistance = planeDistance(prev, plane);
    bool prevInside = prevDistance >= 0.0f;
    for (int i = 0; i < n; ++i) {
        const float d = planeDistance(in[i], plane);
        const bool inside = d >= 0.0f;
        if (prevInside != inside) {
            const float den = __fadd_rn(prevDistance, -d);
            if (den == 0.0f || !isfinite(den)) return -1;
            const float amount = __fdiv_rn(prevDistance, den);
            if (!isfinite(amount)) return -1;
            out[m++] = lerp(prev, in[i], amount);
        }
        if (inside) out[m++] = in[i];
        prev = in[i];
        prevDistance = d;
        prevInside = inside;
    }
    return m;
}

struct ScreenVertex {
    double x, y, depth, rw;
    float c[4];
};

__device__ __forceinline__ double edge(const ScreenVertex& a, const ScreenVertex& b, double x, double y) {
    return __dsub_rn(__dmul_rn(__dsub_rn(b.x, a.x), __dsub_rn(y, a.y)), __dmul_rn(__dsub_rn(b.y, a.y), __dsub_rn(x, a.x)));
}

__device__ __forceinline__ bool topLeft(const ScreenVertex& a, const ScreenVertex& b) {
    const double dx = __dsub_rn(b.x, a.x), dy = __dsub_rn(b.y, a.y);
    return dy < 0.0 || (dy == 0.0 && dx > 0.0);
}

__device__ bool toScreen(const ClipVertex* t, double w, double h, ScreenVertex* s) {
    for (int i = 0; i < 3; ++i) {
        const float cw = t[i].p[3];
        if (!isfinite(cw) || cw <= 1.0e-7f) return false;
        const float x = __fdiv_rn(t[i].p[0], cw), y = __fdiv_rn(t[i].p[1], cw), z = __fdiv_rn(t[i].p[2], cw);
        if (!isfinite(x) || !isfinite(y) || !isfinite(z)) return false;
        s[i].x = __dmul_rn(__dadd_rn(__dmul_rn(static_cast<double>(x), 0.5), 0.5), w);
        s[i].y = __dmul_rn(__dsub_rn(0.5, __dmul_rn(static_cast<double>(y), 0.5)), h);
        s[i].depth = z;
        s[i].rw = __ddiv_rn(1.0, static_cast<double>(cw));
#pragma unroll
        for (int k = 0; k < 4; ++k) s[i].c[k] = t[i].c[k];
    }
    const double area = edge(s[0], s[1], s[2].x, s[2].y);
    if (!isfinite(area) || fabs(area) <= 1.0e-12) return false;
    if (area < 0.0) {
        const ScreenVertex keep = s[1];
        s[1] = s[2];
        s[2] = keep;
    }
    return true;
}

// std::min / std::max over an initializer list of three: the first of equal
// values wins, as on the host.
__device__ __forceinline__ double min3(double a, double b, double c) {
    double r = a;
    if (b < r) r = b;
    if (c < r) r = c;
    return r;
}
__device__ __forceinline__ double max3(double a, double b, double c) {
    double r = a;
    if (r < b) r = b;
    if (r < c) r = c;
    return r;
}

__device__ bool pack(const ScreenVertex* v, std::int64_t w, std::int64_t h, RasterTriangle& t) {
    const double minX = min3(v[0].x, v[1].x, v[2].x), maxX = max3(v[0].x, v[1].x, v[2].x);
    const double minY = min3(v[0].y, v[1].y, v[2].y), maxY = max3(v[0].y, v[1].y, v[2].y);
    auto x0 = static_cast<std::int64_t>(ceil(__dsub_rn(minX, 0.5)));
    auto x1 = static_cast<std::int64_t>(floor(__dsub_rn(maxX, 0.5)));
    auto y0 = static_cast<std::int64_t>(ceil(__dsub_rn(minY, 0.5)));
    auto y1 = static_cast<std::int64_t>(floor(__dsub_rn(maxY, 0.5)));
    x0 = x0 < 0 ? 0 : x0;
    y0 = y0 < 0 ? 0 : y0;
    x1 = x1 > w - 1 ? w - 1 : x1;
    y1 = y1 > h - 1 ? h - 1 : y1;
    if (x0 > x1 || y0 > y1) return false;
    for (int i = 0; i < 3; ++i) {
        t.x[i] = v[i].x;
        t.y[i] = v[i].y;
        t.depth[i] = v[i].depth;
        t.rw[i] = v[i].rw;
#pragma unroll
        for (int k = 0; k < 4; ++k) t.color[i][k] = v[i].c[k];
    }
    t.area = edge(v[0], v[1], v[2].x, v[2].y);
    t.x0 = static_cast<std::int32_t>(x0);
    t.x1 = static_cast<std::int32_t>(x1);
    t.y0 = static_cast<std::int32_t>(y0);
    t.y1 = static_cast<std::int32_t>(y1);
    t.inclusive = (topLeft(v[1], v[2]) ? 1u : 0u) | (topLeft(v[2], v[0]) ? 2u : 0u) | (topLeft(v[0], v[1]) ? 4u : 0u);
    t.pad[0] = t.pad[1] = t.pad[2] = 0;
    return true;
}

// Clips input triangle t and sets up its fan. COUNT: kept[t] = screen
// triangles it yields, post-clip fan triangles summed into meta. Otherwise
// writes them at out[offsets[t]...] in fan order.
template <bool COUNT>
__global__ void __launch_bounds__(kThreads) clipKernel(const ClipVertex* __restrict__ clip, std::uint64_t vertices,
                                                       const std::int64_t* __restrict__ indices,
                                                       std::uint64_t triangles, double w, double h,
                                                       std::uint32_t* __restrict__ kept,
                                                       const std::uint64_t* __restrict__ offsets,
                                                       RasterTriangle* __restrict__ out, Meta* __restrict__ meta) {
    const std::uint64_t t = static_cast<std::uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
    std::uint32_t fans = 0, count = 0;
    bool failed = false;
    if (t < triangles) {
        ClipVertex poly[2][16];
        int n = 3;
        for (int c = 0; c < 3; ++c) {
            const std::int64_t index = indices[t * 3 + c];  // validated on the host: 0 <= index < vertices
            poly[0][c] = clip[static_cast<std::uint64_t>(index) < vertices ? index : 0];
        }
        int cur = 0;
        for (int plane = 0; plane < 6 && n >= 3; ++plane) {
            n = clipPlane(poly[cur], n, plane, poly[cur ^ 1]);
            if (n < 0) {
                failed = true;
                break;
            }
            cur ^= 1;
        }
        if (!failed && n >= 3) {
            std::uint64_t slot = COUNT ? 0 : offsets[t];
            for (int c = 1; c + 1 < n; ++c) {
                ++fans;
                const ClipVertex tri[3] = {poly[cur][0], poly[cur][c], poly[cur][c + 1]};
                ScreenVertex s[3];
                RasterTriangle packed;
                if (toScreen(tri, w, h, s) && pack(s, static_cast<std::int64_t>(w), static_cast<std::int64_t>(h), packed)) {
                    if constexpr (!COUNT) out[slot++] = packed;
                    ++count;
                }
            }
        }
        if constexpr (COUNT) kept[t] = count;
    }
    if constexpr (COUNT) {
        const unsigned warpFans = __reduce_add_sync(0xffffffffu, fans);
        if (threadIdx.x % 32 == 0 && warpFans) atomicAdd(&meta->postClip, static_cast<unsigned long long>(warpFans));
        if (__any_sync(0xffffffffu, failed) && threadIdx.x % 32 == 0) atomicOr(&meta->flags, kFlagClip);
    }
}

// ---- exclusive prefix sums (u32 or u64 in, u64 out) ----

constexpr unsigned kScanItems = 4 * kThreads;  // per block

template <class In>
__global__ void __launch_bounds__(kThreads) scanBlocks(const In* __restrict__ in, std::uint64_t n,
                                                       std::uint64_t* __restrict__ out,
                                                       std::uint64_t* __restrict__ blockSums) {
    __shared__ std::uint64_t warpTotals[kThreads / 32];
    const unsigned lane = threadIdx.x % 32, warp = threadIdx.x / 32;
    const std::uint64_t base = static_cast<std::uint64_t>(blockIdx.x) * kScanItems + threadIdx.x * 4ull;
    std::uint64_t v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = base + j < n ? static_cast<std::uint64_t>(in[base + j]) : 0;
    const std::uint64_t mine = v[0] + v[1] + v[2] + v[3];
    std::uint64_t x = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const std::uint64_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= static_cast<unsigned>(o)) x += y;
    }
    if (lane == 31) warpTotals[warp] = x;
    __syncthreads();
    std::uint64_t before = 0;
    for (unsigned w = 0; w < warp; ++w) before += warpTotals[w];
    std::uint64_t run = before + x - mine;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        if (base + j < n) out[base + j] = run;
        run += v[j];
    }
    if (threadIdx.x == kThreads - 1) blockSums[blockIdx.x] = before + x;
}

__global__ void __launch_bounds__(kThreads) addBlockOffsets(std::uint64_t* __restrict__ out, std::uint64_t n,
                                                            const std::uint64_t* __restrict__ offsets) {
    const std::uint64_t i = static_cast<std::uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (i < n) out[i] += offsets[i / kScanItems];
}

template <class In>
__global__ void lastTotal(const In* __restrict__ in, const std::uint64_t* __restrict__ out, std::uint64_t n,
                          Meta* __restrict__ meta) {
    meta->total = n ? out[n - 1] + static_cast<std::uint64_t>(in[n - 1]) : 0;
}

void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) fail(Category::Runtime, "GPU-RUNTIME", std::string(what) + ": " + cudaGetErrorString(e));
}

unsigned blocksFor(std::uint64_t n, std::uint64_t per) { return static_cast<unsigned>((n + per - 1) / per); }

// The pool's next buffer, grown to at least `bytes` (16 at least); counts
// the growths in `allocations`.
void* take(ScratchPool& pool, std::size_t bytes, int device, std::uint64_t& allocations) {
    if (pool.next == pool.buffers.size()) pool.buffers.push_back(std::make_unique<DeviceBuffer>());
    DeviceBuffer& b = *pool.buffers[pool.next++];
    if (b.reserve(bytes < 16 ? 16 : bytes, device)) ++allocations;
    return b.ptr;
}

// out[i] = sum of in[0..i), meta->total = sum of in; temporaries come from
// `pool`.
template <class In>
void exclusiveScan(const In* in, std::uint64_t n, std::uint64_t* out, Meta* meta, int device, cudaStream_t stream,
                   ScratchPool& pool, DevicePrepared& counts, bool total = true) {
    std::uint64_t& launches = counts.launches;
    if (n == 0) {
        if (total) check(cudaMemsetAsync(&meta->total, 0, sizeof meta->total, stream), "cudaMemsetAsync(scan)");
        return;
    }
    const unsigned blocks = blocksFor(n, kScanItems);
    auto* s = static_cast<std::uint64_t*>(take(pool, static_cast<std::size_t>(blocks) * 8, device, counts.allocations));
    scanBlocks<In><<<blocks, kThreads, 0, stream>>>(in, n, out, s);
    check(cudaGetLastError(), "scan");
    ++launches;
    if (blocks > 1) {
        auto* o = static_cast<std::uint64_t*>(take(pool, static_cast<std::size_t>(blocks) * 8, device, counts.allocations));
        exclusiveScan<std::uint64_t>(s, blocks, o, meta, device, stream, pool, counts, false);
        addBlockOffsets<<<blocksFor(n, kThreads), kThreads, 0, stream>>>(out, n, o);
        check(cudaGetLastError(), "scan offsets");
        ++launches;
    }
    if (total) {
        lastTotal<In><<<1, 1, 0, stream>>>(in, out, n, meta);
        check(cudaGetLastError(), "scan total");
        ++launches;
    }
}

// ---- tile binning ----

__device__ __forceinline__ void tileRange(const RasterTriangle* t, std::int32_t& tx0, std::int32_t& ty0,
                                          std::int32_t& nx, std::int32_t& ny) {
    // (x0 sits at byte 152 of the 192-byte record: 8-byte aligned only.)
    const int2 xs = *reinterpret_cast<const int2*>(&t->x0);  // x0, x1
    const int2 ys = *reinterpret_cast<const int2*>(&t->y0);  // y0, y1
    tx0 = xs.x / kTile;
    ty0 = ys.x / kTile;
    nx = xs.y / kTile - tx0 + 1;
    ny = ys.y / kTile - ty0 + 1;
}

// One warp per chunk of screen triangles, walked in order. COUNT:
// cells[chunk][tile] += 1 per triangle touching the tile; otherwise
// lists[cells[chunk][tile]++] = triangle (cells hold the list cursors). The
// lanes split each triangle's tiles, which are distinct, and __syncwarp
// orders consecutive triangles.
template <bool COUNT>
__global__ void __launch_bounds__(kThreads) binKernel(const RasterTriangle* __restrict__ triangles,
                                                      std::uint64_t count, std::uint64_t chunks,
                                                      std::uint64_t perChunk, std::uint32_t tilesX,
                                                      std::uint64_t tiles, std::uint32_t* __restrict__ cells,
                                                      std::uint32_t* __restrict__ lists) {
    const std::uint64_t chunk = (static_cast<std::uint64_t>(blockIdx.x) * kThreads + threadIdx.x) / 32;
    const unsigned lane = threadIdx.x % 32;
    if (chunk >= chunks) return;
    std::uint32_t* row = cells + chunk * tiles;
    const std::uint64_t begin = chunk * perChunk;
    const std::uint64_t end = begin + perChunk < count ? begin + perChunk : count;
    for (std::uint64_t i = begin; i < end; ++i) {
        std::int32_t tx0, ty0, nx, ny;
        tileRange(triangles + i, tx0, ty0, nx, ny);
        const std::uint32_t cellsInBox = static_cast<std::uint32_t>(nx) * static_cast<std::uint32_t>(ny);
        for (std::uint32_t k = lane; k < cellsInBox; k += 32) {
            const std::uint64_t tile =
                static_cast<std::uint64_t>(ty0 + static_cast<std::int32_t>(k / nx)) * tilesX + tx0 + k % nx;
            if constexpr (COUNT) ++row[tile];
            else lists[row[tile]++] = static_cast<std::uint32_t>(i);
        }
        __syncwarp();
    }
}

// Per tile: cells[c][tile] = entries of chunks before c (exclusive, chunk
// order), totals[tile] = entries of the tile.
__global__ void __launch_bounds__(kThreads) chunkPrefix(std::uint32_t* __restrict__ cells, std::uint64_t chunks,
                                                        std::uint64_t tiles, std::uint64_t* __restrict__ totals) {
    const std::uint64_t tile = static_cast<std::uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (tile >= tiles) return;
    std::uint64_t run = 0;
    for (std::uint64_t c = 0; c < chunks; ++c) {
        const std::uint32_t v = cells[c * tiles + tile];
        cells[c * tiles + tile] = static_cast<std::uint32_t>(run);
        run += v;
    }
    totals[tile] = run;
}

// cells[c][tile] += start[tile]; tileOffsets[tile] = start[tile], and the
// closing entry tileOffsets[tiles] = total.
__global__ void __launch_bounds__(kThreads) addTileStarts(std::uint32_t* __restrict__ cells, std::uint64_t chunks,
                                                          std::uint64_t tiles, const std::uint64_t* __restrict__ start,
                                                          std::uint32_t* __restrict__ tileOffsets,
                                                          const Meta* __restrict__ meta) {
    const std::uint64_t i = static_cast<std::uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (i < chunks * tiles) cells[i] += static_cast<std::uint32_t>(start[i % tiles]);
    if (i < tiles) tileOffsets[i] = static_cast<std::uint32_t>(start[i]);
    if (i == 0) tileOffsets[tiles] = static_cast<std::uint32_t>(meta->total);
}

} // namespace

DevicePrepared prepareOnDevice(const Scene& scene, const float* positions, const float* colors,
                               const std::int64_t* indices, int device, cudaStream_t stream,
                               DeviceBuffer& triangles, DeviceBuffer& tileOffsets, DeviceBuffer& tileLists,
                               ScratchPool& pool) {
    DevicePrepared result;
    const std::uint64_t vertices = scene.vertices, inputs = scene.triangles;
    pool.next = 0;
    auto scratch = [&](std::size_t bytes) { return take(pool, bytes, device, result.allocations); };
    auto* meta = static_cast<Meta*>(scratch(sizeof(Meta)));
    check(cudaMemsetAsync(meta, 0, sizeof(Meta), stream), "cudaMemsetAsync(meta)");
    Meta host{};

    // Transform every vertex, then clip and count each triangle's fan.
    auto* clip = static_cast<ClipVertex*>(scratch(vertices * sizeof(ClipVertex)));
    Matrix mvp;
    for (int k = 0; k < 16; ++k) mvp.m[k] = scene.mvp[k];
    if (vertices) {
        transformKernel<<<std::min<unsigned>(blocksFor(vertices, kThreads), 148u * 16u), kThreads, 0, stream>>>(
            positions, colors, vertices, mvp, clip, meta);
        check(cudaGetLastError(), "transform");
        ++result.launches;
    }
    auto* kept = static_cast<std::uint32_t*>(scratch(inputs * 4));
    auto* offsets = static_cast<std::uint64_t*>(scratch(inputs * 8));
    const double w = static_cast<double>(scene.width), h = static_cast<double>(scene.height);
    if (inputs) {
        clipKernel<true><<<blocksFor(inputs, kThreads), kThreads, 0, stream>>>(clip, vertices, indices, inputs, w, h, kept,
                                                                               nullptr, nullptr, meta);
        check(cudaGetLastError(), "clip (count)");
        ++result.launches;
    }
    exclusiveScan<std::uint32_t>(kept, inputs, offsets, meta, device, stream, pool, result);
    check(cudaMemcpyAsync(&host, meta, sizeof host, cudaMemcpyDeviceToHost, stream), "cudaMemcpyAsync(meta)");
    check(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
    // The host pipeline's failure order: transform, clip, triangle count,
    // tile count, list entries.
    if (host.flags & kFlagTransform) {
        result.failure = "TH019-NONFINITE-TRANSFORMED";
        return result;
    }
    if (host.flags & kFlagClip) {
        result.failure = "TH019-CLIP-NUMERIC";
        return result;
    }
    result.postClipTriangles = host.postClip;
    result.count = host.total;
    const std::uint64_t tiles = static_cast<std::uint64_t>(scene.tilesX) * scene.tilesY;
    if (result.count > std::numeric_limits<std::uint32_t>::max() || tiles >= std::numeric_limits<std::uint32_t>::max()) {
        result.failure = "TH019-FRAMEBUFFER-SIZE";
        return result;
    }

    // Screen triangles in submission order.
    triangles.reserve(std::max<std::size_t>(16, result.count * sizeof(RasterTriangle)), device);
    if (result.count) {
        clipKernel<false><<<blocksFor(inputs, kThreads), kThreads, 0, stream>>>(
            clip, vertices, indices, inputs, w, h, nullptr, offsets, static_cast<RasterTriangle*>(triangles.ptr), meta);
        check(cudaGetLastError(), "clip (write)");
        ++result.launches;
    }

    // Tile lists.
    tileOffsets.reserve((tiles + 1) * 4, device);
    if (result.count == 0 || tiles == 0) {
        check(cudaMemsetAsync(tileOffsets.ptr, 0, (tiles + 1) * 4, stream), "cudaMemsetAsync(tile offsets)");
        tileLists.reserve(16, device);
        check(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
        return result;
    }
    // Chunks: about 64 triangles per warp, at most 1024, and at most 2^26
    // (chunk, tile) cells.
    std::uint64_t chunks = std::min<std::uint64_t>(1024, std::max<std::uint64_t>(1, result.count / 64));
    chunks = std::max<std::uint64_t>(1, std::min<std::uint64_t>(chunks, (1ull << 26) / tiles));
    const std::uint64_t perChunk = (result.count + chunks - 1) / chunks;
    chunks = (result.count + perChunk - 1) / perChunk;
    auto* cells = static_cast<std::uint32_t*>(scratch(chunks * tiles * 4));
    auto* totals = static_cast<std::uint64_t*>(scratch(tiles * 8));
    auto* starts = static_cast<std::uint64_t*>(scratch(tiles * 8));
    check(cudaMemsetAsync(cells, 0, chunks * tiles * 4, stream), "cudaMemsetAsync(cells)");
    const auto* tri = static_cast<const RasterTriangle*>(triangles.ptr);
    const unsigned binBlocks = blocksFor(chunks * 32, kThreads);
    binKernel<true><<<binBlocks, kThreads, 0, stream>>>(tri, result.count, chunks, perChunk, scene.tilesX, tiles, cells,
                                                        nullptr);
    check(cudaGetLastError(), "bin (count)");
    ++result.launches;
    chunkPrefix<<<blocksFor(tiles, kThreads), kThreads, 0, stream>>>(cells, chunks, tiles, totals);
    check(cudaGetLastError(), "bin (chunk prefix)");
    ++result.launches;
    exclusiveScan<std::uint64_t>(totals, tiles, starts, meta, device, stream, pool, result);
    check(cudaMemcpyAsync(&host, meta, sizeof host, cudaMemcpyDeviceToHost, stream), "cudaMemcpyAsync(meta)");
    check(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
    if (host.total >= std::numeric_limits<std::uint32_t>::max()) {
        result.failure = "TH019-FRAMEBUFFER-SIZE";
        return result;
    }
    tileLists.reserve(std::max<std::size_t>(16, host.total * 4), device);
    addTileStarts<<<blocksFor(std::max(chunks * tiles, tiles), kThreads), kThreads, 0, stream>>>(
        cells, chunks, tiles, starts, static_cast<std::uint32_t*>(tileOffsets.ptr), meta);
    check(cudaGetLastError(), "bin (tile starts)");
    ++result.launches;
    binKernel<false><<<binBlocks, kThreads, 0, stream>>>(tri, result.count, chunks, perChunk, scene.tilesX, tiles, cells,
                                                         static_cast<std::uint32_t*>(tileLists.ptr));
    check(cudaGetLastError(), "bin (fill)");
    ++result.launches;
    return result;
}

} // namespace thb::graphics
