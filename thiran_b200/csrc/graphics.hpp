// GPU renderer of the reference's software rasterizer
// (src/graphics/v0/Graphics.cpp, GPU backend src/graphics/v0/GraphicsGpu.cpp).
//
// Validation runs on the host before any driver call, as the reference's
// prepareRender does (Graphics.cpp:374-421). The f32 vertex transform,
// homogeneous clipping, screen setup and binning of screen triangles into
// 16x16-pixel tiles (submission order within each tile) run on the GPU
// (prep.cu) with every operation rounded on its own, so the post-clip
// triangles are the same bits as the reference's CPU path; prepare() is the
// same pipeline on host threads. The rasterizer runs on the GPU: one thread
// per pixel walks its tile's list in order with the reference's f64
// edge / barycentric / perspective-correct arithmetic and strict-less depth
// test, so colour, depth and both pixel counters equal the sequential CPU
// result. (The reference's GPU kernel walks every triangle for every pixel.)
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

namespace thb {
struct DeviceBuffer;
}

namespace thb::graphics {

constexpr int kTile = 16;

// One screen triangle as the raster kernel reads it (192 bytes).
struct alignas(16) RasterTriangle {
    double x[3], y[3], depth[3], rw[3];  // screen position, NDC depth, 1/w
    double area;                         // edge(v0, v1, v2) after orientation
    float color[3][4];
    std::int32_t x0, x1, y0, y1;         // clamped pixel bounding box
    std::uint32_t inclusive;             // top-left rule, bit k = edge k
    std::uint32_t pad[3];
};
static_assert(sizeof(RasterTriangle) == 192, "raster triangle layout");

struct Prepared {
    std::uint64_t width = 0, height = 0;
    float clear[4] = {0, 0, 0, 0};
    std::uint64_t inputTriangles = 0, postClipTriangles = 0;
    std::vector<RasterTriangle> triangles;
    std::uint32_t tilesX = 0, tilesY = 0;
    std::vector<std::uint32_t> tileOffsets;  // tilesX * tilesY + 1
    std::vector<std::uint32_t> tileLists;    // triangle indices, submission order per tile
};

// Validation (TH019-* ids), transform, clipping, screen setup and binning.
// Matrices are 16 f32, row-major, column-vector convention (P * V * M).
Prepared prepare(const float* positions, std::uint64_t vertices, const std::int64_t* indices,
                 std::uint64_t triangles, const float* colors, const float* model, const float* view,
                 const float* projection, std::uint64_t width, std::uint64_t height, const float* clear);

// The checks of prepare() that precede the transform (the reference's
// validateGeometry / validateFramebuffer and the matrix checks, same ids in
// the same order) and the model-view-projection product P * (V * M).
struct Scene {
    std::uint64_t width = 0, height = 0, vertices = 0, triangles = 0;
    float clear[4] = {0, 0, 0, 0};
    float mvp[16] = {};
    std::uint32_t tilesX = 0, tilesY = 0;
};
Scene validate(const float* positions, std::uint64_t vertices, const std::int64_t* indices, std::uint64_t triangles,
               const float* colors, const float* model, const float* view, const float* projection,
               std::uint64_t width, std::uint64_t height, const float* clear);

// Transform, clipping, screen setup and binning of a validated scene on the
// GPU (prep.cu): the same triangles, tile offsets and lists as prepare(),
// bit for bit. positions [vertices][3], colors [vertices][4] and indices
// [triangles][3] are device memory. The three outputs are device buffers
// the raster kernel reads. Synchronises `stream` twice (to size the
// triangle array and the tile lists).
struct DevicePrepared {
    std::uint64_t postClipTriangles = 0;
    std::uint64_t count = 0;  // screen triangles after setup
    const char* failure = nullptr;  // TH019 id found on the device, or null
    std::uint64_t launches = 0;     // kernels launched
    std::uint64_t allocations = 0;  // scratch buffers that had to grow
};
// Device scratch buffers kept from call to call: each call takes them in
// the same request order and grows one only when it is too small.
struct ScratchPool {
    std::vector<std::unique_ptr<thb::DeviceBuffer>> buffers;
    std::size_t next = 0;
};
DevicePrepared prepareOnDevice(const Scene& scene, const float* positions, const float* colors,
                               const std::int64_t* indices, int device, cudaStream_t stream,
                               thb::DeviceBuffer& triangles, thb::DeviceBuffer& tileOffsets,
                               thb::DeviceBuffer& tileLists, ScratchPool& pool);

// Rasterizes on `stream`: color [pixels][4], depth [pixels] (device), stats
// (device, 2 x u64: shaded pixels, depth passes; accumulated into).
cudaError_t rasterize(const RasterTriangle* triangles, const std::uint32_t* tileOffsets,
                      const std::uint32_t* tileLists, std::uint32_t tilesX, std::uint32_t tilesY,
                      std::uint32_t width, std::uint32_t height, const float* clear, float* color, float* depth,
                      unsigned long long* stats, cudaStream_t stream);

} // namespace thb::graphics
