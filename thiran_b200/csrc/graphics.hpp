// GPU renderer of the reference's software rasterizer
// (src/graphics/v0/Graphics.cpp, GPU backend src/graphics/v0/GraphicsGpu.cpp).
//
// Split as in the reference: validation, the f32 vertex transform and
// homogeneous clipping run on the host (its prepareRender, shared by its CPU
// and GPU backends, Graphics.cpp:374-421), so the post-clip triangles are the
// same bits as on the CPU. The rasterizer runs on the GPU: screen triangles
// are binned into 16x16-pixel tiles in submission order, and one thread per
// pixel walks its tile's list in that order with the reference's f64
// edge / barycentric / perspective-correct arithmetic and strict-less depth
// test, so colour, depth and both pixel counters equal the sequential CPU
// result. (The reference's GPU kernel walks every triangle for every pixel.)
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

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

// Rasterizes on `stream`: color [pixels][4], depth [pixels] (device), stats
// (device, 2 x u64: shaded pixels, depth passes; accumulated into).
cudaError_t rasterize(const RasterTriangle* triangles, const std::uint32_t* tileOffsets,
                      const std::uint32_t* tileLists, std::uint32_t tilesX, std::uint32_t tilesY,
                      std::uint32_t width, std::uint32_t height, const float* clear, float* color, float* depth,
                      unsigned long long* stats, cudaStream_t stream);

} // namespace thb::graphics
