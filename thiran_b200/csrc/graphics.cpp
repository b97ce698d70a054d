// Host side of the GPU renderer (see graphics.hpp): the reference's
// validation, f32 vertex transform, homogeneous clipping and screen setup
// (src/graphics/v0/Graphics.cpp:102-421), then tile binning. Built with
// -ffp-contract=off so every f32 / f64 operation rounds on its own, as the
// reference's volatile helpers make it (Graphics.cpp:22-41).
#include "graphics.hpp"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <thread>

#include "common.hpp"

namespace thb::graphics {
namespace {

[[noreturn]] void bad(const char* id) { fail(Category::Semantic, id, id); }

bool finite(float v) { return std::isfinite(v); }

struct ClipVertex {
    float p[4];
    float c[4];
};

// Signed distance to clip plane k: left, right, bottom, top, near, far.
float planeDistance(const ClipVertex& v, int k) {
    switch (k) {
    case 0: return v.p[0] + v.p[3];
    case 1: return v.p[3] + -v.p[0];
    case 2: return v.p[1] + v.p[3];
    case 3: return v.p[3] + -v.p[1];
    case 4: return v.p[2];
    default: return v.p[3] + -v.p[2];
    }
}

ClipVertex lerp(const ClipVertex& a, const ClipVertex& b, float t) {
    ClipVertex r;
    for (int k = 0; k < 4; ++k) {
        const float dp = b.p[k] + -a.p[k];
        const float sp = t * dp;
        r.p[k] = a.p[k] + sp;
        const float dc = b.c[k] + -a.c[k];
        const float sc = t * dc;
        r.c[k] = a.c[k] + sc;
    }
    return r;
}

// Worker threads for `items` independent items (1 below 4096; at most
// THB_HOST_THREADS when set, else the hardware threads, 64 at most).
unsigned workerCount(std::uint64_t items) {
    if (items < 4096) return 1;
    unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    if (const char* env = std::getenv("THB_HOST_THREADS")) hw = std::max(1, std::atoi(env));
    return static_cast<unsigned>(std::min<std::uint64_t>({hw, 64u, items / 2048}));
}

// Runs f(worker, begin, end) over `threads` contiguous chunks of [0, items).
// f must not throw.
template <class F>
void parallelChunks(std::uint64_t items, unsigned threads, F&& f) {
    if (threads <= 1) {
        f(0u, 0ull, items);
        return;
    }
    std::vector<std::thread> pool;
    const std::uint64_t per = (items + threads - 1) / threads;
    for (unsigned w = 0; w < threads; ++w) {
        const std::uint64_t begin = std::min<std::uint64_t>(items, w * per);
        const std::uint64_t end = std::min<std::uint64_t>(items, begin + per);
        pool.emplace_back([&f, w, begin, end] { f(w, begin, end); });
    }
    for (auto& t : pool) t.join();
}

// One Sutherland-Hodgman pass (Graphics.cpp:126-149); -1 where the reference
// fails with TH019-CLIP-NUMERIC.
int clipPlane(const ClipVertex* in, int n, int plane, ClipVertex* out) {
    if (n == 0) return 0;
    int m = 0;
    ClipVertex prev = in[n - 1];
    float prevDistance = planeDistance(prev, plane);
    bool prevInside = prevDistance >= 0.0f;
    for (int i = 0; i < n; ++i) {
        const float d = planeDistance(in[i], plane);
        const bool inside = d >= 0.0f;
        if (prevInside != inside) {
            const float den = prevDistance + -d;
            if (den == 0.0f || !finite(den)) return -1;
            const float amount = prevDistance / den;
            if (!finite(amount)) return -1;
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

double edge(const ScreenVertex& a, const ScreenVertex& b, double x, double y) {
    const double first = (b.x - a.x) * (y - a.y);
    const double second = (b.y - a.y) * (x - a.x);
    return first - second;
}

bool topLeft(const ScreenVertex& a, const ScreenVertex& b) {
    const double dx = b.x - a.x, dy = b.y - a.y;
    return dy < 0.0 || (dy == 0.0 && dx > 0.0);
}

// prepareScreenTriangle (Graphics.cpp:348-372).
bool toScreen(const ClipVertex* t, std::uint64_t w, std::uint64_t h, ScreenVertex* s) {
    for (int i = 0; i < 3; ++i) {
        const float cw = t[i].p[3];
        if (!finite(cw) || cw <= 1.0e-7f) return false;
        const float x = t[i].p[0] / cw, y = t[i].p[1] / cw, z = t[i].p[2] / cw;
        if (!finite(x) || !finite(y) || !finite(z)) return false;
        s[i].x = (static_cast<double>(x) * 0.5 + 0.5) * static_cast<double>(w);
        s[i].y = (0.5 - static_cast<double>(y) * 0.5) * static_cast<double>(h);
        s[i].depth = z;
        s[i].rw = 1.0 / static_cast<double>(cw);
        std::memcpy(s[i].c, t[i].c, sizeof s[i].c);
    }
    const double area = edge(s[0], s[1], s[2].x, s[2].y);
    if (!std::isfinite(area) || std::fabs(area) <= 1.0e-12) return false;
    if (area < 0.0) std::swap(s[1], s[2]);
    return true;
}

// The rasterizer's bounding box and edge setup (Graphics.cpp:253-276).
bool pack(const ScreenVertex* v, std::uint64_t w, std::uint64_t h, RasterTriangle& t) {
    const double minX = std::min({v[0].x, v[1].x, v[2].x}), maxX = std::max({v[0].x, v[1].x, v[2].x});
    const double minY = std::min({v[0].y, v[1].y, v[2].y}), maxY = std::max({v[0].y, v[1].y, v[2].y});
    auto x0 = static_cast<std::int64_t>(std::ceil(minX - 0.5)), x1 = static_cast<std::int64_t>(std::floor(maxX - 0.5));
    auto y0 = static_cast<std::int64_t>(std::ceil(minY - 0.5)), y1 = static_cast<std::int64_t>(std::floor(maxY - 0.5));
    x0 = std::max<std::int64_t>(x0, 0);
    y0 = std::max<std::int64_t>(y0, 0);
    x1 = std::min<std::int64_t>(x1, static_cast<std::int64_t>(w) - 1);
    y1 = std::min<std::int64_t>(y1, static_cast<std::int64_t>(h) - 1);
    if (x0 > x1 || y0 > y1) return false;
    std::memset(&t, 0, sizeof t);
    for (int i = 0; i < 3; ++i) {
        t.x[i] = v[i].x;
        t.y[i] = v[i].y;
        t.depth[i] = v[i].depth;
        t.rw[i] = v[i].rw;
        std::memcpy(t.color[i], v[i].c, sizeof t.color[i]);
    }
    t.area = edge(v[0], v[1], v[2].x, v[2].y);
    t.x0 = static_cast<std::int32_t>(x0);
    t.x1 = static_cast<std::int32_t>(x1);
    t.y0 = static_cast<std::int32_t>(y0);
    t.y1 = static_cast<std::int32_t>(y1);
    t.inclusive = (topLeft(v[1], v[2]) ? 1u : 0u) | (topLeft(v[2], v[0]) ? 2u : 0u) | (topLeft(v[0], v[1]) ? 4u : 0u);
    return true;
}

void multiply(const float* a, const float* b, float* out) {
    float r[16];
    for (int row = 0; row < 4; ++row)
        for (int col = 0; col < 4; ++col) {
            float acc = 0.0f;
            for (int k = 0; k < 4; ++k) {
                const float p = a[row * 4 + k] * b[k * 4 + col];
                acc = acc + p;
            }
            r[row * 4 + col] = acc;
        }
    std::memcpy(out, r, sizeof r);
}

} // namespace

Scene validate(const float* positions, std::uint64_t vertices, const std::int64_t* indices, std::uint64_t triangles,
               const float* colors, const float* model, const float* view, const float* projection,
               std::uint64_t width, std::uint64_t height, const float* clear) {
    // validateGeometry (Graphics.cpp:322-342), validateFramebuffer (:210-226).
    // Each check scans its whole array on host threads; the checks keep the
    // reference's order, so the first failing check gives the id.
    if ((vertices && (!positions || !colors)) || (triangles && !indices) || !model || !view || !projection || !clear)
        fail(Category::Validation, "TH019-GEOMETRY-SHAPE", "null geometry, matrix or clear colour");
    auto anyOf = [](std::uint64_t n, auto&& failing) {
        const unsigned threads = workerCount(n);
        std::vector<char> found(std::max(1u, threads), 0);
        parallelChunks(n, threads, [&](unsigned w, std::uint64_t begin, std::uint64_t end) {
            for (std::uint64_t k = begin; k < end; ++k)
                if (failing(k)) {
                    found[w] = 1;
                    return;
                }
        });
        return std::find(found.begin(), found.end(), 1) != found.end();
    };
    if (anyOf(vertices * 3, [&](std::uint64_t k) { return !finite(positions[k]); })) bad("TH019-NONFINITE-VERTEX");
    if (anyOf(vertices * 4, [&](std::uint64_t k) { return !finite(colors[k]) || colors[k] < 0.0f || colors[k] > 1.0f; }))
        bad("TH019-COLOR-RANGE");
    if (anyOf(triangles * 3,
              [&](std::uint64_t k) { return indices[k] < 0 || static_cast<std::uint64_t>(indices[k]) >= vertices; }))
        bad("TH019-INDEX");
    for (int k = 0; k < 4; ++k)
        if (!finite(clear[k]) || clear[k] < 0.0f || clear[k] > 1.0f) bad("TH019-CLEAR-COLOR");
    const auto limit = static_cast<std::uint64_t>(std::numeric_limits<std::int32_t>::max());
    if (width > limit || height > limit) bad("TH019-FRAMEBUFFER-DIMENSION");
    const std::uint64_t pixels = checkedMul(width, height);
    checkedMul(pixels, 16);
    for (int k = 0; k < 16; ++k)
        if (!finite(model[k]) || !finite(view[k]) || !finite(projection[k])) bad("TH019-NONFINITE-MATRIX");

    Scene scene;
    scene.width = width;
    scene.height = height;
    scene.vertices = vertices;
    scene.triangles = triangles;
    std::memcpy(scene.clear, clear, sizeof scene.clear);
    float mv[16];
    multiply(view, model, mv);
    multiply(projection, mv, scene.mvp);
    for (int k = 0; k < 16; ++k)
        if (!finite(mv[k]) || !finite(scene.mvp[k])) bad("TH019-NONFINITE-MATRIX");
    // (Tile counts of 2^32 and more fail with TH019-FRAMEBUFFER-SIZE after
    // clipping, where the triangle count is checked too.)
    scene.tilesX = static_cast<std::uint32_t>(std::min<std::uint64_t>((width + kTile - 1) / kTile, ~0u));
    scene.tilesY = static_cast<std::uint32_t>(std::min<std::uint64_t>((height + kTile - 1) / kTile, ~0u));
    return scene;
}

Prepared prepare(const float* positions, std::uint64_t vertices, const std::int64_t* indices, std::uint64_t triangles,
                 const float* colors, const float* model, const float* view, const float* projection,
                 std::uint64_t width, std::uint64_t height, const float* clear) {
    const Scene scene = validate(positions, vertices, indices, triangles, colors, model, view, projection, width,
                                 height, clear);
    Prepared out;
    out.width = width;
    out.height = height;
    std::memcpy(out.clear, scene.clear, sizeof out.clear);
    out.inputTriangles = triangles;
    const float* mvp = scene.mvp;
    // Transform, clip and bin in contiguous chunks on host threads; chunk
    // results are joined in order, so the output equals a serial pass. The
    // first failure of any chunk is the reference's failure too: every
    // failure here has one id per step (NONFINITE-TRANSFORMED, CLIP-NUMERIC).
    const unsigned threads = workerCount(std::max(vertices, triangles));
    std::vector<ClipVertex> clip(vertices);
    std::vector<char> transformFailed(threads, 0);
    parallelChunks(vertices, threads, [&](unsigned w, std::uint64_t begin, std::uint64_t end) {
        for (std::uint64_t v = begin; v < end; ++v) {
            const float in[4] = {positions[v * 3], positions[v * 3 + 1], positions[v * 3 + 2], 1.0f};
            for (int row = 0; row < 4; ++row) {
                float acc = 0.0f;
                for (int col = 0; col < 4; ++col) {
                    const float p = mvp[row * 4 + col] * in[col];
                    acc = acc + p;
                }
                if (!finite(acc)) transformFailed[w] = 1;
                clip[v].p[row] = acc;
            }
            std::memcpy(clip[v].c, colors + v * 4, sizeof clip[v].c);
        }
    });
    for (char f : transformFailed)
        if (f) bad("TH019-NONFINITE-TRANSFORMED");

    struct Chunk {
        std::vector<RasterTriangle> triangles;
        std::uint64_t postClip = 0;
        bool clipFailed = false;
    };
    std::vector<Chunk> chunks(threads);
    parallelChunks(triangles, threads, [&](unsigned w, std::uint64_t begin, std::uint64_t end) {
        Chunk& chunk = chunks[w];
        ClipVertex poly[2][16];
        for (std::uint64_t t = begin; t < end && !chunk.clipFailed; ++t) {
            int n = 3;
            for (int c = 0; c < 3; ++c) poly[0][c] = clip[static_cast<std::size_t>(indices[t * 3 + c])];
            int cur = 0;
            for (int plane = 0; plane < 6 && n >= 3; ++plane) {
                n = clipPlane(poly[cur], n, plane, poly[cur ^ 1]);
                if (n < 0) {
                    chunk.clipFailed = true;
                    break;
                }
                cur ^= 1;
            }
            if (n < 3) continue;
            for (int c = 1; c + 1 < n; ++c) {
                ++chunk.postClip;
                const ClipVertex tri[3] = {poly[cur][0], poly[cur][c], poly[cur][c + 1]};
                ScreenVertex s[3];
                RasterTriangle packed;
                if (toScreen(tri, width, height, s) && pack(s, width, height, packed)) chunk.triangles.push_back(packed);
            }
        }
    });
    std::uint64_t total = 0;
    for (const auto& c : chunks) {
        if (c.clipFailed) bad("TH019-CLIP-NUMERIC");
        out.postClipTriangles += c.postClip;
        total += c.triangles.size();
    }
    if (total > std::numeric_limits<std::uint32_t>::max()) bad("TH019-FRAMEBUFFER-SIZE");
    out.triangles.reserve(total);
    for (auto& c : chunks) {
        out.triangles.insert(out.triangles.end(), c.triangles.begin(), c.triangles.end());
        std::vector<RasterTriangle>().swap(c.triangles);
    }

    // Tiles of 16x16 pixels; each list keeps submission order: per-chunk
    // counts, offsets = tile-major then chunk-major prefix sums, parallel fill.
    out.tilesX = scene.tilesX;
    out.tilesY = scene.tilesY;
    const std::uint64_t tiles = static_cast<std::uint64_t>(out.tilesX) * out.tilesY;
    if (tiles >= std::numeric_limits<std::uint32_t>::max()) bad("TH019-FRAMEBUFFER-SIZE");
    const std::uint64_t count = out.triangles.size();
    const unsigned binThreads = tiles * workerCount(count) > (64ull << 20) ? 1 : workerCount(count);
    std::vector<std::uint64_t> counts(binThreads * tiles, 0);
    auto forTiles = [&](const RasterTriangle& t, auto&& f) {
        for (std::int32_t ty = t.y0 / kTile; ty <= t.y1 / kTile; ++ty)
            for (std::int32_t tx = t.x0 / kTile; tx <= t.x1 / kTile; ++tx) f(static_cast<std::uint64_t>(ty) * out.tilesX + tx);
    };
    parallelChunks(count, binThreads, [&](unsigned w, std::uint64_t begin, std::uint64_t end) {
        std::uint64_t* c = counts.data() + w * tiles;
        for (std::uint64_t i = begin; i < end; ++i) forTiles(out.triangles[i], [&](std::uint64_t k) { ++c[k]; });
    });
    out.tileOffsets.assign(tiles + 1, 0);
    std::vector<std::uint64_t> starts(binThreads * tiles);
    std::uint64_t entries = 0;
    for (std::uint64_t k = 0; k < tiles; ++k) {
        out.tileOffsets[k] = static_cast<std::uint32_t>(std::min<std::uint64_t>(entries, ~0u));
        for (unsigned w = 0; w < binThreads; ++w) {
            starts[w * tiles + k] = entries;
            entries += counts[w * tiles + k];
        }
    }
    if (entries >= std::numeric_limits<std::uint32_t>::max()) bad("TH019-FRAMEBUFFER-SIZE");
    out.tileOffsets[tiles] = static_cast<std::uint32_t>(entries);
    out.tileLists.resize(entries);
    parallelChunks(count, binThreads, [&](unsigned w, std::uint64_t begin, std::uint64_t end) {
        std::uint64_t* cursor = starts.data() + w * tiles;
        for (std::uint64_t i = begin; i < end; ++i)
            forTiles(out.triangles[i], [&](std::uint64_t k) { out.tileLists[cursor[k]++] = static_cast<std::uint32_t>(i); });
    });
    return out;
}

} // namespace thb::graphics
