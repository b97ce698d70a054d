// extern "C" surface of libthiran_b200.so (declared in include/thiran_b200.h).
#include <chrono>
#include <cmath>
#include <cstring>
#include <fstream>
#include <memory>
#include <thread>

#include <array>

#include "artifact.hpp"
#include "gemm.hpp"
#include "graphics.hpp"
#include "model.hpp"
#include "mlp.hpp"
#include "runtime.hpp"

struct thb_region {
    std::shared_ptr<thb::CompiledRegion> impl;
};

struct thb_pending {
    std::unique_ptr<thb::Pending> impl;
};

struct thb_mlp {
    int device = 0;
    int smCount = 148;
    thb::mlp::Buffers b;
    thb::mlp::GemmTimer timer;
    std::uint32_t reduceEpoch = 0;  // forward/backward passes since the all-reduce was bound
    bool weightsUpdated = false;    // the last pass applied the weight updates in its all-reduce
    // The session's own W, bf16 W and dW buffers (per layer), to which
    // removing a reduction or update binding returns.
    float* ownW[2] = {};
    void* ownWb[2] = {};
    float* ownDw[2] = {};
    std::vector<std::unique_ptr<thb::DeviceBuffer>> owned;
    ~thb_mlp() {
        for (auto& e : timer.events)
            if (e) cudaEventDestroy(e);
    }
    void* alloc(std::size_t bytes) {
        owned.push_back(std::make_unique<thb::DeviceBuffer>());
        owned.back()->reserve(bytes, device);
        return owned.back()->ptr;
    }
};

namespace {

using namespace thb;

template <class F>
int guarded(char* failure, std::uint64_t cap, F&& body) noexcept {
    try {
        return body();
    } catch (const Failure& f) {
        writeText(failure, cap, f.text());
        return f.status();
    } catch (const std::exception& e) {
        writeText(failure, cap, std::string("GPU-INTERNAL: ") + e.what());
        return THB_STATUS_UNKNOWN;
    } catch (...) {
        writeText(failure, cap, "GPU-INTERNAL: unknown native failure");
        return THB_STATUS_UNKNOWN;
    }
}

void cudaCheck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) fail(Category::Runtime, "GPU-RUNTIME", std::string(what) + ": " + cudaGetErrorString(e));
}

// Validates the argument records against the region's Input nodes (the
// preflight of src/backend/v0/NativeGpu.cpp:73-106) and binds them. In host
// mode tensors are uploaded into the region's input buffers; identical host
// storages are uploaded once (NativeGpu.cpp:961-971).
std::vector<Value> bind(CompiledRegion& region, const thb_abi_arg* args, std::uint64_t argc, bool hostMode,
                        cudaStream_t stream, thb_evidence& ev, std::uint64_t* distinctReads) {
    const Region& r = region.region();
    if (argc != r.inputs.size()) fail(Category::Unsupported, "GPU-INPUT-ARITY", "GPU input arity mismatch");
    if (argc && !args) fail(Category::Validation, "GPU-INPUT-ARITY", "argument array is null");
    std::vector<Value> values(argc);
    for (std::uint64_t i = 0; i < argc; ++i) {
        const Node& node = r.at(r.inputs[i]);
        const thb_abi_arg& a = args[i];
        Value& v = values[i];
        if (a.kind == THB_KIND_TENSOR) {
            if (!node.tensor()) fail(Category::Unsupported, "GPU-INPUT-TYPE", "tensor supplied for scalar GPU input");
            if (a.dtype != static_cast<std::uint32_t>(node.dtype))
                fail(Category::Unsupported, "GPU-INPUT-TYPE", "tensor dtype disagrees with the region input");
            if (a.rank != node.rank || !a.shape)
                fail(Category::Unsupported, "GPU-INPUT-SHAPE", "tensor rank disagrees with the region input");
            std::uint64_t count = 1;
            for (std::uint32_t d = 0; d < a.rank; ++d) {
                if (node.extent[d] >= 0 && a.shape[d] != static_cast<std::uint64_t>(node.extent[d]))
                    fail(Category::Unsupported, "GPU-INPUT-SHAPE", "tensor extent disagrees with the region input");
                count = checkedMul(count, a.shape[d]);
                v.shape[d] = a.shape[d];
            }
            if (count != a.count) fail(Category::Unsupported, "GPU-INPUT-SHAPE", "element count disagrees with shape");
            if (a.reserved & 1u)
                fail(Category::Unsupported, "GPU-UNSUPPORTED-LAYOUT",
                     "native GPU requires materialized offset-zero contiguous row-major tensors");
            if (count && !a.data) fail(Category::Unsupported, "GPU-INPUT-SHAPE", "tensor data pointer is null");
            v.tensor = true;
            v.onDevice = true;
            v.dtype = node.dtype;
            v.rank = a.rank;
            v.data = const_cast<void*>(a.data);
        } else if (a.kind == THB_KIND_SCALAR) {
            if (node.tensor()) fail(Category::Unsupported, "GPU-INPUT-TYPE", "scalar supplied for tensor GPU input");
            if (a.dtype != static_cast<std::uint32_t>(node.dtype) || a.count != 1 || !a.data)
                fail(Category::Unsupported, "GPU-INPUT-TYPE", "scalar dtype disagrees with the region input");
            v.dtype = node.dtype;
            if (node.dtype == DType::I64) std::memcpy(&v.i64, a.data, 8);
            else std::memcpy(&v.f32, a.data, 4);
        } else {
            fail(Category::Unsupported, "GPU-INPUT-TYPE", "argument kind is neither scalar nor tensor");
        }
    }
    std::uint64_t reads = 0;
    if (hostMode) {
        // Host pointer -> (device copy, bytes copied). A later argument at the
        // same address reuses the copy only when the copy covers all of it.
        std::map<const void*, std::pair<void*, std::size_t>> uploaded;
        for (std::uint64_t i = 0; i < argc; ++i) {
            Value& v = values[i];
            if (!v.tensor) continue;
            const void* host = v.data;
            auto found = uploaded.find(host);
            if (found != uploaded.end() && v.bytes() && v.bytes() <= found->second.second) {
                v.data = found->second.first;
                continue;
            }
            ++reads;
            DeviceBuffer& buffer = region.inputBuffer(i);
            if (buffer.reserve(v.bytes(), region.device())) {
                ++ev.allocation_count;
                ev.allocation_bytes_requested += v.bytes();
            }
            if (v.bytes()) {
                cudaCheck(cudaMemcpyAsync(buffer.ptr, host, v.bytes(), cudaMemcpyHostToDevice, stream),
                          "cudaMemcpyAsync(upload)");
                ++ev.host_to_device_copies;
                ev.host_to_device_bytes += v.bytes();
                ++ev.input_storage_uploads;
            }
            if (v.bytes() > uploaded[host].second) uploaded[host] = {buffer.ptr, v.bytes()};
            v.data = buffer.ptr;
        }
    }
    if (distinctReads) *distinctReads = reads;
    return values;
}

void checkOutputCount(const Value& out, std::uint64_t outputCount, bool needBuffer, const void* output) {
    const std::uint64_t want = out.count();
    if (outputCount != want)
        fail(Category::Unsupported, "GPU-OUTPUT-SHAPE",
             "output buffer holds " + std::to_string(outputCount) + " elements, region output has " + std::to_string(want));
    if (needBuffer && want && !output) fail(Category::Unsupported, "GPU-OUTPUT-SHAPE", "output pointer is null");
}

// Copies a completed output into host memory (host scalars directly,
// device values through `stream`).
void downloadOutput(const Value& out, void* host, cudaStream_t stream, thb_evidence& ev) {
    if (out.tensor || out.onDevice) {
        if (out.bytes() && host) {
            cudaCheck(cudaMemcpyAsync(host, out.data, out.bytes(), cudaMemcpyDeviceToHost, stream), "cudaMemcpyAsync(result)");
            ++ev.device_to_host_copies;
            ev.device_to_host_bytes += out.bytes();
            ++ev.result_downloads;
        }
    } else if (host) {
        if (out.dtype == DType::I64) std::memcpy(host, &out.i64, 8);
        else std::memcpy(host, &out.f32, 4);
    }
}

bool pinnedHost(const void* p) {
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return attr.type == cudaMemoryTypeHost;
}

// Chunked, three-stream execution of a row-local region over pinned host
// buffers (see CompiledRegion::Lane). Returns false, having done nothing,
// when the region or the buffers do not qualify.
bool executePipelined(CompiledRegion& r, const std::vector<Value>& host, void* output, std::uint64_t outputCount,
                      cudaStream_t stream, thb_evidence& ev, std::uint32_t* stagedErrors) {
    constexpr std::size_t kMinBytes = 64ull << 20;
    // Bytes (inputs + output) per chunk; THB_CHUNK_MB overrides 48 MiB.
    static const std::size_t kChunkBytes = [] {
        const char* e = std::getenv("THB_CHUNK_MB");
        const long mb = e ? std::atol(e) : 0;
        return static_cast<std::size_t>(mb > 0 ? mb : 48) << 20;
    }();
    if (!r.rowLocal() || host.empty() || !output) return false;
    const Node& outNode = r.region().at(r.region().output);
    const std::uint64_t rows = host[0].shape[0];
    if (!host[0].tensor || rows == 0) return false;
    std::size_t total = 0, rowBytes = 0;
    for (const Value& v : host) {
        if (!v.tensor || v.shape[0] != rows || !pinnedHost(v.data)) return false;
        total += v.bytes();
        rowBytes += v.bytes() / rows;
    }
    if (outputCount % rows) return false;
    const std::size_t outRowBytes = static_cast<std::size_t>(outputCount / rows) * width(outNode.dtype);
    total += outRowBytes * rows;
    rowBytes += outRowBytes;
    if (total < kMinBytes || !pinnedHost(output)) return false;

    const std::uint64_t chunkRows = std::max<std::uint64_t>(1, kChunkBytes / rowBytes);
    cudaEvent_t cleared = r.lane(0).done;
    r.clearErrors(stream);
    cudaCheck(cudaEventRecord(cleared, stream), "cudaEventRecord(clear)");
    for (std::size_t k = 0; k < CompiledRegion::kLanes; ++k)
        cudaCheck(cudaStreamWaitEvent(r.lane(k).stream, cleared, 0), "cudaStreamWaitEvent");
    std::size_t used = 0;
    for (std::uint64_t start = 0, chunk = 0; start < rows; start += chunkRows, ++chunk) {
        const std::uint64_t n = std::min(chunkRows, rows - start);
        auto& lane = r.lane(chunk);
        used = std::max<std::size_t>(used, chunk + 1);
        std::vector<Value> part = host;
        for (std::size_t i = 0; i < host.size(); ++i) {
            const std::size_t rb = host[i].bytes() / rows;
            if (lane.inputs[i]->reserve(rb * chunkRows, r.device())) {
                ++ev.allocation_count;
                ev.allocation_bytes_requested += rb * chunkRows;
            }
            cudaCheck(cudaMemcpyAsync(lane.inputs[i]->ptr, static_cast<const char*>(host[i].data) + start * rb, rb * n,
                                      cudaMemcpyHostToDevice, lane.stream),
                      "cudaMemcpyAsync(upload chunk)");
            ++ev.host_to_device_copies;
            ev.host_to_device_bytes += rb * n;
            part[i].data = lane.inputs[i]->ptr;
            part[i].shape[0] = n;
        }
        if (lane.output.reserve(outRowBytes * chunkRows, r.device())) {
            ++ev.allocation_count;
            ev.allocation_bytes_requested += outRowBytes * chunkRows;
        }
        r.run(part, lane.stream, ev, lane.output.ptr, [&](const Value& o) {
            if (o.count() != n * (outputCount / rows))
                fail(Category::Unsupported, "GPU-OUTPUT-SHAPE", "output buffer size disagrees with the region output");
        });
        cudaCheck(cudaMemcpyAsync(static_cast<char*>(output) + start * outRowBytes, lane.output.ptr, outRowBytes * n,
                                  cudaMemcpyDeviceToHost, lane.stream),
                  "cudaMemcpyAsync(download chunk)");
        ++ev.device_to_host_copies;
        ev.device_to_host_bytes += outRowBytes * n;
    }
    ev.input_storage_uploads += host.size();
    ++ev.result_downloads;
    for (std::size_t k = 0; k < std::min(used, CompiledRegion::kLanes); ++k) {
        auto& lane = r.lane(k);
        cudaCheck(cudaEventRecord(lane.done, lane.stream), "cudaEventRecord(lane)");
        cudaCheck(cudaStreamWaitEvent(stream, lane.done, 0), "cudaStreamWaitEvent(lane)");
    }
    r.copyErrors(stream, stagedErrors);
    return true;
}

void waitEvent(cudaEvent_t event, std::uint64_t timeoutMs) {
    const auto start = std::chrono::steady_clock::now();
    unsigned sleepUs = 20;
    for (;;) {
        const cudaError_t e = cudaEventQuery(event);
        if (e == cudaSuccess) return;
        if (e != cudaErrorNotReady) cudaCheck(e, "cudaEventQuery");
        if (timeoutMs && std::chrono::steady_clock::now() - start > std::chrono::milliseconds(timeoutMs))
            fail(Category::Runtime, "GPU-TIMEOUT", "pending GPU execution did not complete in time");
        std::this_thread::sleep_for(std::chrono::microseconds(sleepUs));
        sleepUs = std::min(sleepUs * 2, 1000u);
    }
}

} // namespace

extern "C" {

int thb_backend_built(void) { return 1; }

uint32_t thb_abi_version(void) { return THB_ABI_VERSION; }

int thb_probe(int device, thb_device_info* out) {
    if (!out) return THB_STATUS_ABI;
    std::memset(out, 0, sizeof *out);
    out->backend_built = 1;
    out->selected_device = -1;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess) {
        cudaGetLastError();
        writeText(out->error_code, sizeof out->error_code, "GPU-DRIVER-NOT-FOUND");
        writeText(out->name, sizeof out->name, cudaGetErrorString(e));
        return THB_STATUS_BACKEND;
    }
    out->driver_loaded = 1;
    int version = 0;
    cudaDriverGetVersion(&version);
    out->driver_version = version;
    out->device_count = count;
    if (device < 0 || device >= count) {
        writeText(out->error_code, sizeof out->error_code, "GPU-INVALID-DEVICE");
        return THB_STATUS_BACKEND;
    }
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
        cudaGetLastError();
        writeText(out->error_code, sizeof out->error_code, "GPU-INVALID-DEVICE");
        return THB_STATUS_BACKEND;
    }
    out->device_available = 1;
    out->selected_device = device;
    out->compute_major = prop.major;
    out->compute_minor = prop.minor;
    out->sm_count = prop.multiProcessorCount;
    writeText(out->name, sizeof out->name, prop.name);
    return THB_STATUS_OK;
}

int thb_region_compile(const thb_region_desc* desc, thb_plan_options options, int device, thb_region** out,
                       char* failure, uint64_t cap) {
    return guarded(failure, cap, [&] {
        if (!desc || !out) fail(Category::Validation, "GPU-INVALID-REGION", "region descriptor or result is null");
        *out = nullptr;
        PlanOptions opts;
        opts.enableReuse = options.enable_reuse != 0;
        opts.enableFusion = options.enable_fusion != 0;
        auto impl = std::make_shared<CompiledRegion>(*desc, opts, device);
        *out = new thb_region{std::move(impl)};
        return THB_STATUS_OK;
    });
}

void thb_region_release(thb_region* region) { delete region; }

// ---- artifacts ------------------------------------------------------------------------

struct thb_artifact {
    thb::artifact::Artifact impl;
};

int thb_artifact_load(const void* bytes, uint64_t size, thb_artifact** out, char* failure, uint64_t cap) {
    return guarded(failure, cap, [&] {
        if (!out || (!bytes && size)) fail(Category::Validation, "ARTIFACT-IO", "null artifact bytes or result");
        *out = nullptr;
        auto a = std::make_unique<thb_artifact>();
        a->impl = thb::artifact::load(std::string(static_cast<const char*>(bytes), static_cast<std::size_t>(size)));
        *out = a.release();
        return THB_STATUS_OK;
    });
}

int thb_artifact_load_file(const char* path, thb_artifact** out, char* failure, uint64_t cap) {
    return guarded(failure, cap, [&] {
        if (!path || !out) fail(Category::Validation, "ARTIFACT-IO", "null path or result");
        *out = nullptr;
        std::ifstream in(path, std::ios::binary | std::ios::ate);
        if (!in) fail(Category::Validation, "ARTIFACT-IO", std::string("cannot open ") + path);
        const auto end = in.tellg();
        // The reference's file limit: payload + region + 4 MiB of manifest.
        if (end < 0 || static_cast<std::uint64_t>(end) > (512ull << 20) + (64ull << 20) + (4ull << 20))
            fail(Category::Validation, "ARTIFACT-IO", "file size exceeds V0 limit");
        std::string bytes(static_cast<std::size_t>(end), '\0');
        in.seekg(0);
        if (!bytes.empty() && !in.read(bytes.data(), end)) fail(Category::Validation, "ARTIFACT-IO", "short file read");
        auto a = std::make_unique<thb_artifact>();
        a->impl = thb::artifact::load(bytes);
        *out = a.release();
        return THB_STATUS_OK;
    });
}

void thb_artifact_release(thb_artifact* artifact) { delete artifact; }

int thb_artifact_inspect(const thb_artifact* artifact, char* buffer, uint64_t capacity, uint64_t* needed) {
    if (!artifact) return THB_STATUS_ABI;
    try {
        const std::string text = thb::artifact::inspect(artifact->impl);
        if (needed) *needed = text.size() + 1;
        writeText(buffer, capacity, text);
        return (capacity >= text.size() + 1 || !buffer) ? THB_STATUS_OK : THB_STATUS_ABI;
    } catch (...) {
        return THB_STATUS_UNKNOWN;
    }
}

int thb_artifact_compile(const thb_artifact* artifact, int device, thb_region** out, char* failure, uint64_t cap) {
    return guarded(failure, cap, [&] {
        if (!artifact || !out) fail(Category::Validation, "ARTIFACT-IO", "null artifact or result");
        *out = nullptr;
        const auto& a = artifact->impl;
        PlanOptions opts;
        opts.enableReuse = a.manifest.enableReuse;
        opts.enableFusion = a.manifest.enableFusion;
        const std::string* cubin = a.engineCubin.empty() ? nullptr : &a.engineCubin;
        auto impl = std::make_shared<CompiledRegion>(a.region, opts, device, cubin);
        *out = new thb_region{std::move(impl)};
        return THB_STATUS_OK;
    });
}

// ---- renderer ---------------------------------------------------------------------------

namespace {

// Per-device state of thb_render: its stream, the uploaded geometry, the
// prepared triangles and tile lists, the framebuffer and the preparation's
// scratch, all reused by the next call. The workspaces live for the
// process, like the driver context they belong to.
struct RenderWorkspace {
    std::mutex mutex;
    cudaStream_t stream = nullptr;
    DeviceBuffer positions, colors, indices, triangles, offsets, lists, color, depth, counters;
    thb::graphics::ScratchPool pool;
};

RenderWorkspace& renderWorkspace(int device) {
    static std::mutex guard;
    static std::map<int, RenderWorkspace*> workspaces;
    std::lock_guard<std::mutex> lock(guard);
    RenderWorkspace*& w = workspaces[device];
    if (!w) w = new RenderWorkspace();
    return *w;
}

} // namespace

int thb_render(int device, const float* positions, uint64_t vertices, const int64_t* indices, uint64_t triangles,
               const float* colors, const float* model, const float* view, const float* projection, uint64_t width,
               uint64_t height, const float* clear, float* color, float* depth, uint64_t* stats, thb_evidence* evidence,
               char* failure, uint64_t cap) {
    thb_evidence ev{};
    const int status = guarded(failure, cap, [&] {
        namespace gfx = thb::graphics;
        const float zero[4] = {0, 0, 0, 0};
        // The transform, clipping, setup and binning run on the GPU unless
        // THB_RENDER_PREP=host (the same pipeline on host threads).
        static const bool hostPrep = [] {
            const char* e = std::getenv("THB_RENDER_PREP");
            return e && std::strcmp(e, "host") == 0;
        }();
        // Validation first: invalid geometry fails before any driver call.
        gfx::Prepared p;
        gfx::Scene scene;
        if (hostPrep)
            p = gfx::prepare(positions, vertices, indices, triangles, colors, model, view, projection, width, height,
                             clear ? clear : zero);
        else
            scene = gfx::validate(positions, vertices, indices, triangles, colors, model, view, projection, width,
                                  height, clear ? clear : zero);
        const std::uint64_t pixels = width * height;
        if (pixels && (!color || !depth)) fail(Category::Validation, "TH019-FRAMEBUFFER-TENSOR", "null output buffer");
        useDevice(device);
        // The device's render workspace: stream and buffers kept from call to
        // call (grown when a frame needs more), one render at a time.
        RenderWorkspace& ws = renderWorkspace(device);
        std::lock_guard<std::mutex> lock(ws.mutex);
        if (!ws.stream)
            cudaCheck(cudaStreamCreateWithFlags(&ws.stream, cudaStreamNonBlocking), "cudaStreamCreateWithFlags");
        cudaStream_t stream = ws.stream;
        DeviceBuffer &tri = ws.triangles, &offsets = ws.offsets, &lists = ws.lists, &colorBuf = ws.color,
                     &depthBuf = ws.depth, &counters = ws.counters;
        auto upload = [&](DeviceBuffer& b, const void* host, std::size_t bytes) {
            if (!bytes) return;
            if (b.reserve(bytes, device)) {
                ++ev.allocation_count;
                ev.allocation_bytes_requested += bytes;
            }
            cudaCheck(cudaMemcpyAsync(b.ptr, host, bytes, cudaMemcpyHostToDevice, stream), "cudaMemcpyAsync(render input)");
            ++ev.host_to_device_copies;
            ev.host_to_device_bytes += bytes;
        };
        std::uint64_t postClip = 0;
        if (hostPrep) {
            upload(tri, p.triangles.data(), p.triangles.size() * sizeof(gfx::RasterTriangle));
            upload(offsets, p.tileOffsets.data(), p.tileOffsets.size() * sizeof(std::uint32_t));
            upload(lists, p.tileLists.data(), p.tileLists.size() * sizeof(std::uint32_t));
            postClip = p.postClipTriangles;
        } else {
            upload(ws.positions, positions, vertices * 3 * sizeof(float));
            upload(ws.colors, colors, vertices * 4 * sizeof(float));
            upload(ws.indices, indices, triangles * 3 * sizeof(std::int64_t));
            const gfx::DevicePrepared d = gfx::prepareOnDevice(
                scene, static_cast<const float*>(ws.positions.ptr), static_cast<const float*>(ws.colors.ptr),
                static_cast<const std::int64_t*>(ws.indices.ptr), device, stream, tri, offsets, lists, ws.pool);
            if (d.failure) fail(Category::Semantic, d.failure, d.failure);
            ev.kernel_launches += d.launches;
            ev.allocation_count += d.allocations;
            ev.synchronizations += 2;
            postClip = d.postClipTriangles;
            p.tilesX = scene.tilesX;
            p.tilesY = scene.tilesY;
            std::memcpy(p.clear, scene.clear, sizeof p.clear);
        }
        if (counters.reserve(2 * sizeof(unsigned long long), device)) ++ev.allocation_count;
        cudaCheck(cudaMemsetAsync(counters.ptr, 0, 2 * sizeof(unsigned long long), stream), "cudaMemsetAsync");
        if (pixels) {
            if (colorBuf.reserve(pixels * 16, device)) {
                ++ev.allocation_count;
                ev.allocation_bytes_requested += pixels * 16;
            }
            if (depthBuf.reserve(pixels * 4, device)) {
                ++ev.allocation_count;
                ev.allocation_bytes_requested += pixels * 4;
            }
            cudaCheck(gfx::rasterize(static_cast<const gfx::RasterTriangle*>(tri.ptr),
                                     static_cast<const std::uint32_t*>(offsets.ptr),
                                     static_cast<const std::uint32_t*>(lists.ptr), p.tilesX, p.tilesY,
                                     static_cast<std::uint32_t>(width), static_cast<std::uint32_t>(height), p.clear,
                                     static_cast<float*>(colorBuf.ptr), static_cast<float*>(depthBuf.ptr),
                                     static_cast<unsigned long long*>(counters.ptr), stream),
                      "raster launch");
            ++ev.kernel_launches;
            cudaCheck(cudaMemcpyAsync(color, colorBuf.ptr, pixels * 16, cudaMemcpyDeviceToHost, stream), "cudaMemcpyAsync(color)");
            cudaCheck(cudaMemcpyAsync(depth, depthBuf.ptr, pixels * 4, cudaMemcpyDeviceToHost, stream), "cudaMemcpyAsync(depth)");
            ev.device_to_host_copies += 2;
            ev.device_to_host_bytes += pixels * 20;
        }
        unsigned long long counts[2] = {0, 0};
        cudaCheck(cudaMemcpyAsync(counts, counters.ptr, sizeof counts, cudaMemcpyDeviceToHost, stream), "cudaMemcpyAsync(stats)");
        cudaCheck(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
        ++ev.synchronizations;
        if (stats) {
            stats[0] = triangles;
            stats[1] = postClip;
            stats[2] = counts[0];
            stats[3] = counts[1];
        }
        return THB_STATUS_OK;
    });
    if (evidence) *evidence = ev;
    return status;
}

// ---- model bundles ----------------------------------------------------------------------

struct thb_model {
    thb::model::Bundle impl;
};

struct thb_model_session {
    std::shared_ptr<CompiledRegion> region;
    std::vector<std::int64_t> sources;                      // per artifact slot (model::slotSources)
    std::vector<thb::model::StoredValue> parameters;        // host copies (scalars are passed by value)
    std::vector<std::unique_ptr<DeviceBuffer>> resident;    // per parameter: its tensor in HBM
    std::vector<std::unique_ptr<DeviceBuffer>> publicSlots; // per artifact slot: public upload buffer
    std::vector<thb::artifact::Type> publicTypes;
    std::uint64_t residentBytes = 0;
};

static int loadModel(const std::string& bytes, const char* identity, thb_model** out) {
    const std::string expected = identity ? identity : "";
    auto m = std::make_unique<thb_model>();
    m->impl = thb::model::load(bytes, identity ? &expected : nullptr);
    *out = m.release();
    return THB_STATUS_OK;
}

int thb_model_load(const void* bytes, uint64_t size, const char* identity, thb_model** out, char* failure,
                   uint64_t cap) {
    return guarded(failure, cap, [&] {
        if (!out || (!bytes && size)) fail(Category::Validation, "MODEL-IO", "null bundle bytes or result");
        *out = nullptr;
        return loadModel(std::string(static_cast<const char*>(bytes), static_cast<std::size_t>(size)), identity, out);
    });
}

int thb_model_load_file(const char* path, const char* identity, thb_model** out, char* failure, uint64_t cap) {
    return guarded(failure, cap, [&] {
        if (!path || !out) fail(Category::Validation, "MODEL-IO", "null path or result");
        *out = nullptr;
        std::ifstream in(path, std::ios::binary | std::ios::ate);
        if (!in) fail(Category::Validation, "MODEL-IO", std::string("cannot open ") + path);
        const auto end = in.tellg();
        if (end < 0 || static_cast<std::uint64_t>(end) > (2ull << 30))
            fail(Category::Validation, "MODEL-IO", "file size exceeds V0 limit");
        std::string bytes(static_cast<std::size_t>(end), '\0');
        in.seekg(0);
        if (!bytes.empty() && !in.read(bytes.data(), end)) fail(Category::Validation, "MODEL-IO", "short file read");
        return loadModel(bytes, identity, out);
    });
}

void thb_model_release(thb_model* model) { delete model; }

int thb_model_inspect(const thb_model* model, char* buffer, uint64_t capacity, uint64_t* needed) {
    if (!model) return THB_STATUS_ABI;
    try {
        const std::string text = thb::model::inspect(model->impl);
        if (needed) *needed = text.size() + 1;
        writeText(buffer, capacity, text);
        return (capacity >= text.size() + 1 || !buffer) ? THB_STATUS_OK : THB_STATUS_ABI;
    } catch (...) {
        return THB_STATUS_UNKNOWN;
    }
}

int thb_model_compile(const thb_model* model, int device, thb_model_session** out, thb_evidence* evidence,
                      char* failure, uint64_t cap) {
    thb_evidence ev{};
    const int status = guarded(failure, cap, [&] {
        if (!model || !out) fail(Category::Validation, "MODEL-IO", "null model or result");
        *out = nullptr;
        const auto& b = model->impl;
        auto s = std::make_unique<thb_model_session>();
        s->sources = thb::model::slotSources(b);  // MODEL-BACKEND-UNAVAILABLE without a GPU artifact
        const auto& a = *b.gpu;
        PlanOptions opts;
        opts.enableReuse = a.manifest.enableReuse;
        opts.enableFusion = a.manifest.enableFusion;
        const std::string* cubin = a.engineCubin.empty() ? nullptr : &a.engineCubin;
        s->region = std::make_shared<CompiledRegion>(a.region, opts, device, cubin);
        s->publicTypes = b.publicInputs;
        s->publicSlots.resize(s->sources.size());
        // Frozen parameters go to HBM once; every later call reuses them.
        for (const auto& p : b.parameters) {
            s->parameters.push_back(p.value);
            s->resident.push_back(std::make_unique<DeviceBuffer>());
            if (p.value.kind != 2 || p.value.bytes.empty()) continue;
            s->resident.back()->reserve(p.value.bytes.size(), device);
            ++ev.allocation_count;
            ev.allocation_bytes_requested += p.value.bytes.size();
            cudaCheck(cudaMemcpy(s->resident.back()->ptr, p.value.bytes.data(), p.value.bytes.size(),
                                 cudaMemcpyHostToDevice),
                      "cudaMemcpy(parameter)");
            ++ev.host_to_device_copies;
            ev.host_to_device_bytes += p.value.bytes.size();
            s->residentBytes += p.value.bytes.size();
        }
        *out = s.release();
        return THB_STATUS_OK;
    });
    if (evidence) *evidence = ev;
    return status;
}

void thb_model_session_release(thb_model_session* session) { delete session; }

int thb_model_execute(thb_model_session* s, const thb_abi_arg* args, uint64_t argc, void* output,
                      uint64_t outputCount, thb_evidence* evidence, char* failure, uint64_t cap) {
    thb_evidence ev{};
    const int status = guarded(failure, cap, [&] {
        if (!s) fail(Category::Validation, "MODEL-IO", "null model session");
        if (argc != s->publicTypes.size())
            fail(Category::Validation, "MODEL-PUBLIC-INPUT-COUNT", "public inference input count mismatch");
        if (argc && !args) fail(Category::Validation, "MODEL-PUBLIC-INPUT-COUNT", "argument array is null");
        // validateRuntimeValue (src/model/v0/ModelBundle.cpp:86-110).
        for (uint64_t i = 0; i < argc; ++i) {
            const auto& t = s->publicTypes[i];
            const thb_abi_arg& a = args[i];
            const std::string where = "public input " + std::to_string(i) + ": ";
            if (a.kind != t.kind) fail(Category::Validation, "MODEL-PUBLIC-INPUT-ABI", where + "kind mismatch");
            if (a.dtype != t.dtype || a.rank != t.rank)
                fail(Category::Validation, "MODEL-PUBLIC-INPUT-ABI", where + "dtype/rank mismatch");
            for (std::size_t d = 0; d < t.extents.size(); ++d)
                if (t.extents[d] && (!a.shape || a.shape[d] != *t.extents[d]))
                    fail(Category::Validation, "MODEL-PUBLIC-INPUT-ABI", where + "shape mismatch");
            if (a.reserved & 1u) fail(Category::Validation, "MODEL-PUBLIC-INPUT-ABI", where + "non-contiguous layout");
        }
        CompiledRegion& r = *s->region;
        std::lock_guard<std::mutex> lock(r.mutex);
        r.planEvidence(ev);
        cudaCheck(cudaSetDevice(r.device()), "cudaSetDevice");
        cudaStream_t stream = r.stream();
        // Artifact-slot arguments: public tensors uploaded into their slot
        // buffers, parameters from HBM, scalars by value.
        std::vector<thb_abi_arg> slotArgs(s->sources.size());
        std::vector<std::array<std::uint64_t, 2>> shapes(s->sources.size());
        for (std::size_t k = 0; k < s->sources.size(); ++k) {
            thb_abi_arg& d = slotArgs[k];
            const std::int64_t src = s->sources[k];
            if (src >= 0) {
                d = args[src];
                if (d.kind == THB_KIND_TENSOR) {
                    const std::uint64_t bytes = d.count * (d.dtype == THB_DTYPE_I64 ? 8 : 4);
                    if (!s->publicSlots[k]) s->publicSlots[k] = std::make_unique<DeviceBuffer>();
                    if (s->publicSlots[k]->reserve(bytes, r.device())) {
                        ++ev.allocation_count;
                        ev.allocation_bytes_requested += bytes;
                    }
                    if (bytes) {
                        if (!d.data) fail(Category::Validation, "MODEL-PUBLIC-INPUT-ABI", "tensor data pointer is null");
                        cudaCheck(cudaMemcpyAsync(s->publicSlots[k]->ptr, d.data, bytes, cudaMemcpyHostToDevice, stream),
                                  "cudaMemcpyAsync(public input)");
                        ++ev.host_to_device_copies;
                        ev.host_to_device_bytes += bytes;
                        ++ev.input_storage_uploads;
                    }
                    d.data = s->publicSlots[k]->ptr;
                }
            } else {
                const std::size_t p = static_cast<std::size_t>(-1 - src);
                const auto& v = s->parameters[p];
                d.kind = v.kind;
                d.dtype = v.dtype;
                d.rank = static_cast<std::uint32_t>(v.shape.size());
                d.reserved = 0;
                d.count = 1;
                for (std::size_t a = 0; a < v.shape.size(); ++a) {
                    shapes[k][a] = v.shape[a];
                    d.count *= v.shape[a];
                }
                d.shape = shapes[k].data();
                d.data = v.kind == 2 ? s->resident[p]->ptr : static_cast<const void*>(v.bytes.data());
            }
        }
        auto inputs = bind(r, slotArgs.data(), slotArgs.size(), false, stream, ev, nullptr);
        r.clearErrors(stream);
        ++ev.submitted_operations;
        Value out = r.run(inputs, stream, ev, nullptr,
                          [&](const Value& o) { checkOutputCount(o, outputCount, true, output); });
        downloadOutput(out, output, stream, ev);
        std::vector<std::uint32_t> words(std::max<std::size_t>(1, r.errorWordCount()));
        PinnedBuffer staged;
        staged.reserve(words.size() * sizeof(std::uint32_t));
        r.copyErrors(stream, static_cast<std::uint32_t*>(staged.ptr));
        cudaCheck(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
        ++ev.synchronizations;
        ++ev.observations;
        std::memcpy(words.data(), staged.ptr, words.size() * sizeof(std::uint32_t));
        const std::string id = r.firstFailure(words.data());
        if (!id.empty()) fail(Category::Semantic, id, id);
        return THB_STATUS_OK;
    });
    if (evidence) *evidence = ev;
    return status;
}

int thb_artifact_build(const thb_region_desc* desc, thb_plan_options options, void* buffer, uint64_t capacity,
                       uint64_t* needed, char* failure, uint64_t cap) {
    return guarded(failure, cap, [&] {
        if (!desc || !needed) fail(Category::Validation, "ARTIFACT-INVALID-REGION", "null region or size result");
        PlanOptions opts;
        opts.enableReuse = options.enable_reuse != 0;
        opts.enableFusion = options.enable_fusion != 0;
        const std::string bytes = thb::artifact::build(importRegion(*desc), opts);
        *needed = bytes.size();
        if (!buffer) return THB_STATUS_OK;
        if (capacity < bytes.size()) fail(Category::Validation, "ARTIFACT-IO", "artifact buffer too small");
        std::memcpy(buffer, bytes.data(), bytes.size());
        return THB_STATUS_OK;
    });
}

int thb_region_execute(thb_region* region, const thb_abi_arg* args, uint64_t argc, void* output, uint64_t outputCount,
                       thb_evidence* evidence, char* failure, uint64_t cap) {
    thb_evidence ev{};
    const int status = guarded(failure, cap, [&] {
        if (!region) fail(Category::Validation, "GPU-INVALID-REGION", "region handle is null");
        CompiledRegion& r = *region->impl;
        std::lock_guard<std::mutex> lock(r.mutex);
        r.planEvidence(ev);
        cudaCheck(cudaSetDevice(r.device()), "cudaSetDevice");
        cudaStream_t stream = r.stream();
        std::uint64_t reads = 0;
        std::vector<std::uint32_t> words(std::max<std::size_t>(1, r.errorWordCount()));
        PinnedBuffer staged;
        staged.reserve(words.size() * sizeof(std::uint32_t));
        ++ev.submitted_operations;
        const auto hostValues = bind(r, args, argc, false, stream, ev, &reads);
        bool pipelined = false;
        if (r.rowLocal())
            pipelined = executePipelined(r, hostValues, output, outputCount, stream, ev,
                                         static_cast<std::uint32_t*>(staged.ptr));
        if (!pipelined) {
            auto inputs = bind(r, args, argc, true, stream, ev, &reads);
            r.clearErrors(stream);
            Value out = r.run(inputs, stream, ev, nullptr,
                              [&](const Value& o) { checkOutputCount(o, outputCount, true, output); });
            downloadOutput(out, output, stream, ev);
            r.copyErrors(stream, static_cast<std::uint32_t*>(staged.ptr));
        }
        ++ev.event_records;
        cudaCheck(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
        ++ev.synchronizations;
        ++ev.observations;
        ev.released_reservations = reads + 1;
        ev.retained_planner_allocations = 0;
        std::memcpy(words.data(), staged.ptr, words.size() * sizeof(std::uint32_t));
        const std::string id = r.firstFailure(words.data());
        if (!id.empty()) fail(Category::Semantic, id, id);
        return THB_STATUS_OK;
    });
    if (evidence) *evidence = ev;
    return status;
}

int thb_region_submit(thb_region* region, const thb_abi_arg* args, uint64_t argc, thb_pending** out,
                      thb_evidence* evidence, char* failure, uint64_t cap) {
    thb_evidence ev{};
    const int status = guarded(failure, cap, [&] {
        if (!region || !out) fail(Category::Validation, "GPU-INVALID-REGION", "region handle or result is null");
        *out = nullptr;
        CompiledRegion& r = *region->impl;
        std::lock_guard<std::mutex> lock(r.mutex);
        r.planEvidence(ev);
        cudaCheck(cudaSetDevice(r.device()), "cudaSetDevice");
        cudaStream_t stream = r.stream();
        auto pending = std::make_unique<Pending>();
        pending->region = region->impl;
        auto inputs = bind(r, args, argc, true, stream, ev, &pending->reads);
        r.clearErrors(stream);
        ++ev.submitted_operations;
        Value result = r.run(inputs, stream, ev);
        pending->result = result;
        if (result.tensor || result.onDevice) {
            pending->outputBytes = result.bytes();
            pending->output.reserve(result.bytes());
            downloadOutput(result, pending->output.ptr, stream, ev);
        }
        pending->errors.reserve(std::max<std::size_t>(1, r.errorWordCount()) * sizeof(std::uint32_t));
        r.copyErrors(stream, static_cast<std::uint32_t*>(pending->errors.ptr));
        cudaCheck(cudaEventCreateWithFlags(&pending->done, cudaEventDisableTiming), "cudaEventCreate");
        cudaCheck(cudaEventRecord(pending->done, stream), "cudaEventRecord");
        ++ev.event_records;
        ++ev.stream_submissions;
        ev.pending_operations = 1;
        ev.active_read_reservations = pending->reads;
        ev.active_write_reservations = 1;
        pending->evidence = ev;
        *out = new thb_pending{std::move(pending)};
        return THB_STATUS_OK;
    });
    if (evidence) *evidence = ev;
    return status;
}

int thb_pending_state(const thb_pending* pending) {
    if (!pending || !pending->impl) return -1;
    if (pending->impl->observed) return 1;
    return cudaEventQuery(pending->impl->done) == cudaSuccess ? 1 : 0;
}

int thb_pending_observe(thb_pending* handle, void* output, uint64_t outputCount, uint64_t timeoutMs,
                        thb_evidence* evidence, char* failure, uint64_t cap) {
    if (!handle || !handle->impl) {
        writeText(failure, cap, "GPU-INVALID-PENDING: pending handle is null");
        return THB_STATUS_ABI;
    }
    Pending& p = *handle->impl;
    const int status = guarded(failure, cap, [&] {
        if (!p.observed) {
            cudaCheck(cudaSetDevice(p.region->device()), "cudaSetDevice");
            waitEvent(p.done, timeoutMs);
            p.observed = true;
            ++p.evidence.synchronizations;
            ++p.evidence.observations;
            p.evidence.pending_operations = 0;
            p.evidence.active_read_reservations = 0;
            p.evidence.active_write_reservations = 0;
            p.evidence.released_reservations = p.reads + 1;
            p.evidence.retained_planner_allocations = 0;
            const std::string id = p.region->firstFailure(static_cast<const std::uint32_t*>(p.errors.ptr));
            if (!id.empty()) {
                p.status = THB_STATUS_SEMANTIC;
                p.failureText = id;
            }
        }
        if (p.status != THB_STATUS_OK) fail(Category::Semantic, p.failureText, p.failureText);
        checkOutputCount(p.result, outputCount, true, output);
        if (p.result.tensor || p.result.onDevice) {
            if (p.outputBytes) std::memcpy(output, p.output.ptr, p.outputBytes);
        } else if (output) {
            if (p.result.dtype == DType::I64) std::memcpy(output, &p.result.i64, 8);
            else std::memcpy(output, &p.result.f32, 4);
        }
        return THB_STATUS_OK;
    });
    if (evidence) *evidence = p.evidence;
    return status;
}

void thb_pending_release(thb_pending* handle) {
    if (!handle) return;
    if (handle->impl && !handle->impl->observed) {
        Pending& p = *handle->impl;
        try {
            cudaSetDevice(p.region->device());
            cudaEventSynchronize(p.done);
            const std::string id = p.region->firstFailure(static_cast<const std::uint32_t*>(p.errors.ptr));
            if (!id.empty()) recordUnobserved(id);
        } catch (...) {
            recordUnobserved("GPU-DRAIN-FAILURE");
        }
    }
    delete handle;
}

uint64_t thb_take_unobserved_errors(char* buffer, uint64_t capacity) {
    const auto ids = takeUnobserved();
    std::string text;
    for (std::size_t i = 0; i < ids.size(); ++i) text += (i ? "\n" : "") + ids[i];
    writeText(buffer, capacity, text);
    return ids.size();
}

int thb_region_launch(thb_region* region, const thb_abi_arg* args, uint64_t argc, void* output, uint64_t outputCount,
                      void* stream, char* failure, uint64_t cap) {
    return guarded(failure, cap, [&] {
        if (!region) fail(Category::Validation, "GPU-INVALID-REGION", "region handle is null");
        CompiledRegion& r = *region->impl;
        std::lock_guard<std::mutex> lock(r.mutex);
        thb_evidence ev{};
        auto inputs = bind(r, args, argc, false, static_cast<cudaStream_t>(stream), ev, nullptr);
        const Node& outNode = r.region().at(r.region().output);
        auto s = static_cast<cudaStream_t>(stream);
        Value out = r.run(inputs, s, ev, outNode.tensor() ? output : nullptr,
                          [&](const Value& o) { checkOutputCount(o, outputCount, true, output); });
        if (!outNode.tensor()) {
            // A scalar result (for example a full-tensor Sum) is copied into
            // the caller's one-element device buffer.
            const std::size_t w = width(out.dtype);
            if (out.onDevice)
                cudaCheck(cudaMemcpyAsync(output, out.data, w, cudaMemcpyDeviceToDevice, s), "cudaMemcpyAsync(scalar)");
            else
                cudaCheck(cudaMemcpy(output, out.dtype == DType::I64 ? static_cast<const void*>(&out.i64)
                                                                     : static_cast<const void*>(&out.f32),
                                     w, cudaMemcpyHostToDevice),
                          "cudaMemcpy(scalar)");
        }
        return THB_STATUS_OK;
    });
}

int thb_region_check_errors(thb_region* region, void* stream, char* failure, uint64_t cap) {
    return guarded(failure, cap, [&] {
        if (!region) fail(Category::Validation, "GPU-INVALID-REGION", "region handle is null");
        CompiledRegion& r = *region->impl;
        std::lock_guard<std::mutex> lock(r.mutex);
        cudaCheck(cudaSetDevice(r.device()), "cudaSetDevice");
        auto s = static_cast<cudaStream_t>(stream);
        PinnedBuffer staged;
        staged.reserve(std::max<std::size_t>(1, r.errorWordCount()) * sizeof(std::uint32_t));
        r.copyErrors(s, static_cast<std::uint32_t*>(staged.ptr));
        r.clearErrors(s);
        cudaCheck(cudaStreamSynchronize(s), "cudaStreamSynchronize");
        const std::string id = r.firstFailure(static_cast<const std::uint32_t*>(staged.ptr));
        if (!id.empty()) fail(Category::Semantic, id, id);
        return THB_STATUS_OK;
    });
}

int thb_gemm_bf16(int device, const thb_gemm_desc* desc, void* stream, char* failure, uint64_t cap) {
    return guarded(failure, cap, [&] {
        if (!desc) fail(Category::Validation, "GPU-GEMM-ARGUMENT", "GEMM descriptor is null");
        const DeviceInfo& info = useDevice(device);
        gemm::Problem q;
        q.m = desc->m;
        q.n = desc->n;
        q.k = desc->k;
        q.a = desc->a;
        q.aMajorMN = desc->a_major == THB_MAJOR_MN;
        q.lda = desc->lda;
        q.b = desc->b;
        q.bMajorMN = desc->b_major == THB_MAJOR_MN;
        q.ldb = desc->ldb;
        q.c = desc->c;
        q.ldc = desc->ldc;
        q.epilogue = static_cast<int>(desc->epilogue);
        q.aux = desc->aux;
        q.ldAux = desc->ld_aux;
        q.c2 = desc->c_f32_copy;
        if (desc->a_major > THB_MAJOR_MN || desc->b_major > THB_MAJOR_MN)
            fail(Category::Validation, "GPU-GEMM-ARGUMENT", "operand major must be THB_MAJOR_K or THB_MAJOR_MN");
        if (const char* bad = gemm::validate(q)) fail(Category::Validation, "GPU-GEMM-ARGUMENT", bad);
        cudaCheck(gemm::run(q, info.smCount, deviceStatus(device), static_cast<cudaStream_t>(stream)), "tcgen05 GEMM launch");
        return THB_STATUS_OK;
    });
}

int thb_device_check_status(int device, void* stream, char* failure, uint64_t cap) {
    return guarded(failure, cap, [&] {
        std::uint32_t* word = deviceStatus(device);
        auto s = static_cast<cudaStream_t>(stream);
        std::uint32_t host = 0;
        cudaCheck(cudaMemcpyAsync(&host, word, sizeof host, cudaMemcpyDeviceToHost, s), "cudaMemcpyAsync(status)");
        cudaCheck(cudaMemsetAsync(word, 0, sizeof host, s), "cudaMemsetAsync(status)");
        cudaCheck(cudaStreamSynchronize(s), "cudaStreamSynchronize");
        if (host) fail(Category::Runtime, statusText(host), "a kernel reported status " + std::to_string(host));
        return THB_STATUS_OK;
    });
}

int thb_mlp_create(int device, uint64_t batch, uint64_t globalBatch, uint64_t in, uint64_t hidden, uint64_t out,
                   thb_mlp** session, char* failure, uint64_t cap) {
    return guarded(failure, cap, [&] {
        if (!session) fail(Category::Validation, "GPU-MLP-ARGUMENT", "session result pointer is null");
        *session = nullptr;
        if (!batch || !in || !hidden || !out || globalBatch < batch)
            fail(Category::Validation, "GPU-MLP-ARGUMENT", "MLP extents must be positive and global_batch >= batch");
        if (batch % 8 || in % 8 || hidden % 8 || out % 8)
            fail(Category::Validation, "GPU-MLP-ARGUMENT", "MLP extents must be multiples of 8 (16-byte rows)");
        const DeviceInfo& info = useDevice(device);
        auto s = std::make_unique<thb_mlp>();
        s->device = device;
        s->smCount = info.smCount;
        auto& b = s->b;
        b.batch = batch;
        b.globalBatch = globalBatch;
        b.in = in;
        b.hidden = hidden;
        b.out = out;
        b.w1 = static_cast<float*>(s->alloc(in * hidden * 4));
        b.w2 = static_cast<float*>(s->alloc(hidden * out * 4));
        b.w1b = s->alloc(in * hidden * 2);
        b.w2b = s->alloc(hidden * out * 2);
        b.xb = s->alloc(batch * in * 2);
        b.h = s->alloc(batch * hidden * 2);
        b.y = static_cast<float*>(s->alloc(batch * out * 4));
        b.dy = s->alloc(batch * out * 2);
        b.dh = s->alloc(batch * hidden * 2);
        b.dw1 = static_cast<float*>(s->alloc(in * hidden * 4));
        b.dw2 = static_cast<float*>(s->alloc(hidden * out * 4));
        b.lossPartials = static_cast<double*>(s->alloc(mlp::lossPartialCount(batch, out, info.smCount) * 8));
        b.lossSum = static_cast<double*>(s->alloc(8));
        s->ownW[0] = b.w1;
        s->ownW[1] = b.w2;
        s->ownWb[0] = b.w1b;
        s->ownWb[1] = b.w2b;
        s->ownDw[0] = b.dw1;
        s->ownDw[1] = b.dw2;
        *session = s.release();
        return THB_STATUS_OK;
    });
}

void thb_mlp_release(thb_mlp* session) { delete session; }

int thb_mlp_set_weights(thb_mlp* s, const float* w1, const float* w2, void* stream, char* failure, uint64_t cap) {
    return guarded(failure, cap, [&] {
        if (!s || !w1 || !w2) fail(Category::Validation, "GPU-MLP-ARGUMENT", "null session or weights");
        useDevice(s->device);
        auto st = static_cast<cudaStream_t>(stream);
        const auto& b = s->b;
        cudaCheck(cudaMemcpyAsync(b.w1, w1, b.in * b.hidden * 4, cudaMemcpyDeviceToDevice, st), "cudaMemcpyAsync(W1)");
        cudaCheck(cudaMemcpyAsync(b.w2, w2, b.hidden * b.out * 4, cudaMemcpyDeviceToDevice, st), "cudaMemcpyAsync(W2)");
        cudaCheck(mlp::castToBf16(b.w1, b.w1b, b.in * b.hidden, s->smCount, st), "cast W1");
        cudaCheck(mlp::castToBf16(b.w2, b.w2b, b.hidden * b.out, s->smCount, st), "cast W2");
        return THB_STATUS_OK;
    });
}

namespace {

// Forward, loss and backward; with `lr`, the weight updates run in the
// all-reduce of the weight-gradient GEMMs (thb_mlp_forward_backward_update).
int forwardBackwardCall(thb_mlp* s, const float* x, const float* t, const float* lr, void* stream, char* failure,
                        uint64_t cap) {
    return guarded(failure, cap, [&] {
        if (!s || !x || !t) fail(Category::Validation, "GPU-MLP-ARGUMENT", "null session or data");
        if ((reinterpret_cast<std::uintptr_t>(x) | reinterpret_cast<std::uintptr_t>(t)) % 16)
            fail(Category::Validation, "GPU-MLP-ARGUMENT", "x and t must be 16-byte aligned");
        if (lr && !(s->b.dw1Reduce.update.paramPeers[0] && s->b.dw2Reduce.update.paramPeers[0]))
            fail(Category::Validation, "GPU-MLP-ARGUMENT",
                 "the fused update needs thb_mlp_bind_reduction and thb_mlp_bind_update for both layers");
        if (!lr && (s->b.dw1Reduce.compact || s->b.dw2Reduce.compact))
            fail(Category::Validation, "GPU-MLP-ARGUMENT",
                 "a bf16 sharded reduction applies the optimizer step in the reduction: "
                 "call thb_mlp_forward_backward_update");
        useDevice(s->device);
        // Each step's announcements raise every signal word by `world`.
        ++s->reduceEpoch;
        s->b.dw1Reduce.target = s->b.dw1Reduce.world * s->reduceEpoch;
        s->b.dw2Reduce.target = s->b.dw2Reduce.world * s->reduceEpoch;
        cudaCheck(mlp::forwardBackward(s->b, x, t, s->smCount, deviceStatus(s->device), static_cast<cudaStream_t>(stream),
                                       &s->timer, lr),
                  "MLP forward/backward");
        s->weightsUpdated = lr != nullptr;
        return THB_STATUS_OK;
    });
}

} // namespace

int thb_mlp_forward_backward(thb_mlp* s, const float* x, const float* t, void* stream, char* failure, uint64_t cap) {
    return forwardBackwardCall(s, x, t, nullptr, stream, failure, cap);
}

int thb_mlp_forward_backward_update(thb_mlp* s, const float* x, const float* t, float lr, void* stream, char* failure,
                                    uint64_t cap) {
    return forwardBackwardCall(s, x, t, &lr, stream, failure, cap);
}

int thb_mlp_apply_sgd(thb_mlp* s, float lr, void* stream, char* failure, uint64_t cap) {
    return guarded(failure, cap, [&] {
        if (!s) fail(Category::Validation, "GPU-MLP-ARGUMENT", "null session");
        useDevice(s->device);
        // After a fused-update pass only the biases are left.
        cudaCheck(mlp::applySgd(s->b, lr, s->smCount, static_cast<cudaStream_t>(stream), !s->weightsUpdated),
                  "MLP SGD");
        s->weightsUpdated = false;
        return THB_STATUS_OK;
    });
}

int thb_mlp_step(thb_mlp* s, const float* x, const float* t, float lr, void* stream, char* failure, uint64_t cap) {
    return guarded(failure, cap, [&] {
        if (!s || !x || !t) fail(Category::Validation, "GPU-MLP-ARGUMENT", "null session or data");
        if ((reinterpret_cast<std::uintptr_t>(x) | reinterpret_cast<std::uintptr_t>(t)) % 16)
            fail(Category::Validation, "GPU-MLP-ARGUMENT", "x and t must be 16-byte aligned");
        if (s->b.dw1Reduce.cPeers[0] || s->b.dw2Reduce.cPeers[0])
            fail(Category::Validation, "GPU-MLP-ARGUMENT",
                 "thb_mlp_step is the single-device step; a session with a bound gradient all-reduce runs "
                 "thb_mlp_forward_backward, a barrier, then thb_mlp_apply_sgd");
        useDevice(s->device);
        const auto st = static_cast<cudaStream_t>(stream);
        // The weight updates run in the dW GEMM epilogues; the biases follow.
        cudaCheck(mlp::forwardBackward(s->b, x, t, s->smCount, deviceStatus(s->device), st, &s->timer, &lr),
                  "MLP step");
        cudaCheck(mlp::applySgd(s->b, lr, s->smCount, st, false), "MLP bias update");
        return THB_STATUS_OK;
    });
}

int thb_mlp_buffer(thb_mlp* s, uint32_t which, void** pointer, uint64_t* elements) {
    if (!s || !pointer) return THB_STATUS_ABI;
    const auto& b = s->b;
    switch (which) {
    case THB_MLP_W1: *pointer = b.w1; if (elements) *elements = b.in * b.hidden; break;
    case THB_MLP_W2: *pointer = b.w2; if (elements) *elements = b.hidden * b.out; break;
    case THB_MLP_DW1: *pointer = b.dw1; if (elements) *elements = b.in * b.hidden; break;
    case THB_MLP_DW2: *pointer = b.dw2; if (elements) *elements = b.hidden * b.out; break;
    case THB_MLP_Y: *pointer = b.y; if (elements) *elements = b.batch * b.out; break;
    case THB_MLP_H: *pointer = b.h; if (elements) *elements = b.batch * b.hidden; break;
    case THB_MLP_LOSS_SUM: *pointer = b.lossSum; if (elements) *elements = 1; break;
    case THB_MLP_B1: *pointer = b.b1; if (elements) *elements = b.b1 ? b.hidden : 0; break;
    case THB_MLP_B2: *pointer = b.b2; if (elements) *elements = b.b1 ? b.out : 0; break;
    case THB_MLP_DB1: *pointer = b.db1; if (elements) *elements = b.b1 ? b.hidden : 0; break;
    case THB_MLP_DB2: *pointer = b.db2; if (elements) *elements = b.b1 ? b.out : 0; break;
    default: return THB_STATUS_ABI;
    }
    return THB_STATUS_OK;
}

int thb_mlp_set_biases(thb_mlp* s, const float* b1, const float* b2, void* stream, char* failure, uint64_t cap) {
    return guarded(failure, cap, [&] {
        if (!s) fail(Category::Validation, "GPU-MLP-ARGUMENT", "null session");
        if (!b1 != !b2) fail(Category::Validation, "GPU-MLP-ARGUMENT", "give both biases or neither");
        useDevice(s->device);
        auto st = static_cast<cudaStream_t>(stream);
        auto& b = s->b;
        if (!b.b1) {
            b.b1 = static_cast<float*>(s->alloc(b.hidden * 4));
            b.b2 = static_cast<float*>(s->alloc(b.out * 4));
            // db1 and db2 adjacent, so one collective call can reduce both.
            b.db1 = static_cast<float*>(s->alloc((b.hidden + b.out) * 4));
            b.db2 = b.db1 + b.hidden;
            b.dyColSums = static_cast<float*>(s->alloc(mlp::lossRowChunks(b.batch, b.out, s->smCount) * b.out * 4));
            b.dhColSums = static_cast<float*>(s->alloc(gemm::colSumRows(b.batch) * b.hidden * 4));
        }
        if (b1) {
            cudaCheck(cudaMemcpyAsync(b.b1, b1, b.hidden * 4, cudaMemcpyDeviceToDevice, st), "cudaMemcpyAsync(b1)");
            cudaCheck(cudaMemcpyAsync(b.b2, b2, b.out * 4, cudaMemcpyDeviceToDevice, st), "cudaMemcpyAsync(b2)");
        } else {
            cudaCheck(cudaMemsetAsync(b.b1, 0, b.hidden * 4, st), "cudaMemsetAsync(b1)");
            cudaCheck(cudaMemsetAsync(b.b2, 0, b.out * 4, st), "cudaMemsetAsync(b2)");
        }
        if (b.vb1) {
            cudaCheck(cudaMemsetAsync(b.vb1, 0, b.hidden * 4, st), "cudaMemsetAsync(vb1)");
            cudaCheck(cudaMemsetAsync(b.vb2, 0, b.out * 4, st), "cudaMemsetAsync(vb2)");
        }
        return THB_STATUS_OK;
    });
}

int thb_mlp_set_momentum(thb_mlp* s, float momentum, void* stream, char* failure, uint64_t cap) {
    return guarded(failure, cap, [&] {
        if (!s) fail(Category::Validation, "GPU-MLP-ARGUMENT", "null session");
        // The reference's optimizer checks (Training.cpp OPT05 / OPT06).
        if (!std::isfinite(momentum) || momentum < 0.0f)
            fail(Category::Semantic, "OPT05", "momentum must be finite and non-negative");
        if (momentum >= 1.0f) fail(Category::Semantic, "OPT06", "momentum must be below 1");
        useDevice(s->device);
        auto st = static_cast<cudaStream_t>(stream);
        auto& b = s->b;
        if (momentum > 0.0f && !b.vw1) {
            b.vw1 = static_cast<float*>(s->alloc(b.in * b.hidden * 4));
            b.vw2 = static_cast<float*>(s->alloc(b.hidden * b.out * 4));
            b.vb1 = static_cast<float*>(s->alloc(b.hidden * 4));
            b.vb2 = static_cast<float*>(s->alloc(b.out * 4));
        }
        if (b.vw1) {  // velocities start at zero (ZeroLike, Training.cpp state init)
            cudaCheck(cudaMemsetAsync(b.vw1, 0, b.in * b.hidden * 4, st), "cudaMemsetAsync(vW1)");
            cudaCheck(cudaMemsetAsync(b.vw2, 0, b.hidden * b.out * 4, st), "cudaMemsetAsync(vW2)");
            cudaCheck(cudaMemsetAsync(b.vb1, 0, b.hidden * 4, st), "cudaMemsetAsync(vb1)");
            cudaCheck(cudaMemsetAsync(b.vb2, 0, b.out * 4, st), "cudaMemsetAsync(vb2)");
        }
        b.momentum = momentum;
        return THB_STATUS_OK;
    });
}

int thb_mlp_enable_timing(thb_mlp* s, int enabled) {
    if (!s) return THB_STATUS_ABI;
    if (enabled && !s->timer.events[0]) {
        if (cudaSetDevice(s->device) != cudaSuccess) return THB_STATUS_BACKEND;
        for (auto& e : s->timer.events)
            if (cudaEventCreate(&e) != cudaSuccess) return THB_STATUS_BACKEND;
    }
    s->timer.enabled = enabled != 0;
    s->timer.used = 0;
    s->timer.launches = 0;
    return THB_STATUS_OK;
}

int thb_mlp_read_timing(thb_mlp* s, double* gemmMs, uint64_t* gemmLaunches) {
    if (!s || !gemmMs || !gemmLaunches) return THB_STATUS_ABI;
    double total = 0.0;
    for (unsigned k = 0; k + 1 < s->timer.used; k += 2) {
        if (cudaEventSynchronize(s->timer.events[k + 1]) != cudaSuccess) return THB_STATUS_BACKEND;
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, s->timer.events[k], s->timer.events[k + 1]) != cudaSuccess) return THB_STATUS_BACKEND;
        total += ms;
    }
    *gemmMs = total;
    *gemmLaunches = s->timer.launches;
    s->timer.used = 0;
    s->timer.launches = 0;
    return THB_STATUS_OK;
}

namespace {

// Removes layer `layer`'s update binding, if any: the layer's W and bf16 W
// return to the session's own buffers (the caller copies the weights in with
// thb_mlp_set_weights), so the bound ones may be freed afterwards.
void dropUpdate(thb_mlp* s, int layer) {
    auto& r = layer == 0 ? s->b.dw1Reduce : s->b.dw2Reduce;
    if (!r.update.paramPeers[0]) return;
    (layer == 0 ? s->b.w1 : s->b.w2) = s->ownW[layer];
    (layer == 0 ? s->b.w1b : s->b.w2b) = s->ownWb[layer];
    r.update = thb::gemm::ReduceUpdate{};
}

} // namespace

int thb_mlp_bind_reduction(thb_mlp* s, uint32_t which, void* const* peers, void* multicast, uint32_t* const* flagPeers,
                           uint32_t rank, uint32_t world) {
    if (!s || (which != THB_MLP_DW1 && which != THB_MLP_DW2)) return THB_STATUS_ABI;
    const int layer = which == THB_MLP_DW1 ? 0 : 1;
    thb::gemm::AllReduce r;
    if (peers) {
        if (!flagPeers || world == 0 || world > static_cast<uint32_t>(thb::gemm::kMaxRanks) || rank >= world ||
            reinterpret_cast<std::uintptr_t>(multicast) % 16)
            return THB_STATUS_ABI;
        for (uint32_t k = 0; k < world; ++k) {
            if (!peers[k] || !flagPeers[k] || reinterpret_cast<std::uintptr_t>(peers[k]) % 16 ||
                reinterpret_cast<std::uintptr_t>(flagPeers[k]) % 4)
                return THB_STATUS_ABI;
            r.cPeers[k] = peers[k];
            r.flagsPeers[k] = flagPeers[k];
        }
        r.cMulticast = multicast;
        r.rank = rank;
        r.world = world;
    }
    auto& bound = which == THB_MLP_DW1 ? s->b.dw1Reduce : s->b.dw2Reduce;
    float*& dw = which == THB_MLP_DW1 ? s->b.dw1 : s->b.dw2;
    dropUpdate(s, layer);
    if (peers) dw = static_cast<float*>(peers[rank]);
    else if (bound.cPeers[0]) dw = s->ownDw[layer];  // back to the local store
    bound = r;
    s->reduceEpoch = 0;  // fresh (zeroed) signal words
    return THB_STATUS_OK;
}

int thb_mlp_bind_update(thb_mlp* s, uint32_t which, float* const* paramPeers, void* paramMulticast,
                        void* const* copyPeers, void* copyMulticast) {
    if (!s || (which != THB_MLP_W1 && which != THB_MLP_W2)) return THB_STATUS_ABI;
    auto& r = which == THB_MLP_W1 ? s->b.dw1Reduce : s->b.dw2Reduce;
    if (!paramPeers) {
        dropUpdate(s, which == THB_MLP_W1 ? 0 : 1);
        return THB_STATUS_OK;
    }
    if (!r.cPeers[0] || !copyPeers) return THB_STATUS_ABI;
    if (!r.cMulticast != !paramMulticast || !paramMulticast != !copyMulticast) return THB_STATUS_ABI;
    if (reinterpret_cast<std::uintptr_t>(paramMulticast) % 16 || reinterpret_cast<std::uintptr_t>(copyMulticast) % 16)
        return THB_STATUS_ABI;
    thb::gemm::ReduceUpdate u;
    for (uint32_t k = 0; k < r.world; ++k) {
        if (!paramPeers[k] || !copyPeers[k] || reinterpret_cast<std::uintptr_t>(paramPeers[k]) % 16 ||
            reinterpret_cast<std::uintptr_t>(copyPeers[k]) % 16)
            return THB_STATUS_ABI;
        u.paramPeers[k] = paramPeers[k];
        u.copyPeers[k] = copyPeers[k];
    }
    u.paramMulticast = static_cast<float*>(paramMulticast);
    u.copyMulticast = copyMulticast;
    (which == THB_MLP_W1 ? s->b.w1 : s->b.w2) = paramPeers[r.rank];
    (which == THB_MLP_W1 ? s->b.w1b : s->b.w2b) = copyPeers[r.rank];
    r.update = u;
    return THB_STATUS_OK;
}

int thb_mlp_set_reduction_format(thb_mlp* s, uint32_t which, uint32_t format) {
    if (!s || (which != THB_MLP_DW1 && which != THB_MLP_DW2) ||
        (format != THB_REDUCE_F32 && format != THB_REDUCE_BF16_SHARDED))
        return THB_STATUS_ABI;
    auto& r = which == THB_MLP_DW1 ? s->b.dw1Reduce : s->b.dw2Reduce;
    if (format == THB_REDUCE_BF16_SHARDED && !r.cPeers[0]) return THB_STATUS_ABI;
    r.compact = format == THB_REDUCE_BF16_SHARDED;
    return THB_STATUS_OK;
}

int thb_mlp_gather_parameters(thb_mlp* s, uint32_t which, void* stream, char* failure, uint64_t cap) {
    return guarded(failure, cap, [&] {
        if (!s || (which != THB_MLP_W1 && which != THB_MLP_W2))
            fail(Category::Validation, "GPU-MLP-ARGUMENT", "null session or not a weight (THB_MLP_W1 / W2)");
        const bool first = which == THB_MLP_W1;
        const auto& r = first ? s->b.dw1Reduce : s->b.dw2Reduce;
        if (!r.update.paramPeers[0])
            fail(Category::Validation, "GPU-MLP-ARGUMENT", "no parameter binding (thb_mlp_bind_update) to gather from");
        // The weight-gradient GEMM whose tile owners hold the parameters.
        gemm::Problem q;
        q.m = first ? s->b.in : s->b.hidden;
        q.n = first ? s->b.hidden : s->b.out;
        q.k = s->b.batch;
        q.ldc = q.n;
        q.epilogue = gemm::kEpiAllReduceF32;
        q.reduce = r;
        q.reduce.update.enabled = true;
        useDevice(s->device);
        cudaCheck(gemm::gatherOwned(q, s->smCount, static_cast<cudaStream_t>(stream)), "gather parameters");
        return THB_STATUS_OK;
    });
}

uint64_t thb_mlp_reduction_flag_words(thb_mlp* s, uint32_t which) {
    if (!s) return 0;
    if (which == THB_MLP_DW1) return 4 * thb::gemm::tileCount(s->b.in, s->b.hidden);
    if (which == THB_MLP_DW2) return 4 * thb::gemm::tileCount(s->b.hidden, s->b.out);
    return 0;
}

int thb_mlp_bind(thb_mlp* s, uint32_t which, void* pointer) {
    if (!s || !pointer || reinterpret_cast<std::uintptr_t>(pointer) % 16) return THB_STATUS_ABI;
    auto& b = s->b;
    switch (which) {
    case THB_MLP_W1: b.w1 = static_cast<float*>(pointer); break;
    case THB_MLP_W2: b.w2 = static_cast<float*>(pointer); break;
    case THB_MLP_DW1: b.dw1 = static_cast<float*>(pointer); break;
    case THB_MLP_DW2: b.dw2 = static_cast<float*>(pointer); break;
    case THB_MLP_Y: b.y = static_cast<float*>(pointer); break;
    case THB_MLP_H: b.h = pointer; break;
    case THB_MLP_LOSS_SUM: b.lossSum = static_cast<double*>(pointer); break;
    case THB_MLP_B1: if (!b.b1) return THB_STATUS_ABI; b.b1 = static_cast<float*>(pointer); break;
    case THB_MLP_B2: if (!b.b1) return THB_STATUS_ABI; b.b2 = static_cast<float*>(pointer); break;
    case THB_MLP_DB1: if (!b.b1) return THB_STATUS_ABI; b.db1 = static_cast<float*>(pointer); break;
    case THB_MLP_DB2: if (!b.b1) return THB_STATUS_ABI; b.db2 = static_cast<float*>(pointer); break;
    default: return THB_STATUS_ABI;
    }
    return THB_STATUS_OK;
}

static int writeOut(const std::string& text, char* buffer, uint64_t capacity, uint64_t* needed) {
    if (needed) *needed = text.size() + 1;
    writeText(buffer, capacity, text);
    return (capacity >= text.size() + 1 || !buffer) ? THB_STATUS_OK : THB_STATUS_ABI;
}

int thb_region_emit_source(const thb_region* region, char* buffer, uint64_t capacity, uint64_t* needed) {
    if (!region) return THB_STATUS_ABI;
    return writeOut(region->impl->source(), buffer, capacity, needed);
}

int thb_region_dump_plan(const thb_region* region, char* buffer, uint64_t capacity, uint64_t* needed) {
    if (!region) return THB_STATUS_ABI;
    return writeOut(region->impl->region().dump() + region->impl->plan().dump(region->impl->region()), buffer,
                    capacity, needed);
}

int thb_region_describe(const thb_region_desc* desc, thb_plan_options options, uint32_t what, char* buffer,
                        uint64_t capacity, uint64_t* needed, uint64_t* counts, char* failure, uint64_t cap) {
    return guarded(failure, cap, [&] {
        if (!desc) fail(Category::Validation, "GPU-INVALID-REGION", "region descriptor is null");
        const Region region = importRegion(*desc);
        PlanOptions opts;
        opts.enableReuse = options.enable_reuse != 0;
        opts.enableFusion = options.enable_fusion != 0;
        const Plan plan = buildPlan(region, opts);
        std::vector<GroupKernel> kernels;
        const std::string source = generateSource(region, plan, kernels);
        if (counts) {
            counts[0] = plan.groups.size();
            counts[1] = 0;
            counts[2] = 0;
            for (const auto& g : plan.groups) {
                counts[1] += g.fused;
                counts[2] += g.kind != GroupKind::Index;
            }
        }
        std::string text;
        if (what == THB_DESCRIBE_PLAN) text = region.dump() + plan.dump(region);
        else if (what == THB_DESCRIBE_SOURCE) text = source;
        else if (what == THB_DESCRIBE_CUBIN) text = std::to_string(kernels.empty() ? 0 : compileCubin(source).size());
        else fail(Category::Validation, "GPU-DESCRIBE", "unknown describe selector");
        return writeOut(text, buffer, capacity, needed);
    });
}

int thb_region_plan_counts(const thb_region* region, uint64_t* fusionGroups, uint64_t* fusedGroups, uint64_t* kernels) {
    if (!region) return THB_STATUS_ABI;
    const Plan& plan = region->impl->plan();
    std::uint64_t fused = 0, launches = 0;
    for (const auto& g : plan.groups) {
        fused += g.fused;
        launches += g.kind != GroupKind::Index;
    }
    if (fusionGroups) *fusionGroups = plan.groups.size();
    if (fusedGroups) *fusedGroups = fused;
    if (kernels) *kernels = launches;
    return THB_STATUS_OK;
}

} // extern "C"
