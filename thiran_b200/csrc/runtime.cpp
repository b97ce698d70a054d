// Persistent device runtime (see runtime.hpp).
#include "runtime.hpp"

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <utility>

#include "gemm.hpp"
#include "kernels.hpp"
#include "mlp.hpp"

namespace thb {

namespace {

void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) fail(Category::Runtime, "GPU-RUNTIME", std::string(what) + ": " + cudaGetErrorString(e));
}

std::mutex deviceMutex;
std::map<int, DeviceInfo> deviceInfos;

std::mutex unobservedMutex;
std::vector<std::string> unobservedErrors;

struct BulkShape {
    std::uint32_t stages = 0;
    std::uint32_t tileBytes = 0;
};

// Ring geometry of a group's bulk-copy entry for `arity` tensor inputs: two
// stages, tiles of the largest multiple of 4 KiB up to 48 KiB for which the
// (2 * arity + 2) tiles fit in 200 KiB of shared memory (48 KiB for one
// input, 32 KiB for two: the 2^28 f32 chain measured 341 us per launch with
// 48 KiB against 344 with 32 KiB, and 351-358 with 3-4 stages or 24 KiB).
// On B200 two stages of 32 KiB ran the 8192^2 i64 region at ~238 us per
// launch whatever the placement of its three arrays, where the 128-bit
// vector kernel took ~270-290 us; 16 KiB tiles (2-4 stages) took ~325 us and
// 8 KiB tiles ~515 us (the per-tile barriers dominate).
// THB_BULK=off keeps the vector kernel; THB_BULK=<stages>,<KiB> sets the
// shape.
bool bulkShape(std::size_t arity, BulkShape& s) {
    static const std::pair<int, int> choice = [] {
        const char* e = std::getenv("THB_BULK");
        if (!e || !*e) return std::pair<int, int>{0, 0};
        int stages = 0, kib = 0;
        if (std::sscanf(e, "%d,%d", &stages, &kib) == 2 && stages > 0 && kib > 0) return std::pair<int, int>{stages, kib};
        return std::pair<int, int>{-1, 0};
    }();
    if (choice.first < 0 || arity == 0) return false;
    if (choice.first > 0) {
        s.stages = static_cast<std::uint32_t>(choice.first);
        s.tileBytes = static_cast<std::uint32_t>(choice.second) * 1024u;
    } else {
        constexpr std::uint64_t kBudget = 200u * 1024u, kTile = 49152, kStep = 4096;
        s.stages = 2;
        const std::uint64_t tiles = 2 * arity + 2;
        s.tileBytes = static_cast<std::uint32_t>(std::min<std::uint64_t>(kTile, kBudget / tiles / kStep * kStep));
        if (s.tileBytes < kStep) return false;
    }
    return s.stages >= 1 && s.stages <= kBulkMaxStages && s.tileBytes >= 256 && s.tileBytes % 16 == 0;
}

} // namespace

DeviceBuffer::~DeviceBuffer() {
    if (ptr) {
        int previous = -1;
        cudaGetDevice(&previous);
        cudaSetDevice(device);
        cudaFree(ptr);
        if (previous >= 0) cudaSetDevice(previous);
    }
}

bool DeviceBuffer::reserve(std::size_t want, int ordinal) {
    if (ptr && bytes >= want) return false;
    // The buffer lands on `ordinal` whatever the calling thread's current
    // device is; that device is restored afterwards.
    int previous = -1;
    cudaGetDevice(&previous);
    if (previous != ordinal) check(cudaSetDevice(ordinal), "cudaSetDevice");
    if (ptr) {
        cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
    }
    device = ordinal;
    const std::size_t rounded = std::max<std::size_t>(256, (want + 255) / 256 * 256);
    const cudaError_t e = cudaMalloc(&ptr, rounded);
    if (previous >= 0 && previous != ordinal) cudaSetDevice(previous);
    if (e != cudaSuccess) {
        ptr = nullptr;
        cudaGetLastError();  // an allocation failure is not left for a later launch check
    }
    check(e, "cudaMalloc");
    bytes = rounded;
    return true;
}

PinnedBuffer::~PinnedBuffer() {
    if (ptr) cudaFreeHost(ptr);
}

void PinnedBuffer::reserve(std::size_t want) {
    if (ptr && bytes >= want) return;
    if (ptr) cudaFreeHost(ptr);
    ptr = nullptr;
    bytes = 0;
    const std::size_t rounded = std::max<std::size_t>(64, want);
    check(cudaMallocHost(&ptr, rounded), "cudaMallocHost");
    bytes = rounded;
}

const DeviceInfo& useDevice(int ordinal) {
    std::lock_guard<std::mutex> lock(deviceMutex);
    int count = 0;
    const cudaError_t e = cudaGetDeviceCount(&count);
    if (e == cudaErrorInsufficientDriver || e == cudaErrorNoDevice || e == cudaErrorInitializationError ||
        e == cudaErrorSystemDriverMismatch || e == cudaErrorCompatNotSupportedOnDevice) {
        cudaGetLastError();
        fail(Category::BackendUnavailable, "GPU-DRIVER-NOT-FOUND", std::string("CUDA driver/device unavailable: ") +
                                                                        cudaGetErrorString(e));
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        fail(Category::BackendUnavailable, "GPU-DRIVER-NOT-FOUND", cudaGetErrorString(e));
    }
    if (ordinal < 0 || ordinal >= count)
        fail(Category::InvalidDevice, "GPU-INVALID-DEVICE", "device ordinal " + std::to_string(ordinal) +
                                                                 " outside [0," + std::to_string(count) + ")");
    check(cudaSetDevice(ordinal), "cudaSetDevice");
    auto found = deviceInfos.find(ordinal);
    if (found == deviceInfos.end()) {
        cudaDeviceProp prop{};
        check(cudaGetDeviceProperties(&prop, ordinal), "cudaGetDeviceProperties");
        if (prop.major < 10)
            fail(Category::Unsupported, "GPU-UNSUPPORTED-DEVICE",
                 std::string("this engine is built for sm_100a (B200); device is ") + prop.name);
        DeviceInfo info;
        info.ordinal = ordinal;
        info.smCount = prop.multiProcessorCount;
        info.major = prop.major;
        info.minor = prop.minor;
        info.maxSmemOptin = static_cast<int>(prop.sharedMemPerBlockOptin);
        found = deviceInfos.emplace(ordinal, info).first;
    }
    return found->second;
}

std::uint32_t* deviceStatus(int ordinal) {
    static std::mutex statusMutex;
    static std::map<int, std::unique_ptr<DeviceBuffer>> words;
    useDevice(ordinal);
    std::lock_guard<std::mutex> lock(statusMutex);
    auto& word = words[ordinal];
    if (!word) {
        word = std::make_unique<DeviceBuffer>();
        word->reserve(sizeof(std::uint32_t), ordinal);
        check(cudaMemset(word->ptr, 0, word->bytes), "cudaMemset(status)");
    }
    return static_cast<std::uint32_t*>(word->ptr);
}

std::string statusText(std::uint32_t word) {
    if (word & 32u) return "GPU-KERNEL-DRAIN-TIMEOUT";  // copies in flight outlived the CTA
    if (word & 16u) return "GPU-KERNEL-TIMEOUT";
    if (word & 1u) return "TH-SPEC-I64-OVERFLOW";
    if (word & 2u) return "TH021-DIVIDE-BY-ZERO";
    return "GPU-KERNEL-STATUS";
}

void recordUnobserved(const std::string& id) {
    std::lock_guard<std::mutex> lock(unobservedMutex);
    unobservedErrors.push_back(id);
}

std::vector<std::string> takeUnobserved() {
    std::lock_guard<std::mutex> lock(unobservedMutex);
    std::vector<std::string> out;
    out.swap(unobservedErrors);
    return out;
}

Pending::~Pending() {
    if (done) cudaEventDestroy(done);
}

// ---- compiled region --------------------------------------------------------

CompiledRegion::CompiledRegion(const thb_region_desc& desc, PlanOptions options, int device)
    : CompiledRegion(importRegion(desc), options, device, nullptr) {}

CompiledRegion::CompiledRegion(Region region, PlanOptions options, int device, const std::string* prebuiltCubin)
    : region_(std::move(region)), plan_(buildPlan(region_, options)), device_(device) {
    // Planning and code generation need no device: a malformed region fails
    // before any driver call (NativeGpuTests.cpp:175-198 contract).
    source_ = generateSource(region_, plan_, kernels_);
    info_ = &useDevice(device);
    if (!kernels_.empty())
        module_ = compileAndLoad(source_, device, kernels_, moduleJitted_, moduleLoaded_, prebuiltCubin);
    check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreateWithFlags");
    errors_.reserve(std::max<std::size_t>(1, plan_.groups.size()) * sizeof(std::uint32_t) + 64, device_);
    check(cudaMemsetAsync(errors_.ptr, 0, errors_.bytes, stream_), "cudaMemsetAsync");
    check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");

    // Row-local: one kernel group; every other node is an Input tensor or an
    // Alias; the group's operation keeps rows independent.
    rowLocal_ = plan_.groups.size() == 1 && region_.at(region_.output).tensor();
    for (const auto& n : region_.nodes) {
        if (n.op == Op::Input) rowLocal_ = rowLocal_ && n.tensor();
        else if (n.op == Op::Alias) continue;
        else if (isElementwise(n.op) || n.op == Op::Softmax || n.op == Op::RowMax) continue;
        else if (n.op == Op::Sum) rowLocal_ = rowLocal_ && n.axis == 1;
        else rowLocal_ = false;
    }
}

CompiledRegion::~CompiledRegion() {
    int previous = -1;
    cudaGetDevice(&previous);
    cudaSetDevice(device_);
    for (auto& l : lanes_) {
        if (l.stream) {
            cudaStreamSynchronize(l.stream);
            cudaStreamDestroy(l.stream);
        }
        if (l.done) cudaEventDestroy(l.done);
    }
    if (stream_) {
        cudaStreamSynchronize(stream_);
        cudaStreamDestroy(stream_);
    }
    if (previous >= 0) cudaSetDevice(previous);
}

CompiledRegion::Lane& CompiledRegion::lane(std::size_t k) {
    if (!lanesReady_) {
        lanesReady_ = true;
        for (auto& l : lanes_) {
            check(cudaStreamCreateWithFlags(&l.stream, cudaStreamNonBlocking), "cudaStreamCreateWithFlags(lane)");
            check(cudaEventCreateWithFlags(&l.done, cudaEventDisableTiming), "cudaEventCreate(lane)");
            for (std::size_t i = 0; i < region_.inputs.size(); ++i) l.inputs.push_back(std::make_unique<DeviceBuffer>());
        }
    }
    return lanes_[k % kLanes];
}

DeviceBuffer& CompiledRegion::inputBuffer(std::size_t position) {
    auto& slot = inputs_[position];
    if (!slot) slot = std::make_unique<DeviceBuffer>();
    return *slot;
}

void CompiledRegion::clearErrors(cudaStream_t stream) {
    check(cudaMemsetAsync(errors_.ptr, 0, errorWordCount() * sizeof(std::uint32_t), stream), "cudaMemsetAsync(errors)");
}

void CompiledRegion::copyErrors(cudaStream_t stream, std::uint32_t* host) {
    check(cudaMemcpyAsync(host, errors_.ptr, errorWordCount() * sizeof(std::uint32_t), cudaMemcpyDeviceToHost, stream),
          "cudaMemcpyAsync(errors)");
}

std::string CompiledRegion::firstFailure(const std::uint32_t* words) const {
    for (std::size_t g = 0; g < plan_.groups.size(); ++g) {
        if (!words[g]) continue;
        // Group error codes: bit 0 = checked i64 overflow, bit 1 = recipe
        // divide by zero (the reference's error words 1 and 2,
        // src/backend/v0/NativeGpu.cpp:1123-1125).
        return statusText(words[g]);
    }
    return {};
}

void CompiledRegion::planEvidence(thb_evidence& ev) const {
    ev.logical_tensor_values = plan_.values.size();
    ev.physical_slots = plan_.slots.size();
    ev.fusion_groups = plan_.groups.size();
    ev.logical_intermediates = 0;
    for (const auto& n : region_.nodes)
        if (n.tensor() && n.op != Op::Input && n.op != Op::Alias && n.id != region_.output) ++ev.logical_intermediates;
    ev.materialized_intermediates = 0;
    for (const auto& v : plan_.values)
        if (v.value == v.root && v.materialized && v.klass == ValueClass::Temporary) ++ev.materialized_intermediates;
    ev.physical_temporary_slots = 0;
    ev.reused_slot_assignments = 0;
    for (const auto& s : plan_.slots) {
        if (s.reusable && !s.external) ++ev.physical_temporary_slots;
        std::uint64_t roots = 0;
        for (auto id : s.values) {
            const ValuePlan* v = plan_.value(id);
            roots += v && v->value == v->root;
        }
        if (roots > 1) ev.reused_slot_assignments += roots - 1;
    }
    ev.fused_kernel_groups = 0;
    for (const auto& g : plan_.groups) ev.fused_kernel_groups += g.fused;
    ev.module_loads = moduleLoaded_ ? 1 : 0;
    ev.driver_jit_loads = moduleJitted_ ? 1 : 0;
}

void* CompiledRegion::slotPointer(std::uint32_t value, std::size_t bytes, thb_evidence& ev) {
    const ValuePlan* v = plan_.value(value);
    if (!v || !v->slot)
        fail(Category::Unsupported, "GPU-INVALID-PLAN", "materialized tensor v" + std::to_string(value) + " has no slot");
    if (outputOverride_ && v->root == outputRoot_) return outputOverride_;
    auto& buffer = slots_[*v->slot];
    if (!buffer) buffer = std::make_unique<DeviceBuffer>();
    if (buffer->reserve(bytes, device_)) {
        ++ev.allocation_count;
        ev.allocation_bytes_requested += bytes;
    }
    touched_.insert(*v->slot);
    return buffer->ptr;
}

void CompiledRegion::launchElementwise(const FusionGroup& group, const std::vector<const Value*>& operands,
                                       const std::vector<const Value*>& scalars, Value& out, cudaStream_t stream,
                                       thb_evidence& ev) {
    GroupKernel* kernel = nullptr;
    for (auto& k : kernels_)
        if (k.group == group.id) kernel = &k;
    if (!kernel) fail(Category::Unsupported, "GPU-INVALID-PLAN", "fusion group has no generated kernel");
    const std::uint64_t n = out.count();
    if (n == 0) return;
    bool aligned = (reinterpret_cast<std::uintptr_t>(out.data) % 16) == 0;
    for (const Value* v : operands) aligned = aligned && (reinterpret_cast<std::uintptr_t>(v->data) % 16) == 0;
    const unsigned lanes = group.dtype == DType::F32 ? 4 : 2;
    const std::uint64_t work = aligned ? std::max<std::uint64_t>(1, n / lanes) : n;
    const std::uint64_t perBlock = static_cast<std::uint64_t>(kBlock) * (aligned ? kUnroll : 1);
    // One full resident wave (SMs x resident CTAs per SM) of the grid-stride
    // kernel: measured 1-2 % faster than two waves on the 8192^2 i64 region
    // (interleaved medians, 12 rounds of 20 back-to-back launches).
    const std::uint64_t cap =
        static_cast<std::uint64_t>(info_->smCount) * (aligned ? kernel->vectorResident : kernel->scalarResident);
    const unsigned blocks = static_cast<unsigned>(std::max<std::uint64_t>(1, std::min(cap, (work + perBlock - 1) / perBlock)));
    std::vector<void*> args;
    void* outPtr = out.data;
    std::vector<const void*> inPtrs;
    for (const Value* v : operands) inPtrs.push_back(v->data);
    std::uint64_t count = n;
    std::uint32_t* errorWord = static_cast<std::uint32_t*>(errors_.ptr) + (group.id - 1);
    args.push_back(&outPtr);
    for (auto& p : inPtrs) args.push_back(&p);
    // Runtime scalar operands, by value, in the group's parameter order.
    std::vector<std::int64_t> scalarI64(scalars.size());
    std::vector<float> scalarF32(scalars.size());
    for (std::size_t i = 0; i < scalars.size(); ++i) {
        if (scalars[i]->onDevice)
            fail(Category::Unsupported, "GPU-UNSUPPORTED-OP", "device-computed scalars cannot feed an elementwise chain");
        scalarI64[i] = scalars[i]->i64;
        scalarF32[i] = scalars[i]->f32;
        args.push_back(group.dtype == DType::I64 ? static_cast<void*>(&scalarI64[i]) : static_cast<void*>(&scalarF32[i]));
    }
    args.push_back(&count);
    args.push_back(&errorWord);
    // Large aligned groups stream through the bulk-copy pipeline: at least
    // one whole tile per SM, in one resident wave of persistent CTAs.
    BulkShape shape;
    const std::uint64_t elementBytes = group.dtype == DType::F32 ? 4 : 8;
    if (aligned && kernel->bulkKernel && bulkShape(kernel->arity, shape)) {
        std::uint32_t tile = static_cast<std::uint32_t>(shape.tileBytes / elementBytes);
        std::uint32_t stages = shape.stages;
        const std::uint64_t smem = (static_cast<std::uint64_t>(stages) * kernel->arity + 2) * shape.tileBytes;
        const std::uint64_t tiles = n / tile;
        if (tiles >= static_cast<std::uint64_t>(info_->smCount) && smem <= static_cast<std::uint64_t>(info_->maxSmemOptin)) {
            if (kernel->bulkSmemAllowed < smem) {
                check(cudaFuncSetAttribute(kernel->bulkKernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem)),
                      "cudaFuncSetAttribute(bulk)");
                kernel->bulkSmemAllowed = static_cast<std::uint32_t>(smem);
            }
            if (kernel->bulkResidentSmem != smem) {
                int resident = 0;
                if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, kernel->bulkKernel, kBlock, smem) !=
                        cudaSuccess ||
                    resident < 1) {
                    (void)cudaGetLastError();
                    resident = 1;
                }
                kernel->bulkResident = static_cast<std::uint32_t>(resident);
                kernel->bulkResidentSmem = static_cast<std::uint32_t>(smem);
            }
            const unsigned bulkBlocks = static_cast<unsigned>(
                std::min<std::uint64_t>(tiles, static_cast<std::uint64_t>(info_->smCount) * kernel->bulkResident));
            args.push_back(&stages);
            args.push_back(&tile);
            check(cudaLaunchKernel(kernel->bulkKernel, dim3(bulkBlocks), dim3(kBlock), args.data(), smem, stream),
                  "cudaLaunchKernel(fusion-group, bulk)");
            ++ev.kernel_launches;
            ++ev.stream_submissions;
            return;
        }
    }
    const void* fn = aligned ? kernel->vectorKernel : kernel->scalarKernel;
    check(cudaLaunchKernel(fn, dim3(blocks), dim3(kBlock), args.data(), 0, stream), "cudaLaunchKernel(fusion-group)");
    ++ev.kernel_launches;
    ++ev.stream_submissions;
}

void CompiledRegion::launchReduction(const FusionGroup& group, const Value& in, Value& out, cudaStream_t stream,
                                     thb_evidence& ev) {
    const Node& node = region_.at(group.nodes.front());
    const float* x = static_cast<const float*>(in.data);
    float* y = static_cast<float*>(out.data);
    const std::uint64_t rows = in.rank == 2 ? in.shape[0] : 1;
    const std::uint64_t cols = in.rank == 2 ? in.shape[1] : in.shape[0];
    if (in.count() == 0) {
        if (out.count()) check(cudaMemsetAsync(out.data, 0, out.bytes(), stream), "cudaMemsetAsync(empty-sum)");
        return;
    }
    std::uint32_t* status = static_cast<std::uint32_t*>(errors_.ptr) + (group.id - 1);
    cudaError_t e = cudaSuccess;
    switch (node.op) {
    case Op::Softmax: e = kernels::softmaxRowsF32(x, y, rows, cols, info_->smCount, stream, status); break;
    case Op::RowMax: e = kernels::maxRowsF32(x, y, rows, cols, info_->smCount, stream, status); break;
    case Op::Sum:
        if (node.dtype == DType::I64) {
            const auto* xi = static_cast<const std::int64_t*>(in.data);
            auto* yi = static_cast<std::int64_t*>(out.data);
            if (in.rank == 1) {
                const std::size_t bytes = kernels::sumAllI64ScratchBytes(in.count(), info_->smCount);
                auto& scratch = scalars_[0x80000000u | group.id];
                if (!scratch) scratch = std::make_unique<DeviceBuffer>();
                if (scratch->reserve(bytes, device_)) {
                    ++ev.allocation_count;
                    ev.allocation_bytes_requested += bytes;
                }
                e = kernels::sumAllI64(xi, in.count(), scratch->ptr, yi, info_->smCount, stream, status);
            } else if (node.axis == 1) {
                e = kernels::sumRowsI64(xi, yi, rows, cols, info_->smCount, stream, status);
            } else {
                e = kernels::sumColsI64(xi, yi, rows, cols, stream, status);
            }
        } else if (in.rank == 1) {
            const std::uint32_t parts = kernels::sumAllPartialCount(in.count(), info_->smCount);
            auto& scratch = scalars_[0x80000000u | group.id];
            if (!scratch) scratch = std::make_unique<DeviceBuffer>();
            if (scratch->reserve(parts * sizeof(double), device_)) {
                ++ev.allocation_count;
                ev.allocation_bytes_requested += parts * sizeof(double);
            }
            e = kernels::sumAllF32(x, in.count(), static_cast<double*>(scratch->ptr), parts, nullptr, y,
                                   info_->smCount, stream, status);
        } else if (node.axis == 1) {
            e = kernels::sumRowsF32(x, y, rows, cols, info_->smCount, stream, status);
        } else {
            e = kernels::sumColsF32(x, y, rows, cols, info_->smCount, stream);
        }
        break;
    default: fail(Category::Unsupported, "GPU-UNSUPPORTED-OP", "reduction group holds a non-reduction node");
    }
    check(e, "reduction launch");
    ++ev.kernel_launches;
    ++ev.stream_submissions;
}

void* CompiledRegion::scratch(std::uint32_t key, std::size_t bytes, thb_evidence& ev) {
    auto& buffer = scalars_[key];
    if (!buffer) buffer = std::make_unique<DeviceBuffer>();
    if (buffer->reserve(bytes, device_)) {
        ++ev.allocation_count;
        ev.allocation_bytes_requested += bytes;
    }
    return buffer->ptr;
}

void CompiledRegion::launchKernel(const FusionGroup& group, const std::vector<const Value*>& in, Value& out,
                                  cudaStream_t stream, thb_evidence& ev) {
    const Node& node = region_.at(group.nodes.front());
    std::uint32_t* status = static_cast<std::uint32_t*>(errors_.ptr) + (group.id - 1);
    const int sms = info_->smCount;
    auto launched = [&](cudaError_t e, const char* what) {
        check(e, what);
        ++ev.kernel_launches;
        ++ev.stream_submissions;
    };
    if (out.count() == 0) return;
    switch (node.op) {
    case Op::ZeroLike:
        check(cudaMemsetAsync(out.data, 0, out.bytes(), stream), "cudaMemsetAsync(zero-like)");
        ++ev.stream_submissions;
        return;
    case Op::Transpose:
        launched(kernels::transpose(in[0]->data, out.data, in[0]->shape[0], in[0]->shape[1], width(in[0]->dtype), sms,
                                    stream),
                 "transpose launch");
        return;
    case Op::BroadcastToShape:
        if (in[0]->rank == 0) {  // scalar source: host value or device scalar
            launched(kernels::fillF32(in[0]->onDevice ? static_cast<const float*>(in[0]->data) : nullptr, in[0]->f32,
                                      static_cast<float*>(out.data), out.count(), sms, stream),
                     "broadcast fill");
            return;
        }
        launched(kernels::broadcastF32(static_cast<const float*>(in[0]->data), static_cast<float*>(out.data),
                                       out.rank == 2 ? out.shape[0] : 1, out.rank == 2 ? out.shape[1] : out.shape[0],
                                       out.rank == 2 ? node.axis : 0, sms, stream),
                 "broadcast launch");
        return;
    case Op::ReduceToShape: {
        const Value& src = *in[0];
        const float* x = static_cast<const float*>(src.data);
        float* y = static_cast<float*>(out.data);
        const std::uint64_t rows = src.rank == 2 ? src.shape[0] : 1;
        const std::uint64_t cols = src.rank == 2 ? src.shape[1] : src.shape[0];
        if (out.count() == src.count()) {  // nothing to reduce
            check(cudaMemcpyAsync(out.data, src.data, src.bytes(), cudaMemcpyDeviceToDevice, stream), "reduce copy");
            ++ev.device_to_device_copies;
            ev.device_to_device_bytes += src.bytes();
            return;
        }
        if (out.count() == 1) {
            const std::uint32_t parts = kernels::sumAllPartialCount(src.count(), sms);
            double* partials = static_cast<double*>(scratch(0x20000000u | group.id, parts * sizeof(double), ev));
            launched(kernels::sumAllF32(x, src.count(), partials, parts, nullptr, y, sms, stream), "reduce sum");
            return;
        }
        const bool keepRows = out.rank == 2 ? (out.shape[1] == 1) : false;
        if (keepRows) launched(kernels::sumRowsF32(x, y, rows, cols, sms, stream, status), "reduce rows");
        else launched(kernels::sumColsF32(x, y, rows, cols, sms, stream), "reduce columns");
        return;
    }
    case Op::MatMul: {
        const Value& a = *in[0];
        const Value& b = *in[1];
        const std::uint64_t m = a.shape[0], k = a.shape[1], n = b.shape[1];
        if (k == 0) {  // empty sums: acc stays 0 (Evaluator.cpp:135-141)
            check(cudaMemsetAsync(out.data, 0, out.bytes(), stream), "cudaMemsetAsync(matmul k=0)");
            ++ev.stream_submissions;
            return;
        }
        if (node.dtype == DType::I64) {
            launched(kernels::matmulCheckedI64(static_cast<const std::int64_t*>(a.data),
                                               static_cast<const std::int64_t*>(b.data),
                                               static_cast<std::int64_t*>(out.data), m, k, n, status, stream),
                     "matmul i64 launch");
            return;
        }
        if (node.axis == THB_MATMUL_EXACT) {
            launched(kernels::matmulExactF32(static_cast<const float*>(a.data), static_cast<const float*>(b.data),
                                             static_cast<float*>(out.data), m, k, n, stream),
                     "matmul exact launch");
            return;
        }
        // Tensor cores: bf16 operands with 16-byte row strides. K and N are
        // padded to multiples of 8 with zeros (exact zero products).
        const std::uint64_t kp = (k + 7) / 8 * 8, np = (n + 7) / 8 * 8;
        void* a16 = scratch(0x30000000u | group.id, m * kp * 2, ev);
        void* b16 = scratch(0x38000000u | group.id, kp * np * 2, ev);
        if (kp == k) launched(mlp::castToBf16(static_cast<const float*>(a.data), a16, m * k, sms, stream), "matmul cast A");
        else launched(kernels::castPadBf16(static_cast<const float*>(a.data), a16, m, k, m, kp, sms, stream),
                      "matmul cast A");
        if (kp == k && np == n)
            launched(mlp::castToBf16(static_cast<const float*>(b.data), b16, k * n, sms, stream), "matmul cast B");
        else launched(kernels::castPadBf16(static_cast<const float*>(b.data), b16, k, n, kp, np, sms, stream),
                      "matmul cast B");
        gemm::Problem q;
        q.m = m; q.n = n; q.k = kp;
        q.a = a16; q.lda = kp;
        q.b = b16; q.bMajorMN = true; q.ldb = np;
        q.c = out.data; q.ldc = n; q.epilogue = gemm::kEpiF32;
        if (const char* bad = gemm::validate(q)) fail(Category::Unsupported, "GPU-UNSUPPORTED-SHAPE", bad);
        launched(gemm::run(q, sms, status, stream), "matmul launch");
        return;
    }
    default: fail(Category::Unsupported, "GPU-UNSUPPORTED-OP", "kernel group holds an unexpected node");
    }
}

Value CompiledRegion::run(const std::vector<Value>& inputs, cudaStream_t stream, thb_evidence& ev,
                          void* outputOverride, const std::function<void(const Value&)>& onShapes) {
    check(cudaSetDevice(device_), "cudaSetDevice");
    touched_.clear();
    outputOverride_ = outputOverride;
    const Node& outputNode = region_.at(region_.output);
    outputRoot_ = outputNode.tensor() ? region_.canonical(region_.output) : 0;
    if (outputRoot_) {
        const ValuePlan* rootPlan = plan_.value(outputRoot_);
        if (rootPlan) outputRoot_ = rootPlan->root;
    }
    if (inputs.size() != region_.inputs.size())
        fail(Category::Unsupported, "GPU-INPUT-ARITY", "GPU input arity mismatch");
    std::map<std::uint32_t, Value> values;
    for (std::size_t i = 0; i < inputs.size(); ++i) values[region_.inputs[i]] = inputs[i];

    // Pass 1: runtime shapes and every host-side check, before any launch.
    std::map<std::uint32_t, Value> shapes = values;
    for (const auto& n : region_.nodes) {
        if (n.op == Op::Input) continue;
        Value v;
        v.dtype = n.dtype;
        v.rank = n.rank;
        v.tensor = n.tensor();
        auto dep = [&](std::size_t k) -> const Value& { return shapes.at(region_.canonical(n.dependencies.at(k))); };
        switch (n.op) {
        case Op::Integer: v.i64 = n.integer; break;
        case Op::Float: v.f32 = n.floating; break;
        case Op::TensorLiteral:
            for (std::uint32_t a = 0; a < n.rank; ++a) v.shape[a] = static_cast<std::uint64_t>(n.extent[a]);
            break;
        case Op::Alias: v = dep(0); break;
        case Op::Copy: case Op::Negate: case Op::Relu: case Op::Softmax:
            v.shape[0] = dep(0).shape[0]; v.shape[1] = dep(0).shape[1]; break;
        case Op::Transpose:
            v.shape[0] = dep(0).shape[1]; v.shape[1] = dep(0).shape[0]; break;
        case Op::MatMul: {
            const Value& a = dep(0);
            const Value& b = dep(1);
            if (a.shape[1] != b.shape[0])
                fail(Category::Semantic, "TH-SPEC-SHAPE", "matmul inner extents differ");
            v.shape[0] = a.shape[0]; v.shape[1] = b.shape[1];
            break;
        }
        case Op::BroadcastToShape: {
            const Value& src = dep(0);
            const Value& ref = dep(1);
            // The source is the target with `axis` removed (Evaluator.cpp:278-309).
            const std::uint64_t kept = ref.rank == 2 ? ref.shape[n.axis == 0 ? 1 : 0] : 1;
            if (src.rank + 1 != ref.rank || (ref.rank == 2 && src.shape[0] != kept))
                fail(Category::Semantic, "TH-SPEC-BROADCAST", "broadcast source does not match the target");
            v.shape[0] = ref.shape[0]; v.shape[1] = ref.shape[1];
            break;
        }
        case Op::ReduceToShape: {
            const Value& src = dep(0);
            const Value& ref = dep(1);
            // Target axes of extent 1 (or missing leading axes) are summed
            // (Evaluator.cpp:258-277).
            const std::uint32_t delta = src.rank - ref.rank;
            for (std::uint32_t d = 0; d < ref.rank; ++d)
                if (ref.shape[d] != 1 && ref.shape[d] != src.shape[d + delta])
                    fail(Category::Semantic, "TH-SPEC-BROADCAST", "reduce target does not match the source");
            v.shape[0] = ref.shape[0]; v.shape[1] = ref.shape[1];
            break;
        }
        case Op::ZeroLike:
            v.shape[0] = dep(0).shape[0]; v.shape[1] = dep(0).shape[1]; break;
        case Op::Add: case Op::Subtract: case Op::ElementMultiply: case Op::Extension: case Op::ExtensionGradient: {
            // The result takes the first tensor operand's shape; scalar
            // operands broadcast.
            std::size_t first = 0;
            while (first + 1 < n.dependencies.size() && !dep(first).tensor) ++first;
            const Value& a = dep(first);
            for (std::size_t k = 0; k < n.dependencies.size(); ++k) {
                const Value& b = dep(k);
                if (!b.tensor) continue;
                if (b.rank != a.rank || b.shape[0] != a.shape[0] || b.shape[1] != a.shape[1])
                    fail(Category::Unsupported, "GPU-RUNTIME-SHAPE",
                         "runtime fused elementwise inputs require equal dtype and shape");
            }
            v.shape[0] = a.shape[0]; v.shape[1] = a.shape[1];
            break;
        }
        case Op::Sum: {
            const Value& a = dep(0);
            if (a.rank == 2) v.shape[0] = n.axis == 1 ? a.shape[0] : a.shape[1];
            break;
        }
        case Op::RowMax: {
            const Value& a = dep(0);
            if (a.shape[1] == 0 && a.shape[0] != 0)
                fail(Category::Semantic, "TH-SPEC-EMPTY-REDUCTION", "max over an empty row");
            v.shape[0] = a.shape[0];
            break;
        }
        case Op::Index: {
            const Value& a = dep(0);
            std::uint64_t linear = 0;
            for (std::size_t axis = 0; axis < n.indices.size(); ++axis) {
                const Value& c = shapes.at(region_.canonical(n.indices[axis]));
                if (c.onDevice)
                    fail(Category::Unsupported, "GPU-DYNAMIC-INDEX", "device-computed index coordinates are unsupported");
                if (c.i64 < 0 || static_cast<std::uint64_t>(c.i64) >= a.shape[axis])
                    fail(Category::Semantic, "TH-SPEC-BOUNDS", "GPU index is out of bounds");
                linear = linear * a.shape[axis] + static_cast<std::uint64_t>(c.i64);
            }
            v.i64 = static_cast<std::int64_t>(linear);  // linear offset, used in pass 2
            v.onDevice = true;
            break;
        }
        default: fail(Category::Unsupported, "GPU-UNSUPPORTED-OP", std::string("no GPU lowering for ") + opName(n.op));
        }
        for (std::uint32_t a = 0; a < n.rank; ++a)
            if (n.extent[a] >= 0 && static_cast<std::uint64_t>(n.extent[a]) != v.shape[a])
                fail(Category::Unsupported, "GPU-RUNTIME-SHAPE", "runtime shape disagrees with the region's shape fact");
        shapes[n.id] = v;
    }
    if (onShapes) onShapes(shapes.at(region_.output));

    // Pass 2: materialise and launch in region order.
    std::set<std::uint32_t> launched;
    for (const auto& n : region_.nodes) {
        if (n.op == Op::Input) continue;
        Value v = shapes.at(n.id);
        switch (n.op) {
        case Op::Integer: case Op::Float: break;
        case Op::Alias: {
            // An alias of a fused intermediate names a value that is never
            // materialized (src/backend/v0/NativeGpu.cpp:984-988 skips it the same way).
            auto found = values.find(region_.canonical(n.dependencies.at(0)));
            if (found == values.end()) continue;
            v = found->second;
            break;
        }
        case Op::TensorLiteral: {
            v.data = slotPointer(n.id, v.bytes(), ev);
            bool device = false;
            for (auto d : n.dependencies) device = device || values.at(d).onDevice;
            if (device) {
                const std::size_t w = width(n.dtype);
                for (std::size_t k = 0; k < n.dependencies.size(); ++k) {
                    const Value& s = values.at(n.dependencies[k]);
                    if (s.onDevice)
                        check(cudaMemcpyAsync(static_cast<char*>(v.data) + k * w, s.data, w, cudaMemcpyDeviceToDevice, stream),
                              "cudaMemcpyAsync(literal)");
                    else
                        check(cudaMemcpyAsync(static_cast<char*>(v.data) + k * w,
                                              n.dtype == DType::I64 ? static_cast<const void*>(&s.i64)
                                                                    : static_cast<const void*>(&s.f32),
                                              w, cudaMemcpyHostToDevice, stream),
                              "cudaMemcpyAsync(literal)");
                    ++ev.device_to_device_copies;
                    ev.device_to_device_bytes += w;
                }
            } else if (v.bytes()) {
                std::vector<unsigned char> host(v.bytes());
                for (std::size_t k = 0; k < n.dependencies.size(); ++k) {
                    const Value& s = values.at(n.dependencies[k]);
                    if (n.dtype == DType::I64) std::memcpy(host.data() + 8 * k, &s.i64, 8);
                    else std::memcpy(host.data() + 4 * k, &s.f32, 4);
                }
                check(cudaMemcpyAsync(v.data, host.data(), host.size(), cudaMemcpyHostToDevice, stream),
                      "cudaMemcpyAsync(literal)");
                ++ev.host_to_device_copies;
                ev.host_to_device_bytes += host.size();
            }
            break;
        }
        case Op::Copy: {
            const Value& src = values.at(region_.canonical(n.dependencies.at(0)));
            v.data = v.bytes() ? slotPointer(n.id, v.bytes(), ev) : nullptr;
            if (v.bytes()) {
                check(cudaMemcpyAsync(v.data, src.data, v.bytes(), cudaMemcpyDeviceToDevice, stream), "cudaMemcpyAsync(copy)");
                ++ev.device_to_device_copies;
                ev.device_to_device_bytes += v.bytes();
                ++ev.stream_submissions;
            }
            break;
        }
        case Op::Index: {
            const Value& src = values.at(region_.canonical(n.dependencies.at(0)));
            auto& buffer = scalars_[n.id];
            if (!buffer) buffer = std::make_unique<DeviceBuffer>();
            if (buffer->reserve(8, device_)) ++ev.allocation_count;
            const std::size_t w = width(src.dtype);
            check(cudaMemcpyAsync(buffer->ptr, static_cast<const char*>(src.data) + static_cast<std::size_t>(v.i64) * w, w,
                                  cudaMemcpyDeviceToDevice, stream),
                  "cudaMemcpyAsync(index)");
            ++ev.device_to_device_copies;
            ev.device_to_device_bytes += w;
            v.data = buffer->ptr;
            v.onDevice = true;
            break;
        }
        default: {
            const FusionGroup* group = plan_.groupFor(n.id);
            if (!group) fail(Category::Unsupported, "GPU-INVALID-PLAN", "kernel node outside every group");
            // Only the group's first node launches; the others (fused
            // intermediates and the terminal) are produced by that launch.
            if (group->nodes.front() != n.id || !launched.insert(group->id).second) continue;
            const Value& shape = shapes.at(group->output);
            Value out = shape;
            if (out.rank == 0) {  // scalar reduction result lives in a device scalar buffer
                auto& buffer = scalars_[group->output];
                if (!buffer) buffer = std::make_unique<DeviceBuffer>();
                if (buffer->reserve(8, device_)) ++ev.allocation_count;
                out.data = buffer->ptr;
                out.onDevice = true;
            } else {
                out.data = out.bytes() ? slotPointer(group->output, out.bytes(), ev) : nullptr;
            }
            if (group->kind == GroupKind::Elementwise) {
                std::vector<const Value*> operands;
                for (auto id : group->inputs) operands.push_back(&values.at(id));
                std::vector<const Value*> scalars;
                for (auto id : group->scalars) scalars.push_back(&values.at(id));
                launchElementwise(*group, operands, scalars, out, stream, ev);
            } else if (group->kind == GroupKind::Kernel) {
                std::vector<const Value*> operands;
                for (auto d : n.dependencies) operands.push_back(&values.at(region_.canonical(d)));
                launchKernel(*group, operands, out, stream, ev);
            } else {
                launchReduction(*group, values.at(region_.canonical(n.dependencies.at(0))), out, stream, ev);
            }
            values[group->output] = out;
            continue;
        }
        }
        values[n.id] = v;
    }
    ev.planner_owned_allocations = 0;
    for (auto id : touched_) ev.planner_owned_allocations += !plan_.slots.at(id - 1).external;
    ev.retained_planner_allocations = ev.planner_owned_allocations;
    Value result = values.at(region_.output);
    if (outputOverride && result.tensor && result.data != outputOverride && result.bytes()) {
        check(cudaMemcpyAsync(outputOverride, result.data, result.bytes(), cudaMemcpyDeviceToDevice, stream),
              "cudaMemcpyAsync(output)");
        ++ev.device_to_device_copies;
        ev.device_to_device_bytes += result.bytes();
        result.data = outputOverride;
    }
    outputOverride_ = nullptr;
    return result;
}

} // namespace thb
