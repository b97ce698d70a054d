// Persistent device runtime of the B200 engine.
//
// The reference creates a context, stream and module and allocates every slot
// on each call (NativeGpuPendingState, src/backend/v0/NativeGpu.cpp:849-907,
// submitWork :951-1119). Here a compiled region owns, for its lifetime, one
// non-blocking stream, its loaded module, a pool of device slot buffers sized
// on first use, pinned staging, and one 32-bit error word per fusion group.
// Launches are stream-ordered; only observation synchronises.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <functional>
#include <map>
#include <set>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "codegen.hpp"
#include "region.hpp"

namespace thb {

struct DeviceBuffer {
    void* ptr = nullptr;
    std::size_t bytes = 0;
    int device = -1;
    DeviceBuffer() = default;
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    ~DeviceBuffer();
    // Ensures capacity >= bytes; returns true when a new allocation was made.
    bool reserve(std::size_t bytes, int device);
};

struct PinnedBuffer {
    void* ptr = nullptr;
    std::size_t bytes = 0;
    PinnedBuffer() = default;
    PinnedBuffer(const PinnedBuffer&) = delete;
    PinnedBuffer& operator=(const PinnedBuffer&) = delete;
    ~PinnedBuffer();
    void reserve(std::size_t bytes);
};

// Device properties cached per ordinal.
struct DeviceInfo {
    int ordinal = 0;
    int smCount = 148;
    int major = 0, minor = 0;
    int maxSmemOptin = 232448;  // dynamic shared memory a block may opt into
};

// Selects `ordinal` as the current device after validating it; throws
// GPU-DRIVER-NOT-FOUND / GPU-INVALID-DEVICE.
const DeviceInfo& useDevice(int ordinal);

// Per-device 32-bit status word latched by kernels launched outside a
// region (bit 4 = a bounded wait expired). Allocated zeroed on first use.
std::uint32_t* deviceStatus(int ordinal);
// Text of a nonzero status word.
std::string statusText(std::uint32_t word);

// A runtime value during one execution.
struct Value {
    bool tensor = false;
    bool onDevice = false;  // tensor: always; scalar: produced by Index on the device
    DType dtype = DType::F32;
    std::uint32_t rank = 0;
    std::uint64_t shape[2] = {0, 0};
    void* data = nullptr;   // device pointer (tensors, device scalars)
    std::int64_t i64 = 0;   // host scalar
    float f32 = 0.0f;       // host scalar
    std::uint64_t count() const { return rank == 0 ? 1 : (rank == 1 ? shape[0] : shape[0] * shape[1]); }
    std::size_t bytes() const { return static_cast<std::size_t>(count()) * width(dtype); }
};

class CompiledRegion {
public:
    CompiledRegion(const thb_region_desc&, PlanOptions, int device);
    // From an imported region (an artifact's); `prebuiltCubin`, when given,
    // is the cubin of exactly the source this region generates.
    CompiledRegion(Region region, PlanOptions, int device, const std::string* prebuiltCubin);
    ~CompiledRegion();

    const Region& region() const { return region_; }
    const Plan& plan() const { return plan_; }
    const std::string& source() const { return source_; }
    int device() const { return device_; }
    cudaStream_t stream() const { return stream_; }

    // Runs the plan on `stream` over already-bound inputs (device tensors or
    // host scalars). Returns the output value (device tensor, device scalar or
    // host scalar). Every shape/bounds check happens before the first launch.
    // `outputOverride` (optional) is a device buffer that receives the region
    // output instead of the output slot; `onShapes` (optional) sees the output
    // description after shape inference and may throw to stop before launch.
    Value run(const std::vector<Value>& inputs, cudaStream_t stream, thb_evidence& evidence,
              void* outputOverride = nullptr, const std::function<void(const Value&)>& onShapes = {});

    // Error words: clear (stream-ordered), copy to host (stream-ordered).
    void clearErrors(cudaStream_t stream);
    void copyErrors(cudaStream_t stream, std::uint32_t* host);
    std::size_t errorWordCount() const { return plan_.groups.size(); }
    // First failing group in region order, or empty.
    std::string firstFailure(const std::uint32_t* words) const;

    void planEvidence(thb_evidence& evidence) const;

    // Upload buffers for host-mode inputs, one per input position.
    DeviceBuffer& inputBuffer(std::size_t position);
    std::mutex mutex;

    // Chunked host execution: a row-local region (one kernel group whose
    // output rows depend only on the same input rows) runs chunk by chunk on
    // three streams, so the host->device copy of chunk k+1, the kernel on
    // chunk k and the device->host copy of chunk k-1 overlap.
    struct Lane {
        cudaStream_t stream = nullptr;
        cudaEvent_t done = nullptr;
        std::vector<std::unique_ptr<DeviceBuffer>> inputs;
        DeviceBuffer output;
    };
    static constexpr std::size_t kLanes = 3;
    bool rowLocal() const { return rowLocal_; }
    Lane& lane(std::size_t k);

private:
    void launchElementwise(const FusionGroup&, const std::vector<const Value*>& operands,
                           const std::vector<const Value*>& scalars, Value& out, cudaStream_t stream,
                           thb_evidence& evidence);
    void launchReduction(const FusionGroup&, const Value& operand, Value& out, cudaStream_t stream,
                         thb_evidence& evidence);
    void launchKernel(const FusionGroup&, const std::vector<const Value*>& operands, Value& out,
                      cudaStream_t stream, thb_evidence& evidence);
    void* scratch(std::uint32_t key, std::size_t bytes, thb_evidence& evidence);
    void* slotPointer(std::uint32_t value, std::size_t bytes, thb_evidence& evidence);

    Region region_;
    Plan plan_;
    int device_ = 0;
    const DeviceInfo* info_ = nullptr;
    std::string source_;
    std::vector<GroupKernel> kernels_;
    std::shared_ptr<Module> module_;
    bool moduleJitted_ = false, moduleLoaded_ = false;
    cudaStream_t stream_ = nullptr;
    DeviceBuffer errors_;
    std::map<std::uint32_t, std::unique_ptr<DeviceBuffer>> slots_;
    std::map<std::uint32_t, std::unique_ptr<DeviceBuffer>> scalars_;
    std::map<std::size_t, std::unique_ptr<DeviceBuffer>> inputs_;
    std::set<std::uint32_t> touched_;      // slots used by the current run
    bool rowLocal_ = false;
    bool lanesReady_ = false;
    Lane lanes_[kLanes];
    void* outputOverride_ = nullptr;
    std::uint32_t outputRoot_ = 0;
};

// One submitted execution (PendingGpuExecution, NativeGpu.hpp:107-137).
struct Pending {
    std::shared_ptr<CompiledRegion> region;
    cudaEvent_t done = nullptr;
    PinnedBuffer output;      // staged tensor output
    PinnedBuffer errors;      // staged error words
    Value result;             // output description
    std::size_t outputBytes = 0;
    thb_evidence evidence{};
    bool observed = false;
    int status = THB_STATUS_OK;
    std::string failureText;
    std::uint64_t reads = 0;  // distinct input storages
    ~Pending();
};

void recordUnobserved(const std::string& id);
std::vector<std::string> takeUnobserved();

} // namespace thb
