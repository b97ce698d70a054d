// Full-tensor f32 sum that allocates nothing.
//
// Some hosts that embed this library own every byte of device memory through
// their own allocator and do not let a component call cudaMalloc / cudaFree
// (those calls can synchronise the whole device and fragment the host's
// pool). Such a caller passes its input and output buffers and cannot give
// the reduction any scratch. This entry point keeps the reduction's block
// partials in a fixed array compiled into the library instead: kMaxPartials
// f64 values (32 KiB) of device memory that every GPU loading the library
// holds until the process exits, plus one u32 status word the kernels raise
// when a bounded wait runs out.
//
// The reduction is the same two-pass kernel pair as the region Sum path
// (kernels::sumAllF32 in reduce.cu, same fixed grid), so both give
// identical results for the same input.
#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <mutex>
#include <string>

#include "kernels.hpp"
#include "runtime.hpp"

namespace thb::noalloc {

constexpr std::uint32_t kMaxPartials = 4096;

// The shared scratch: one f64 partial per block of pass 1. In host code the
// name is only a stand-in; kernels receive the device address obtained with
// cudaGetSymbolAddress below.
static __device__ __align__(256) double gSumScratch[kMaxPartials];
// Status word of the call in flight: bit 4 (16) a bounded wait ran out, bit 5
// (32) the copies in flight could not be drained after that. Cleared by every
// call before its launches.
static __device__ __align__(4) std::uint32_t gSumStatus;

namespace {

struct Scratch {
    double* partials = nullptr;
    std::uint32_t* status = nullptr;
};

std::mutex addressMutex;
std::map<int, Scratch> addresses;  // device ordinal -> device addresses of the static arrays

// Resolves the device addresses of gSumScratch and gSumStatus once per
// device, with that device current. The addresses stay valid for the life of
// the device's primary context: a host that resets the device
// (cudaDeviceReset) after the first call must not call this entry point
// again. Throws on failure.
Scratch scratchAddress(int device) {
    std::lock_guard<std::mutex> lock(addressMutex);
    auto found = addresses.find(device);
    if (found != addresses.end()) return found->second;
    Scratch s;
    cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.partials), gSumScratch);
    if (e != cudaSuccess || !s.partials)
        fail(Category::Runtime, "GPU-NOALLOC-SETUP",
             std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.status), gSumStatus);
    if (e != cudaSuccess || !s.status)
        fail(Category::Runtime, "GPU-NOALLOC-SETUP",
             std::string("cudaGetSymbolAddress(status): ") + cudaGetErrorString(e));
    addresses.emplace(device, s);
    return s;
}

} // namespace

} // namespace thb::noalloc

extern "C" int thb_sum_all_f32_noalloc(int device, const float* x, uint64_t n, float* outF32, double* outF64,
                                       void* stream, char* failure, uint64_t cap) {
    using namespace thb;
    try {
        if ((n && !x) || (!outF32 && !outF64))
            fail(Category::Validation, "GPU-NOALLOC-ARGUMENT", "input is null or no output was given");
        const DeviceInfo& info = useDevice(device);  // also makes `device` current
        const std::uint32_t parts = kernels::sumAllPartialCount(n, info.smCount);
        if (parts > noalloc::kMaxPartials)
            fail(Category::Validation, "GPU-NOALLOC-SIZE",
                 "this reduction needs " + std::to_string(parts) + " block partials; the static scratch holds " +
                     std::to_string(noalloc::kMaxPartials));
        const noalloc::Scratch scratch = noalloc::scratchAddress(device);
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        cudaError_t e = cudaMemsetAsync(scratch.status, 0, sizeof(std::uint32_t), s);
        if (e == cudaSuccess)
            e = kernels::sumAllF32(x, n, scratch.partials, parts, outF64, outF32, info.smCount, s, scratch.status);
        if (e != cudaSuccess)
            fail(Category::Runtime, "GPU-RUNTIME", std::string("full-sum launch: ") + cudaGetErrorString(e));
        // The call returns the result's status: wait for the stream and read
        // the status word (into host memory; nothing is allocated).
        std::uint32_t word = 0;
        e = cudaMemcpyAsync(&word, scratch.status, sizeof word, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess)
            fail(Category::Runtime, "GPU-RUNTIME", std::string("full-sum status read: ") + cudaGetErrorString(e));
        if (word) fail(Category::Runtime, statusText(word), "a bounded wait of the full sum ran out; the outputs are invalid");
        return THB_STATUS_OK;
    } catch (const Failure& f) {
        writeText(failure, cap, f.text());
        return f.status();
    } catch (const std::exception& ex) {
        writeText(failure, cap, std::string("GPU-INTERNAL: ") + ex.what());
        return THB_STATUS_UNKNOWN;
    }
}
