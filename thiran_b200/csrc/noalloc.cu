// Full-tensor f32 sum that allocates nothing.
//
// Some hosts that embed this library own every byte of device memory through
// their own allocator and do not let a component call cudaMalloc / cudaFree
// (those calls can synchronise the whole device and fragment the host's
// pool). Such a caller passes its input and output buffers and cannot give
// the reduction any scratch. This entry point keeps the reduction's block
// partials in a fixed array compiled into the library instead: kMaxPartials
// f64 values (32 KiB) of device memory that every GPU loading the library
// holds until the process exits.
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

namespace {

std::mutex addressMutex;
std::map<int, double*> addresses;  // device ordinal -> device address of gSumScratch

// Resolves the scratch's device address once per device, with that device
// current. Throws on failure.
double* scratchAddress(int device) {
    std::lock_guard<std::mutex> lock(addressMutex);
    auto found = addresses.find(device);
    if (found != addresses.end()) return found->second;
    double* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), gSumScratch);
    if (e != cudaSuccess || !ptr)
        fail(Category::Runtime, "GPU-NOALLOC-SETUP",
             std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    addresses.emplace(device, ptr);
    return ptr;
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
        double* scratch = noalloc::scratchAddress(device);
        const cudaError_t e =
            kernels::sumAllF32(x, n, scratch, parts, outF64, outF32, info.smCount, static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess)
            fail(Category::Runtime, "GPU-RUNTIME", std::string("full-sum launch: ") + cudaGetErrorString(e));
        return THB_STATUS_OK;
    } catch (const Failure& f) {
        writeText(failure, cap, f.text());
        return f.status();
    } catch (const std::exception& ex) {
        writeText(failure, cap, std::string("GPU-INTERNAL: ") + ex.what());
        return THB_STATUS_UNKNOWN;
    }
}
