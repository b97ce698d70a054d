// CUDA source generation for elementwise fusion groups and NVRTC compilation.
//
// The reference emits one PTX entry per fusion group (groupPtx,
// src/backend/v0/NativeGpu.cpp:473-588): one element per thread, scalar loads,
// IR-ordered add/sub/mul.rn.f32, inlined extension recipes with a divide-by-
// zero flag, checked i64 arithmetic that sets an error word. This engine keeps
// the same arithmetic contract but generates CUDA C++ for a grid-stride,
// 128-bit vectorised, streaming-cache kernel and compiles it once per region
// shape for sm_100a; the compiled module is cached by the digest of its text.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "region.hpp"

namespace thb {

// Elements moved per 128-bit access and accesses in flight per thread.
constexpr unsigned kBlock = 256;
constexpr unsigned kUnroll = 4;

struct GroupKernel {
    std::uint32_t group = 0;
    DType dtype = DType::F32;
    std::size_t arity = 0;          // number of tensor inputs
    std::string vectorName, scalarName;
    void* vectorKernel = nullptr;   // cudaKernel_t
    void* scalarKernel = nullptr;
    unsigned vectorResident = 4;    // resident CTAs per SM at kBlock threads
    unsigned scalarResident = 4;
    // Bulk-copy pipelined entry (groups with tensor inputs; null when the
    // module lacks it): extra arguments (stages, tile elements), dynamic
    // shared memory (stages * arity + 2) * tile * element size.
    std::string bulkName;
    void* bulkKernel = nullptr;
    std::uint32_t bulkSmemAllowed = 0;  // dynamic shared memory the entry is configured for
    std::uint32_t bulkResident = 1;     // resident CTAs per SM at bulkResidentSmem
    std::uint32_t bulkResidentSmem = 0;
};

// Most ring stages of the bulk entry.
constexpr unsigned kBulkMaxStages = 8;

struct Module;  // compiled NVRTC library (opaque)

// Generates the CUDA source for every elementwise group of `plan`, in group
// order. `kernels` receives one record per generated group.
std::string generateSource(const Region&, const Plan&, std::vector<GroupKernel>& kernels);

// Compiles `source` for sm_100a with NVRTC (or takes it from the in-process /
// on-disk cache, or from `prebuiltCubin`, an artifact's cubin of this exact
// source) and loads it on the current device. Fills the kernel handles.
// `jitted` reports whether NVRTC ran (a cache miss).
std::shared_ptr<Module> compileAndLoad(const std::string& source, int device,
                                       std::vector<GroupKernel>& kernels, bool& jitted, bool& loaded,
                                       const std::string* prebuiltCubin = nullptr);

std::uint64_t fnv1a(const std::string&);

// NVRTC compilation only (no device): returns the sm_100a cubin.
std::string compileCubin(const std::string& source);

} // namespace thb
