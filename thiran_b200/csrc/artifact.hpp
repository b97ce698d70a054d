// `.tha` native artifacts: the reference's container
// (src/artifact/v0/NativeArtifacts.cpp:547-572, loadArtifactBytes :1100-1140)
// read and written by this engine.
//
// The container is kept byte-compatible: "THIRAN16", a little-endian
// manifest, the serialized TensorRegion (:244-331) and a payload. Reference
// GPU artifacts (payload kind 2, generated PTX) load and run here: their
// region is verified (size, FNV-1a digest, region rules) and planned onto this
// engine's kernels; the PTX payload is integrity-checked but not executed.
// The engine adds payload kind 3: the region's generated CUDA source and its
// sm_100a cubin, so loading one needs no NVRTC run. Engine-only region ops
// (Sum, MatMul, ... numbered from 32) may appear only in kind-3 artifacts;
// their axis travels in the node's optional integer field.
#pragma once

#include <cstdint>
#include <optional>
#include <string>
#include <vector>

#include "region.hpp"

namespace thb::artifact {

constexpr std::uint8_t kBackendCpu = 1, kBackendGpu = 2;          // NativeBackend
constexpr std::uint8_t kPayloadElf = 1, kPayloadPtx = 2;          // PayloadKind
constexpr std::uint8_t kPayloadB200 = 3;                          // engine addition
constexpr const char* kReferenceGpuTarget = "ptx60-sm50-min-cc50";
constexpr const char* kReferenceGpuRuntime = "native-runtime-abi=1;libcuda.so.1;driver-ptx-jit;min-cc=5.0";
constexpr const char* kReferenceCpuRuntime = "native-runtime-abi=1;system-cxx-runtime";
constexpr const char* kEngineTarget = "sm_100a";
constexpr const char* kEngineRuntime = "thiran-b200-runtime-abi=1;libcudart;sm_100a";

// ArtifactType (include/artifact/v0/NativeArtifacts.hpp:24-30).
struct Type {
    std::uint8_t kind = 1;   // 1 scalar, 2 tensor
    std::uint8_t dtype = 0;  // 1 i64, 2 f32
    std::uint32_t rank = 0;
    std::vector<std::optional<std::uint64_t>> extents;
};

struct Manifest {
    std::uint32_t formatVersion = 0, compilerAbiVersion = 1, runtimeAbiVersion = 1;
    std::uint8_t backend = kBackendGpu, payloadKind = kPayloadB200;
    bool enableReuse = true, enableFusion = true;
    std::string target, runtimeRequirement, entryName;
    std::vector<Type> parameters;
    Type result;
    std::string planDigest;
    std::uint64_t regionSize = 0;
    std::string regionDigest;
    std::uint64_t payloadSize = 0;
    std::string payloadDigest;
};

struct Artifact {
    Manifest manifest;
    Region region;
    std::string payload;
    // Kind 3: the payload's generated source and cubin.
    std::string engineSource, engineCubin;
};

// "fnv1a64:%016x" of bytes (digestBytes, NativeArtifacts.cpp:948-957).
std::string digest(const std::string& bytes);

// Parses and validates an artifact; throws Failure(Validation, "ARTIFACT-...")
// with the reference's error ids. CPU artifacts (ELF payload) are accepted
// only with `acceptCpu` (a model bundle checks their signature; they never
// execute here).
Artifact load(const std::string& bytes, bool acceptCpu = false);

// Builds a kind-3 artifact of `region` (device-free: NVRTC only).
std::string build(const Region& region, PlanOptions options);

// Manifest, region and plan as JSON text.
std::string inspect(const Artifact&);

} // namespace thb::artifact
