// Reference-side binding of the B200 engine: the C++ a Thiran maintainer
// adds to the reference tree so that `--backend gpu` runs on
// libthiran_b200.so. It compiles against the reference's own headers
// (include/backend/v0/NativeGpu.hpp, include/semantic/v0/Ir.hpp) and the
// engine's C ABI (include/thiran_b200.h), and keeps the reference's types on
// its side of the boundary.
//
// Entry points (plus probeNativeGpu and loadAndExecuteArtifact below):
//  - lowerFunction: a function of a verified semantic module becomes an
//    engine region. It admits what extractStrictRegion admits
//    (src/backend/v0/TensorRegion.cpp:230-447) and also the operations the
//    reference rejects there ("MatMul / Sum / Transpose / AD helper lowering
//    deferred", :424-431): Matmul, Sum, Transpose (and its borrowed view),
//    StopGradient, ZeroLike, ReduceToShape and BroadcastToShape, scalar
//    Multiply, trailing-axis broadcasts of a rank-1 operand, and a returned
//    tuple (one element per region). Autodiff's generated backward functions
//    (src/autodiff/v0/Autodiff.cpp:72-294) are such functions.
//  - executeNativeGpu: the body of the reference's executeNativeGpu
//    (NativeGpu.hpp:219-222) over the engine, same signature. It lives in
//    namespace b200 here because this build also links the reference's own
//    definition; in the reference tree it replaces that definition.
#pragma once

#include "analysis/v0/Ownership.hpp"
#include "artifact/v0/NativeArtifacts.hpp"
#include "backend/v0/NativeGpu.hpp"
#include "semantic/v0/Ir.hpp"
#include "thiran_b200.h"

#include <cstdint>
#include <deque>
#include <memory>
#include <optional>
#include <string>
#include <vector>

namespace thiran::v0::backend::b200 {

// How f32 Matmul nodes run: the reference's sequential f32 sums, bit-exact on
// the CUDA cores, or bf16 operands on the tensor cores (f32 accumulation).
enum class MatmulMode { Exact, TensorCores };

// Engine records of one region, with the storage they point into.
struct LoweredRegion {
    std::string name;
    std::vector<thb_region_node> nodes;
    std::deque<std::vector<std::uint32_t>> lists;   // dependencies and index coordinates
    std::vector<std::uint32_t> inputs;
    struct Operation {                              // an extension operation as thb_operation
        std::string name, version;
        std::vector<thb_scalar_node> forward;
        std::deque<std::vector<thb_scalar_node>> gradientNodes;
        std::vector<thb_scalar_recipe> gradients;
        thb_derivative derivative{};
        thb_operation record{};
    };
    std::deque<Operation> operations;
    thb_region_desc desc{};
    std::string coverage;  // one line per lowered operation
};

struct LoweringResult {
    std::unique_ptr<LoweredRegion> region;
    std::string diagnostic;  // "BACKEND-UNSUPPORTED: ..." when region is null
    bool ok() const { return region != nullptr; }
};

// Lowers `name` from `module` (verified, one function of that name). When the
// function returns a tuple, `element` selects the tuple element the region
// computes; otherwise it must be 0.
LoweringResult lowerFunction(const semantic::Module& module, const std::string& name, std::size_t element = 0,
                             MatmulMode matmul = MatmulMode::Exact);

// The reference's own region (extractStrictRegion's subset) as engine records.
std::unique_ptr<LoweredRegion> lowerRegion(const TensorRegion& region);

// Runs a lowered region on `device` with host inputs: the same contract as
// executeNativeGpu (inputs uploaded, result downloaded before return, checked
// failures as GpuError with the reference's ids, no fallback).
GpuExecutionResult executeLowered(const LoweredRegion& region, const std::vector<GpuValue>& inputs, int device,
                                  PhysicalPlanOptions options) noexcept;

// executeNativeGpu (NativeGpu.hpp:219-222) over the engine.
GpuExecutionResult executeNativeGpu(const TensorRegion& region, const std::vector<GpuValue>& inputs, int device,
                                    PhysicalPlanOptions options) noexcept;

// probeNativeGpu (NativeGpu.hpp:102) over the engine.
GpuDeviceInfo probeNativeGpu(int device) noexcept;

// The GPU branch of artifact::loadAndExecuteArtifact
// (include/artifact/v0/NativeArtifacts.hpp:138-139), which `thiran run
// --backend gpu <file.tha>` reaches: the reference's loader validates the
// container (digests, signature, region), and a GPU artifact's region runs
// on the engine (its PTX payload is digest-checked by the loader but not
// executed). A CPU artifact is refused with ARTIFACT-BACKEND (the reference
// keeps running those itself). Artifacts this engine built (payload kind 3,
// an sm_100a cubin) are outside the reference's loader; engine-aware callers
// load them with thb_artifact_load_file. Failures come back as ArtifactError
// with the reference's ids.
artifact::ArtifactExecutionResult loadAndExecuteArtifact(const std::string& path,
                                                         const std::vector<artifact::ArtifactValue>& inputs,
                                                         int device) noexcept;

} // namespace thiran::v0::backend::b200
