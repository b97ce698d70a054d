// `.thm` model bundles (src/model/v0/ModelBundle.cpp) read by this engine and
// executed on device-resident frozen parameters.
//
// The container is the reference's: "THIRANMB", format and runtime-ABI
// versions, payload size and FNV-1a 64 digest, then the payload (identity,
// entry, parameter digest, frozen parameters in the persistence format,
// public ABI, bindings, one or two embedded `.tha` artifacts;
// serializeBundle / loadModelBundle, :139-178, :362-430). Validation follows
// validateModelBundle (:242-326) with its MODEL-* ids.
//
// Execution differs from the reference's submitModelGpu (:461-474), which
// binds every frozen parameter as a host value and uploads it on each call:
// here a compiled model uploads the parameters once, keeps them in HBM, and
// each call uploads only the public inputs.
#pragma once

#include <cstdint>
#include <optional>
#include <string>
#include <vector>

#include "artifact.hpp"

namespace thb::model {

// persistence::StoredValue (include/persistence/v0/Persistence.hpp:21-27).
struct StoredValue {
    std::uint8_t kind = 2;   // 1 scalar, 2 tensor
    std::uint8_t dtype = 2;  // 1 i64, 2 f32
    std::vector<std::uint64_t> shape;
    std::string bytes;
};

struct Parameter {
    std::uint64_t id = 0;
    std::string name;
    StoredValue value;
};

struct Bundle {
    std::string identity, entry, parameterDigest;
    std::vector<Parameter> parameters;
    std::vector<artifact::Type> publicInputs;
    artifact::Type result;
    std::vector<std::pair<std::uint32_t, std::uint32_t>> publicBindings;     // public index -> artifact slot
    std::vector<std::pair<std::uint64_t, std::uint32_t>> parameterBindings;  // parameter id -> artifact slot
    std::optional<artifact::Artifact> gpu;  // the embedded GPU artifact
    bool hasCpu = false;                    // an embedded CPU artifact (not executed here)
};

// Parses and validates; throws Failure(Validation, "MODEL-...").
Bundle load(const std::string& bytes, const std::string* expectedIdentity);

// The artifact input slot -> source of every input: a public input index
// (>= 0) or a parameter (-1 - position in `parameters`).
std::vector<std::int64_t> slotSources(const Bundle&);

std::string inspect(const Bundle&);

} // namespace thb::model
