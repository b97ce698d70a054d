// shim_driver: exercises the reference-side binding (NativeGpuB200.cpp) from
// the command line. It parses and analyses a V0 program with the reference's
// own front end, lowers functions with the shim and runs them on the engine.
//
//   shim_driver lower <program.th> <function> [element] [exact|tensor]
//       prints the lowered region (one line per node: id op dtype rank
//       extents deps axis) or the BACKEND-UNSUPPORTED diagnostic; no device.
//   shim_driver run <program.th> <function> <element> <exact|tensor> <device> <out.bin> [in.bin ...]
//       lowerFunction + executeLowered; writes the result.
//   shim_driver native <program.th> <function> <device> <out.bin> [in.bin ...]
//       the reference's extractStrictGpu region through b200::executeNativeGpu.
//   shim_driver artifact <file.tha> <device> <out.bin> [in.bin ...]
//       loadAndExecuteArtifact: the reference's loader, the region on the engine.
//   shim_driver vjp <program.th> <function> <exact|tensor> <device> <out-prefix> <cotangent.bin> [in.bin ...]
//       autodiff::differentiate over every parameter; the generated forward
//       function runs on the engine one tuple element (primal, saved values)
//       per region, then the generated backward function one gradient per
//       region. Writes <prefix>primal.bin and <prefix>grad<k>.bin, and the
//       reference's executeVjpWithPrimal results as <prefix>ref_primal.bin /
//       <prefix>ref_grad<k>.bin.
//
// Each run prints one JSON line: {"status":"ok"} or
// {"status":"error","code":...,"category":...}.
// Tensor files: "THB1", u32 dtype (1 i64, 2 f32), u32 rank, u64 shape[rank],
// little-endian elements; rank 0 is a scalar.
//
// Programs may call `research_chain` (((x*1.5+0.25)*x - x)*0.5 + x with its
// derivative) and `research_square_linear` (x*x + x, derivative 2x + 1).
#include "NativeGpuB200.hpp"

#include "autodiff/v0/Autodiff.hpp"
#include "backend/v0/TensorRegion.hpp"
#include "extension/v0/Extension.hpp"
#include "frontend/v0/Parser.hpp"
#include "semantic/v0/Analyzer.hpp"
#include "semantic/v0/Evaluator.hpp"
#include "semantic/v0/Verifier.hpp"

#include <cstring>
#include <fstream>
#include <iostream>
#include <optional>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

using namespace thiran::v0;
namespace s = thiran::v0::semantic;
namespace e = thiran::v0::extension;
namespace b = thiran::v0::backend;
namespace g = thiran::v0::backend::b200;

namespace {

// The two example extension operations (recipes as in examples/research_extension
// and the f32 chain), with their gradient recipes over (x, y, dz).
using Op = e::ScalarOpcode;
constexpr e::ScalarNodeV0 kChain[] = {
    {Op::Input, 0, 0, 0, 0.0f}, {Op::ConstantF32, 0, 0, 0, 1.5f}, {Op::Multiply, 0, 1, 0, 0.0f},
    {Op::ConstantF32, 0, 0, 0, 0.25f}, {Op::Add, 2, 3, 0, 0.0f}, {Op::Multiply, 4, 0, 0, 0.0f},
    {Op::Subtract, 5, 0, 0, 0.0f}, {Op::ConstantF32, 0, 0, 0, 0.5f}, {Op::Multiply, 6, 7, 0, 0.0f},
    {Op::Add, 8, 0, 0, 0.0f},
};
constexpr e::ScalarNodeV0 kChainGradient[] = {
    {Op::Input, 0, 0, 0, 0.0f}, {Op::ConstantF32, 0, 0, 0, 1.5f}, {Op::Multiply, 0, 1, 0, 0.0f},
    {Op::ConstantF32, 0, 0, 0, 0.25f}, {Op::Add, 2, 3, 0, 0.0f}, {Op::Add, 4, 2, 0, 0.0f},
    {Op::ConstantF32, 0, 0, 0, 1.0f}, {Op::Subtract, 5, 6, 0, 0.0f}, {Op::ConstantF32, 0, 0, 0, 0.5f},
    {Op::Multiply, 7, 8, 0, 0.0f}, {Op::Add, 9, 6, 0, 0.0f}, {Op::Input, 0, 0, 2, 0.0f},
    {Op::Multiply, 11, 10, 0, 0.0f},
};
constexpr e::ScalarRecipeV0 kChainGradients[] = {{kChainGradient, 13, 12, 3}};
constexpr e::DerivativeV0 kChainDerivative{1, 1, false, kChainGradients, 1};
constexpr e::ScalarNodeV0 kSquareLinear[] = {
    {Op::Input, 0, 0, 0, 0.0f}, {Op::Multiply, 0, 0, 0, 0.0f}, {Op::Add, 1, 0, 0, 0.0f}};
constexpr e::ScalarNodeV0 kSquareLinearGradient[] = {
    {Op::Input, 0, 0, 2, 0.0f}, {Op::ConstantF32, 0, 0, 0, 2.0f}, {Op::Input, 0, 0, 0, 0.0f},
    {Op::Multiply, 1, 2, 0, 0.0f}, {Op::ConstantF32, 0, 0, 0, 1.0f}, {Op::Add, 3, 4, 0, 0.0f},
    {Op::Multiply, 0, 5, 0, 0.0f}};
constexpr e::ScalarRecipeV0 kSquareLinearGradients[] = {{kSquareLinearGradient, 7, 6, 3}};
constexpr e::DerivativeV0 kSquareLinearDerivative{1, 1, false, kSquareLinearGradients, 1};
constexpr e::OperationDescriptorV0 kOperations[] = {
    {"research_chain", "1.0.0", 1, 1, 2, 0, true, e::EffectV0::Pure,
     e::BackendV0::Reference | e::BackendV0::Cpu | e::BackendV0::Gpu, true, {kChain, 10, 9, 1}, &kChainDerivative},
    {"research_square_linear", "1.0.0", 1, 1, 2, 0, true, e::EffectV0::Pure,
     e::BackendV0::Reference | e::BackendV0::Cpu | e::BackendV0::Gpu, true, {kSquareLinear, 3, 2, 1},
     &kSquareLinearDerivative},
};
constexpr e::ExtensionDescriptorV0 kExtension{e::extensionAbiVersion, "org.thiran.b200.shim", "1.0.0", kOperations, 2,
                                              nullptr};

std::string readText(const std::string& path) {
    std::ifstream in(path);
    if (!in) throw std::runtime_error("cannot read " + path);
    std::ostringstream out;
    out << in.rdbuf();
    return out.str();
}

s::Module compile(const std::string& text, e::ExtensionRegistry& registry) {
    auto parsed = parse(text, "<shim>");
    if (!parsed.module) throw std::runtime_error("parse failed: " + parsed.diagnostics.front().format());
    auto analyzed = s::analyze(*parsed.module, registry);
    if (!analyzed.module) throw std::runtime_error("analysis failed: " + analyzed.diagnostics.front().format());
    if (!s::verify(*analyzed.module).ok) throw std::runtime_error("semantic verifier failed");
    return *analyzed.module;
}

b::GpuValue readValue(const std::string& path) {
    std::ifstream in(path, std::ios::binary);
    if (!in) throw std::runtime_error("cannot read " + path);
    char magic[4];
    std::uint32_t dtype = 0, rank = 0;
    in.read(magic, 4);
    in.read(reinterpret_cast<char*>(&dtype), 4);
    in.read(reinterpret_cast<char*>(&rank), 4);
    if (std::memcmp(magic, "THB1", 4) != 0) throw std::runtime_error("bad tensor file " + path);
    std::vector<std::uint64_t> shape(rank);
    std::uint64_t count = 1;
    for (auto& extent : shape) {
        in.read(reinterpret_cast<char*>(&extent), 8);
        count *= extent;
    }
    if (rank == 0) {
        if (dtype == 1) { std::int64_t v = 0; in.read(reinterpret_cast<char*>(&v), 8); return b::GpuValue{v}; }
        float v = 0; in.read(reinterpret_cast<char*>(&v), 4); return b::GpuValue{v};
    }
    if (dtype == 1) {
        std::vector<std::int64_t> values(count);
        in.read(reinterpret_cast<char*>(values.data()), static_cast<std::streamsize>(count * 8));
        return b::GpuValue{storage::Tensor::materializeI64(shape, values)};
    }
    std::vector<float> values(count);
    in.read(reinterpret_cast<char*>(values.data()), static_cast<std::streamsize>(count * 4));
    return b::GpuValue{storage::Tensor::materializeF32(shape, values)};
}

void writeHeader(std::ofstream& out, std::uint32_t dtype, const std::vector<std::uint64_t>& shape) {
    out.write("THB1", 4);
    const std::uint32_t rank = static_cast<std::uint32_t>(shape.size());
    out.write(reinterpret_cast<const char*>(&dtype), 4);
    out.write(reinterpret_cast<const char*>(&rank), 4);
    for (auto extent : shape) out.write(reinterpret_cast<const char*>(&extent), 8);
}

void writeValue(const std::string& path, const b::GpuValue& value) {
    std::ofstream out(path, std::ios::binary);
    if (const auto* i = std::get_if<std::int64_t>(&value)) { writeHeader(out, 1, {}); out.write(reinterpret_cast<const char*>(i), 8); return; }
    if (const auto* f = std::get_if<float>(&value)) { writeHeader(out, 2, {}); out.write(reinterpret_cast<const char*>(f), 4); return; }
    const auto& t = std::get<storage::Tensor>(value);
    if (t.descriptor().dtype == storage::DType::I64) {
        const auto v = t.logicalI64Values();
        writeHeader(out, 1, t.descriptor().shape);
        out.write(reinterpret_cast<const char*>(v.data()), static_cast<std::streamsize>(v.size() * 8));
    } else {
        const auto v = t.logicalF32Values();
        writeHeader(out, 2, t.descriptor().shape);
        out.write(reinterpret_cast<const char*>(v.data()), static_cast<std::streamsize>(v.size() * 4));
    }
}

// Reference runtime values (Evaluator) as GpuValues.
b::GpuValue fromRuntime(const s::RuntimeValue& v) {
    if (const auto* i = std::get_if<std::int64_t>(&v.data)) return b::GpuValue{*i};
    if (const auto* f = std::get_if<float>(&v.data)) return b::GpuValue{*f};
    const auto& t = std::get<s::RuntimeTensor>(v.data);
    std::vector<std::uint64_t> shape(t.shape.begin(), t.shape.end());
    return t.dtype == s::TypeKind::I64 ? b::GpuValue{storage::Tensor::materializeI64(shape, t.values)}
                                       : b::GpuValue{storage::Tensor::materializeF32(shape, t.f32Values)};
}

s::RuntimeValue toRuntime(const b::GpuValue& v) {
    if (const auto* i = std::get_if<std::int64_t>(&v)) return s::RuntimeValue{*i};
    if (const auto* f = std::get_if<float>(&v)) return s::RuntimeValue{*f};
    const auto& t = std::get<storage::Tensor>(v);
    std::vector<std::int64_t> shape(t.descriptor().shape.begin(), t.descriptor().shape.end());
    if (t.descriptor().dtype == storage::DType::I64)
        return s::RuntimeValue{s::RuntimeTensor{s::TypeKind::I64, shape, t.logicalI64Values(), {}}};
    return s::RuntimeValue{s::RuntimeTensor{s::TypeKind::F32, shape, {}, t.logicalF32Values()}};
}

const char* categoryName(b::GpuErrorCategory c) {
    switch (c) {
    case b::GpuErrorCategory::ValidationFailure: return "ValidationFailure";
    case b::GpuErrorCategory::BackendUnavailable: return "BackendUnavailable";
    case b::GpuErrorCategory::InvalidDevice: return "InvalidDevice";
    case b::GpuErrorCategory::BackendUnsupported: return "BackendUnsupported";
    case b::GpuErrorCategory::RuntimeFailure: return "RuntimeFailure";
    case b::GpuErrorCategory::SemanticFailure: return "SemanticFailure";
    }
    return "Unknown";
}

int report(const b::GpuExecutionResult& r) {
    if (r.ok()) {
        std::cout << "{\"status\":\"ok\",\"kernel_launches\":" << r.evidence.kernelLaunches << "}\n";
        return 0;
    }
    std::cout << "{\"status\":\"error\",\"code\":\"" << r.error->code << "\",\"category\":\""
              << categoryName(r.error->category) << "\"}\n";
    return 0;
}

g::MatmulMode modeOf(const std::string& s) {
    if (s == "exact") return g::MatmulMode::Exact;
    if (s == "tensor") return g::MatmulMode::TensorCores;
    throw std::runtime_error("matmul mode must be exact or tensor");
}

const s::Function& functionById(const s::Module& m, s::FunctionId id) {
    for (const auto& f : m.functions) if (f.id == id) return f;
    throw std::runtime_error("no function @" + std::to_string(id));
}

std::size_t tupleSize(const s::Type& t) { return t.kind == s::TypeKind::Tuple ? t.elements.size() : 1; }

// Reverse mode over every parameter of `name` (autodiff::differentiate,
// src/autodiff/v0/Autodiff.cpp:72-294).
autodiff::DifferentiationResult differentiateAll(const s::Module& module, const std::string& name) {
    const auto facts = analysis::analyze(module);
    if (!facts.ok()) throw std::runtime_error("ownership analysis failed");
    const s::Function* fn = nullptr;
    for (const auto& candidate : module.functions) if (candidate.name == name) fn = &candidate;
    if (!fn) throw std::runtime_error("no function " + name);
    autodiff::ReverseModeRequest request;
    request.function = fn->id;
    for (std::size_t k = 0; k < fn->parameters.size(); ++k) request.wrtParameters.push_back(k);
    auto diff = autodiff::differentiate(module, facts, request);
    if (!diff.ok()) throw std::runtime_error("differentiate failed");
    return diff;
}

} // namespace

int main(int argc, char** argv) {
    try {
        if (argc < 4) {
            std::cerr << "usage: shim_driver lower|run|native|vjp <program.th> <function> ...\n";
            return 64;
        }
        const std::string mode = argv[1];
        if (mode == "artifact") {
            // shim_driver artifact <file.tha> <device> <out.bin> [in.bin ...]
            if (argc < 5) throw std::runtime_error("artifact needs a device and an output path");
            std::vector<b::GpuValue> inputs;
            for (int k = 5; k < argc; ++k) inputs.push_back(readValue(argv[k]));
            const auto r = g::loadAndExecuteArtifact(argv[2], inputs, std::stoi(argv[3]));
            if (!r.ok()) {
                std::cout << "{\"status\":\"error\",\"code\":\"" << r.error->code << "\"}\n";
                return 0;
            }
            writeValue(argv[4], *r.value);
            std::cout << "{\"status\":\"ok\",\"kernel_launches\":"
                      << (r.gpuEvidence ? r.gpuEvidence->kernelLaunches : 0) << "}\n";
            return 0;
        }
        e::ExtensionRegistry registry;
        if (auto r = registry.registerExtension(kExtension); !r.ok()) throw std::runtime_error(r.message);
        const s::Module module = compile(readText(argv[2]), registry);
        const std::string function = argv[3];
        if (mode == "lower") {
            const std::size_t element = argc > 4 ? std::stoull(argv[4]) : 0;
            // <fn>@forward / <fn>@backward: autodiff's generated functions.
            const auto suffix = function.find('@');
            std::optional<autodiff::DifferentiationResult> diff;
            std::string name = function;
            if (suffix != std::string::npos) {
                diff = differentiateAll(module, function.substr(0, suffix));
                const bool forward = function.substr(suffix + 1) == "forward";
                name = functionById(*diff->module, forward ? diff->forwardFunction : diff->backwardFunction).name;
            }
            const auto lowered = g::lowerFunction(diff ? *diff->module : module, name, element,
                                                  argc > 5 ? modeOf(argv[5]) : g::MatmulMode::Exact);
            if (!lowered.ok()) {
                std::cout << lowered.diagnostic << "\n";
                return 0;
            }
            const auto& r = *lowered.region;
            std::cout << "region " << r.name << " inputs";
            for (auto i : r.inputs) std::cout << ' ' << i;
            std::cout << " output " << r.desc.output << "\n";
            for (const auto& n : r.nodes) {
                std::cout << "node " << n.id << " op=" << n.op << " dtype=" << n.dtype << " rank=" << n.rank
                          << " extent=" << n.extent[0] << "," << n.extent[1] << " deps=";
                for (std::uint32_t k = 0; k < n.dependency_count; ++k) std::cout << (k ? "," : "") << n.dependencies[k];
                std::cout << " axis=" << n.axis << "\n";
            }
            // The engine's verifier and planner (device-free).
            std::uint64_t needed = 0, counts[3] = {};
            char failure[1024] = {};
            const int status = thb_region_describe(&r.desc, {1, 1}, THB_DESCRIBE_PLAN, nullptr, 0, &needed, counts,
                                                   failure, sizeof failure);
            if (status != THB_STATUS_OK) std::cout << "verifier " << failure << "\n";
            else std::cout << "plan groups=" << counts[0] << " fused=" << counts[1] << " kernels=" << counts[2] << "\n";
            return 0;
        }
        if (mode == "run") {
            if (argc < 8) throw std::runtime_error("run needs element, mode, device and an output path");
            const auto lowered = g::lowerFunction(module, function, std::stoull(argv[4]), modeOf(argv[5]));
            if (!lowered.ok()) {
                std::cout << "{\"status\":\"error\",\"code\":\"" << lowered.diagnostic << "\"}\n";
                return 0;
            }
            std::vector<b::GpuValue> inputs;
            for (int k = 8; k < argc; ++k) inputs.push_back(readValue(argv[k]));
            const auto result = g::executeLowered(*lowered.region, inputs, std::stoi(argv[6]), {});
            if (result.ok()) writeValue(argv[7], *result.value);
            return report(result);
        }
        if (mode == "native") {
            if (argc < 6) throw std::runtime_error("native needs a device and an output path");
            const auto facts = analysis::analyze(module);
            const auto extracted = b::extractStrictGpu(module, facts, function, false);
            if (!extracted.ok()) {
                std::cout << "{\"status\":\"error\",\"code\":\"" << extracted.diagnostic << "\"}\n";
                return 0;
            }
            std::vector<b::GpuValue> inputs;
            for (int k = 6; k < argc; ++k) inputs.push_back(readValue(argv[k]));
            const auto result = g::executeNativeGpu(*extracted.region, inputs, std::stoi(argv[4]), {});
            if (result.ok()) writeValue(argv[5], *result.value);
            return report(result);
        }
        if (mode == "vjp") {
            if (argc < 8) throw std::runtime_error("vjp needs mode, device, prefix and cotangent");
            const auto matmul = modeOf(argv[4]);
            const int device = std::stoi(argv[5]);
            const std::string prefix = argv[6];
            const auto cotangent = readValue(argv[7]);
            std::vector<b::GpuValue> inputs;
            for (int k = 8; k < argc; ++k) inputs.push_back(readValue(argv[k]));
            const auto diff = differentiateAll(module, function);
            const auto& generated = *diff.module;
            const auto& forward = functionById(generated, diff.forwardFunction);
            const auto& backward = functionById(generated, diff.backwardFunction);
            // Forward: primal and every saved value, one region each.
            std::vector<b::GpuValue> saves;
            b::GpuValue primal{0.0f};
            for (std::size_t k = 0; k < tupleSize(forward.result); ++k) {
                const auto lowered = g::lowerFunction(generated, forward.name, k, matmul);
                if (!lowered.ok()) {
                    std::cout << "{\"status\":\"error\",\"code\":\"" << lowered.diagnostic << "\"}\n";
                    return 0;
                }
                const auto r = g::executeLowered(*lowered.region, inputs, device, {});
                if (!r.ok()) return report(r);
                if (k == 0) primal = *r.value;
                else saves.push_back(*r.value);
            }
            saves.push_back(cotangent);
            const std::size_t gradients = tupleSize(backward.result);
            std::vector<b::GpuValue> grads;
            for (std::size_t k = 0; k < gradients; ++k) {
                const auto lowered = g::lowerFunction(generated, backward.name, k, matmul);
                if (!lowered.ok()) {
                    std::cout << "{\"status\":\"error\",\"code\":\"" << lowered.diagnostic << "\"}\n";
                    return 0;
                }
                const auto r = g::executeLowered(*lowered.region, saves, device, {});
                if (!r.ok()) return report(r);
                grads.push_back(*r.value);
            }
            writeValue(prefix + "primal.bin", primal);
            for (std::size_t k = 0; k < grads.size(); ++k) writeValue(prefix + "grad" + std::to_string(k) + ".bin", grads[k]);
            // The reference's own reverse mode on the same inputs.
            std::vector<s::RuntimeValue> args;
            for (const auto& v : inputs) args.push_back(toRuntime(v));
            const auto ref = autodiff::executeVjpWithPrimal(diff, args, toRuntime(cotangent));
            if (!ref.ok()) throw std::runtime_error("executeVjpWithPrimal: " + ref.errorId);
            writeValue(prefix + "ref_primal.bin", fromRuntime(*ref.primal));
            if (const auto* tuple = std::get_if<s::RuntimeTuple>(&ref.gradients->data)) {
                for (std::size_t k = 0; k < tuple->size(); ++k)
                    writeValue(prefix + "ref_grad" + std::to_string(k) + ".bin", fromRuntime((*tuple)[k]));
            } else {
                writeValue(prefix + "ref_grad0.bin", fromRuntime(*ref.gradients));
            }
            std::cout << "{\"status\":\"ok\",\"gradients\":" << grads.size() << "}\n";
            return 0;
        }
        throw std::runtime_error("unknown mode " + mode);
    } catch (const std::exception& failure) {
        std::cout << "{\"status\":\"error\",\"code\":\"DRIVER\",\"message\":\"" << failure.what() << "\"}\n";
        return 1;
    }
}
