// ref_driver — runs the REFERENCE implementation (compiled from its own
// sources by oracle/Makefile) to pin the oracle and to build the timed
// reference CPU path. TEST INFRASTRUCTURE ONLY; nothing in thiran_b200/ uses it.
//
//   ref_driver eval <program.th> <function> <out.bin> [in.bin ...]
//       semantic::evaluateCall (src/semantic/v0/Evaluator.cpp:634); prints
//       {"status":"ok"} or {"status":"error","error_id":...}.
//   ref_driver emit <program.th> <function> <out.cpp>
//       extractStrictNative + emitCpp20 (src/backend/v0/NativeCpu.cpp:368-375)
//       with an extern "C" thiran_ref_entry wrapper that follows
//       thiran_v0_entry (src/artifact/v0/NativeArtifacts.cpp:631-700) but takes
//       its tensor shapes from the arguments.
//   ref_driver plan <program.th> <function> [nofusion]
//       prints the region and buildPhysicalPlan dump (PhysicalPlan.cpp:366).
//   ref_driver tha <program.th> <function> <out.tha> [nofusion]
//       writes the reference's GPU artifact of the region: buildGpuAot
//       (src/artifact/v0/NativeArtifacts.cpp:1056-1097), THIRAN16 manifest,
//       serialized region and its generated PTX payload.
//   ref_driver thm <program.th> <function> <out.thm> <public-count> <in.bin ...>
//       writes the reference's model bundle (createModelBundle /
//       writeModelBundle, src/model/v0/ModelBundle.cpp:328-360): the first
//       <public-count> inputs are public, the rest frozen parameters (ids 1..,
//       names p1..) with the given values; one GPU artifact specialised to
//       these shapes (specializeEntry, NativeArtifacts.cpp:891-922).
//   ref_driver render <positions.bin> <indices.bin> <colors.bin> <model.bin>
//                     <view.bin> <projection.bin> <width> <height> <out-prefix>
//       graphics::render (src/graphics/v0/Graphics.cpp:574-596) with a zero
//       clear colour; writes <prefix>color.bin / <prefix>depth.bin and prints
//       the statistics, or the TH019-* failure id.
//
// Programs may call the extension operations `research_chain` (the
// ((x*1.5+0.25)*x - x)*0.5 + x recipe) and `research_square_linear` (x*x + x).
//
// Tensor files: "THB1", u32 dtype (1 i64, 2 f32), u32 rank, u64 shape[rank],
// little-endian elements; rank 0 is a scalar.
#include "artifact/v0/NativeArtifacts.hpp"
#include "autodiff/v0/Autodiff.hpp"
#include "graphics/v0/Graphics.hpp"
#include "model/v0/ModelBundle.hpp"
#include "backend/v0/NativeCpu.hpp"
#include "backend/v0/PhysicalPlan.hpp"
#include "extension/v0/Extension.hpp"
#include "frontend/v0/Parser.hpp"
#include "semantic/v0/Analyzer.hpp"
#include "semantic/v0/Evaluator.hpp"
#include "semantic/v0/Verifier.hpp"

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iostream>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

using namespace thiran::v0;
namespace s = thiran::v0::semantic;
namespace b = thiran::v0::backend;
namespace e = thiran::v0::extension;

namespace {

constexpr e::ScalarNodeV0 chainNodes[] = {
    {e::ScalarOpcode::Input, 0, 0, 0, 0.0f},       // 0 x
    {e::ScalarOpcode::ConstantF32, 0, 0, 0, 1.5f}, // 1
    {e::ScalarOpcode::Multiply, 0, 1, 0, 0.0f},    // 2 x*1.5
    {e::ScalarOpcode::ConstantF32, 0, 0, 0, 0.25f},// 3
    {e::ScalarOpcode::Add, 2, 3, 0, 0.0f},         // 4 +0.25
    {e::ScalarOpcode::Multiply, 4, 0, 0, 0.0f},    // 5 *x
    {e::ScalarOpcode::Subtract, 5, 0, 0, 0.0f},    // 6 -x
    {e::ScalarOpcode::ConstantF32, 0, 0, 0, 0.5f}, // 7
    {e::ScalarOpcode::Multiply, 6, 7, 0, 0.0f},    // 8 *0.5
    {e::ScalarOpcode::Add, 8, 0, 0, 0.0f},         // 9 +x
};
// d/dx of the chain, over (x, y, dz): dz * ((((x*1.5 + 0.25) + x*1.5) - 1) * 0.5 + 1)
constexpr e::ScalarNodeV0 chainGradientNodes[] = {
    {e::ScalarOpcode::Input, 0, 0, 0, 0.0f},        // 0 x
    {e::ScalarOpcode::ConstantF32, 0, 0, 0, 1.5f},  // 1
    {e::ScalarOpcode::Multiply, 0, 1, 0, 0.0f},     // 2 x*1.5
    {e::ScalarOpcode::ConstantF32, 0, 0, 0, 0.25f}, // 3
    {e::ScalarOpcode::Add, 2, 3, 0, 0.0f},          // 4 x*1.5+0.25
    {e::ScalarOpcode::Add, 4, 2, 0, 0.0f},          // 5 + x*1.5
    {e::ScalarOpcode::ConstantF32, 0, 0, 0, 1.0f},  // 6
    {e::ScalarOpcode::Subtract, 5, 6, 0, 0.0f},     // 7 - 1
    {e::ScalarOpcode::ConstantF32, 0, 0, 0, 0.5f},  // 8
    {e::ScalarOpcode::Multiply, 7, 8, 0, 0.0f},     // 9 * 0.5
    {e::ScalarOpcode::Add, 9, 6, 0, 0.0f},          // 10 + 1
    {e::ScalarOpcode::Input, 0, 0, 2, 0.0f},        // 11 dz
    {e::ScalarOpcode::Multiply, 11, 10, 0, 0.0f},   // 12 dz * (...)
};
constexpr e::ScalarRecipeV0 chainGradients[] = {{chainGradientNodes, 13, 12, 3}};
constexpr e::DerivativeV0 chainDerivative{1, 1, false, chainGradients, 1};
constexpr e::ScalarNodeV0 squareLinearNodes[] = {
    {e::ScalarOpcode::Input, 0, 0, 0, 0.0f},
    {e::ScalarOpcode::Multiply, 0, 0, 0, 0.0f},
    {e::ScalarOpcode::Add, 1, 0, 0, 0.0f},
};
// The example extension's gradient (examples/research_extension): dz * (2x + 1).
constexpr e::ScalarNodeV0 squareLinearGradientNodes[] = {
    {e::ScalarOpcode::Input, 0, 0, 2, 0.0f},
    {e::ScalarOpcode::ConstantF32, 0, 0, 0, 2.0f},
    {e::ScalarOpcode::Input, 0, 0, 0, 0.0f},
    {e::ScalarOpcode::Multiply, 1, 2, 0, 0.0f},
    {e::ScalarOpcode::ConstantF32, 0, 0, 0, 1.0f},
    {e::ScalarOpcode::Add, 3, 4, 0, 0.0f},
    {e::ScalarOpcode::Multiply, 0, 5, 0, 0.0f},
};
constexpr e::ScalarRecipeV0 squareLinearGradients[] = {{squareLinearGradientNodes, 7, 6, 3}};
constexpr e::DerivativeV0 squareLinearDerivative{1, 1, false, squareLinearGradients, 1};
constexpr e::OperationDescriptorV0 operations[] = {
    {"research_chain", "1.0.0", 1, 1, 2, 0, true, e::EffectV0::Pure,
     e::BackendV0::Reference | e::BackendV0::Cpu | e::BackendV0::Gpu, true, {chainNodes, 10, 9, 1}, &chainDerivative},
    {"research_square_linear", "1.0.0", 1, 1, 2, 0, true, e::EffectV0::Pure,
     e::BackendV0::Reference | e::BackendV0::Cpu | e::BackendV0::Gpu, true, {squareLinearNodes, 3, 2, 1},
     &squareLinearDerivative},
};
constexpr e::ExtensionDescriptorV0 descriptor{e::extensionAbiVersion, "org.thiran.b200.oracle", "1.0.0", operations, 2,
                                             nullptr};

std::string readText(const std::string& path) {
    std::ifstream in(path);
    if (!in) throw std::runtime_error("cannot read " + path);
    std::ostringstream out;
    out << in.rdbuf();
    return out.str();
}

s::Module compile(const std::string& text, e::ExtensionRegistry& registry) {
    auto parsed = parse(text, "<oracle>");
    if (!parsed.module) throw std::runtime_error("parse failed: " + parsed.diagnostics.front().format());
    auto analyzed = s::analyze(*parsed.module, registry);
    if (!analyzed.module) throw std::runtime_error("analysis failed: " + analyzed.diagnostics.front().format());
    if (!s::verify(*analyzed.module).ok) throw std::runtime_error("semantic verifier failed");
    return *analyzed.module;
}

s::RuntimeValue readValue(const std::string& path) {
    std::ifstream in(path, std::ios::binary);
    if (!in) throw std::runtime_error("cannot read " + path);
    char magic[4];
    std::uint32_t dtype = 0, rank = 0;
    in.read(magic, 4);
    in.read(reinterpret_cast<char*>(&dtype), 4);
    in.read(reinterpret_cast<char*>(&rank), 4);
    if (std::memcmp(magic, "THB1", 4) != 0) throw std::runtime_error("bad tensor file " + path);
    std::vector<std::int64_t> shape(rank);
    std::uint64_t count = 1;
    for (auto& extent : shape) {
        std::uint64_t v = 0;
        in.read(reinterpret_cast<char*>(&v), 8);
        extent = static_cast<std::int64_t>(v);
        count *= v;
    }
    if (rank == 0) {
        if (dtype == 1) { std::int64_t v; in.read(reinterpret_cast<char*>(&v), 8); return s::RuntimeValue{v}; }
        float v; in.read(reinterpret_cast<char*>(&v), 4); return s::RuntimeValue{v};
    }
    if (dtype == 1) {
        std::vector<std::int64_t> values(count);
        in.read(reinterpret_cast<char*>(values.data()), static_cast<std::streamsize>(count * 8));
        return s::RuntimeValue{s::RuntimeTensor{s::TypeKind::I64, shape, values, {}}};
    }
    std::vector<float> values(count);
    in.read(reinterpret_cast<char*>(values.data()), static_cast<std::streamsize>(count * 4));
    return s::RuntimeValue{s::RuntimeTensor{s::TypeKind::F32, shape, {}, values}};
}

void writeValue(const std::string& path, const s::RuntimeValue& value) {
    std::ofstream out(path, std::ios::binary);
    auto header = [&](std::uint32_t dtype, const std::vector<std::int64_t>& shape) {
        out.write("THB1", 4);
        const std::uint32_t rank = static_cast<std::uint32_t>(shape.size());
        out.write(reinterpret_cast<const char*>(&dtype), 4);
        out.write(reinterpret_cast<const char*>(&rank), 4);
        for (auto extent : shape) {
            const std::uint64_t v = static_cast<std::uint64_t>(extent);
            out.write(reinterpret_cast<const char*>(&v), 8);
        }
    };
    if (const auto* i = std::get_if<std::int64_t>(&value.data)) { header(1, {}); out.write(reinterpret_cast<const char*>(i), 8); return; }
    if (const auto* f = std::get_if<float>(&value.data)) { header(2, {}); out.write(reinterpret_cast<const char*>(f), 4); return; }
    const auto& t = std::get<s::RuntimeTensor>(value.data);
    if (t.dtype == s::TypeKind::I64) {
        header(1, t.shape);
        out.write(reinterpret_cast<const char*>(t.values.data()), static_cast<std::streamsize>(t.values.size() * 8));
    } else {
        header(2, t.shape);
        out.write(reinterpret_cast<const char*>(t.f32Values.data()), static_cast<std::streamsize>(t.f32Values.size() * 4));
    }
}

b::TensorRegion extract(const s::Module& module, const std::string& name) {
    auto facts = analysis::analyze(module);
    if (!facts.ok()) throw std::runtime_error("ownership analysis failed");
    auto lowered = b::extractStrictNative(module, facts, name, false);
    if (!lowered.ok()) throw std::runtime_error(lowered.diagnostic);
    return *lowered.region;
}

// The extern "C" wrapper appended to the emitted region source.
std::string wrapper(const b::TensorRegion& region) {
    std::ostringstream out;
    out << "\n#include <cstring>\n"
           "extern \"C\" {\n"
           "struct RefAbiArg { std::uint32_t kind,dtype,rank,reserved; const std::uint64_t* shape; const void* data; "
           "std::uint64_t count; };\n"
           "static void ref_error(char* o,std::uint64_t cap,const char* t){if(!o||!cap)return;std::strncpy(o,t,cap-1);o[cap-1]=0;}\n"
           "int thiran_ref_entry(const RefAbiArg* args,std::uint64_t argc,void* output,std::uint64_t output_count,"
           "char* failure,std::uint64_t failure_cap) noexcept {\n try {\n";
    out << "  if(argc!=" << region.inputs.size() << "ULL){ref_error(failure,failure_cap,\"ARGUMENT-COUNT\");return 1;}\n";
    for (std::size_t k = 0; k < region.inputs.size(); ++k) {
        const b::RegionNode* node = nullptr;
        for (const auto& n : region.nodes) if (n.id == region.inputs[k]) node = &n;
        const bool tensor = node->type.kind == s::TypeKind::Tensor;
        const bool i64 = tensor ? node->type.elements[0].kind == s::TypeKind::I64 : node->type.kind == s::TypeKind::I64;
        const char* scalar = i64 ? "std::int64_t" : "float";
        if (tensor) {
            out << "  std::vector<std::uint64_t> shape_" << k << "(args[" << k << "].shape,args[" << k << "].shape+args["
                << k << "].rank);\n"
                << "  std::vector<" << scalar << "> values_" << k << "; if(args[" << k << "].count){auto p=static_cast<const "
                << scalar << "*>(args[" << k << "].data); values_" << k << ".assign(p,p+args[" << k << "].count);}\n"
                << "  Tensor input_" << k << "=Tensor::materialize" << (i64 ? "I64" : "F32") << "(shape_" << k << ",values_"
                << k << ");\n";
        } else {
            out << "  " << scalar << " input_" << k << "=*static_cast<const " << scalar << "*>(args[" << k << "].data);\n";
        }
    }
    out << "  auto result=native_f" << region.function << "(";
    for (std::size_t k = 0; k < region.inputs.size(); ++k) out << (k ? "," : "") << "input_" << k;
    out << ");\n";
    const bool tensorOut = region.outputType.kind == s::TypeKind::Tensor;
    const bool i64Out = tensorOut ? region.outputType.elements[0].kind == s::TypeKind::I64
                                  : region.outputType.kind == s::TypeKind::I64;
    if (tensorOut) {
        out << "  auto values=result." << (i64Out ? "logicalI64Values" : "logicalF32Values") << "();\n"
            << "  if(values.size()!=output_count){ref_error(failure,failure_cap,\"RESULT-SHAPE\");return 1;}\n"
            << "  if(output_count)std::memcpy(output,values.data(),output_count*sizeof(values[0]));\n";
    } else {
        out << "  *static_cast<" << (i64Out ? "std::int64_t" : "float") << "*>(output)=result;\n";
    }
    out << "  return 0;\n } catch(const SemanticFailure& e){ref_error(failure,failure_cap,e.id);return 2;}\n"
           " catch(const std::exception& e){ref_error(failure,failure_cap,e.what());return 3;}\n"
           " catch(...){ref_error(failure,failure_cap,\"unknown\");return 4;}\n}\n}\n";
    return out.str();
}

} // namespace

int main(int argc, char** argv) {
    try {
        if (argc < 4) {
            std::cerr << "usage: ref_driver eval|emit|plan <program.th> <function> ...\n";
            return 64;
        }
        const std::string mode = argv[1];
        if (mode == "render") {
            if (argc < 11) throw std::runtime_error("render needs six tensors, width, height and a prefix");
            auto tensor = [&](int k) {
                const auto value = readValue(argv[k]);
                const auto& t = std::get<s::RuntimeTensor>(value.data);
                std::vector<std::uint64_t> shape(t.shape.begin(), t.shape.end());
                return t.dtype == s::TypeKind::I64 ? storage::Tensor::materializeI64(shape, t.values)
                                                   : storage::Tensor::materializeF32(shape, t.f32Values);
            };
            try {
                const auto frame = graphics::render(tensor(2), tensor(3), tensor(4), tensor(5), tensor(6), tensor(7),
                                                    std::stoull(argv[8]), std::stoull(argv[9]));
                const std::string prefix = argv[10];
                auto dump = [&](const storage::Tensor& t, const std::string& path) {
                    const auto values = t.logicalF32Values();
                    std::vector<std::int64_t> shape(t.descriptor().shape.begin(), t.descriptor().shape.end());
                    writeValue(path, s::RuntimeValue{s::RuntimeTensor{s::TypeKind::F32, shape, {}, values}});
                };
                dump(frame.framebuffer.color(), prefix + "color.bin");
                dump(frame.framebuffer.depth(), prefix + "depth.bin");
                const auto& st = frame.statistics;
                std::cout << "{\"status\":\"ok\",\"stats\":[" << st.inputTriangleCount << "," << st.postClipTriangleCount
                          << "," << st.shadedPixelCount << "," << st.depthPassCount << "]}\n";
            } catch (const std::exception& failure) {
                std::cout << "{\"status\":\"error\",\"error_id\":\"" << failure.what() << "\"}\n";
            }
            return 0;
        }
        e::ExtensionRegistry registry;
        if (auto r = registry.registerExtension(descriptor); !r.ok()) throw std::runtime_error(r.message);
        const s::Module module = compile(readText(argv[2]), registry);
        const std::string function = argv[3];
        if (mode == "eval") {
            if (argc < 5) throw std::runtime_error("eval needs an output path");
            std::vector<s::RuntimeValue> inputs;
            for (int k = 5; k < argc; ++k) inputs.push_back(readValue(argv[k]));
            const auto result = s::evaluateCall(module, function, inputs);
            if (!result.ok || !result.value) {
                std::cout << result.format() << "\n";
                return 0;
            }
            writeValue(argv[4], *result.value);
            std::cout << "{\"status\":\"ok\"}\n";
            return 0;
        }
        if (mode == "emit") {
            if (argc < 5) throw std::runtime_error("emit needs an output path");
            const auto region = extract(module, function);
            std::ofstream out(argv[4]);
            out << b::emitCpp20(region, false, wrapper(region));
            return 0;
        }
        if (mode == "vjp") {
            // ref_driver vjp <program> <fn> <out-prefix> <cotangent.bin> <inputs...>
            // Reverse mode over every parameter (autodiff::differentiate,
            // src/autodiff/v0/Autodiff.cpp:72-294) executed by
            // executeVjpWithPrimal (:379-393); writes <prefix>primal.bin and
            // <prefix>grad<k>.bin.
            if (argc < 6) throw std::runtime_error("vjp needs an output prefix and a cotangent");
            const auto facts = analysis::analyze(module);
            if (!facts.ok()) throw std::runtime_error("ownership analysis failed");
            const s::Function* fn = nullptr;
            for (const auto& candidate : module.functions)
                if (candidate.name == function) fn = &candidate;
            if (!fn) throw std::runtime_error("no function " + function);
            thiran::v0::autodiff::ReverseModeRequest request;
            request.function = fn->id;
            for (std::size_t k = 0; k < fn->parameters.size(); ++k) request.wrtParameters.push_back(k);
            const auto diff = thiran::v0::autodiff::differentiate(module, facts, request);
            if (!diff.ok())
                throw std::runtime_error("differentiate: " +
                                         (diff.diagnostics.empty() ? std::string("failed") : diff.diagnostics.front().code));
            if (std::getenv("THB_DUMP_BACKWARD")) std::cerr << diff.dump() << s::dump(*diff.module);
            std::vector<s::RuntimeValue> inputs;
            for (int k = 6; k < argc; ++k) inputs.push_back(readValue(argv[k]));
            const auto result = thiran::v0::autodiff::executeVjpWithPrimal(diff, inputs, readValue(argv[5]));
            if (!result.ok()) {
                std::cout << "{\"status\":\"error\",\"error_id\":\"" << result.errorId << "\"}\n";
                return 0;
            }
            const std::string prefix = argv[4];
            writeValue(prefix + "primal.bin", *result.primal);
            if (const auto* tuple = std::get_if<s::RuntimeTuple>(&result.gradients->data)) {
                for (std::size_t k = 0; k < tuple->size(); ++k) writeValue(prefix + "grad" + std::to_string(k) + ".bin", (*tuple)[k]);
            } else {
                writeValue(prefix + "grad0.bin", *result.gradients);
            }
            std::cout << "{\"status\":\"ok\"}\n";
            return 0;
        }
        if (mode == "plan") {
            const auto region = extract(module, function);
            b::PhysicalPlanOptions options;
            if (argc > 4 && std::string(argv[4]) == "nofusion") options.enableFusion = false;
            auto plan = b::buildPhysicalPlan(region, b::PhysicalDevice::Gpu, options);
            if (!plan.ok()) throw std::runtime_error(plan.errors.front());
            std::cout << region.dump() << plan.plan->dump();
            return 0;
        }
        if (mode == "tha") {
            if (argc < 5) throw std::runtime_error("tha needs an output path");
            const auto region = extract(module, function);
            artifact::ArtifactBuildOptions options;
            options.output = argv[4];
            if (argc > 5 && std::string(argv[5]) == "nofusion") options.planning.enableFusion = false;
            const auto built = artifact::buildGpuAot(region, options);
            if (!built.success)
                throw std::runtime_error(built.error ? built.error->code + ": " + built.error->message : "build failed");
            std::cout << "{\"status\":\"ok\"}\n";
            return 0;
        }
        if (mode == "thm") {
            if (argc < 6) throw std::runtime_error("thm needs an output path and a public-input count");
            const auto region = extract(module, function);
            const std::size_t publicCount = std::stoul(argv[5]);
            std::vector<artifact::ArtifactValue> values;
            std::vector<persistence::StoredParameter> parameters;
            for (int k = 6; k < argc; ++k) {
                const auto value = readValue(argv[k]);
                const auto* tensor = std::get_if<s::RuntimeTensor>(&value.data);
                if (!tensor) throw std::runtime_error("thm inputs must be tensors");
                std::vector<std::uint64_t> shape(tensor->shape.begin(), tensor->shape.end());
                persistence::StoredValue stored;
                stored.kind = persistence::StoredValueKind::Tensor;
                stored.shape = shape;
                if (tensor->dtype == s::TypeKind::I64) {
                    values.emplace_back(storage::Tensor::materializeI64(shape, tensor->values));
                    stored.dtype = storage::DType::I64;
                    const auto* p = reinterpret_cast<const std::byte*>(tensor->values.data());
                    stored.bytes.assign(p, p + tensor->values.size() * 8);
                } else {
                    values.emplace_back(storage::Tensor::materializeF32(shape, tensor->f32Values));
                    stored.dtype = storage::DType::F32;
                    const auto* p = reinterpret_cast<const std::byte*>(tensor->f32Values.data());
                    stored.bytes.assign(p, p + tensor->f32Values.size() * 4);
                }
                const std::size_t index = static_cast<std::size_t>(k - 6);
                if (index >= publicCount)
                    parameters.push_back({index - publicCount + 1, "p" + std::to_string(index - publicCount + 1), stored});
            }
            const std::string temporary = std::string(argv[4]) + ".artifact.tmp";
            artifact::ArtifactBuildOptions options;
            options.output = temporary;
            options.specializedEntry = artifact::specializeEntry(region, values);
            const auto built = artifact::buildGpuAot(region, options);
            if (!built.success)
                throw std::runtime_error(built.error ? built.error->code + ": " + built.error->message : "build failed");
            auto loaded = artifact::loadArtifact(temporary);
            std::remove(temporary.c_str());
            if (!loaded.ok()) throw std::runtime_error("artifact reload: " + loaded.error->code);
            model::DeploymentSnapshot snapshot;
            snapshot.modelIdentity = "research-model@1";
            snapshot.inferenceEntry = loaded.artifact->manifest.entry.name;
            snapshot.parameters = parameters;
            const auto& entry = loaded.artifact->manifest.entry;
            for (std::size_t i = 0; i < entry.parameters.size(); ++i) {
                if (i < publicCount) {
                    snapshot.publicInputs.push_back(entry.parameters[i]);
                    snapshot.publicBindings.push_back({static_cast<std::uint32_t>(i), static_cast<std::uint32_t>(i)});
                } else {
                    snapshot.parameterBindings.push_back({i - publicCount + 1, static_cast<std::uint32_t>(i)});
                }
            }
            snapshot.result = entry.result;
            snapshot.parameterDigest = persistence::parameterDigest(parameters);
            auto bundle = model::createModelBundle(snapshot, {{snapshot.modelIdentity, *loaded.artifact}});
            if (!bundle.ok()) throw std::runtime_error("bundle: " + bundle.error->code + " " + bundle.error->message);
            const auto written = model::writeModelBundle(*bundle.bundle, argv[4]);
            if (!written.ok()) throw std::runtime_error("bundle write: " + written.error->code);
            std::cout << "{\"status\":\"ok\"}\n";
            return 0;
        }
        throw std::runtime_error("unknown mode " + mode);
    } catch (const std::exception& error) {
        std::cerr << "ref_driver: " << error.what() << "\n";
        return 2;
    }
}
