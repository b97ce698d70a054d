// Reference-side binding of the B200 engine (see NativeGpuB200.hpp).
#include "NativeGpuB200.hpp"

#include <algorithm>
#include <cstring>
#include <map>
#include <set>
#include <variant>

namespace thiran::v0::backend::b200 {
namespace {

using semantic::TypeKind;

bool isTensor(const semantic::Type& t) { return t.kind == TypeKind::Tensor; }

TypeKind elementKind(const semantic::Type& t) {
    return isTensor(t) ? (t.elements.empty() ? TypeKind::Invalid : t.elements.front().kind) : t.kind;
}

std::optional<std::uint32_t> engineDtype(const semantic::Type& t) {
    switch (elementKind(t)) {
    case TypeKind::I64: return THB_DTYPE_I64;
    case TypeKind::F32: return THB_DTYPE_F32;
    default: return std::nullopt;
    }
}

// A node before pruning and renumbering. Keys are semantic value ids; nodes
// the lowering inserts get keys from kSynthetic up.
constexpr std::uint32_t kSynthetic = 0x80000000u;

struct Pending {
    std::uint32_t key = 0;
    std::uint32_t op = THB_OP_UNSUPPORTED;
    std::uint32_t dtype = THB_DTYPE_F32;
    std::uint32_t rank = 0;
    std::int64_t extent[2] = {-1, -1};
    std::vector<std::uint32_t> deps, indices;
    std::int64_t integer = 0;
    float floating = 0.0f;
    std::int32_t axis = 0;
    const extension::Operation* extension = nullptr;
};

struct Failure {
    std::string reason;
};

const thb_operation* convertOperation(LoweredRegion& out, const extension::Operation& op) {
    for (auto& existing : out.operations)
        if (existing.name == op.name && existing.version == op.semanticVersion) return &existing.record;
    auto& rec = out.operations.emplace_back();
    rec.name = op.name;
    rec.version = op.semanticVersion;
    auto convertNodes = [](const extension::ScalarRecipe& r) {
        std::vector<thb_scalar_node> nodes;
        for (const auto& n : r.nodes)
            nodes.push_back({static_cast<std::uint8_t>(n.opcode), n.left, n.right, n.input, n.constant});
        return nodes;
    };
    rec.forward = convertNodes(op.forward);
    rec.record.name = rec.name.c_str();
    rec.record.semantic_version = rec.version.c_str();
    rec.record.arity = op.arity;
    rec.record.minimum_rank = op.minimumRank;
    rec.record.maximum_rank = op.maximumRank;
    rec.record.result_like_input = op.resultLikeInput;
    rec.record.same_shape = op.sameShape ? 1 : 0;
    rec.record.effect = static_cast<std::uint8_t>(op.effect);
    rec.record.backends = op.backends;
    rec.record.fusible = op.fusible ? 1 : 0;
    rec.record.forward = {rec.forward.data(), rec.forward.size(), op.forward.root, op.forward.inputCount};
    if (op.derivative) {
        for (const auto& g : op.derivative->gradients) {
            const auto& nodes = rec.gradientNodes.emplace_back(convertNodes(g));
            rec.gradients.push_back({nodes.data(), nodes.size(), g.root, g.inputCount});
        }
        rec.derivative = {op.derivative->differentiableInputs, op.derivative->savedInputs,
                          static_cast<std::uint8_t>(op.derivative->savesOutput ? 1 : 0), rec.gradients.data(),
                          rec.gradients.size()};
        rec.record.derivative = &rec.derivative;
    }
    return &rec.record;
}

// Keeps the inputs and every node the output depends on, in their order,
// and renumbers them 1..n; fills the region's C records.
std::unique_ptr<LoweredRegion> finish(std::unique_ptr<LoweredRegion> out, const std::vector<Pending>& nodes,
                                      const std::vector<std::uint32_t>& inputs, std::uint32_t output,
                                      std::uint32_t function) {
    std::map<std::uint32_t, const Pending*> byKey;
    for (const auto& n : nodes) byKey[n.key] = &n;
    std::set<std::uint32_t> live(inputs.begin(), inputs.end());
    std::vector<std::uint32_t> work{output};
    while (!work.empty()) {
        const std::uint32_t k = work.back();
        work.pop_back();
        if (!live.insert(k).second && k != output) continue;
        live.insert(k);
        const auto found = byKey.find(k);
        if (found == byKey.end()) continue;  // the verifier reports it
        for (auto d : found->second->deps) if (!live.count(d)) work.push_back(d);
        for (auto d : found->second->indices) if (!live.count(d)) work.push_back(d);
    }
    std::map<std::uint32_t, std::uint32_t> id;
    for (const auto& n : nodes)
        if (live.count(n.key)) id.emplace(n.key, static_cast<std::uint32_t>(id.size() + 1));
    auto mapped = [&](std::uint32_t k) {
        const auto found = id.find(k);
        return found == id.end() ? 0u : found->second;  // 0: undefined (verifier TRV03)
    };
    for (const auto& n : nodes) {
        if (!live.count(n.key)) continue;
        thb_region_node c{};
        c.id = mapped(n.key);
        c.op = n.op;
        c.dtype = n.dtype;
        c.rank = n.rank;
        c.extent[0] = n.extent[0];
        c.extent[1] = n.extent[1];
        auto& deps = out->lists.emplace_back();
        for (auto d : n.deps) deps.push_back(mapped(d));
        auto& idx = out->lists.emplace_back();
        for (auto d : n.indices) idx.push_back(mapped(d));
        c.dependencies = deps.empty() ? nullptr : deps.data();
        c.dependency_count = static_cast<std::uint32_t>(deps.size());
        c.indices = idx.empty() ? nullptr : idx.data();
        c.index_count = static_cast<std::uint32_t>(idx.size());
        c.integer = n.integer;
        c.floating = n.floating;
        c.axis = n.axis;
        c.extension = n.extension ? convertOperation(*out, *n.extension) : nullptr;
        out->nodes.push_back(c);
    }
    for (auto k : inputs) out->inputs.push_back(mapped(k));
    out->desc.function = function;
    out->desc.name = out->name.c_str();
    out->desc.nodes = out->nodes.data();
    out->desc.node_count = static_cast<std::uint32_t>(out->nodes.size());
    out->desc.inputs = out->inputs.data();
    out->desc.input_count = static_cast<std::uint32_t>(out->inputs.size());
    out->desc.output = mapped(output);
    return out;
}

void setShape(Pending& p, const semantic::Type& type, const semantic::ShapeFact& shape) {
    p.rank = isTensor(type) ? type.rank : 0;
    for (std::uint32_t a = 0; a < p.rank && a < 2; ++a)
        p.extent[a] = a < shape.extents.size() && shape.extents[a] ? *shape.extents[a] : -1;
}

GpuError toError(int status, const char* text) {
    const std::string t(text ? text : "");
    const std::string code = t.substr(0, t.find(": "));
    GpuErrorCategory category = GpuErrorCategory::RuntimeFailure;
    if (status == THB_STATUS_SEMANTIC) category = GpuErrorCategory::SemanticFailure;
    else if (code == "GPU-DRIVER-NOT-FOUND" || code == "GPU-BACKEND-NOT-BUILT") category = GpuErrorCategory::BackendUnavailable;
    else if (code == "GPU-INVALID-DEVICE") category = GpuErrorCategory::InvalidDevice;
    else if (code == "GPU-INPUT-ARITY" || code == "GPU-INPUT-TYPE" || code == "GPU-INVALID-REGION")
        category = GpuErrorCategory::ValidationFailure;
    else if (status == THB_STATUS_ABI) category = GpuErrorCategory::BackendUnsupported;
    return {category, code, t};
}

void copyEvidence(const thb_evidence& e, GpuExecutionEvidence& r) {
    r.allocationCount = e.allocation_count;
    r.allocationBytesRequested = e.allocation_bytes_requested;
    r.hostToDeviceCopies = e.host_to_device_copies;
    r.hostToDeviceBytes = e.host_to_device_bytes;
    r.deviceToHostCopies = e.device_to_host_copies;
    r.deviceToHostBytes = e.device_to_host_bytes;
    r.deviceToDeviceCopies = e.device_to_device_copies;
    r.deviceToDeviceBytes = e.device_to_device_bytes;
    r.moduleLoads = e.module_loads;
    r.driverJitLoads = e.driver_jit_loads;
    r.inputStorageUploads = e.input_storage_uploads;
    r.resultDownloads = e.result_downloads;
    r.kernelLaunches = e.kernel_launches;
    r.synchronizations = e.synchronizations;
    r.submittedOperations = e.submitted_operations;
    r.pendingOperations = e.pending_operations;
    r.activeReadReservations = e.active_read_reservations;
    r.activeWriteReservations = e.active_write_reservations;
    r.streamSubmissions = e.stream_submissions;
    r.eventRecords = e.event_records;
    r.observations = e.observations;
    r.droppedDrains = e.dropped_drains;
    r.releasedReservations = e.released_reservations;
    r.logicalTensorValues = e.logical_tensor_values;
    r.logicalIntermediates = e.logical_intermediates;
    r.materializedIntermediates = e.materialized_intermediates;
    r.physicalSlots = e.physical_slots;
    r.physicalTemporarySlots = e.physical_temporary_slots;
    r.reusedSlotAssignments = e.reused_slot_assignments;
    r.fusionGroups = e.fusion_groups;
    r.fusedKernelGroups = e.fused_kernel_groups;
    r.plannerOwnedAllocations = e.planner_owned_allocations;
    r.retainedPlannerAllocations = e.retained_planner_allocations;
}

// Runtime extents of every node from the argument shapes: the rules the
// engine applies before its first launch (elementwise results take their
// first tensor operand's shape; scalar operands broadcast).
std::vector<std::uint64_t> outputShape(const LoweredRegion& r, const std::vector<std::vector<std::uint64_t>>& argShapes) {
    std::map<std::uint32_t, std::vector<std::uint64_t>> shape;
    for (std::size_t k = 0; k < r.inputs.size() && k < argShapes.size(); ++k) shape[r.inputs[k]] = argShapes[k];
    auto dep = [&](const thb_region_node& n, std::uint32_t k) -> const std::vector<std::uint64_t>& {
        static const std::vector<std::uint64_t> none;
        if (k >= n.dependency_count) return none;
        const auto found = shape.find(n.dependencies[k]);
        return found == shape.end() ? none : found->second;
    };
    for (const auto& n : r.nodes) {
        if (n.op == THB_OP_INPUT) continue;
        std::vector<std::uint64_t> s;
        switch (n.op) {
        case THB_OP_INTEGER: case THB_OP_FLOAT: case THB_OP_INDEX: break;
        case THB_OP_TENSOR_LITERAL:
            for (std::uint32_t a = 0; a < n.rank; ++a) s.push_back(static_cast<std::uint64_t>(n.extent[a]));
            break;
        case THB_OP_SUM: {
            const auto& a = dep(n, 0);
            for (std::size_t d = 0; d < a.size(); ++d) if (static_cast<std::int32_t>(d) != n.axis) s.push_back(a[d]);
            break;
        }
        case THB_OP_ROW_MAX: if (!dep(n, 0).empty()) s = {dep(n, 0)[0]}; break;
        case THB_OP_TRANSPOSE: if (dep(n, 0).size() == 2) s = {dep(n, 0)[1], dep(n, 0)[0]}; break;
        case THB_OP_MATMUL:
            if (dep(n, 0).size() == 2 && dep(n, 1).size() == 2) s = {dep(n, 0)[0], dep(n, 1)[1]};
            break;
        case THB_OP_BROADCAST_TO_SHAPE: case THB_OP_REDUCE_TO_SHAPE: s = dep(n, 1); break;
        default:
            for (std::uint32_t k = 0; k < n.dependency_count; ++k)
                if (!dep(n, k).empty()) { s = dep(n, k); break; }
            break;
        }
        shape[n.id] = s;
    }
    return shape[r.desc.output];
}

} // namespace

LoweringResult lowerFunction(const semantic::Module& module, const std::string& name, std::size_t element,
                             MatmulMode matmul) {
    LoweringResult result;
    auto out = std::make_unique<LoweredRegion>();
    out->name = name;
    try {
        auto fail = [&](const std::string& reason) -> void { throw Failure{reason}; };
        const semantic::Function* function = nullptr;
        std::size_t matches = 0;
        for (const auto& candidate : module.functions)
            if (candidate.name == name) { function = &candidate; ++matches; }
        if (!function || matches != 1) fail("exactly one named function required");

        std::vector<Pending> nodes;
        std::vector<std::uint32_t> inputs;
        std::map<semantic::BindingId, semantic::ValueId> bindings;
        std::map<semantic::ValueId, std::size_t> position;             // key -> index in nodes
        std::map<semantic::ValueId, std::vector<semantic::ValueId>> tuples;
        std::uint32_t synthetic = kSynthetic;
        std::optional<semantic::ValueId> returned;
        auto at = [&](semantic::ValueId v) -> const Pending& {
            const auto found = position.find(v);
            if (found == position.end()) fail("operand %" + std::to_string(v) + " is not a region value");
            return nodes[found->second];
        };
        auto push = [&](Pending p) {
            position[p.key] = nodes.size();
            out->coverage += std::to_string(p.op) + '\n';
            nodes.push_back(std::move(p));
        };

        for (const auto& parameter : function->parameters) {
            if (parameter.access != semantic::AccessMode::Read) fail("parameter access mode");
            const auto dtype = engineDtype(parameter.type);
            if (!dtype) fail("parameter type " + semantic::typeName(parameter.type));
            Pending p;
            p.key = parameter.id;
            p.op = THB_OP_INPUT;
            p.dtype = *dtype;
            setShape(p, parameter.type, parameter.shape);
            push(p);
            inputs.push_back(parameter.id);
            bindings[parameter.binding] = parameter.id;
        }

        for (const auto& step : function->body.steps) {
            if (const auto* check = std::get_if<semantic::Check>(&step)) {
                // Bounds, broadcast, matmul and extension shape checks are
                // enforced by the engine before its first launch; a slice
                // check has no engine counterpart.
                if (check->kind == semantic::CheckKind::Slice) fail("Slice check");
                continue;
            }
            if (const auto* write = std::get_if<semantic::BindingWrite>(&step)) {
                if (!write->declaration) fail("mutable rebinding");
                bindings[write->binding] = write->value;
                continue;
            }
            if (const auto* flow = std::get_if<semantic::Flow>(&step)) {
                if (flow->kind != semantic::Flow::Kind::Return || !flow->value) fail("non-return flow");
                returned = *flow->value;
                continue;
            }
            if (std::holds_alternative<semantic::Structured>(step)) fail("structured control flow");
            const auto& in = std::get<semantic::Instruction>(step);
            if (in.op == semantic::Op::Tuple) {
                tuples[in.id] = in.operands;
                continue;
            }
            Pending p;
            p.key = in.id;
            const auto dtype = engineDtype(in.type);
            if (!dtype) fail("value type " + semantic::typeName(in.type));
            p.dtype = *dtype;
            setShape(p, in.type, in.shape);
            p.deps.assign(in.operands.begin(), in.operands.end());
            // Elementwise operands: a rank-1 tensor against a rank-2 tensor
            // broadcasts along the leading axis (the Evaluator aligns
            // trailing axes, Evaluator.cpp:95-124): made explicit as a
            // BroadcastToShape node.
            auto elementwise = [&](std::uint32_t op) {
                if (in.operands.size() != 2) fail("elementwise arity");
                p.op = op;
                const Pending& a = at(in.operands[0]);
                const Pending& b = at(in.operands[1]);
                if (a.rank && b.rank && a.rank != b.rank) {
                    const bool aLow = a.rank < b.rank;
                    const Pending& low = aLow ? a : b;
                    const Pending& high = aLow ? b : a;
                    if (low.rank != 1 || high.rank != 2 || low.dtype != THB_DTYPE_F32)
                        fail("broadcast outside the rank-1 into rank-2 f32 form");
                    Pending bc;
                    bc.key = synthetic++;
                    bc.op = THB_OP_BROADCAST_TO_SHAPE;
                    bc.dtype = THB_DTYPE_F32;
                    bc.rank = 2;
                    bc.extent[0] = high.extent[0];
                    bc.extent[1] = high.extent[1];
                    bc.deps = {low.key, high.key};
                    bc.axis = 0;
                    p.deps[aLow ? 0 : 1] = bc.key;
                    push(bc);
                }
            };
            switch (in.op) {
            case semantic::Op::Integer: p.op = THB_OP_INTEGER; p.integer = in.integer.value_or(0); break;
            case semantic::Op::Float: p.op = THB_OP_FLOAT; p.floating = in.floating.value_or(0.0f); break;
            case semantic::Op::TensorLiteral: p.op = THB_OP_TENSOR_LITERAL; break;
            case semantic::Op::LoadBinding: {
                const auto found = bindings.find(in.binding);
                if (found == bindings.end()) fail("unknown binding");
                p.op = THB_OP_ALIAS;
                p.deps = {found->second};
                break;
            }
            case semantic::Op::StopGradient: p.op = THB_OP_ALIAS; break;
            case semantic::Op::Copy: p.op = THB_OP_COPY; break;
            case semantic::Op::Negate: p.op = THB_OP_NEGATE; break;
            case semantic::Op::Add: elementwise(THB_OP_ADD); break;
            case semantic::Op::Subtract: elementwise(THB_OP_SUBTRACT); break;
            case semantic::Op::ElementMultiply: elementwise(THB_OP_ELEMENT_MULTIPLY); break;
            case semantic::Op::Multiply:
                // Scalar * scalar or scalar * tensor; tensor * tensor is Matmul.
                elementwise(THB_OP_ELEMENT_MULTIPLY);
                if (at(in.operands[0]).rank && at(in.operands[1]).rank) fail("tensor Multiply");
                break;
            case semantic::Op::Extension:
                if (!in.extensionOperation) fail("missing extension descriptor");
                if (!(in.extensionOperation->backends & extension::Gpu)) fail("extension without the GPU backend");
                p.op = THB_OP_EXTENSION;
                p.extension = &*in.extensionOperation;
                break;
            case semantic::Op::Index:
                p.op = THB_OP_INDEX;
                for (const auto& s : in.selectors) {
                    if (s.slice || !s.index) fail("slice Index");
                    p.indices.push_back(*s.index);
                }
                break;
            case semantic::Op::Matmul:
                p.op = THB_OP_MATMUL;
                p.axis = matmul == MatmulMode::Exact ? THB_MATMUL_EXACT : THB_MATMUL_TENSOR;
                if (p.dtype == THB_DTYPE_I64) p.axis = THB_MATMUL_TENSOR;  // i64: always checked, mode unused
                break;
            case semantic::Op::Sum:
                // sum(A, axis): the axis travels as an operand and in `axis`.
                p.op = THB_OP_SUM;
                p.deps = {in.operands.at(0)};
                p.axis = static_cast<std::int32_t>(in.axis);
                break;
            case semantic::Op::Transpose: p.op = THB_OP_TRANSPOSE; break;
            case semantic::Op::ZeroLike: p.op = THB_OP_ZERO_LIKE; break;
            case semantic::Op::ReduceToShape: p.op = THB_OP_REDUCE_TO_SHAPE; break;
            case semantic::Op::BroadcastToShape:
                p.op = THB_OP_BROADCAST_TO_SHAPE;
                p.axis = static_cast<std::int32_t>(in.axis);
                break;
            default: fail("operation " + std::to_string(static_cast<int>(in.op)));
            }
            push(std::move(p));
        }
        if (!returned) fail("no returned value");
        semantic::ValueId output = *returned;
        const auto tuple = tuples.find(output);
        if (tuple != tuples.end()) {
            if (element >= tuple->second.size()) fail("tuple element out of range");
            output = tuple->second[element];
        } else if (element != 0) {
            fail("the function does not return a tuple");
        }
        if (!position.count(output)) fail("returned value is not a region value");
        semantic::ValueId root = output;  // through Alias nodes (let bindings, parameter loads)
        while (at(root).op == THB_OP_ALIAS) root = at(root).deps.at(0);
        if (std::find(inputs.begin(), inputs.end(), root) != inputs.end()) {
            // A returned parameter: the region copies it into its output.
            Pending copy = at(output);
            if (!copy.rank) fail("a returned scalar parameter");
            copy.key = synthetic++;
            copy.op = THB_OP_COPY;
            copy.deps = {output};
            push(copy);
            output = copy.key;
        }
        result.region = finish(std::move(out), nodes, inputs, output, function->id);
    } catch (const Failure& f) {
        result.diagnostic = "BACKEND-UNSUPPORTED: " + f.reason;
    }
    return result;
}

std::unique_ptr<LoweredRegion> lowerRegion(const TensorRegion& region) {
    auto out = std::make_unique<LoweredRegion>();
    out->name = region.name;
    std::vector<Pending> nodes;
    for (const auto& n : region.nodes) {
        Pending p;
        p.key = n.id;
        p.op = static_cast<std::uint32_t>(n.op);  // RegionOp numbering is the engine's
        p.dtype = engineDtype(n.type).value_or(0);
        setShape(p, n.type, n.shape);
        p.deps.assign(n.dependencies.begin(), n.dependencies.end());
        p.indices.assign(n.indices.begin(), n.indices.end());
        p.integer = n.integer.value_or(0);
        p.floating = n.floating.value_or(0.0f);
        if (n.extensionOperation) p.extension = &*n.extensionOperation;
        nodes.push_back(std::move(p));
    }
    std::vector<std::uint32_t> inputs(region.inputs.begin(), region.inputs.end());
    return finish(std::move(out), nodes, inputs, region.output, region.function);
}

GpuExecutionResult executeLowered(const LoweredRegion& region, const std::vector<GpuValue>& inputs, int device,
                                  PhysicalPlanOptions options) noexcept {
    GpuExecutionResult result;
    try {
        char failure[1024] = {};
        // Host arguments: scalars by value, tensors as their logical values
        // (contiguous row-major; a view is marked and refused by the engine
        // with GPU-UNSUPPORTED-LAYOUT, NativeGpu.cpp:94-96).
        std::deque<std::vector<std::uint64_t>> shapes;
        std::deque<std::vector<std::int64_t>> i64s;
        std::deque<std::vector<float>> f32s;
        std::deque<std::int64_t> iScalars;
        std::deque<float> fScalars;
        std::vector<thb_abi_arg> args;
        std::vector<std::vector<std::uint64_t>> argShapes;
        for (const auto& v : inputs) {
            thb_abi_arg a{};
            if (const auto* i = std::get_if<std::int64_t>(&v)) {
                a.kind = THB_KIND_SCALAR; a.dtype = THB_DTYPE_I64; a.data = &iScalars.emplace_back(*i); a.count = 1;
                argShapes.emplace_back();
            } else if (const auto* f = std::get_if<float>(&v)) {
                a.kind = THB_KIND_SCALAR; a.dtype = THB_DTYPE_F32; a.data = &fScalars.emplace_back(*f); a.count = 1;
                argShapes.emplace_back();
            } else {
                const auto& t = std::get<storage::Tensor>(v);
                const auto& d = t.descriptor();
                const auto& shape = shapes.emplace_back(d.shape);
                argShapes.push_back(d.shape);
                a.kind = THB_KIND_TENSOR;
                a.rank = static_cast<std::uint32_t>(shape.size());
                a.shape = shape.data();
                a.reserved = (t.isView() || !t.isContiguousRowMajor() || d.elementOffset) ? 1u : 0u;
                if (d.dtype == storage::DType::I64) {
                    const auto& values = i64s.emplace_back(t.logicalI64Values());
                    a.dtype = THB_DTYPE_I64; a.data = values.data(); a.count = values.size();
                } else if (d.dtype == storage::DType::F32) {
                    const auto& values = f32s.emplace_back(t.logicalF32Values());
                    a.dtype = THB_DTYPE_F32; a.data = values.data(); a.count = values.size();
                } else {
                    a.dtype = 0;  // refused with GPU-INPUT-TYPE
                }
            }
            args.push_back(a);
        }
        thb_region* compiled = nullptr;
        int s = thb_region_compile(&region.desc, {options.enableReuse ? 1u : 0u, options.enableFusion ? 1u : 0u},
                                   device, &compiled, failure, sizeof failure);
        if (s != THB_STATUS_OK) {
            result.error = toError(s, failure);
            return result;
        }
        const thb_region_node* out = nullptr;
        for (const auto& n : region.nodes) if (n.id == region.desc.output) out = &n;
        const auto shape = outputShape(region, argShapes);
        std::uint64_t count = 1;
        for (auto e : shape) count *= e;
        thb_evidence ev{};
        const bool i64 = out && out->dtype == THB_DTYPE_I64;
        std::vector<std::int64_t> iOut(i64 ? count : 0);
        std::vector<float> fOut(i64 ? 0 : count);
        s = thb_region_execute(compiled, args.data(), args.size(), i64 ? static_cast<void*>(iOut.data()) : fOut.data(),
                               count, &ev, failure, sizeof failure);
        thb_region_release(compiled);
        copyEvidence(ev, result.evidence);
        if (s != THB_STATUS_OK) {
            result.error = toError(s, failure);
            return result;
        }
        if (!out || out->rank == 0) {
            if (i64) result.value = GpuValue{iOut.at(0)};
            else result.value = GpuValue{fOut.at(0)};
        } else if (i64) {
            result.value = GpuValue{storage::Tensor::materializeI64(shape, iOut)};
        } else {
            result.value = GpuValue{storage::Tensor::materializeF32(shape, fOut)};
        }
    } catch (const std::exception& e) {
        result.value.reset();
        result.error = GpuError{GpuErrorCategory::RuntimeFailure, "GPU-INTERNAL", e.what()};
    }
    return result;
}

GpuExecutionResult executeNativeGpu(const TensorRegion& region, const std::vector<GpuValue>& inputs, int device,
                                    PhysicalPlanOptions options) noexcept {
    try {
        const auto lowered = lowerRegion(region);
        return executeLowered(*lowered, inputs, device, options);
    } catch (const std::exception& e) {
        GpuExecutionResult result;
        result.error = GpuError{GpuErrorCategory::RuntimeFailure, "GPU-INTERNAL", e.what()};
        return result;
    }
}

GpuDeviceInfo probeNativeGpu(int device) noexcept {
    GpuDeviceInfo info;
    thb_device_info d{};
    thb_probe(device, &d);
    info.backendBuilt = d.backend_built != 0;
    info.driverLoaded = d.driver_loaded != 0;
    info.deviceAvailable = d.device_available != 0;
    info.deviceCount = d.device_count;
    info.selectedDevice = d.selected_device;
    info.driverVersion = d.driver_version;
    info.computeMajor = d.compute_major;
    info.computeMinor = d.compute_minor;
    info.name = d.name;
    if (d.error_code[0]) info.error = GpuError{GpuErrorCategory::BackendUnavailable, d.error_code, d.error_code};
    return info;
}

artifact::ArtifactExecutionResult loadAndExecuteArtifact(const std::string& path,
                                                         const std::vector<artifact::ArtifactValue>& inputs,
                                                         int device) noexcept {
    artifact::ArtifactExecutionResult result;
    try {
        auto loaded = artifact::loadArtifact(path);
        if (!loaded.ok()) {
            result.error = loaded.error;
            return result;
        }
        const auto& a = *loaded.artifact;
        if (a.manifest.backend != artifact::NativeBackend::Gpu) {
            result.error = artifact::ArtifactError{artifact::ArtifactErrorCategory::Execution, "ARTIFACT-BACKEND",
                                                   "not a GPU artifact"};
            return result;
        }
        auto run = b200::executeNativeGpu(a.region, inputs, device, a.manifest.planning);
        result.gpuEvidence = run.evidence;
        if (!run.ok()) {
            result.error = artifact::ArtifactError{artifact::ArtifactErrorCategory::Execution, run.error->code,
                                                   run.error->message};
            return result;
        }
        result.value = std::move(run.value);
    } catch (const std::exception& e) {
        result.value.reset();
        result.error = artifact::ArtifactError{artifact::ArtifactErrorCategory::Execution, "GPU-INTERNAL", e.what()};
    }
    return result;
}

} // namespace thiran::v0::backend::b200
