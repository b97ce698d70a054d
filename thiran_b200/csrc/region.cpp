// Region import, verification and physical planning (see region.hpp).
#include "region.hpp"

#include <algorithm>
#include <cmath>
#include <iomanip>
#include <sstream>

namespace thb {

const char* opName(Op op) {
    switch (op) {
    case Op::Input: return "Input";
    case Op::Integer: return "Integer";
    case Op::Float: return "Float";
    case Op::TensorLiteral: return "TensorLiteral";
    case Op::Alias: return "Alias";
    case Op::Copy: return "Copy";
    case Op::Negate: return "Negate";
    case Op::Add: return "Add";
    case Op::Subtract: return "Subtract";
    case Op::ElementMultiply: return "ElementMultiply";
    case Op::Extension: return "Extension";
    case Op::Index: return "Index";
    case Op::Unsupported: return "Unsupported";
    case Op::Sum: return "Sum";
    case Op::RowMax: return "RowMax";
    case Op::Softmax: return "Softmax";
    case Op::Relu: return "Relu";
    case Op::ExtensionGradient: return "ExtensionGradient";
    case Op::Transpose: return "Transpose";
    case Op::MatMul: return "MatMul";
    case Op::BroadcastToShape: return "BroadcastToShape";
    case Op::ReduceToShape: return "ReduceToShape";
    case Op::ZeroLike: return "ZeroLike";
    }
    return "Unsupported";
}

bool isElementwise(Op op) {
    return op == Op::Negate || op == Op::Add || op == Op::Subtract || op == Op::ElementMultiply ||
           op == Op::Extension || op == Op::Relu || op == Op::ExtensionGradient;
}

bool isReduction(Op op) { return op == Op::Sum || op == Op::RowMax || op == Op::Softmax; }

bool isKernelOp(Op op) {
    return op == Op::Transpose || op == Op::MatMul || op == Op::BroadcastToShape || op == Op::ReduceToShape ||
           op == Op::ZeroLike;
}

// ---- operation descriptors ---------------------------------------------------

namespace {

bool validVersion(const std::string& v) {
    if (v.empty()) return false;
    for (char c : v)
        if (!(c == '.' || c == '-' || c == '+' || c == '_' || (c >= '0' && c <= '9') ||
              (c >= 'A' && c <= 'Z') || (c >= 'a' && c <= 'z')))
            return false;
    return true;
}

struct Fnv {
    std::uint64_t h = 1469598103934665603ULL;
    void byte(std::uint8_t b) { h ^= b; h *= 1099511628211ULL; }
    template <class T> void value(T v) {
        unsigned char raw[sizeof(T)];
        std::memcpy(raw, &v, sizeof(T));
        for (unsigned char b : raw) byte(b);
    }
    void text(const std::string& s) { value<std::uint64_t>(s.size()); for (unsigned char c : s) byte(c); }
    void recipe(const Recipe& r) {
        value(r.inputCount); value(r.root); value<std::uint64_t>(r.nodes.size());
        for (const auto& n : r.nodes) { byte(n.opcode); value(n.left); value(n.right); value(n.input); value(n.constant); }
    }
};

Recipe importRecipe(const thb_scalar_recipe& raw) {
    Recipe r;
    r.root = raw.root;
    r.inputCount = raw.input_count;
    if (raw.nodes && raw.node_count <= 4096)
        for (std::size_t i = 0; i < raw.node_count; ++i) {
            const auto& n = raw.nodes[i];
            r.nodes.push_back({n.opcode, n.left, n.right, n.input, n.constant});
        }
    else if (raw.node_count > 4096)
        r.nodes.resize(257);  // rejected by validateRecipe
    return r;
}

} // namespace

std::string validateRecipe(const Recipe& recipe, std::uint32_t inputs, bool allowDivide) {
    if (recipe.inputCount != inputs) return "recipe input count disagrees with schema";
    if (recipe.nodes.empty() || recipe.nodes.size() > 256 || recipe.root >= recipe.nodes.size())
        return "recipe node/root count is invalid";
    for (std::size_t i = 0; i < recipe.nodes.size(); ++i) {
        const auto& n = recipe.nodes[i];
        switch (n.opcode) {
        case THB_SCALAR_INPUT:
            if (n.input >= inputs) return "recipe input reference is out of range";
            break;
        case THB_SCALAR_CONSTANT_F32:
            if (!std::isfinite(n.constant)) return "recipe constant must be finite";
            break;
        case THB_SCALAR_NEGATE:
            if (n.left >= i) return "recipe unary dependency is not earlier";
            break;
        case THB_SCALAR_ADD:
        case THB_SCALAR_SUBTRACT:
        case THB_SCALAR_MULTIPLY:
            if (n.left >= i || n.right >= i) return "recipe dependency is not earlier";
            break;
        case THB_SCALAR_DIVIDE:
            if (!allowDivide) return "division requires MayTrap";
            if (n.left >= i || n.right >= i) return "recipe dependency is not earlier";
            break;
        default: return "recipe opcode is invalid";
        }
    }
    return {};
}

std::string validateOperation(const Operation& op) {
    if (op.name.empty() || !validVersion(op.semanticVersion)) return "operation identity field is missing or malformed";
    if (op.arity == 0 || op.arity > 8 || op.resultLikeInput >= op.arity) return "operation arity/result rule is invalid";
    if (op.minimumRank < 1 || op.maximumRank > 2 || op.minimumRank > op.maximumRank) return "operation rank contract is invalid";
    if (!op.sameShape) return "V0 requires same-shape operands";
    if ((op.backends & THB_BACKEND_REFERENCE) == 0 ||
        (op.backends & ~std::uint32_t(THB_BACKEND_REFERENCE | THB_BACKEND_CPU | THB_BACKEND_GPU)) != 0)
        return "operation backend contract is invalid";
    if (op.effect != THB_EFFECT_PURE && op.effect != THB_EFFECT_MAY_TRAP) return "operation effect is invalid";
    if (op.fusible && (op.effect != THB_EFFECT_PURE || (op.backends & (THB_BACKEND_CPU | THB_BACKEND_GPU)) == 0))
        return "fusibility requires pure native lowering";
    if (auto bad = validateRecipe(op.forward, op.arity, op.effect == THB_EFFECT_MAY_TRAP); !bad.empty()) return bad;
    if (op.derivative) {
        const std::uint64_t mask = (1ULL << op.arity) - 1ULL;
        if ((op.derivative->differentiableInputs & ~mask) || (op.derivative->savedInputs & ~mask))
            return "derivative input/save mask is invalid";
        if (op.derivative->gradients.size() != op.arity) return "derivative gradient count disagrees with arity";
        for (std::size_t i = 0; i < op.derivative->gradients.size(); ++i) {
            const auto& g = op.derivative->gradients[i];
            const bool differentiable = (op.derivative->differentiableInputs >> i) & 1ULL;
            if (differentiable && g.nodes.empty()) return "differentiable input has no gradient recipe";
            if (!differentiable && !g.nodes.empty()) return "non-differentiable input has a gradient recipe";
            if (!g.nodes.empty())
                if (auto bad = validateRecipe(g, op.arity + 2, false); !bad.empty()) return bad;
        }
    }
    return {};
}

std::string canonicalIdentity(const Operation& op) {
    return op.extensionId + "::" + op.name + "@" + op.semanticVersion + "/abi" + std::to_string(op.abiVersion);
}

std::string descriptorDigest(const Operation& op) {
    Fnv h;
    h.text(op.extensionId); h.text(op.extensionVersion); h.text(op.name); h.text(op.semanticVersion);
    h.value(op.abiVersion); h.value(op.arity); h.value(op.minimumRank); h.value(op.maximumRank);
    h.value(op.resultLikeInput); h.byte(op.sameShape); h.byte(op.effect); h.value(op.backends); h.byte(op.fusible);
    h.recipe(op.forward);
    h.byte(op.derivative.has_value());
    if (op.derivative) {
        h.value(op.derivative->differentiableInputs); h.value(op.derivative->savedInputs);
        h.byte(op.derivative->savesOutput); h.value<std::uint64_t>(op.derivative->gradients.size());
        for (const auto& g : op.derivative->gradients) h.recipe(g);
    }
    std::ostringstream out;
    out << "fnv1a64:" << std::hex << std::setw(16) << std::setfill('0') << h.h;
    return out.str();
}

Operation importOperation(const thb_operation& raw) {
    Operation op;
    op.name = raw.name ? raw.name : "";
    op.semanticVersion = raw.semantic_version ? raw.semantic_version : "";
    op.arity = raw.arity;
    op.minimumRank = raw.minimum_rank;
    op.maximumRank = raw.maximum_rank;
    op.resultLikeInput = raw.result_like_input;
    op.sameShape = raw.same_shape != 0;
    op.effect = raw.effect;
    op.backends = raw.backends;
    op.fusible = raw.fusible != 0;
    op.forward = importRecipe(raw.forward);
    if (raw.derivative) {
        Derivative d;
        d.differentiableInputs = raw.derivative->differentiable_inputs;
        d.savedInputs = raw.derivative->saved_inputs;
        d.savesOutput = raw.derivative->saves_output != 0;
        if (raw.derivative->gradients && raw.derivative->gradient_count <= 8)
            for (std::size_t i = 0; i < raw.derivative->gradient_count; ++i)
                d.gradients.push_back(importRecipe(raw.derivative->gradients[i]));
        op.derivative = std::move(d);
    }
    op.digest = engineDigest(op);
    return op;
}

std::string engineDigest(const Operation& op) {
    Fnv h;
    h.text(op.name); h.text(op.semanticVersion); h.value(op.arity); h.value(op.minimumRank);
    h.value(op.maximumRank); h.value(op.resultLikeInput); h.byte(op.sameShape); h.byte(op.effect);
    h.value(op.backends); h.byte(op.fusible); h.recipe(op.forward);
    std::ostringstream out;
    out << "fnv1a64:" << std::hex << h.h;
    return out.str();
}

// ---- region IR ------------------------------------------------------------------

bool Node::knownShapeMismatch(const Node& o) const {
    if (rank != o.rank) return true;
    for (std::uint32_t a = 0; a < rank; ++a)
        if (extent[a] >= 0 && o.extent[a] >= 0 && extent[a] != o.extent[a]) return true;
    return false;
}

bool Node::sameShapeFact(const Node& o) const {
    if (rank != o.rank) return false;
    for (std::uint32_t a = 0; a < rank; ++a)
        if (extent[a] != o.extent[a]) return false;
    return true;
}

const Node* Region::find(std::uint32_t id) const {
    for (const auto& n : nodes)
        if (n.id == id) return &n;
    return nullptr;
}

const Node& Region::at(std::uint32_t id) const {
    const Node* n = find(id);
    if (!n) fail(Category::Unsupported, "GPU-INVALID-REGION", "region value v" + std::to_string(id) + " is absent");
    return *n;
}

std::size_t Region::position(std::uint32_t id) const {
    for (std::size_t i = 0; i < nodes.size(); ++i)
        if (nodes[i].id == id) return i;
    fail(Category::Unsupported, "GPU-INVALID-REGION", "region value v" + std::to_string(id) + " is absent");
}

std::uint32_t Region::canonical(std::uint32_t id) const {
    std::set<std::uint32_t> seen;
    while (seen.insert(id).second) {
        const Node* n = find(id);
        if (!n || n->op != Op::Alias || n->dependencies.size() != 1) break;
        id = n->dependencies.front();
    }
    return id;
}

std::string Region::dump() const {
    std::ostringstream out;
    out << "region f" << function << ' ' << name << '\n';
    for (const auto& n : nodes) {
        out << "  v" << n.id << ' ' << opName(n.op) << ' ' << dtypeName(n.dtype);
        if (n.rank) {
            out << " [";
            for (std::uint32_t a = 0; a < n.rank; ++a) {
                if (a) out << ',';
                if (n.extent[a] >= 0) out << n.extent[a]; else out << '?';
            }
            out << ']';
        }
        for (auto d : n.dependencies) out << " v" << d;
        for (auto i : n.indices) out << " [v" << i << ']';
        if (n.op == Op::Integer) out << " =" << n.integer;
        if (n.op == Op::Float) out << " =" << n.floating << 'f';
        if (isReduction(n.op)) out << " axis=" << n.axis;
        if (n.extension) out << " extension=" << n.extension->name << '@' << n.extension->semanticVersion
                             << " digest=" << n.extension->digest;
        out << '\n';
    }
    out << "  output v" << output << '\n';
    return out.str();
}

Region importRegion(const thb_region_desc& desc) {
    Region r;
    r.function = desc.function;
    r.name = desc.name ? desc.name : "";
    if (desc.node_count && !desc.nodes) fail(Category::Validation, "GPU-INVALID-REGION", "node array is null");
    if (desc.input_count && !desc.inputs) fail(Category::Validation, "GPU-INVALID-REGION", "input array is null");
    r.nodes.reserve(desc.node_count);
    for (std::uint32_t i = 0; i < desc.node_count; ++i) {
        const auto& raw = desc.nodes[i];
        Node n;
        n.id = raw.id;
        n.op = static_cast<Op>(raw.op);
        switch (raw.op) {
        case THB_OP_INPUT: case THB_OP_INTEGER: case THB_OP_FLOAT: case THB_OP_TENSOR_LITERAL:
        case THB_OP_ALIAS: case THB_OP_COPY: case THB_OP_NEGATE: case THB_OP_ADD: case THB_OP_SUBTRACT:
        case THB_OP_ELEMENT_MULTIPLY: case THB_OP_EXTENSION: case THB_OP_INDEX: case THB_OP_SUM:
        case THB_OP_ROW_MAX: case THB_OP_SOFTMAX: case THB_OP_RELU: case THB_OP_EXTENSION_GRADIENT:
        case THB_OP_TRANSPOSE: case THB_OP_MATMUL: case THB_OP_BROADCAST_TO_SHAPE: case THB_OP_REDUCE_TO_SHAPE:
        case THB_OP_ZERO_LIKE:
            break;
        default: n.op = Op::Unsupported;
        }
        if (raw.dtype != THB_DTYPE_I64 && raw.dtype != THB_DTYPE_F32)
            fail(Category::Unsupported, "GPU-INVALID-REGION", "region dtype must be i64 or f32");
        n.dtype = static_cast<DType>(raw.dtype);
        n.rank = raw.rank;
        if (n.rank > 2) fail(Category::Unsupported, "GPU-INVALID-REGION", "region tensors are rank 1 or 2");
        n.extent[0] = raw.extent[0];
        n.extent[1] = raw.extent[1];
        if (raw.dependency_count && !raw.dependencies)
            fail(Category::Validation, "GPU-INVALID-REGION", "dependency array is null");
        n.dependencies.assign(raw.dependencies, raw.dependencies + raw.dependency_count);
        if (raw.index_count && !raw.indices) fail(Category::Validation, "GPU-INVALID-REGION", "index array is null");
        n.indices.assign(raw.indices, raw.indices + raw.index_count);
        n.integer = raw.integer;
        n.floating = raw.floating;
        n.axis = raw.axis;
        if (raw.extension) n.extension = std::make_shared<const Operation>(importOperation(*raw.extension));
        r.nodes.push_back(std::move(n));
    }
    r.inputs.assign(desc.inputs, desc.inputs + desc.input_count);
    r.output = desc.output;
    return r;
}

// ---- verifier -------------------------------------------------------------------

std::vector<std::string> verifyRegion(const Region& region) {
    std::vector<std::string> errors;
    std::set<std::uint32_t> all, seen;
    for (const auto& n : region.nodes)
        if (!all.insert(n.id).second || n.id == 0) errors.push_back("TRV01 duplicate/zero region value ID");
    auto numericTensor = [](const Node& n) { return n.rank == 1 || n.rank == 2; };
    for (const auto& n : region.nodes) {
        for (auto d : n.dependencies) {
            if (!all.count(d)) errors.push_back("TRV02 unknown dependency");
            else if (!seen.count(d)) errors.push_back("TRV03 use before definition");
        }
        for (auto d : n.indices) {
            if (!all.count(d)) errors.push_back("TRV02 unknown index dependency");
            else if (!seen.count(d)) errors.push_back("TRV03 index use before definition");
        }
        auto dep = [&](std::size_t i) -> const Node* {
            return i < n.dependencies.size() ? region.find(n.dependencies[i]) : nullptr;
        };
        switch (n.op) {
        case Op::Add: case Op::Subtract: case Op::ElementMultiply: {
            if (!numericTensor(n)) errors.push_back("TRV04 elementwise result is not Tensor<i64/f32,R>");
            const Node* l = dep(0); const Node* r = dep(1);
            // Tensor (x) tensor of one type, or tensor (x) scalar of the same
            // element type: the scalar broadcasts (Evaluator.cpp:95-124); the
            // reference's native extractor rejects the scalar form.
            const bool both = l && r && numericTensor(*l) && numericTensor(*r) && l->sameType(*r) && l->sameType(n);
            const bool scalarRight = l && r && numericTensor(*l) && r->rank == 0 && r->dtype == l->dtype && l->sameType(n);
            const bool scalarLeft = l && r && numericTensor(*r) && l->rank == 0 && l->dtype == r->dtype && r->sameType(n);
            if (n.dependencies.size() != 2 || !(both || scalarRight || scalarLeft))
                errors.push_back("TRV05 elementwise input type mismatch");
            if (both && (l->knownShapeMismatch(*r) || n.knownShapeMismatch(*l)))
                errors.push_back("TRV06 elementwise known shape mismatch");
            if (scalarRight && n.knownShapeMismatch(*l)) errors.push_back("TRV06 elementwise known shape mismatch");
            if (scalarLeft && n.knownShapeMismatch(*r)) errors.push_back("TRV06 elementwise known shape mismatch");
            break;
        }
        case Op::Extension: {
            bool ok = n.extension != nullptr;
            if (ok) {
                const auto& op = *n.extension;
                ok = validateOperation(op).empty() && n.dependencies.size() == op.arity &&
                     numericTensor(n) && n.rank >= op.minimumRank && n.rank <= op.maximumRank &&
                     n.dtype == DType::F32;
                for (auto d : n.dependencies) {
                    const Node* in = region.find(d);
                    ok = ok && in && in->sameType(n) && !in->knownShapeMismatch(n);
                }
            }
            if (!ok) errors.push_back("TRV11 malformed extension operation");
            break;
        }
        case Op::Negate: case Op::Relu: {
            const Node* in = dep(0);
            if (n.dependencies.size() != 1 || !in || !numericTensor(n) || !in->sameType(n) || in->knownShapeMismatch(n) ||
                (n.op == Op::Relu && n.dtype != DType::F32))
                errors.push_back(std::string("TRV10 malformed ") + opName(n.op));
            break;
        }
        case Op::Index: {
            const Node* in = dep(0);
            if (!in || !numericTensor(*in) || n.indices.size() != in->rank)
                errors.push_back("TRV07 Index non-tensor/full-rank input");
            if (!in || n.rank != 0 || n.dtype != in->dtype) errors.push_back("TRV08 Index result dtype mismatch");
            for (auto i : n.indices) {
                const Node* c = region.find(i);
                if (c && !(c->rank == 0 && c->dtype == DType::I64)) errors.push_back("TRV07 Index coordinate not i64");
            }
            break;
        }
        case Op::Sum: {
            const Node* in = dep(0);
            // f32 (f64-accumulated) or i64 (exact, checked) operands.
            bool ok = n.dependencies.size() == 1 && in && numericTensor(*in) &&
                      (in->dtype == DType::F32 || in->dtype == DType::I64) && n.dtype == in->dtype && n.axis >= 0 &&
                      static_cast<std::uint32_t>(n.axis) < in->rank && n.rank + 1 == in->rank;
            if (ok && n.rank == 1) {
                const std::int64_t kept = in->extent[n.axis == 0 ? 1 : 0];
                ok = n.extent[0] < 0 || kept < 0 || n.extent[0] == kept;
            }
            if (!ok) errors.push_back("TRV12 malformed Sum");
            break;
        }
        case Op::RowMax: {
            const Node* in = dep(0);
            bool ok = n.dependencies.size() == 1 && in && in->rank == 2 && in->dtype == DType::F32 &&
                      n.dtype == DType::F32 && n.rank == 1 && n.axis == 1 &&
                      (n.extent[0] < 0 || in->extent[0] < 0 || n.extent[0] == in->extent[0]);
            if (!ok) errors.push_back("TRV12 malformed RowMax");
            break;
        }
        case Op::Softmax: {
            const Node* in = dep(0);
            bool ok = n.dependencies.size() == 1 && in && numericTensor(*in) && in->sameType(n) &&
                      n.dtype == DType::F32 && !in->knownShapeMismatch(n) &&
                      n.axis == static_cast<std::int32_t>(n.rank) - 1;
            if (!ok) errors.push_back("TRV12 malformed Softmax");
            break;
        }
        case Op::ExtensionGradient: {
            // deps: arity primals, the primal result, the output cotangent;
            // axis selects the differentiable operand (Autodiff.cpp:231-270).
            bool ok = n.extension && n.extension->derivative && validateOperation(*n.extension).empty() &&
                      n.dtype == DType::F32 && numericTensor(n) && n.axis >= 0 &&
                      static_cast<std::uint32_t>(n.axis) < n.extension->arity &&
                      n.dependencies.size() == n.extension->arity + 2u;
            if (ok) {
                const auto& d = *n.extension->derivative;
                ok = ((d.differentiableInputs >> n.axis) & 1ULL) &&
                     static_cast<std::size_t>(n.axis) < d.gradients.size() && !d.gradients[n.axis].nodes.empty();
                for (auto id : n.dependencies) {
                    const Node* in = region.find(id);
                    ok = ok && in && in->sameType(n) && !in->knownShapeMismatch(n);
                }
            }
            if (!ok) errors.push_back("TRV11 malformed extension gradient");
            break;
        }
        case Op::Transpose: {
            const Node* in = dep(0);
            bool ok = n.dependencies.size() == 1 && in && in->rank == 2 && n.rank == 2 && in->dtype == n.dtype;
            ok = ok && (n.extent[0] < 0 || in->extent[1] < 0 || n.extent[0] == in->extent[1]) &&
                 (n.extent[1] < 0 || in->extent[0] < 0 || n.extent[1] == in->extent[0]);
            if (!ok) errors.push_back("TRV12 malformed Transpose");
            break;
        }
        case Op::MatMul: {
            const Node* a = dep(0); const Node* b = dep(1);
            // f32 (tensor-core or exact mode) or checked i64 operands.
            bool ok = n.dependencies.size() == 2 && a && b && a->rank == 2 && b->rank == 2 && n.rank == 2 &&
                      (n.dtype == DType::F32 || n.dtype == DType::I64) && a->dtype == n.dtype &&
                      b->dtype == n.dtype && (n.axis == THB_MATMUL_TENSOR || n.axis == THB_MATMUL_EXACT);
            ok = ok && (a->extent[1] < 0 || b->extent[0] < 0 || a->extent[1] == b->extent[0]) &&
                 (n.extent[0] < 0 || a->extent[0] < 0 || n.extent[0] == a->extent[0]) &&
                 (n.extent[1] < 0 || b->extent[1] < 0 || n.extent[1] == b->extent[1]);
            if (!ok) errors.push_back("TRV12 malformed MatMul");
            break;
        }
        case Op::BroadcastToShape: {
            const Node* v = dep(0); const Node* ref = dep(1);
            bool ok = n.dependencies.size() == 2 && v && ref && v->dtype == DType::F32 && ref->dtype == DType::F32 &&
                      n.dtype == DType::F32 && numericTensor(*ref) && n.sameType(*ref) && !n.knownShapeMismatch(*ref) &&
                      n.axis >= 0 && static_cast<std::uint32_t>(n.axis) < ref->rank && v->rank + 1 == ref->rank;
            if (!ok) errors.push_back("TRV12 malformed BroadcastToShape");
            break;
        }
        case Op::ReduceToShape: {
            const Node* v = dep(0); const Node* ref = dep(1);
            bool ok = n.dependencies.size() == 2 && v && ref && v->dtype == DType::F32 && ref->dtype == DType::F32 &&
                      n.dtype == DType::F32 && numericTensor(*v) && n.rank == ref->rank && ref->rank <= v->rank &&
                      !n.knownShapeMismatch(*ref);
            if (!ok) errors.push_back("TRV12 malformed ReduceToShape");
            break;
        }
        case Op::ZeroLike: {
            const Node* ref = dep(0);
            bool ok = n.dependencies.size() == 1 && ref && n.dtype == DType::F32 && n.rank == ref->rank &&
                      !n.knownShapeMismatch(*ref);
            if (!ok) errors.push_back("TRV12 malformed ZeroLike");
            break;
        }
        case Op::Unsupported: errors.push_back("TRV10 unsupported operation admitted"); break;
        case Op::Input: break;
        case Op::TensorLiteral: {
            bool known = numericTensor(n);
            std::uint64_t count = 1;
            for (std::uint32_t a = 0; known && a < n.rank; ++a) {
                if (n.extent[a] < 0) { known = false; break; }
                std::uint64_t next = 0;
                if (__builtin_mul_overflow(count, static_cast<std::uint64_t>(n.extent[a]), &next)) {
                    errors.push_back("TRV10 tensor literal element-count overflow");
                    known = false;
                    break;
                }
                count = next;
            }
            if (!known) errors.push_back("TRV10 malformed tensor literal");
            else if (count != n.dependencies.size()) errors.push_back("TRV10 tensor literal element count mismatch");
            for (auto d : n.dependencies) {
                const Node* c = region.find(d);
                if (c && !(c->rank == 0 && c->dtype == n.dtype)) errors.push_back("TRV10 tensor literal element dtype mismatch");
            }
            break;
        }
        case Op::Alias: {
            const Node* in = dep(0);
            if (n.dependencies.size() != 1 || !in || !in->sameType(n)) errors.push_back("TRV10 malformed alias");
            break;
        }
        case Op::Copy: {
            const Node* in = dep(0);
            if (n.dependencies.size() != 1 || !in || !numericTensor(n) || !in->sameType(n) || in->knownShapeMismatch(n))
                errors.push_back("TRV10 malformed Copy");
            break;
        }
        case Op::Integer:
            if (n.rank != 0 || n.dtype != DType::I64) errors.push_back("TRV10 malformed integer");
            break;
        case Op::Float:
            if (n.rank != 0 || n.dtype != DType::F32) errors.push_back("TRV10 malformed float");
            break;
        }
        seen.insert(n.id);
    }
    if (!all.count(region.output) || region.output == 0) errors.push_back("TRV09 missing region output");
    for (auto id : region.inputs) {
        const Node* n = region.find(id);
        if (!n || n->op != Op::Input) errors.push_back("TRV09 region input is not an Input node");
    }
    return errors;
}

// ---- physical plan --------------------------------------------------------------

const ValuePlan* Plan::value(std::uint32_t id) const {
    for (const auto& v : values)
        if (v.value == id) return &v;
    return nullptr;
}

const FusionGroup* Plan::groupFor(std::uint32_t id) const {
    for (const auto& g : groups)
        if (std::find(g.nodes.begin(), g.nodes.end(), id) != g.nodes.end()) return &g;
    return nullptr;
}

namespace {

bool fusibleNode(const Node& n) {
    if (!isElementwise(n.op)) return false;
    if (n.op != Op::Extension) return true;
    return n.extension && n.extension->fusible && n.extension->effect == THB_EFFECT_PURE;
}

bool kernelNode(const Node& n) {
    return isElementwise(n.op) || isReduction(n.op) || isKernelOp(n.op) || n.op == Op::Index;
}

// Consumers of each canonical value, looking through Alias nodes
// (fusionConsumers, src/backend/v0/PhysicalPlan.cpp:78-87).
std::map<std::uint32_t, std::vector<std::uint32_t>> consumers(const Region& region) {
    std::map<std::uint32_t, std::vector<std::uint32_t>> uses;
    for (const auto& n : region.nodes) {
        if (n.op == Op::Alias) continue;
        for (auto d : n.dependencies) uses[region.canonical(d)].push_back(n.id);
    }
    return uses;
}

// makeFusionGroups (src/backend/v0/PhysicalPlan.cpp:170-225): a new kernel
// node joins the most recent group only when that group's tail is an
// elementwise node of identical type and shape whose single consumer is this
// node, the tail is not the region output, and no other operand of this node
// was produced after the group began.
std::vector<FusionGroup> makeGroups(const Region& region, const PlanOptions& options) {
    const auto uses = consumers(region);
    const std::uint32_t output = region.canonical(region.output);
    std::vector<FusionGroup> groups;
    for (const auto& current : region.nodes) {
        if (!kernelNode(current)) continue;
        bool extend = false;
        if (options.enableFusion && fusibleNode(current) && !groups.empty() &&
            groups.back().kind == GroupKind::Elementwise) {
            const FusionGroup& prior = groups.back();
            const Node& tail = region.at(prior.nodes.back());
            if (fusibleNode(tail) && tail.id != output && tail.sameType(current) && tail.sameShapeFact(current)) {
                auto use = uses.find(tail.id);
                const bool oneConsumer = use != uses.end() && use->second.size() == 1 && use->second.front() == current.id;
                std::size_t occurrences = 0;
                bool intervening = false;
                const std::size_t groupStart = region.position(prior.nodes.front());
                for (auto d : current.dependencies) {
                    const auto c = region.canonical(d);
                    if (c == tail.id) ++occurrences;
                    // Scalars are kernel constants/parameters, not materialised tensors.
                    else if (region.at(c).tensor() && region.position(c) > groupStart) intervening = true;
                }
                extend = oneConsumer && occurrences == 1 && !intervening;
            }
        }
        if (extend) {
            auto& g = groups.back();
            g.nodes.push_back(current.id);
            g.output = current.id;
            g.fused = true;
        } else {
            FusionGroup g;
            g.id = static_cast<std::uint32_t>(groups.size() + 1);
            g.kind = isElementwise(current.op) ? GroupKind::Elementwise
                   : isReduction(current.op) ? GroupKind::Reduction
                   : isKernelOp(current.op) ? GroupKind::Kernel : GroupKind::Index;
            g.nodes = {current.id};
            g.output = current.id;
            g.dtype = current.op == Op::Index ? region.at(region.canonical(current.dependencies.at(0))).dtype : current.dtype;
            groups.push_back(std::move(g));
        }
    }
    for (auto& g : groups) {
        std::set<std::uint32_t> inside(g.nodes.begin(), g.nodes.end()), seenInputs;
        for (auto id : g.nodes) {
            const Node& n = region.at(id);
            if (n.dtype == DType::I64 && g.kind == GroupKind::Elementwise) g.mayTrap = true;
            if (n.op == Op::Extension && n.extension && n.extension->effect == THB_EFFECT_MAY_TRAP) g.mayTrap = true;
            if (g.kind == GroupKind::Index) continue;
            for (auto d : n.dependencies) {
                const auto c = region.canonical(d);
                if (inside.count(c) || !seenInputs.insert(c).second) continue;
                const Node& operand = region.at(c);
                if (operand.tensor()) g.inputs.push_back(c);
                else if (operand.op != Op::Integer && operand.op != Op::Float) g.scalars.push_back(c);
            }
        }
    }
    return groups;
}

} // namespace

Plan buildPlan(const Region& region, PlanOptions options) {
    const auto errors = verifyRegion(region);
    if (!errors.empty()) fail(Category::Unsupported, "GPU-INVALID-REGION", errors.front());
    Plan plan;
    plan.options = options;
    plan.groups = makeGroups(region, options);

    std::set<std::uint32_t> fusedIntermediate;
    for (const auto& g : plan.groups)
        if (g.nodes.size() > 1) fusedIntermediate.insert(g.nodes.begin(), g.nodes.end() - 1);

    // Roots: aliases share their source's physical root (roots(),
    // PhysicalPlan.cpp:235-254).
    std::map<std::uint32_t, std::uint32_t> root;
    for (const auto& n : region.nodes) {
        if (!n.tensor()) continue;
        root[n.id] = n.op == Op::Alias ? root.at(n.dependencies.front()) : n.id;
    }
    const std::uint32_t outputRoot = region.at(region.output).tensor() ? root.at(region.output) : 0;
    const std::size_t end = region.nodes.size();

    // Lifetimes: from the first definition of a root to its last use, or to the
    // region end for the output root (requiredLifetime, PhysicalPlan.cpp:256-279).
    auto lifetime = [&](std::uint32_t r) {
        std::size_t first = region.position(r), last = first;
        for (std::size_t p = 0; p < region.nodes.size(); ++p) {
            const Node& n = region.nodes[p];
            for (auto d : n.dependencies)
                if (root.count(d) && root.at(d) == r) last = std::max(last, p);
            for (auto d : n.indices)
                if (root.count(d) && root.at(d) == r) last = std::max(last, p);
        }
        if (r == outputRoot) last = end;
        return std::pair<std::size_t, std::size_t>(first, last);
    };

    for (const auto& n : region.nodes) {
        if (!n.tensor()) continue;
        ValuePlan v;
        v.value = n.id;
        v.root = root.at(n.id);
        std::tie(v.definition, v.lastUse) = lifetime(v.root);
        bool zero = false;
        for (std::uint32_t a = 0; a < n.rank; ++a) zero = zero || n.extent[a] == 0;
        v.materialized = !fusedIntermediate.count(n.id) && !fusedIntermediate.count(v.root);
        if (zero) v.klass = ValueClass::ZeroSize;
        else if (!v.materialized) v.klass = ValueClass::FusedIntermediate;
        else if (n.op == Op::Alias) v.klass = ValueClass::Alias;
        else if (n.id == region.output || v.root == outputRoot) v.klass = ValueClass::Output;
        else if (n.op == Op::Input) v.klass = ValueClass::External;
        else v.klass = ValueClass::Temporary;
        v.reusable = v.materialized && !zero && options.enableReuse && v.klass == ValueClass::Temporary && v.value == v.root;
        plan.values.push_back(v);
    }

    // Slot assignment: a reusable root takes the first reusable slot with an
    // identical requirement whose resident roots do not overlap its lifetime.
    auto overlaps = [](const ValuePlan& a, const ValuePlan& b) {
        return !(a.lastUse < b.definition || b.lastUse < a.definition);
    };
    for (auto& v : plan.values) {
        if (v.value != v.root || !v.materialized || v.klass == ValueClass::ZeroSize) continue;
        const Node& n = region.at(v.value);
        Slot* chosen = nullptr;
        if (v.reusable) {
            for (auto& s : plan.slots) {
                if (!s.reusable || s.dtype != n.dtype || s.rank != n.rank || s.extent[0] != n.extent[0] ||
                    s.extent[1] != n.extent[1])
                    continue;
                bool clash = false;
                for (auto other : s.values) {
                    const ValuePlan* o = nullptr;
                    for (const auto& candidate : plan.values)
                        if (candidate.value == other) o = &candidate;
                    if (o && o->root == o->value && overlaps(*o, v)) { clash = true; break; }
                }
                if (!clash) { chosen = &s; break; }
            }
        }
        if (!chosen) {
            Slot s;
            s.id = static_cast<std::uint32_t>(plan.slots.size() + 1);
            s.dtype = n.dtype;
            s.rank = n.rank;
            s.extent[0] = n.extent[0];
            s.extent[1] = n.extent[1];
            s.external = n.op == Op::Input;
            s.reusable = v.reusable;
            plan.slots.push_back(s);
            chosen = &plan.slots.back();
        }
        v.slot = chosen->id;
        chosen->values.push_back(v.value);
    }
    for (auto& v : plan.values) {
        if (v.value == v.root || !v.materialized) continue;
        for (const auto& r : plan.values)
            if (r.value == v.root) v.slot = r.slot;
        if (v.slot) plan.slots.at(*v.slot - 1).values.push_back(v.value);
    }
    return plan;
}

std::string Plan::dump(const Region& region) const {
    static const char* names[] = {"external", "temporary", "output", "alias", "fused-intermediate", "zero-size"};
    std::ostringstream out;
    out << "physical-plan f" << region.function << " device=gpu reuse=" << (options.enableReuse ? "on" : "off")
        << " fusion=" << (options.enableFusion ? "on" : "off") << '\n';
    for (const auto& v : values)
        out << "  value v" << v.value << " root=v" << v.root << " class=" << names[static_cast<int>(v.klass)]
            << " lifetime=[" << v.definition << ',' << v.lastUse << ']'
            << " materialized=" << (v.materialized ? "yes" : "no") << " reusable=" << (v.reusable ? "yes" : "no")
            << " slot=" << (v.slot ? std::to_string(*v.slot) : "none") << '\n';
    for (const auto& s : slots) {
        out << "  slot s" << s.id << " dtype=" << dtypeName(s.dtype) << " external=" << (s.external ? "yes" : "no")
            << " reusable=" << (s.reusable ? "yes" : "no") << " values=";
        for (std::size_t i = 0; i < s.values.size(); ++i) out << (i ? "," : "") << 'v' << s.values[i];
        out << '\n';
    }
    for (const auto& g : groups) {
        out << "  group g" << g.id << " nodes=";
        for (std::size_t i = 0; i < g.nodes.size(); ++i) out << (i ? "," : "") << 'v' << g.nodes[i];
        out << " output=v" << g.output << " fused=" << (g.fused ? "yes" : "no") << '\n';
    }
    return out.str();
}

} // namespace thb
