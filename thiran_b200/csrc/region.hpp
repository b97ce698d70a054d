// Host-side TensorRegion IR, verifier and physical planner of the B200 engine.
//
// The IR carries the same facts as the reference's RegionNode / TensorRegion
// (include/backend/v0/TensorRegion.hpp:14-57); the planner produces the same
// kinds of decisions as buildPhysicalPlan (src/backend/v0/PhysicalPlan.cpp:
// 366-482): fusion groups of single-consumer elementwise chains, value
// classes, lifetimes and reusable device slots. Engine-side reductions
// (Sum / RowMax / Softmax) become their own kernel groups.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <optional>
#include <set>
#include <string>
#include <vector>

#include "common.hpp"

namespace thb {

enum class Op : std::uint32_t {
    Input = THB_OP_INPUT,
    Integer = THB_OP_INTEGER,
    Float = THB_OP_FLOAT,
    TensorLiteral = THB_OP_TENSOR_LITERAL,
    Alias = THB_OP_ALIAS,
    Copy = THB_OP_COPY,
    Negate = THB_OP_NEGATE,
    Add = THB_OP_ADD,
    Subtract = THB_OP_SUBTRACT,
    ElementMultiply = THB_OP_ELEMENT_MULTIPLY,
    Extension = THB_OP_EXTENSION,
    Index = THB_OP_INDEX,
    Unsupported = THB_OP_UNSUPPORTED,
    Sum = THB_OP_SUM,
    RowMax = THB_OP_ROW_MAX,
    Softmax = THB_OP_SOFTMAX,
    Relu = THB_OP_RELU,
    ExtensionGradient = THB_OP_EXTENSION_GRADIENT,
    Transpose = THB_OP_TRANSPOSE,
    MatMul = THB_OP_MATMUL,
    BroadcastToShape = THB_OP_BROADCAST_TO_SHAPE,
    ReduceToShape = THB_OP_REDUCE_TO_SHAPE,
    ZeroLike = THB_OP_ZERO_LIKE,
};

const char* opName(Op op);

struct ScalarNode {
    std::uint8_t opcode = THB_SCALAR_INPUT;
    std::uint32_t left = 0, right = 0, input = 0;
    float constant = 0.0f;
};

struct Recipe {
    std::vector<ScalarNode> nodes;
    std::uint32_t root = 0;
    std::uint32_t inputCount = 0;
};

struct Derivative {
    std::uint64_t differentiableInputs = 0, savedInputs = 0;
    bool savesOutput = false;
    std::vector<Recipe> gradients;
};

// A validated copy of an operation descriptor (OperationDescriptorV0).
struct Operation {
    std::string name, semanticVersion;
    std::uint32_t arity = 0, minimumRank = 1, maximumRank = 2, resultLikeInput = 0;
    bool sameShape = true;
    std::uint8_t effect = THB_EFFECT_PURE;
    std::uint32_t backends = 0;
    bool fusible = false;
    Recipe forward;
    std::optional<Derivative> derivative;
    std::string digest;  // FNV-1a over the descriptor fields
    // Registry identity (include/extension/v0/Extension.hpp:81-93): carried
    // by artifacts. Descriptors passed in directly get extensionId "inline".
    std::string extensionId = "inline", extensionVersion = "1.0.0";
    std::uint32_t abiVersion = 1;
};

// "<extension>::<name>@<version>/abi<N>" (src/extension/v0/Extension.cpp:203).
std::string canonicalIdentity(const Operation&);
// FNV-1a 64 over the identity and descriptor fields in the reference's order
// (operationDigest, src/extension/v0/Extension.cpp:135-149), "fnv1a64:%016x".
std::string descriptorDigest(const Operation&);

// Validation of a descriptor; the rules of validateRecipe / validateOperation
// (src/extension/v0/Extension.cpp:51-133). Returns an empty string when valid.
std::string validateRecipe(const Recipe&, std::uint32_t inputs, bool allowDivide);
std::string validateOperation(const Operation&);
Operation importOperation(const thb_operation&);
// The engine's short descriptor digest (`Operation::digest`: name, version,
// contract and forward recipe), shown in region dumps.
std::string engineDigest(const Operation&);

struct Node {
    std::uint32_t id = 0;
    Op op = Op::Unsupported;
    DType dtype = DType::F32;
    std::uint32_t rank = 0;          // 0 = scalar
    std::int64_t extent[2] = {-1, -1};
    std::vector<std::uint32_t> dependencies;
    std::vector<std::uint32_t> indices;
    std::int64_t integer = 0;
    float floating = 0.0f;
    std::int32_t axis = 0;
    std::shared_ptr<const Operation> extension;

    bool tensor() const { return rank > 0; }
    bool sameType(const Node& o) const { return dtype == o.dtype && rank == o.rank; }
    bool knownShapeMismatch(const Node& o) const;
    bool sameShapeFact(const Node& o) const;
};

struct Region {
    std::uint32_t function = 0;
    std::string name;
    std::vector<Node> nodes;
    std::vector<std::uint32_t> inputs;
    std::uint32_t output = 0;

    const Node* find(std::uint32_t id) const;
    const Node& at(std::uint32_t id) const;
    std::size_t position(std::uint32_t id) const;
    std::uint32_t canonical(std::uint32_t id) const;  // follows Alias chains
    std::string dump() const;
};

Region importRegion(const thb_region_desc&);

// verifyRegion (src/backend/v0/TensorRegion.cpp:103-228): returns the list of
// TRVnn errors, empty when the region is well formed.
std::vector<std::string> verifyRegion(const Region&);

// Elementwise groups get a generated kernel; Reduction and Kernel groups run
// one precompiled kernel (reductions, transpose, matmul, broadcast).
enum class GroupKind { Elementwise, Reduction, Index, Kernel };

struct FusionGroup {
    std::uint32_t id = 0;
    GroupKind kind = GroupKind::Elementwise;
    std::vector<std::uint32_t> nodes;
    std::vector<std::uint32_t> inputs;  // canonical external tensor operands, first-use order
    std::vector<std::uint32_t> scalars; // runtime scalar operands (kernel parameters); literals are constants
    std::uint32_t output = 0;
    DType dtype = DType::F32;
    bool fused = false;
    bool mayTrap = false;  // i64 checks or a MayTrap recipe: needs an error word
};

enum class ValueClass { External, Temporary, Output, Alias, FusedIntermediate, ZeroSize };

struct ValuePlan {
    std::uint32_t value = 0, root = 0;
    ValueClass klass = ValueClass::Temporary;
    std::size_t definition = 0, lastUse = 0;
    bool materialized = true;
    bool reusable = false;
    std::optional<std::uint32_t> slot;
};

struct Slot {
    std::uint32_t id = 0;
    DType dtype = DType::F32;
    std::uint32_t rank = 0;
    std::int64_t extent[2] = {-1, -1};
    bool external = false;
    bool reusable = false;
    std::vector<std::uint32_t> values;
};

struct PlanOptions {
    bool enableReuse = true;
    bool enableFusion = true;
};

struct Plan {
    PlanOptions options;
    std::vector<FusionGroup> groups;
    std::vector<ValuePlan> values;
    std::vector<Slot> slots;

    const ValuePlan* value(std::uint32_t id) const;
    const FusionGroup* groupFor(std::uint32_t id) const;
    std::string dump(const Region&) const;
};

// buildPhysicalPlan for the GPU device. Throws Failure(GPU-INVALID-REGION)
// when the region does not verify.
Plan buildPlan(const Region&, PlanOptions);

bool isElementwise(Op op);
bool isReduction(Op op);
// Transpose, MatMul, BroadcastToShape, ReduceToShape, ZeroLike.
bool isKernelOp(Op op);

} // namespace thb
