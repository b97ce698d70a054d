// `.tha` artifacts (see artifact.hpp). The byte layout follows the
// reference's Writer / Reader (src/artifact/v0/NativeArtifacts.cpp:58-127):
// little-endian u8/u32/u64, texts as u64 length + bytes.
#include "artifact.hpp"

#include <cstring>
#include <iomanip>
#include <limits>
#include <sstream>

#include "codegen.hpp"

namespace thb::artifact {
namespace {

constexpr char kMagic[8] = {'T', 'H', 'I', 'R', 'A', 'N', '1', '6'};
constexpr char kEngineMagic[8] = {'T', 'H', 'B', 'C', 'U', 'B', 'I', 'N'};
constexpr std::uint64_t kMaxString = 1ull << 20;
constexpr std::uint64_t kMaxRegion = 64ull << 20;
constexpr std::uint64_t kMaxPayload = 512ull << 20;
constexpr std::uint64_t kMaxItems = 1ull << 20;
// semantic::TypeKind (include/semantic/v0/Ir.hpp:18).
constexpr std::uint8_t kTypeI64 = 3, kTypeF32 = 6, kTypeTensor = 8;

[[noreturn]] void bad(const std::string& code, const std::string& message) {
    fail(Category::Validation, code, message);
}

class Reader {
public:
    explicit Reader(const std::string& bytes) : bytes_(bytes) {}
    std::uint8_t u8() {
        need(1);
        return static_cast<std::uint8_t>(bytes_[offset_++]);
    }
    std::uint32_t u32() {
        std::uint32_t v = 0;
        for (unsigned s = 0; s < 32; s += 8) v |= static_cast<std::uint32_t>(u8()) << s;
        return v;
    }
    std::uint64_t u64() {
        std::uint64_t v = 0;
        for (unsigned s = 0; s < 64; s += 8) v |= static_cast<std::uint64_t>(u8()) << s;
        return v;
    }
    std::int64_t i64() {
        const std::uint64_t v = u64();
        std::int64_t r;
        std::memcpy(&r, &v, 8);
        return r;
    }
    float f32() {
        const std::uint32_t v = u32();
        float r;
        std::memcpy(&r, &v, 4);
        return r;
    }
    std::string text() {
        const std::uint64_t n = u64();
        if (n > kMaxString) bad("ARTIFACT-LENGTH", "string exceeds V0 limit");
        return raw(n);
    }
    std::string raw(std::uint64_t n) {
        need(n);
        std::string v = bytes_.substr(offset_, static_cast<std::size_t>(n));
        offset_ += static_cast<std::size_t>(n);
        return v;
    }
    std::uint32_t count(std::uint64_t limit, const char* what) {
        const std::uint32_t n = u32();
        if (n > limit) bad("ARTIFACT-REGION", std::string(what) + " exceeds V0 limit");
        return n;
    }
    bool done() const { return offset_ == bytes_.size(); }

private:
    void need(std::uint64_t n) {
        if (n > bytes_.size() || offset_ > bytes_.size() - static_cast<std::size_t>(n))
            bad("ARTIFACT-TRUNCATED", "checked read exceeds artifact size");
    }
    const std::string& bytes_;
    std::size_t offset_ = 0;
};

class Writer {
public:
    void u8(std::uint8_t v) { out_.push_back(static_cast<char>(v)); }
    void u32(std::uint32_t v) {
        for (unsigned s = 0; s < 32; s += 8) u8(static_cast<std::uint8_t>(v >> s));
    }
    void u64(std::uint64_t v) {
        for (unsigned s = 0; s < 64; s += 8) u8(static_cast<std::uint8_t>(v >> s));
    }
    void i64(std::int64_t v) {
        std::uint64_t u;
        std::memcpy(&u, &v, 8);
        u64(u);
    }
    void f32(float v) {
        std::uint32_t u;
        std::memcpy(&u, &v, 4);
        u32(u);
    }
    void text(const std::string& s) {
        u64(s.size());
        out_ += s;
    }
    void raw(const std::string& s) { out_ += s; }
    std::string take() { return std::move(out_); }

private:
    std::string out_;
};

// ---- node types -------------------------------------------------------------------

// semantic::Type: kind u8, rank u32, element count u32, elements.
void readSemanticType(Reader& r, Node& n, unsigned depth = 0) {
    if (depth > 8) bad("ARTIFACT-REGION", "type nesting exceeds V0 limit");
    const std::uint8_t kind = r.u8();
    const std::uint32_t rank = r.u32();
    const std::uint32_t elements = r.count(16, "type arity");
    if (kind == kTypeTensor) {
        if (elements != 1 || rank < 1 || rank > 2) bad("ARTIFACT-REGION", "unsupported tensor type");
        const std::uint8_t element = r.u8();
        const std::uint32_t elementRank = r.u32();
        const std::uint32_t inner = r.count(16, "type arity");
        if (elementRank != 0 || inner != 0 || (element != kTypeI64 && element != kTypeF32))
            bad("ARTIFACT-REGION", "unsupported tensor element type");
        n.dtype = element == kTypeI64 ? DType::I64 : DType::F32;
        n.rank = rank;
    } else if (kind == kTypeI64 || kind == kTypeF32) {
        if (rank != 0 || elements != 0) bad("ARTIFACT-REGION", "scalar type has rank or elements");
        n.dtype = kind == kTypeI64 ? DType::I64 : DType::F32;
        n.rank = 0;
    } else {
        bad("ARTIFACT-REGION", "unsupported node type kind " + std::to_string(kind));
    }
}

void writeSemanticType(Writer& w, DType dtype, std::uint32_t rank) {
    if (dtype != DType::I64 && dtype != DType::F32) bad("ARTIFACT-REGION", "artifacts carry i64 and f32 values only");
    const std::uint8_t element = dtype == DType::I64 ? kTypeI64 : kTypeF32;
    if (rank == 0) {
        w.u8(element);
        w.u32(0);
        w.u32(0);
        return;
    }
    w.u8(kTypeTensor);
    w.u32(rank);
    w.u32(1);
    w.u8(element);
    w.u32(0);
    w.u32(0);
}

Type readArtifactType(Reader& r) {
    Type t;
    t.kind = r.u8();
    t.dtype = r.u8();
    t.rank = r.u32();
    const std::uint32_t n = r.u32();
    if (n > 64) bad("ARTIFACT-SIGNATURE", "rank exceeds V0 limit");
    for (std::uint32_t i = 0; i < n; ++i) {
        if (r.u8()) t.extents.emplace_back(r.u64());
        else t.extents.emplace_back(std::nullopt);
    }
    return t;
}

void writeArtifactType(Writer& w, const Type& t) {
    w.u8(t.kind);
    w.u8(t.dtype);
    w.u32(t.rank);
    w.u32(static_cast<std::uint32_t>(t.extents.size()));
    for (const auto& e : t.extents) {
        w.u8(e.has_value());
        if (e) w.u64(*e);
    }
}

// ArtifactType of a node (artifactType, NativeArtifacts.cpp:872-889).
Type typeOf(const Node& n) {
    Type t;
    t.dtype = n.dtype == DType::I64 ? 1 : 2;
    if (n.rank == 0) return t;
    t.kind = 2;
    t.rank = n.rank;
    for (std::uint32_t a = 0; a < n.rank; ++a) {
        if (n.extent[a] >= 0) t.extents.emplace_back(static_cast<std::uint64_t>(n.extent[a]));
        else t.extents.emplace_back(std::nullopt);
    }
    return t;
}

// ---- extension descriptors ----------------------------------------------------------

Recipe readRecipe(Reader& r) {
    Recipe rec;
    rec.inputCount = r.u32();
    rec.root = r.u32();
    const std::uint32_t n = r.u32();
    if (n > 256) bad("ARTIFACT-REGION", "extension recipe too large");
    for (std::uint32_t i = 0; i < n; ++i) {
        ScalarNode s;
        s.opcode = r.u8();
        s.left = r.u32();
        s.right = r.u32();
        s.input = r.u32();
        s.constant = r.f32();
        rec.nodes.push_back(s);
    }
    return rec;
}

void writeRecipe(Writer& w, const Recipe& rec) {
    w.u32(rec.inputCount);
    w.u32(rec.root);
    w.u32(static_cast<std::uint32_t>(rec.nodes.size()));
    for (const auto& s : rec.nodes) {
        w.u8(s.opcode);
        w.u32(s.left);
        w.u32(s.right);
        w.u32(s.input);
        w.f32(s.constant);
    }
}

// Field order of writeOperation / readOperation (NativeArtifacts.cpp:186-221).
Operation readOperation(Reader& r) {
    Operation op;
    op.extensionId = r.text();
    op.extensionVersion = r.text();
    op.name = r.text();
    op.semanticVersion = r.text();
    op.abiVersion = r.u32();
    op.arity = r.u32();
    op.minimumRank = r.u32();
    op.maximumRank = r.u32();
    op.resultLikeInput = r.u32();
    op.sameShape = r.u8() != 0;
    op.effect = r.u8();
    op.backends = r.u32();
    op.fusible = r.u8() != 0;
    op.forward = readRecipe(r);
    if (r.u8()) {
        Derivative d;
        d.differentiableInputs = r.u64();
        d.savedInputs = r.u64();
        d.savesOutput = r.u8() != 0;
        const std::uint32_t n = r.u32();
        if (n > 8) bad("ARTIFACT-REGION", "extension gradient count too large");
        for (std::uint32_t i = 0; i < n; ++i) d.gradients.push_back(readRecipe(r));
        op.derivative = std::move(d);
    }
    const std::string identity = r.text();
    const std::string digestText = r.text();
    if (auto invalid = validateOperation(op); !invalid.empty()) bad("ARTIFACT-REGION", invalid);
    if (identity != canonicalIdentity(op))
        bad("ARTIFACT-REGION", "canonical operation identity disagrees with descriptor fields");
    if (digestText != descriptorDigest(op)) bad("ARTIFACT-REGION", "extension descriptor digest mismatch");
    op.digest = engineDigest(op);
    return op;
}

void writeOperation(Writer& w, const Operation& op) {
    w.text(op.extensionId);
    w.text(op.extensionVersion);
    w.text(op.name);
    w.text(op.semanticVersion);
    w.u32(op.abiVersion);
    w.u32(op.arity);
    w.u32(op.minimumRank);
    w.u32(op.maximumRank);
    w.u32(op.resultLikeInput);
    w.u8(op.sameShape);
    w.u8(op.effect);
    w.u32(op.backends);
    w.u8(op.fusible);
    writeRecipe(w, op.forward);
    w.u8(op.derivative.has_value());
    if (op.derivative) {
        w.u64(op.derivative->differentiableInputs);
        w.u64(op.derivative->savedInputs);
        w.u8(op.derivative->savesOutput);
        w.u32(static_cast<std::uint32_t>(op.derivative->gradients.size()));
        for (const auto& g : op.derivative->gradients) writeRecipe(w, g);
    }
    w.text(canonicalIdentity(op));
    w.text(descriptorDigest(op));
}

// ---- regions ------------------------------------------------------------------------

std::vector<std::uint32_t> readIds(Reader& r) {
    const std::uint32_t n = r.count(kMaxItems, "collection");
    std::vector<std::uint32_t> ids;
    ids.reserve(n);
    for (std::uint32_t i = 0; i < n; ++i) {
        const std::uint64_t v = r.u64();
        if (v > std::numeric_limits<std::uint32_t>::max()) bad("ARTIFACT-REGION", "identifier overflow");
        ids.push_back(static_cast<std::uint32_t>(v));
    }
    return ids;
}

void writeIds(Writer& w, const std::vector<std::uint32_t>& ids) {
    w.u32(static_cast<std::uint32_t>(ids.size()));
    for (auto id : ids) w.u64(id);
}

// Engine ops keep their axis (reduction axis, broadcast axis, gradient
// operand) in the integer field, which none of them uses otherwise.
bool carriesAxis(Op op) { return static_cast<std::uint32_t>(op) >= THB_OP_SUM; }

// serializeRegion / deserializeRegion (NativeArtifacts.cpp:244-331). Checks,
// provenance, resources and view roots are read and dropped: this engine's
// verifier and kernels re-derive every bounds / overflow / divide check from
// the ops themselves.
Region readRegion(const std::string& bytes, bool allowEngineOps) {
    Reader r(bytes);
    Region region;
    region.function = r.u32();
    region.name = r.text();
    const std::uint32_t count = r.u32();
    if (count == 0 || count > kMaxItems) bad("ARTIFACT-REGION", "invalid node count");
    region.nodes.reserve(count);
    for (std::uint32_t k = 0; k < count; ++k) {
        Node n;
        n.id = r.u32();
        const std::uint8_t op = r.u8();
        const bool reference = op <= THB_OP_UNSUPPORTED;
        const bool engine = op >= THB_OP_SUM && op <= THB_OP_ZERO_LIKE;
        if (!reference && !(engine && allowEngineOps))
            bad("ARTIFACT-REGION", "unknown region op " + std::to_string(op));
        n.op = static_cast<Op>(op);
        readSemanticType(r, n);
        const std::uint32_t extents = r.count(64, "rank");
        if (extents != n.rank) bad("ARTIFACT-REGION", "shape rank disagrees with type");
        for (std::uint32_t a = 0; a < extents; ++a) n.extent[a] = r.u8() ? r.i64() : -1;
        n.dependencies = readIds(r);
        n.indices = readIds(r);
        if (r.u8()) n.integer = r.i64();
        if (r.u8()) n.floating = r.f32();
        if (r.u8()) n.extension = std::make_shared<Operation>(readOperation(r));
        const std::uint32_t checks = r.count(kMaxItems, "check count");
        for (std::uint32_t c = 0; c < checks; ++c) {
            r.u8();
            readIds(r);
            r.text();
            r.u32();
            r.u8();
        }
        r.u8();  // provenance
        const std::uint32_t resources = r.count(kMaxItems, "resource count");
        for (std::uint32_t i = 0; i < resources; ++i) r.u64();
        const std::uint32_t roots = r.count(kMaxItems, "view-root count");
        for (std::uint32_t i = 0; i < roots; ++i) r.u32();
        if (carriesAxis(n.op)) n.axis = static_cast<std::int32_t>(n.integer);
        region.nodes.push_back(std::move(n));
    }
    region.inputs = readIds(r);
    region.output = r.u32();
    Node outputType;
    readSemanticType(r, outputType);
    if (!r.done()) bad("ARTIFACT-REGION", "trailing region metadata");
    const auto errors = verifyRegion(region);
    if (!errors.empty()) bad("ARTIFACT-REGION", errors.front());
    const Node& out = region.at(region.output);
    if (out.dtype != outputType.dtype || out.rank != outputType.rank)
        bad("ARTIFACT-REGION", "output type disagrees with the output node");
    return region;
}

std::string writeRegion(const Region& region) {
    Writer w;
    w.u32(region.function);
    w.text(region.name);
    w.u32(static_cast<std::uint32_t>(region.nodes.size()));
    for (const auto& n : region.nodes) {
        w.u32(n.id);
        w.u8(static_cast<std::uint8_t>(n.op));
        writeSemanticType(w, n.dtype, n.rank);
        w.u32(n.rank);
        for (std::uint32_t a = 0; a < n.rank; ++a) {
            w.u8(n.extent[a] >= 0);
            if (n.extent[a] >= 0) w.i64(n.extent[a]);
        }
        writeIds(w, n.dependencies);
        writeIds(w, n.indices);
        const bool integer = n.op == Op::Integer || carriesAxis(n.op);
        w.u8(integer);
        if (integer) w.i64(carriesAxis(n.op) ? n.axis : n.integer);
        w.u8(n.op == Op::Float);
        if (n.op == Op::Float) w.f32(n.floating);
        w.u8(n.extension != nullptr);
        if (n.extension) writeOperation(w, *n.extension);
        w.u32(0);  // checks
        w.u8(0);   // provenance
        w.u32(0);  // resources
        w.u32(0);  // view roots
    }
    writeIds(w, region.inputs);
    w.u32(region.output);
    const Node& out = region.at(region.output);
    writeSemanticType(w, out.dtype, out.rank);
    return w.take();
}

// validateSignature (NativeArtifacts.cpp:386-421): the entry must describe
// the region's inputs and output.
bool compatible(const Type& entry, const Node& n) {
    const Type base = typeOf(n);
    if (entry.kind != base.kind || entry.dtype != base.dtype || entry.rank != base.rank ||
        entry.extents.size() != base.extents.size())
        return false;
    for (std::size_t a = 0; a < base.extents.size(); ++a)
        if (base.extents[a] && entry.extents[a] != base.extents[a]) return false;
    return true;
}

std::string validType(const Type& t) {
    if (t.dtype != 1 && t.dtype != 2) return "unsupported dtype";
    if (t.kind == 1) return t.rank != 0 || !t.extents.empty() ? "scalar has rank/extents" : "";
    if (t.kind == 2) return (t.rank != 1 && t.rank != 2) || t.extents.size() != t.rank ? "tensor rank/extents mismatch" : "";
    return "unknown value kind";
}

void validateSignature(const Manifest& m, const Region& region) {
    if (m.entryName.empty() || m.entryName != region.name)
        bad("ARTIFACT-ENTRY", "entry name does not match lowered region");
    if (m.parameters.size() != region.inputs.size()) bad("ARTIFACT-SIGNATURE", "parameter count mismatch");
    for (std::size_t i = 0; i < m.parameters.size(); ++i) {
        if (auto e = validType(m.parameters[i]); !e.empty()) bad("ARTIFACT-SIGNATURE", e);
        if (!compatible(m.parameters[i], region.at(region.inputs[i])))
            bad("ARTIFACT-SIGNATURE", "parameter type conflicts with region");
    }
    if (auto e = validType(m.result); !e.empty()) bad("ARTIFACT-SIGNATURE", e);
    if (!compatible(m.result, region.at(region.output)))
        bad("ARTIFACT-SIGNATURE", "result type conflicts with region");
}

std::string planDigest(const Region& region, PlanOptions options) {
    return digest(buildPlan(region, options).dump(region));
}

} // namespace

std::string digest(const std::string& bytes) {
    std::uint64_t h = 1469598103934665603ULL;
    for (unsigned char c : bytes) {
        h ^= c;
        h *= 1099511628211ULL;
    }
    std::ostringstream out;
    out << "fnv1a64:" << std::hex << std::setw(16) << std::setfill('0') << h;
    return out.str();
}

Artifact load(const std::string& bytes, bool acceptCpu) {
    Reader r(bytes);
    for (char expected : kMagic)
        if (r.u8() != static_cast<std::uint8_t>(expected)) bad("ARTIFACT-MAGIC", "missing THIRAN16 header");
    Artifact a;
    Manifest& m = a.manifest;
    m.formatVersion = r.u32();
    m.compilerAbiVersion = r.u32();
    m.runtimeAbiVersion = r.u32();
    m.backend = r.u8();
    m.payloadKind = r.u8();
    m.enableReuse = r.u8() != 0;
    m.enableFusion = r.u8() != 0;
    m.target = r.text();
    m.runtimeRequirement = r.text();
    m.entryName = r.text();
    const std::uint32_t parameters = r.u32();
    if (parameters > 64) bad("ARTIFACT-SIGNATURE", "too many parameters");
    for (std::uint32_t i = 0; i < parameters; ++i) m.parameters.push_back(readArtifactType(r));
    m.result = readArtifactType(r);
    m.planDigest = r.text();
    m.regionSize = r.u64();
    m.regionDigest = r.text();
    m.payloadSize = r.u64();
    m.payloadDigest = r.text();
    if (m.regionSize > kMaxRegion || m.payloadSize > kMaxPayload) bad("ARTIFACT-LENGTH", "payload exceeds V0 limit");
    const std::string regionBytes = r.raw(m.regionSize);
    a.payload = r.raw(m.payloadSize);
    if (!r.done()) bad("ARTIFACT-TRAILING-DATA", "bytes follow declared payload");

    // Manifest checks in the order of validateArtifact (NativeArtifacts.cpp:574-630).
    if (m.formatVersion != 0) bad("ARTIFACT-FORMAT-VERSION", "unsupported artifact format version");
    if (m.compilerAbiVersion != 1) bad("ARTIFACT-COMPILER-ABI", "unsupported compiler/artifact ABI");
    if (m.runtimeAbiVersion != 1) bad("ARTIFACT-RUNTIME-ABI", "unsupported native runtime ABI");
    const bool cpu = m.backend == kBackendCpu;
    if (cpu && !acceptCpu)
        bad("ARTIFACT-BACKEND", "CPU artifacts run on the reference's CPU runtime, not on this GPU engine");
    if (m.backend != kBackendGpu && !cpu) bad("ARTIFACT-BACKEND", "unsupported artifact backend");
    const bool engine = m.payloadKind == kPayloadB200 && !cpu;
    if (cpu ? m.payloadKind != kPayloadElf : (m.payloadKind != kPayloadPtx && !engine))
        bad("ARTIFACT-PAYLOAD-KIND", "payload kind/backend mismatch");
    if (!cpu && m.target != (engine ? kEngineTarget : kReferenceGpuTarget))
        bad("ARTIFACT-TARGET", "artifact target is incompatible with this runtime");
    if (m.runtimeRequirement != (cpu ? kReferenceCpuRuntime : engine ? kEngineRuntime : kReferenceGpuRuntime))
        bad("ARTIFACT-RUNTIME-REQUIREMENT", "artifact runtime requirement is unsupported");
    if (m.regionDigest != digest(regionBytes)) bad("ARTIFACT-REGION-INTEGRITY", "lowered-region size/digest mismatch");
    a.region = readRegion(regionBytes, engine);
    validateSignature(m, a.region);
    if (a.payload.empty()) bad("ARTIFACT-MISSING-PAYLOAD", "artifact payload is empty");
    if (m.payloadDigest != digest(a.payload)) bad("ARTIFACT-PAYLOAD-INTEGRITY", "payload digest mismatch");
    const PlanOptions options{m.enableReuse, m.enableFusion};
    try {
        buildPlan(a.region, options);
    } catch (const Failure&) {
        bad("ARTIFACT-PLAN", "persistent plan cannot be reconstructed");
    }
    if (engine) {
        // The reference's plan digest hashes its own plan text; only the
        // engine's artifacts carry a digest of this planner's plan.
        if (m.planDigest != planDigest(a.region, options))
            bad("ARTIFACT-PLAN-INTEGRITY", "physical plan identity mismatch");
        Reader p(a.payload);
        for (char expected : kEngineMagic)
            if (p.u8() != static_cast<std::uint8_t>(expected)) bad("ARTIFACT-MALFORMED-PAYLOAD", "missing engine payload header");
        if (p.u32() != 1) bad("ARTIFACT-MALFORMED-PAYLOAD", "unsupported engine payload version");
        const std::uint64_t n = p.u64();
        if (n > kMaxPayload) bad("ARTIFACT-LENGTH", "payload exceeds V0 limit");
        a.engineSource = p.raw(n);
        const std::uint64_t c = p.u64();
        if (c > kMaxPayload) bad("ARTIFACT-LENGTH", "payload exceeds V0 limit");
        a.engineCubin = p.raw(c);
        if (!p.done()) bad("ARTIFACT-MALFORMED-PAYLOAD", "trailing payload bytes");
        std::vector<GroupKernel> kernels;
        const Plan plan = buildPlan(a.region, options);
        if (generateSource(a.region, plan, kernels) != a.engineSource)
            bad("ARTIFACT-PAYLOAD-MISMATCH", "engine payload was generated from a different region or engine version");
        if (!kernels.empty() && a.engineCubin.empty()) bad("ARTIFACT-MISSING-PAYLOAD", "engine payload has no cubin");
    }
    return a;
}

std::string build(const Region& region, PlanOptions options) {
    const auto errors = verifyRegion(region);
    if (!errors.empty()) fail(Category::Validation, "ARTIFACT-INVALID-REGION", errors.front());
    for (const auto& n : region.nodes)
        if (n.dtype != DType::I64 && n.dtype != DType::F32)
            fail(Category::Validation, "ARTIFACT-INVALID-REGION", "artifacts carry i64 and f32 values only");
    const Plan plan = buildPlan(region, options);
    std::vector<GroupKernel> kernels;
    const std::string source = generateSource(region, plan, kernels);
    const std::string cubin = kernels.empty() ? std::string() : compileCubin(source);
    Writer payload;
    payload.raw(std::string(kEngineMagic, 8));
    payload.u32(1);
    payload.text(source);
    payload.text(cubin);
    const std::string payloadBytes = payload.take();
    const std::string regionBytes = writeRegion(region);

    Writer w;
    w.raw(std::string(kMagic, 8));
    w.u32(0);
    w.u32(1);
    w.u32(1);
    w.u8(kBackendGpu);
    w.u8(kPayloadB200);
    w.u8(options.enableReuse);
    w.u8(options.enableFusion);
    w.text(kEngineTarget);
    w.text(kEngineRuntime);
    w.text(region.name);
    w.u32(static_cast<std::uint32_t>(region.inputs.size()));
    for (auto id : region.inputs) writeArtifactType(w, typeOf(region.at(id)));
    writeArtifactType(w, typeOf(region.at(region.output)));
    w.text(digest(plan.dump(region)));
    w.u64(regionBytes.size());
    w.text(digest(regionBytes));
    w.u64(payloadBytes.size());
    w.text(digest(payloadBytes));
    w.raw(regionBytes);
    w.raw(payloadBytes);
    return w.take();
}

std::string inspect(const Artifact& a) {
    const Manifest& m = a.manifest;
    auto quote = [](const std::string& s) {
        std::string o = "\"";
        for (char c : s) {
            if (c == '"' || c == '\\') o += '\\';
            if (c == '\n') { o += "\\n"; continue; }
            o += c;
        }
        return o + "\"";
    };
    auto type = [](const Type& t) {
        std::ostringstream o;
        o << "{\"kind\":\"" << (t.kind == 2 ? "tensor" : "scalar") << "\",\"dtype\":\"" << (t.dtype == 1 ? "i64" : "f32")
          << "\",\"rank\":" << t.rank << ",\"extents\":[";
        for (std::size_t i = 0; i < t.extents.size(); ++i) {
            if (i) o << ",";
            if (t.extents[i]) o << *t.extents[i];
            else o << "null";
        }
        o << "]}";
        return o.str();
    };
    const PlanOptions options{m.enableReuse, m.enableFusion};
    const Plan plan = buildPlan(a.region, options);
    std::ostringstream o;
    o << "{\"format_version\":" << m.formatVersion << ",\"backend\":\"" << (m.backend == kBackendGpu ? "gpu" : "cpu")
      << "\",\"payload_kind\":\"" << (m.payloadKind == kPayloadB200 ? "b200-cubin" : m.payloadKind == kPayloadPtx ? "ptx" : "elf")
      << "\",\"target\":" << quote(m.target) << ",\"runtime_requirement\":" << quote(m.runtimeRequirement)
      << ",\"entry\":" << quote(m.entryName) << ",\"parameters\":[";
    for (std::size_t i = 0; i < m.parameters.size(); ++i) o << (i ? "," : "") << type(m.parameters[i]);
    o << "],\"result\":" << type(m.result) << ",\"enable_reuse\":" << (m.enableReuse ? "true" : "false")
      << ",\"enable_fusion\":" << (m.enableFusion ? "true" : "false") << ",\"plan_digest\":" << quote(m.planDigest)
      << ",\"region_size\":" << m.regionSize << ",\"region_digest\":" << quote(m.regionDigest)
      << ",\"payload_size\":" << m.payloadSize << ",\"payload_digest\":" << quote(m.payloadDigest)
      << ",\"nodes\":" << a.region.nodes.size() << ",\"fusion_groups\":" << plan.groups.size()
      << ",\"region\":" << quote(a.region.dump()) << ",\"plan\":" << quote(plan.dump(a.region)) << "}";
    return o.str();
}

} // namespace thb::artifact
