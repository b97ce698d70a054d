// `.thm` model bundles (see model.hpp).
#include "model.hpp"

#include <algorithm>
#include <iomanip>
#include <map>
#include <set>
#include <sstream>

namespace thb::model {
namespace {

constexpr char kMagic[8] = {'T', 'H', 'I', 'R', 'A', 'N', 'M', 'B'};
constexpr std::uint64_t kMaxBundle = 2ull << 30;
constexpr std::uint64_t kMaxEmbedded = 768ull << 20;
constexpr std::uint64_t kMaxItems = 1ull << 16;
constexpr std::uint64_t kMaxString = 1ull << 20;
constexpr std::uint64_t kMaxValue = 64ull << 20;

[[noreturn]] void bad(const std::string& code, const std::string& message) {
    fail(Category::Validation, code, message);
}

// persistence::BinaryReader with the "MODEL" error prefix
// (src/persistence/v0/Persistence.cpp:34-78).
class Reader {
public:
    Reader(const std::string& bytes, std::size_t begin, std::size_t end) : bytes_(bytes), offset_(begin), end_(end) {}
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
    std::string text() {
        const std::uint64_t n = u64();
        if (n > kMaxString) bad("MODEL-LENGTH", "string exceeds V0 limit");
        return raw(n, kMaxString);
    }
    std::string raw(std::uint64_t n, std::uint64_t limit) {
        if (n > limit) bad("MODEL-LENGTH", "byte payload exceeds V0 limit");
        need(n);
        std::string v = bytes_.substr(offset_, static_cast<std::size_t>(n));
        offset_ += static_cast<std::size_t>(n);
        return v;
    }
    std::size_t offset() const { return offset_; }
    bool done() const { return offset_ == end_; }

private:
    void need(std::uint64_t n) {
        if (n > end_ - offset_) bad("MODEL-TRUNCATED", "checked read exceeds file size");
    }
    const std::string& bytes_;
    std::size_t offset_, end_;
};

std::uint64_t fnv(const std::string& bytes, std::size_t begin, std::size_t end) {
    std::uint64_t h = 1469598103934665603ULL;
    for (std::size_t i = begin; i < end; ++i) {
        h ^= static_cast<unsigned char>(bytes[i]);
        h *= 1099511628211ULL;
    }
    return h;
}

std::string validStored(const StoredValue& v) {
    if (v.dtype != 1 && v.dtype != 2) return "unsupported stored dtype";
    const std::uint64_t width = v.dtype == 1 ? 8 : 4;
    if (v.kind == 1) return !v.shape.empty() ? "scalar stored value has a shape"
                          : v.bytes.size() != width ? "scalar stored value has an invalid byte length" : "";
    if (v.kind != 2) return "unknown stored value kind";
    if (v.shape.empty() || v.shape.size() > 2) return "stored tensor rank is outside V0";
    std::uint64_t count = 1;
    for (auto e : v.shape) {
        if (e && count > ~0ull / e) return "stored tensor size arithmetic failed";
        count *= e;
    }
    if (count > ~0ull / width || v.bytes.size() != count * width) return "stored tensor payload length disagrees with shape";
    return "";
}

// readStoredValue (Persistence.cpp:116-128).
StoredValue readStored(Reader& r) {
    StoredValue v;
    v.kind = r.u8();
    v.dtype = r.u8();
    const std::uint32_t rank = r.u32();
    if (rank > 64) bad("PERSISTENCE-RANK", "stored rank exceeds V0 limit");
    for (std::uint32_t a = 0; a < rank; ++a) v.shape.push_back(r.u64());
    v.bytes = r.raw(r.u64(), kMaxValue);
    if (auto e = validStored(v); !e.empty()) bad("PERSISTENCE-VALUE", e);
    return v;
}

void appendU32(std::string& s, std::uint32_t v) {
    for (unsigned k = 0; k < 32; k += 8) s.push_back(static_cast<char>(v >> k));
}
void appendU64(std::string& s, std::uint64_t v) {
    for (unsigned k = 0; k < 64; k += 8) s.push_back(static_cast<char>(v >> k));
}

// parameterDigest (Persistence.cpp:163-168): FNV-1a over the parameters as
// writeStoredParameter lays them out.
std::string parameterDigest(const std::vector<Parameter>& ps) {
    std::string w;
    appendU32(w, static_cast<std::uint32_t>(ps.size()));
    for (const auto& p : ps) {
        appendU64(w, p.id);
        appendU64(w, p.name.size());
        w += p.name;
        w.push_back(static_cast<char>(p.value.kind));
        w.push_back(static_cast<char>(p.value.dtype));
        appendU32(w, static_cast<std::uint32_t>(p.value.shape.size()));
        for (auto e : p.value.shape) appendU64(w, e);
        appendU64(w, p.value.bytes.size());
        w += p.value.bytes;
    }
    return artifact::digest(w);
}

artifact::Type readType(Reader& r) {
    artifact::Type t;
    t.kind = r.u8();
    t.dtype = r.u8();
    t.rank = r.u32();
    const std::uint32_t n = r.u32();
    if (n > 64) bad("MODEL-PUBLIC-ABI", "rank exceeds V0 limit");
    for (std::uint32_t i = 0; i < n; ++i) {
        if (r.u8()) t.extents.emplace_back(r.u64());
        else t.extents.emplace_back(std::nullopt);
    }
    return t;
}

bool sameType(const artifact::Type& a, const artifact::Type& b) {
    return a.kind == b.kind && a.dtype == b.dtype && a.rank == b.rank && a.extents == b.extents;
}

std::string validType(const artifact::Type& t) {
    if (t.dtype != 1 && t.dtype != 2) return "unsupported dtype";
    if (t.kind == 1) return t.rank || !t.extents.empty() ? "scalar has rank/extents" : "";
    if (t.kind == 2) return (t.rank != 1 && t.rank != 2) || t.extents.size() != t.rank ? "tensor rank/extents mismatch" : "";
    return "unknown value kind";
}

artifact::Type storedType(const StoredValue& v) {
    artifact::Type t;
    t.kind = v.kind;
    t.dtype = v.dtype;
    if (v.kind == 2) {
        t.rank = static_cast<std::uint32_t>(v.shape.size());
        for (auto e : v.shape) t.extents.emplace_back(e);
    }
    return t;
}

bool sameEntry(const artifact::Manifest& a, const artifact::Manifest& b) {
    if (a.entryName != b.entryName || a.parameters.size() != b.parameters.size() || !sameType(a.result, b.result))
        return false;
    for (std::size_t i = 0; i < a.parameters.size(); ++i)
        if (!sameType(a.parameters[i], b.parameters[i])) return false;
    return true;
}

// validateModelBundle (ModelBundle.cpp:242-326).
void validate(const Bundle& b, const std::vector<const artifact::Manifest*>& manifests,
              const std::vector<std::string>& artifactIdentities) {
    if (b.identity.empty() || b.entry.empty()) bad("MODEL-IDENTITY", "model/entry identity is empty");
    if (auto e = validType(b.result); !e.empty()) bad("MODEL-PUBLIC-ABI", e);
    for (const auto& t : b.publicInputs)
        if (auto e = validType(t); !e.empty()) bad("MODEL-PUBLIC-ABI", e);
    std::set<std::uint64_t> ids;
    std::set<std::string> names;
    for (const auto& p : b.parameters) {
        if (p.id == 0 || !ids.insert(p.id).second) bad("MODEL-DUPLICATE-PARAMETER", "duplicate/zero ParameterId");
        if (p.name.empty() || !names.insert(p.name).second)
            bad("MODEL-DUPLICATE-PARAMETER", "duplicate/empty parameter name");
        if (auto e = validStored(p.value); !e.empty()) bad("MODEL-PARAMETER-SCHEMA", e);
    }
    if (parameterDigest(b.parameters) != b.parameterDigest)
        bad("MODEL-PARAMETER-DIGEST", "frozen parameter digest mismatch");
    if (manifests.empty()) bad("MODEL-BACKEND-UNAVAILABLE", "bundle contains no native artifact");
    std::set<std::uint8_t> backends;
    const artifact::Manifest* common = nullptr;
    for (std::size_t i = 0; i < manifests.size(); ++i) {
        if (artifactIdentities[i] != b.identity)
            bad("MODEL-ARTIFACT-IDENTITY", "embedded artifact model identity mismatch");
        if (!backends.insert(manifests[i]->backend).second) bad("MODEL-DUPLICATE-BACKEND", "duplicate backend artifact");
        if (manifests[i]->entryName != b.entry) bad("MODEL-ARTIFACT-IDENTITY", "artifact entry identity mismatch");
        if (!common) common = manifests[i];
        else if (!sameEntry(*manifests[i], *common))
            bad("MODEL-ARTIFACT-SIGNATURE", "CPU/GPU artifact signatures disagree");
    }
    if (!sameType(common->result, b.result)) bad("MODEL-PUBLIC-ABI", "artifact result disagrees with public ABI");
    std::set<std::uint32_t> slots, publics;
    for (const auto& [pub, slot] : b.publicBindings) {
        if (pub >= b.publicInputs.size() || slot >= common->parameters.size())
            bad("MODEL-PUBLIC-BINDING", "public binding is out of range");
        if (!publics.insert(pub).second || !slots.insert(slot).second)
            bad("MODEL-DUPLICATE-BINDING", "duplicate public/artifact binding");
        if (!sameType(b.publicInputs[pub], common->parameters[slot]))
            bad("MODEL-PUBLIC-ABI", "public input ABI disagrees with artifact slot");
    }
    if (publics.size() != b.publicInputs.size()) bad("MODEL-MISSING-BINDING", "a public input is not bound");
    std::set<std::uint64_t> bound;
    for (const auto& [id, slot] : b.parameterBindings) {
        if (!ids.count(id)) bad("MODEL-UNEXPECTED-PARAMETER", "binding references unknown ParameterId");
        if (slot >= common->parameters.size()) bad("MODEL-PARAMETER-BINDING", "parameter binding is out of range");
        if (!bound.insert(id).second || !slots.insert(slot).second)
            bad("MODEL-DUPLICATE-BINDING", "duplicate parameter/artifact binding");
        const auto p = std::find_if(b.parameters.begin(), b.parameters.end(), [&](const Parameter& x) { return x.id == id; });
        if (!sameType(storedType(p->value), common->parameters[slot]))
            bad("MODEL-PARAMETER-ABI", "frozen parameter dtype/rank/shape disagrees with artifact slot");
    }
    if (bound.size() != ids.size()) bad("MODEL-MISSING-PARAMETER", "a frozen parameter is not bound");
    if (slots.size() != common->parameters.size()) bad("MODEL-MISSING-BINDING", "an artifact input slot is not bound");
}

} // namespace

Bundle load(const std::string& bytes, const std::string* expectedIdentity) {
    if (bytes.size() > kMaxBundle) bad("MODEL-LENGTH", "bundle exceeds V0 limit");
    Reader head(bytes, 0, bytes.size());
    for (char expected : kMagic)
        if (head.u8() != static_cast<std::uint8_t>(expected)) bad("MODEL-MAGIC", "missing THIRANMB header");
    if (head.u32() != 0) bad("MODEL-FORMAT-VERSION", "unsupported model bundle version");
    if (head.u32() != 1) bad("MODEL-RUNTIME-ABI", "unsupported model runtime ABI");
    const std::uint64_t size = head.u64();
    const std::uint64_t digest = head.u64();
    if (size > kMaxBundle) bad("MODEL-LENGTH", "byte payload exceeds V0 limit");
    const std::size_t begin = head.offset();
    head.raw(size, kMaxBundle);
    if (!head.done()) bad("MODEL-TRAILING-DATA", "bytes follow declared bundle payload");
    const std::size_t end = begin + static_cast<std::size_t>(size);
    if (fnv(bytes, begin, end) != digest) bad("MODEL-BUNDLE-INTEGRITY", "bundle payload digest mismatch");

    Reader r(bytes, begin, end);
    Bundle b;
    b.identity = r.text();
    if (expectedIdentity && b.identity != *expectedIdentity) bad("MODEL-IDENTITY", "unexpected model identity");
    b.entry = r.text();
    b.parameterDigest = r.text();
    const std::uint32_t params = r.u32();
    if (params > kMaxItems) bad("MODEL-LENGTH", "excessive parameter count");
    for (std::uint32_t i = 0; i < params; ++i) {
        Parameter p;
        p.id = r.u64();
        p.name = r.text();
        p.value = readStored(r);
        b.parameters.push_back(std::move(p));
    }
    const std::uint32_t publics = r.u32();
    if (publics > kMaxItems) bad("MODEL-LENGTH", "excessive public input count");
    for (std::uint32_t i = 0; i < publics; ++i) b.publicInputs.push_back(readType(r));
    b.result = readType(r);
    const std::uint32_t pb = r.u32();
    if (pb > kMaxItems) bad("MODEL-LENGTH", "excessive public binding count");
    for (std::uint32_t i = 0; i < pb; ++i) {
        const std::uint32_t pub = r.u32();
        b.publicBindings.emplace_back(pub, r.u32());
    }
    const std::uint32_t qb = r.u32();
    if (qb > kMaxItems) bad("MODEL-LENGTH", "excessive parameter binding count");
    for (std::uint32_t i = 0; i < qb; ++i) {
        const std::uint64_t id = r.u64();
        b.parameterBindings.emplace_back(id, r.u32());
    }
    const std::uint32_t artifacts = r.u32();
    if (artifacts == 0 || artifacts > 2) bad("MODEL-BACKEND-COUNT", "bundle requires one or two artifacts");
    std::vector<artifact::Artifact> loaded;
    std::vector<std::string> identities;
    for (std::uint32_t i = 0; i < artifacts; ++i) {
        identities.push_back(r.text());
        const std::uint8_t declared = r.u8();
        const std::string artifactBytes = r.raw(r.u64(), kMaxEmbedded);
        try {
            loaded.push_back(artifact::load(artifactBytes, true));
        } catch (const Failure& f) {
            bad("MODEL-EMBEDDED-ARTIFACT", f.code() + " " + f.message());
        }
        if (loaded.back().manifest.backend != declared)
            bad("MODEL-ARTIFACT-BACKEND", "embedded backend declaration mismatch");
    }
    if (!r.done()) bad("MODEL-TRAILING-DATA", "bytes follow model bundle state");
    std::vector<const artifact::Manifest*> manifests;
    for (const auto& a : loaded) manifests.push_back(&a.manifest);
    validate(b, manifests, identities);
    for (auto& a : loaded) {
        if (a.manifest.backend == artifact::kBackendGpu) b.gpu = std::move(a);
        else b.hasCpu = true;
    }
    return b;
}

std::vector<std::int64_t> slotSources(const Bundle& b) {
    if (!b.gpu) bad("MODEL-BACKEND-UNAVAILABLE", "GPU artifact is not present; no CPU fallback");
    std::vector<std::int64_t> sources(b.gpu->manifest.parameters.size(), 0);
    for (const auto& [pub, slot] : b.publicBindings) sources[slot] = pub;
    for (const auto& [id, slot] : b.parameterBindings) {
        const auto p = std::find_if(b.parameters.begin(), b.parameters.end(), [&](const Parameter& x) { return x.id == id; });
        sources[slot] = -1 - static_cast<std::int64_t>(p - b.parameters.begin());
    }
    return sources;
}

std::string inspect(const Bundle& b) {
    std::ostringstream o;
    auto quote = [](const std::string& s) {
        std::string q = "\"";
        for (char c : s) {
            if (c == '"' || c == '\\') q += '\\';
            q += c;
        }
        return q + "\"";
    };
    o << "{\"model_identity\":" << quote(b.identity) << ",\"inference_entry\":" << quote(b.entry)
      << ",\"parameter_digest\":" << quote(b.parameterDigest) << ",\"parameters\":[";
    for (std::size_t i = 0; i < b.parameters.size(); ++i) {
        const auto& p = b.parameters[i];
        o << (i ? "," : "") << "{\"id\":" << p.id << ",\"name\":" << quote(p.name) << ",\"dtype\":\""
          << (p.value.dtype == 1 ? "i64" : "f32") << "\",\"shape\":[";
        for (std::size_t a = 0; a < p.value.shape.size(); ++a) o << (a ? "," : "") << p.value.shape[a];
        o << "],\"bytes\":" << p.value.bytes.size() << "}";
    }
    auto type = [](const artifact::Type& t) {
        std::ostringstream s;
        s << "{\"kind\":\"" << (t.kind == 2 ? "tensor" : "scalar") << "\",\"dtype\":\"" << (t.dtype == 1 ? "i64" : "f32")
          << "\",\"rank\":" << t.rank << ",\"extents\":[";
        for (std::size_t i = 0; i < t.extents.size(); ++i) {
            if (i) s << ",";
            if (t.extents[i]) s << *t.extents[i];
            else s << "null";
        }
        s << "]}";
        return s.str();
    };
    o << "],\"public_abi\":[";
    for (std::size_t i = 0; i < b.publicInputs.size(); ++i) o << (i ? "," : "") << type(b.publicInputs[i]);
    o << "],\"result\":" << type(b.result) << ",\"backend_gpu\":" << (b.gpu ? "true" : "false")
      << ",\"backend_cpu\":" << (b.hasCpu ? "true" : "false");
    if (b.gpu)
        o << ",\"gpu_payload_kind\":\"" << (b.gpu->manifest.payloadKind == artifact::kPayloadB200 ? "b200-cubin" : "ptx")
          << "\",\"gpu_payload_digest\":" << quote(b.gpu->manifest.payloadDigest);
    o << "}";
    return o.str();
}

} // namespace thb::model
