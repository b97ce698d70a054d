// CUDA source generation + NVRTC compilation for elementwise fusion groups.
#include "codegen.hpp"

#include <cuda_runtime.h>
#include <nvrtc.h>

#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <iomanip>
#include <mutex>
#include <set>
#include <sstream>
#include <sys/stat.h>
#include <unistd.h>

namespace thb {

struct Module {
    int device = -1;
    cudaLibrary_t library = nullptr;
    ~Module() {
        if (library) {
            int previous = 0;
            if (cudaGetDevice(&previous) == cudaSuccess) {
                cudaSetDevice(device);
                cudaLibraryUnload(library);
                cudaSetDevice(previous);
            }
        }
    }
};

std::uint64_t fnv1a(const std::string& text) {
    std::uint64_t h = 1469598103934665603ULL;
    for (unsigned char c : text) { h ^= c; h *= 1099511628211ULL; }
    return h;
}

namespace {

// Fixed text shared by every generated module: integer typedefs, streaming
// 128-bit loads/stores, and checked i64 arithmetic. The loads carry no L2
// prefetch-size hint: `.L2::256B` measured ~4 % slower on back-to-back
// launches of the 8192^2 i64 region on B200. The i64 overflow tests
// are the standard sign tests (two's complement add/sub) and a high-word test
// for multiply; they match the reference's checked_add/sub/mul/neg semantics
// (src/backend/v0/NativeCpu.cpp:116-132): the operation fails exactly when the
// mathematical result is outside [INT64_MIN, INT64_MAX].
const char* kPrelude = R"CUDA(
typedef unsigned long long thb_u64;
typedef long long thb_i64;
typedef unsigned int thb_u32;
struct __align__(16) thb_f32x4 { float v[4]; };
struct __align__(16) thb_i64x2 { thb_i64 v[2]; };

static __device__ __forceinline__ thb_f32x4 thb_load(const thb_f32x4* p) {
    thb_f32x4 r;
    asm("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
        : "=f"(r.v[0]), "=f"(r.v[1]), "=f"(r.v[2]), "=f"(r.v[3]) : "l"(p));
    return r;
}
static __device__ __forceinline__ thb_i64x2 thb_load(const thb_i64x2* p) {
    thb_i64x2 r;
    asm("ld.global.nc.L1::no_allocate.v2.s64 {%0,%1}, [%2];" : "=l"(r.v[0]), "=l"(r.v[1]) : "l"(p));
    return r;
}
static __device__ __forceinline__ void thb_store(thb_f32x4* p, const thb_f32x4& r) {
    asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};"
                 :: "l"(p), "f"(r.v[0]), "f"(r.v[1]), "f"(r.v[2]), "f"(r.v[3]) : "memory");
}
static __device__ __forceinline__ void thb_store(thb_i64x2* p, const thb_i64x2& r) {
    asm volatile("st.global.cs.v2.s64 [%0], {%1,%2};" :: "l"(p), "l"(r.v[0]), "l"(r.v[1]) : "memory");
}
static __device__ __forceinline__ thb_i64 thb_add(thb_i64 a, thb_i64 b, thb_u32& f) {
    const thb_i64 r = (thb_i64)((thb_u64)a + (thb_u64)b);
    f |= (thb_u32)(((r ^ a) & (r ^ b)) < 0);
    return r;
}
static __device__ __forceinline__ thb_i64 thb_sub(thb_i64 a, thb_i64 b, thb_u32& f) {
    const thb_i64 r = (thb_i64)((thb_u64)a - (thb_u64)b);
    f |= (thb_u32)(((a ^ b) & (r ^ a)) < 0);
    return r;
}
static __device__ __forceinline__ thb_i64 thb_mul(thb_i64 a, thb_i64 b, thb_u32& f) {
    const thb_i64 lo = (thb_i64)((thb_u64)a * (thb_u64)b);
    const thb_i64 hi = __mul64hi(a, b);
    f |= (thb_u32)(hi != (lo >> 63));
    return lo;
}
static __device__ __forceinline__ thb_i64 thb_neg(thb_i64 a, thb_u32& f) {
    f |= (thb_u32)(a == (thb_i64)0x8000000000000000ULL);
    return (thb_i64)(0ULL - (thb_u64)a);
}
static __device__ __forceinline__ float thb_div(float a, float b, thb_u32& f) {
    f |= (b == 0.0f) ? 2u : 0u;
    return __fdiv_rn(a, b);
}
static __device__ __forceinline__ float thb_relu(float a) {
    return (a > 0.0f || a != a) ? a : 0.0f;
}
// Bulk (TMA engine, non-tensor) copies between global and shared memory.
static __device__ __forceinline__ unsigned thb_smem_addr(const void* p) {
    unsigned long long a;
    asm("cvta.to.shared.u64 %0, %1;" : "=l"(a) : "l"(p));
    return (unsigned)a;
}
static __device__ __forceinline__ void thb_bulk_load(void* dst, const void* src, unsigned bytes, unsigned long long* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(thb_smem_addr(dst)), "l"(src), "r"(bytes), "r"(thb_smem_addr(bar)) : "memory");
}
static __device__ __forceinline__ void thb_bulk_store(void* dst, const void* src, unsigned bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
                 :: "l"(dst), "r"(thb_smem_addr(src)), "r"(bytes) : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// True once the mbarrier phase of this parity completed; false after `limit`
// polls (2^26 by default; the caller reports GPU-KERNEL-TIMEOUT). The drain
// after a timeout polls 2^30 times (GPU-KERNEL-DRAIN-TIMEOUT when that runs
// out too).
static __device__ __forceinline__ bool thb_wait_parity(unsigned long long* bar, unsigned parity,
                                                       unsigned limit = 1u << 26) {
    for (unsigned spin = 0; spin < limit; ++spin) {
        unsigned done;
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
                     " selp.u32 %0, 1, 0, p;\n}\n" : "=r"(done) : "r"(thb_smem_addr(bar)), "r"(parity) : "memory");
        if (done) return true;
    }
    return false;
}
)CUDA";

std::string floatLiteral(float value) {
    std::uint32_t bits = 0;
    std::memcpy(&bits, &value, sizeof bits);
    std::ostringstream out;
    out << "__int_as_float(0x" << std::hex << std::setw(8) << std::setfill('0') << bits << ")";
    return out.str();
}

// Emits `thb_g<id>_body`, one scalar function of the group inputs that
// evaluates the group's nodes in region order, each f32 operation rounded
// separately (the build uses -fmad=false, and the explicit _rn intrinsics
// keep every add/sub/mul/div an IEEE round-to-nearest operation).
void emitBody(std::ostringstream& out, const Region& region, const FusionGroup& group) {
    const bool f32 = group.dtype == DType::F32;
    const char* type = f32 ? "float" : "thb_i64";
    std::map<std::uint32_t, std::string> names;
    out << "static __device__ __forceinline__ " << type << " thb_g" << group.id << "_body(";
    for (std::size_t i = 0; i < group.inputs.size(); ++i) {
        out << (i ? ", " : "") << type << " a" << i;
        names[group.inputs[i]] = "a" + std::to_string(i);
    }
    for (std::size_t i = 0; i < group.scalars.size(); ++i) {
        out << ", " << type << " s" << i;
        names[group.scalars[i]] = "s" + std::to_string(i);
    }
    out << ", thb_u32& flag) {\n";
    // Tensor operands and runtime scalars are parameters; Float / Integer
    // literals become exact constants in the generated source.
    auto operand = [&](std::uint32_t id) {
        const std::uint32_t c = region.canonical(id);
        const Node& n = region.at(c);
        if (n.op == Op::Float && !names.count(c)) return floatLiteral(n.floating);
        if (n.op == Op::Integer && !names.count(c)) {
            std::ostringstream lit;
            lit << "(thb_i64)" << static_cast<unsigned long long>(n.integer) << "ULL";
            return lit.str();
        }
        return names.at(c);
    };
    for (auto id : group.nodes) {
        const Node& n = region.at(id);
        const std::string v = "v" + std::to_string(id);
        if (n.op == Op::Extension || n.op == Op::ExtensionGradient) {
            // A gradient recipe reads (primals..., result, cotangent), which
            // are exactly the node's dependencies in order.
            const Recipe& recipe =
                n.op == Op::Extension ? n.extension->forward : n.extension->derivative->gradients.at(n.axis);
            const std::string prefix = "e" + std::to_string(id) + "_";
            for (std::size_t r = 0; r < recipe.nodes.size(); ++r) {
                const ScalarNode& s = recipe.nodes[r];
                out << "    const float " << prefix << r << " = ";
                auto ref = [&](std::uint32_t k) { return prefix + std::to_string(k); };
                switch (s.opcode) {
                case THB_SCALAR_INPUT: out << operand(n.dependencies.at(s.input)); break;
                case THB_SCALAR_CONSTANT_F32: out << floatLiteral(s.constant); break;
                case THB_SCALAR_ADD: out << "__fadd_rn(" << ref(s.left) << ", " << ref(s.right) << ")"; break;
                case THB_SCALAR_SUBTRACT: out << "__fsub_rn(" << ref(s.left) << ", " << ref(s.right) << ")"; break;
                case THB_SCALAR_MULTIPLY: out << "__fmul_rn(" << ref(s.left) << ", " << ref(s.right) << ")"; break;
                case THB_SCALAR_DIVIDE: out << "thb_div(" << ref(s.left) << ", " << ref(s.right) << ", flag)"; break;
                case THB_SCALAR_NEGATE: out << "-" << ref(s.left); break;
                }
                out << ";\n";
            }
            out << "    const float " << v << " = " << prefix << recipe.root << ";\n";
        } else {
            out << "    const " << type << " " << v << " = ";
            const std::string a = operand(n.dependencies.at(0));
            if (f32) {
                switch (n.op) {
                case Op::Negate: out << "-" << a; break;
                case Op::Relu: out << "thb_relu(" << a << ")"; break;
                case Op::Add: out << "__fadd_rn(" << a << ", " << operand(n.dependencies.at(1)) << ")"; break;
                case Op::Subtract: out << "__fsub_rn(" << a << ", " << operand(n.dependencies.at(1)) << ")"; break;
                case Op::ElementMultiply: out << "__fmul_rn(" << a << ", " << operand(n.dependencies.at(1)) << ")"; break;
                default: fail(Category::Unsupported, "GPU-UNSUPPORTED-OP", "non-elementwise node in elementwise group");
                }
            } else {
                switch (n.op) {
                case Op::Negate: out << "thb_neg(" << a << ", flag)"; break;
                case Op::Add: out << "thb_add(" << a << ", " << operand(n.dependencies.at(1)) << ", flag)"; break;
                case Op::Subtract: out << "thb_sub(" << a << ", " << operand(n.dependencies.at(1)) << ", flag)"; break;
                case Op::ElementMultiply: out << "thb_mul(" << a << ", " << operand(n.dependencies.at(1)) << ", flag)"; break;
                default: fail(Category::Unsupported, "GPU-UNSUPPORTED-OP", "non-elementwise node in i64 group");
                }
            }
            out << ";\n";
        }
        names[id] = v;
    }
    out << "    return v" << group.output << ";\n}\n";
}

// Emits the two entry points of one group. The vector kernel requires every
// pointer 16-byte aligned; it streams 128-bit packets in a grid-stride loop,
// kUnroll packets per input in flight per thread, then block 0 finishes the
// n % lanes tail. The scalar kernel is the fallback for unaligned pointers.
void emitKernels(std::ostringstream& out, const FusionGroup& group, const std::string& vectorName,
                 const std::string& scalarName, const std::string& bulkName) {
    const bool f32 = group.dtype == DType::F32;
    const char* type = f32 ? "float" : "thb_i64";
    const char* packet = f32 ? "thb_f32x4" : "thb_i64x2";
    const unsigned lanes = f32 ? 4 : 2;
    const std::size_t k = group.inputs.size();
    auto params = [&]() {
        std::ostringstream p;
        p << type << "* __restrict__ out";
        for (std::size_t i = 0; i < k; ++i) p << ", const " << type << "* __restrict__ in" << i;
        for (std::size_t i = 0; i < group.scalars.size(); ++i) p << ", " << type << " s" << i;
        p << ", thb_u64 n, thb_u32* __restrict__ err";
        return p.str();
    };
    // Runtime scalars are passed through to every body call.
    std::string scalarArgs;
    for (std::size_t i = 0; i < group.scalars.size(); ++i) scalarArgs += "s" + std::to_string(i) + ", ";
    const std::string body = "thb_g" + std::to_string(group.id) + "_body";

    out << "extern \"C\" __global__ void __launch_bounds__(" << kBlock << ") " << vectorName << "(" << params() << ") {\n"
        << "    thb_u32 flag = 0;\n"
        << "    const thb_u64 packets = n / " << lanes << ";\n"
        << "    const thb_u64 stride = (thb_u64)gridDim.x * blockDim.x;\n"
        << "    thb_u64 i = (thb_u64)blockIdx.x * blockDim.x + threadIdx.x;\n"
        << "    " << packet << "* o = (" << packet << "*)out;\n";
    for (std::size_t j = 0; j < k; ++j)
        out << "    const " << packet << "* p" << j << " = (const " << packet << "*)in" << j << ";\n";
    // Main loop: kUnroll packets per input in flight.
    out << "    for (; i + " << (kUnroll - 1) << " * stride < packets; i += " << kUnroll << " * stride) {\n";
    for (std::size_t j = 0; j < k; ++j) out << "        " << packet << " x" << j << "[" << kUnroll << "];\n";
    out << "#pragma unroll\n        for (int u = 0; u < " << kUnroll << "; ++u) {\n";
    for (std::size_t j = 0; j < k; ++j) out << "            x" << j << "[u] = thb_load(p" << j << " + i + u * stride);\n";
    out << "        }\n#pragma unroll\n        for (int u = 0; u < " << kUnroll << "; ++u) {\n"
        << "            " << packet << " r;\n"
        << "#pragma unroll\n            for (int l = 0; l < " << lanes << "; ++l) r.v[l] = " << body << "(";
    for (std::size_t j = 0; j < k; ++j) out << "x" << j << "[u].v[l], ";
    out << scalarArgs << "flag);\n            thb_store(o + i + u * stride, r);\n        }\n    }\n";
    // Remainder packets.
    out << "    for (; i < packets; i += stride) {\n";
    for (std::size_t j = 0; j < k; ++j) out << "        const " << packet << " x" << j << " = thb_load(p" << j << " + i);\n";
    out << "        " << packet << " r;\n#pragma unroll\n        for (int l = 0; l < " << lanes << "; ++l) r.v[l] = "
        << body << "(";
    for (std::size_t j = 0; j < k; ++j) out << "x" << j << ".v[l], ";
    out << scalarArgs << "flag);\n        thb_store(o + i, r);\n    }\n";
    // Tail elements.
    out << "    if (blockIdx.x == 0) {\n"
        << "        const thb_u64 t = packets * " << lanes << " + threadIdx.x;\n"
        << "        if (t < n) out[t] = " << body << "(";
    for (std::size_t j = 0; j < k; ++j) out << "in" << j << "[t], ";
    out << scalarArgs << "flag);\n    }\n"
        << "    if (flag) atomicOr(err, flag);\n}\n";

    out << "extern \"C\" __global__ void __launch_bounds__(" << kBlock << ") " << scalarName << "(" << params() << ") {\n"
        << "    thb_u32 flag = 0;\n"
        << "    const thb_u64 stride = (thb_u64)gridDim.x * blockDim.x;\n"
        << "    for (thb_u64 i = (thb_u64)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)\n"
        << "        out[i] = " << body << "(";
    for (std::size_t j = 0; j < k; ++j) out << "in" << j << "[i], ";
    out << scalarArgs << "flag);\n    if (flag) atomicOr(err, flag);\n}\n";

    if (k == 0 || bulkName.empty()) return;
    // Bulk-copy pipeline: persistent CTAs take whole tiles (tile elements,
    // 16-byte multiple) t = blockIdx.x + j * gridDim.x. Thread 0 keeps a ring
    // of `stages` shared-memory stages full, each holding the tile of every
    // input, with cp.async.bulk loads completing on the stage's mbarrier; all
    // threads compute a tile from shared memory into one of two output tiles,
    // which thread 0 writes back with a bulk store. Elements past the last
    // whole tile take plain loads. Dynamic shared memory:
    // (stages * inputs + 2) * tile elements.
    out << "extern \"C\" __global__ void __launch_bounds__(" << kBlock << ") " << bulkName << "(" << params()
        << ", thb_u32 stages, thb_u32 tile) {\n"
        << "    extern __shared__ __align__(128) unsigned char thb_dyn[];\n"
        << "    __shared__ __align__(8) unsigned long long thb_full[" << kBulkMaxStages << "];\n"
        << "    __shared__ int thb_abort;\n"
        << "    " << type << "* thb_stage = (" << type << "*)thb_dyn;\n"
        << "    " << type << "* thb_out = thb_stage + (thb_u64)stages * " << k << " * tile;\n"
        << "    thb_u32 flag = 0;\n"
        << "    const thb_u64 tiles = n / tile;\n"
        << "    const thb_u64 first = blockIdx.x, step = gridDim.x;\n"
        << "    const thb_u32 tileBytes = tile * (thb_u32)sizeof(" << type << ");\n"
        << "    // Tile t (global index) into stage s; stage s of local tile j is j % stages.\n"
        << "    auto issue = [&](thb_u64 t, thb_u32 s) {\n"
        << "        if (t >= tiles) return;\n"
        << "        asm volatile(\"mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\" :: \"r\"(thb_smem_addr(&thb_full[s])), "
           "\"r\"(" << k << "u * tileBytes) : \"memory\");\n";
    for (std::size_t j = 0; j < k; ++j)
        out << "        thb_bulk_load(thb_stage + ((thb_u64)s * " << k << " + " << j << ") * tile, in" << j
            << " + t * tile, tileBytes, &thb_full[s]);\n";
    out << "    };\n"
        << "    if (threadIdx.x == 0) {\n"
        << "        thb_abort = 0;\n"
        << "        for (thb_u32 s = 0; s < stages; ++s)\n"
        << "            asm volatile(\"mbarrier.init.shared::cta.b64 [%0], 1;\" :: \"r\"(thb_smem_addr(&thb_full[s])) : \"memory\");\n"
        << "        asm volatile(\"fence.mbarrier_init.release.cluster;\" ::: \"memory\");\n"
        << "        for (thb_u32 s = 0; s < stages; ++s) issue(first + s * step, s);\n"
        << "    }\n"
        << "    __syncthreads();\n"
        << "    thb_u32 st = 0, phase = 0, ob = 0;\n"
        << "    for (thb_u64 t = first; t < tiles; t += step) {\n"
        << "        if (threadIdx.x == 0) {\n"
        << "            if (!thb_wait_parity(&thb_full[st], phase)) {\n"
        << "                thb_abort = 1;\n"
        << "                // Loads still in flight land before the CTA exits (bounded).\n"
        << "                thb_u32 s = st, p = phase;\n"
        << "                for (thb_u32 q = 0; q < stages; ++q) {\n"
        << "                    if (t + q * step < tiles && !thb_wait_parity(&thb_full[s], p, 1u << 30)) thb_abort = 2;\n"
        << "                    if (++s == stages) { s = 0; p ^= 1u; }\n"
        << "                }\n"
        << "            }\n"
        << "            asm volatile(\"cp.async.bulk.wait_group.read 1;\" ::: \"memory\");  // output tile of two tiles ago was read\n"
        << "        }\n"
        << "        __syncthreads();\n"
        << "        if (thb_abort) break;\n";
    // (Stage pointers are thb_in<j>: s<j> names the group's runtime scalars.)
    for (std::size_t j = 0; j < k; ++j)
        out << "        const " << packet << "* thb_in" << j << " = (const " << packet << "*)(thb_stage + ((thb_u64)st * "
            << k << " + " << j << ") * tile);\n";
    out << "        " << packet << "* so = (" << packet << "*)(thb_out + (thb_u64)ob * tile);\n"
        << "        for (thb_u32 q = threadIdx.x; q < tile / " << lanes << "; q += blockDim.x) {\n";
    for (std::size_t j = 0; j < k; ++j)
        out << "            const " << packet << " x" << j << " = thb_in" << j << "[q];\n";
    out << "            " << packet << " r;\n#pragma unroll\n            for (int l = 0; l < " << lanes << "; ++l) r.v[l] = "
        << body << "(";
    for (std::size_t j = 0; j < k; ++j) out << "x" << j << ".v[l], ";
    out << scalarArgs << "flag);\n"
        << "            so[q] = r;\n"
        << "        }\n"
        << "        asm volatile(\"fence.proxy.async.shared::cta;\" ::: \"memory\");\n"
        << "        __syncthreads();\n"
        << "        if (threadIdx.x == 0) {\n"
        << "            thb_bulk_store(out + t * tile, so, tileBytes);\n"
        << "            issue(t + (thb_u64)stages * step, st);\n"
        << "        }\n"
        << "        ob ^= 1u;\n"
        << "        if (++st == stages) { st = 0; phase ^= 1u; }\n"
        << "    }\n"
        << "    if (threadIdx.x == 0) asm volatile(\"cp.async.bulk.wait_group 0;\" ::: \"memory\");\n"
        << "    if (thb_abort) {\n"
        << "        flag |= thb_abort == 2 ? 48u : 16u;\n"
        << "    } else {\n"
        << "        const thb_u64 stride = (thb_u64)gridDim.x * blockDim.x;\n"
        << "        for (thb_u64 i = tiles * tile + (thb_u64)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)\n"
        << "            out[i] = " << body << "(";
    for (std::size_t j = 0; j < k; ++j) out << "in" << j << "[i], ";
    out << scalarArgs << "flag);\n"
        << "    }\n"
        << "    if (flag) atomicOr(err, flag);\n}\n";
}

std::string cacheDirectory() {
    if (const char* d = std::getenv("THB_CACHE_DIR")) return d;
    if (const char* h = std::getenv("HOME")) return std::string(h) + "/.cache/thiran_b200";
    return "/tmp/thiran_b200_cache";
}

bool readFile(const std::string& path, std::string& data) {
    std::ifstream in(path, std::ios::binary);
    if (!in) return false;
    std::ostringstream s;
    s << in.rdbuf();
    data = s.str();
    return !data.empty();
}

void writeFileAtomically(const std::string& dir, const std::string& path, const std::string& data) {
    std::string partial;
    std::size_t pos = 0;
    while ((pos = dir.find('/', pos + 1)) != std::string::npos) {
        partial = dir.substr(0, pos);
        ::mkdir(partial.c_str(), 0755);
    }
    ::mkdir(dir.c_str(), 0755);
    const std::string tmp = path + ".tmp" + std::to_string(::getpid());
    {
        std::ofstream out(tmp, std::ios::binary);
        if (!out) return;
        out.write(data.data(), static_cast<std::streamsize>(data.size()));
        if (!out) return;
    }
    std::rename(tmp.c_str(), path.c_str());
}

std::string nvrtcCompile(const std::string& source) {
    nvrtcProgram program = nullptr;
    if (nvrtcCreateProgram(&program, source.c_str(), "thiran_region.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS)
        fail(Category::Runtime, "GPU-NVRTC", "nvrtcCreateProgram failed");
    const char* options[] = {"--gpu-architecture=sm_100a", "-fmad=false", "--std=c++17", "--ftz=false",
                             "--prec-div=true", "--prec-sqrt=true", "-lineinfo"};
    const nvrtcResult status = nvrtcCompileProgram(program, sizeof options / sizeof options[0], options);
    if (status != NVRTC_SUCCESS) {
        std::size_t logSize = 0;
        nvrtcGetProgramLogSize(program, &logSize);
        std::string log(logSize, '\0');
        if (logSize) nvrtcGetProgramLog(program, log.data());
        nvrtcDestroyProgram(&program);
        fail(Category::Runtime, "GPU-NVRTC", std::string(nvrtcGetErrorString(status)) + ": " + log);
    }
    std::size_t size = 0;
    nvrtcGetCUBINSize(program, &size);
    std::string cubin(size, '\0');
    nvrtcGetCUBIN(program, cubin.data());
    nvrtcDestroyProgram(&program);
    return cubin;
}

std::mutex cacheMutex;
std::map<std::pair<std::uint64_t, int>, std::weak_ptr<Module>> liveModules;

} // namespace

std::string compileCubin(const std::string& source) { return nvrtcCompile(source); }

std::string generateSource(const Region& region, const Plan& plan, std::vector<GroupKernel>& kernels) {
    std::ostringstream out;
    out << "// thiran_b200 generated kernels for region f" << region.function << " (" << region.name << ")\n"
        << "// fusion=" << (plan.options.enableFusion ? "on" : "off") << " groups=" << plan.groups.size() << "\n"
        << kPrelude;
    kernels.clear();
    for (const auto& group : plan.groups) {
        if (group.kind != GroupKind::Elementwise) continue;
        GroupKernel k;
        k.group = group.id;
        k.dtype = group.dtype;
        k.arity = group.inputs.size();
        const std::string stem = "thb_f" + std::to_string(region.function) + "_g" + std::to_string(group.id) + "_" +
                                 dtypeName(group.dtype);
        k.vectorName = stem + "_vec";
        k.scalarName = stem + "_scalar";
        if (k.arity > 0) k.bulkName = stem + "_bulk";
        out << "\n// group g" << group.id << ": " << group.nodes.size() << " node(s), " << k.arity << " input(s)\n";
        emitBody(out, region, group);
        emitKernels(out, group, k.vectorName, k.scalarName, k.bulkName);
        kernels.push_back(k);
    }
    return out.str();
}

std::shared_ptr<Module> compileAndLoad(const std::string& source, int device, std::vector<GroupKernel>& kernels,
                                       bool& jitted, bool& loaded, const std::string* prebuiltCubin) {
    jitted = false;
    loaded = false;
    const std::uint64_t digest = fnv1a(source);
    std::lock_guard<std::mutex> lock(cacheMutex);
    std::shared_ptr<Module> module = liveModules[{digest, device}].lock();
    if (!module && prebuiltCubin) {
        // An artifact's cubin of exactly this source: no NVRTC, no disk cache.
        module = std::make_shared<Module>();
        module->device = device;
        const cudaError_t e =
            cudaLibraryLoadData(&module->library, prebuiltCubin->data(), nullptr, nullptr, 0, nullptr, nullptr, 0);
        if (e != cudaSuccess)
            fail(Category::Runtime, "GPU-MODULE-LOAD", std::string("artifact cubin: ") + cudaGetErrorString(e));
        loaded = true;
        liveModules[{digest, device}] = module;
    }
    if (!module) {
        std::ostringstream name;
        name << std::hex << std::setw(16) << std::setfill('0') << digest;
        const std::string dir = cacheDirectory();
        const std::string path = dir + "/" + name.str() + ".sm100a.cubin";
        std::string cubin;
        if (!readFile(path, cubin)) {
            cubin = nvrtcCompile(source);
            jitted = true;
            writeFileAtomically(dir, path, cubin);
        }
        module = std::make_shared<Module>();
        module->device = device;
        cudaError_t e = cudaLibraryLoadData(&module->library, cubin.data(), nullptr, nullptr, 0, nullptr, nullptr, 0);
        if (e != cudaSuccess && !jitted) {
            // A stale or foreign cache entry: rebuild once from source.
            cudaGetLastError();
            cubin = nvrtcCompile(source);
            jitted = true;
            writeFileAtomically(dir, path, cubin);
            e = cudaLibraryLoadData(&module->library, cubin.data(), nullptr, nullptr, 0, nullptr, nullptr, 0);
        }
        if (e != cudaSuccess)
            fail(Category::Runtime, "GPU-MODULE-LOAD", std::string("cudaLibraryLoadData: ") + cudaGetErrorString(e));
        loaded = true;
        liveModules[{digest, device}] = module;
    }
    for (auto& k : kernels) {
        cudaKernel_t v = nullptr, s = nullptr;
        if (cudaLibraryGetKernel(&v, module->library, k.vectorName.c_str()) != cudaSuccess ||
            cudaLibraryGetKernel(&s, module->library, k.scalarName.c_str()) != cudaSuccess)
            fail(Category::Runtime, "GPU-MODULE-LOAD", "generated kernel missing from module: " + k.vectorName);
        k.vectorKernel = reinterpret_cast<void*>(v);
        k.scalarKernel = reinterpret_cast<void*>(s);
        cudaKernel_t bulk = nullptr;
        if (!k.bulkName.empty() && cudaLibraryGetKernel(&bulk, module->library, k.bulkName.c_str()) != cudaSuccess) {
            bulk = nullptr;  // a module built without the bulk entry: the vector kernel serves
            (void)cudaGetLastError();
        }
        k.bulkKernel = reinterpret_cast<void*>(bulk);
        // Resident CTAs per SM, which sizes the launch to one full wave.
        int vr = 0, sr = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&vr, reinterpret_cast<const void*>(v), kBlock, 0) != cudaSuccess)
            vr = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&sr, reinterpret_cast<const void*>(s), kBlock, 0) != cudaSuccess)
            sr = 0;
        (void)cudaGetLastError();
        k.vectorResident = vr > 0 ? static_cast<unsigned>(vr) : 4u;
        k.scalarResident = sr > 0 ? static_cast<unsigned>(sr) : 4u;
    }
    return module;
}

} // namespace thb
