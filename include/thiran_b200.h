/*
 * thiran_b200.h — C ABI of the B200-native execution engine for Thiran's
 * TensorRegion hot path.
 *
 * Every entry point is extern "C", takes plain pointers and sizes, and
 * returns one of the THB_STATUS_* codes below. Failures write a NUL-terminated
 * text into the caller's (failure, failure_cap) buffer; for a checked semantic
 * failure that text is exactly the failure id (for example
 * "TH-SPEC-I64-OVERFLOW"), for every other failure it is "CODE: message".
 * This is the convention of the reference's native CPU artifact entry
 * `thiran_v0_entry` (src/artifact/v0/NativeArtifacts.cpp:631-700).
 *
 * Nothing here ever falls back to a CPU implementation: when the CUDA driver
 * or device is missing the call fails with GPU-DRIVER-NOT-FOUND /
 * GPU-INVALID-DEVICE.
 */
#ifndef THIRAN_B200_H
#define THIRAN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define THB_ABI_VERSION 1u

/* Return codes. 0..4 keep the meaning of thiran_v0_entry's return values
 * (src/artifact/v0/NativeArtifacts.cpp:693-697). */
enum {
    THB_STATUS_OK = 0,
    THB_STATUS_ABI = 1,      /* arity / type / shape / layout / malformed region */
    THB_STATUS_SEMANTIC = 2, /* checked failure; the failure id is in the buffer */
    THB_STATUS_BACKEND = 3,  /* driver / device / launch failure */
    THB_STATUS_UNKNOWN = 4
};

/* Element dtypes. I64 and F32 use the artifact ABI codes
 * (src/artifact/v0/NativeArtifacts.cpp:130-134); BF16 is an engine addition
 * used only for tensor-core GEMM operands. */
enum { THB_DTYPE_I64 = 1, THB_DTYPE_F32 = 2, THB_DTYPE_BF16 = 3 };

/* Value kinds (include/artifact/v0/NativeArtifacts.hpp:22). */
enum { THB_KIND_SCALAR = 1, THB_KIND_TENSOR = 2 };

/* RegionOp, numbered exactly as include/backend/v0/TensorRegion.hpp:14-28. */
enum {
    THB_OP_INPUT = 0,
    THB_OP_INTEGER = 1,
    THB_OP_FLOAT = 2,
    THB_OP_TENSOR_LITERAL = 3,
    THB_OP_ALIAS = 4,
    THB_OP_COPY = 5,
    THB_OP_NEGATE = 6,
    THB_OP_ADD = 7,
    THB_OP_SUBTRACT = 8,
    THB_OP_ELEMENT_MULTIPLY = 9,
    THB_OP_EXTENSION = 10,
    THB_OP_INDEX = 11,
    THB_OP_UNSUPPORTED = 12,
    /* Engine additions. The reference executes these only in its Evaluator
     * (src/semantic/v0/Evaluator.cpp) and rejects them natively
     * (src/backend/v0/TensorRegion.cpp:424-431). */
    THB_OP_SUM = 32,     /* sum(A, axis): Evaluator.cpp:214-251; axis in node.axis */
    THB_OP_ROW_MAX = 33, /* max over the last axis */
    THB_OP_SOFTMAX = 34, /* softmax over the last axis (RegionPythonEmitter.cpp:293-294) */
    THB_OP_RELU = 35,    /* max(x, 0) (PythonExecutorEmitter.cpp:94) */
    /* Reverse-AD operations the reference emits into backward functions and
     * evaluates only in its Evaluator (src/autodiff/v0/Autodiff.cpp:195-294):
     *   EXTENSION_GRADIENT: deps = primal operands..., primal result, output
     *     cotangent; axis = operand index k; evaluates the descriptor's
     *     gradient recipe k elementwise (Autodiff.cpp:231-270);
     *   TRANSPOSE (Evaluator.cpp:200-213); MATMUL (Evaluator.cpp:125-154):
     *     i64 operands with checked multiply and add (TH-SPEC-I64-OVERFLOW);
     *     f32 operands by node.axis: THB_MATMUL_TENSOR computes bf16 x bf16
     *     -> f32 on the tensor cores (any K and N: operands are zero-padded
     *     to 16-byte rows), THB_MATMUL_EXACT the Evaluator's sequential,
     *     separately rounded f32 sums on the CUDA cores (bit-exact);
     *   BROADCAST_TO_SHAPE: deps = value, reference; axis (Evaluator.cpp:278-309);
     *   REDUCE_TO_SHAPE: deps = value, reference (Evaluator.cpp:258-277);
     *   ZERO_LIKE: deps = reference. */
    THB_OP_EXTENSION_GRADIENT = 36,
    THB_OP_TRANSPOSE = 37,
    THB_OP_MATMUL = 38,
    THB_OP_BROADCAST_TO_SHAPE = 39,
    THB_OP_REDUCE_TO_SHAPE = 40,
    THB_OP_ZERO_LIKE = 41
};

/* MatMul modes of f32 operands (node.axis of a THB_OP_MATMUL node). */
enum { THB_MATMUL_TENSOR = 0, THB_MATMUL_EXACT = 1 };

/* Scalar recipe opcodes (include/extension/v0/Extension.hpp:16-17). */
enum {
    THB_SCALAR_INPUT = 1,
    THB_SCALAR_CONSTANT_F32 = 2,
    THB_SCALAR_ADD = 3,
    THB_SCALAR_SUBTRACT = 4,
    THB_SCALAR_MULTIPLY = 5,
    THB_SCALAR_DIVIDE = 6,
    THB_SCALAR_NEGATE = 7
};

/* Operation effects and backend mask (include/extension/v0/Extension.hpp:31-32). */
enum { THB_EFFECT_PURE = 0, THB_EFFECT_MAY_TRAP = 1 };
enum { THB_BACKEND_REFERENCE = 1, THB_BACKEND_CPU = 2, THB_BACKEND_GPU = 4 };

/* Layout-compatible with ScalarNodeV0 / ScalarRecipeV0 / DerivativeV0 /
 * OperationDescriptorV0 (include/extension/v0/Extension.hpp:18-53), so the
 * descriptor an extension plugin returns from thiran_extension_v0() can be
 * passed here unchanged. C++ bool is one byte; uint8_t stands in for it. */
typedef struct thb_scalar_node {
    uint8_t opcode;
    uint32_t left;
    uint32_t right;
    uint32_t input;
    float constant;
} thb_scalar_node;

typedef struct thb_scalar_recipe {
    const thb_scalar_node* nodes;
    size_t node_count;
    uint32_t root;
    uint32_t input_count;
} thb_scalar_recipe;

typedef struct thb_derivative {
    uint64_t differentiable_inputs;
    uint64_t saved_inputs;
    uint8_t saves_output;
    const thb_scalar_recipe* gradients;
    size_t gradient_count;
} thb_derivative;

typedef struct thb_operation {
    const char* name;
    const char* semantic_version;
    uint32_t arity;
    uint32_t minimum_rank;
    uint32_t maximum_rank;
    uint32_t result_like_input;
    uint8_t same_shape;
    uint8_t effect;
    uint32_t backends;
    uint8_t fusible;
    thb_scalar_recipe forward;
    const thb_derivative* derivative;
} thb_operation;

/* One TensorRegion node (RegionNode, include/backend/v0/TensorRegion.hpp:30-47).
 * rank 0 is a scalar of `dtype`; rank 1..2 is a contiguous row-major tensor.
 * An extent of -1 is unknown until execution. */
typedef struct thb_region_node {
    uint32_t id;
    uint32_t op;
    uint32_t dtype;
    uint32_t rank;
    int64_t extent[2];
    const uint32_t* dependencies;
    uint32_t dependency_count;
    const uint32_t* indices;
    uint32_t index_count;
    int64_t integer;
    float floating;
    int32_t axis;
    const thb_operation* extension;
} thb_region_node;

/* TensorRegion (TensorRegion.hpp:49-57). */
typedef struct thb_region_desc {
    uint32_t function;
    const char* name;
    const thb_region_node* nodes;
    uint32_t node_count;
    const uint32_t* inputs;
    uint32_t input_count;
    uint32_t output;
} thb_region_desc;

/* PhysicalPlanOptions (include/backend/v0/PhysicalPlan.hpp:37-41). */
typedef struct thb_plan_options {
    uint32_t enable_reuse;
    uint32_t enable_fusion;
} thb_plan_options;

/* Argument record, layout-identical to ThiranAbiArg
 * (src/artifact/v0/NativeArtifacts.cpp:702-708). For tensors `data` is a host
 * pointer in thb_region_execute / thb_region_submit and a device pointer in
 * thb_region_launch. Bit 0 of `reserved` marks a view / non-contiguous /
 * offset tensor, which is rejected with GPU-UNSUPPORTED-LAYOUT
 * (src/backend/v0/NativeGpu.cpp:94-96). */
typedef struct thb_abi_arg {
    uint32_t kind;
    uint32_t dtype;
    uint32_t rank;
    uint32_t reserved;
    const uint64_t* shape;
    const void* data;
    uint64_t count;
} thb_abi_arg;

/* GpuExecutionEvidence (include/backend/v0/NativeGpu.hpp:52-87), same
 * fields in the same order. Under the persistent runtime moduleLoads and
 * driverJitLoads count cache misses, allocationCount counts pool misses. */
typedef struct thb_evidence {
    uint64_t allocation_count;
    uint64_t allocation_bytes_requested;
    uint64_t host_to_device_copies;
    uint64_t host_to_device_bytes;
    uint64_t device_to_host_copies;
    uint64_t device_to_host_bytes;
    uint64_t device_to_device_copies;
    uint64_t device_to_device_bytes;
    uint64_t module_loads;
    uint64_t driver_jit_loads;
    uint64_t input_storage_uploads;
    uint64_t result_downloads;
    uint64_t kernel_launches;
    uint64_t synchronizations;
    uint64_t submitted_operations;
    uint64_t pending_operations;
    uint64_t active_read_reservations;
    uint64_t active_write_reservations;
    uint64_t stream_submissions;
    uint64_t event_records;
    uint64_t observations;
    uint64_t dropped_drains;
    uint64_t released_reservations;
    uint64_t logical_tensor_values;
    uint64_t logical_intermediates;
    uint64_t materialized_intermediates;
    uint64_t physical_slots;
    uint64_t physical_temporary_slots;
    uint64_t reused_slot_assignments;
    uint64_t fusion_groups;
    uint64_t fused_kernel_groups;
    uint64_t planner_owned_allocations;
    uint64_t retained_planner_allocations;
} thb_evidence;

/* GpuDeviceInfo (include/backend/v0/NativeGpu.hpp:37-48). */
typedef struct thb_device_info {
    int32_t backend_built;
    int32_t driver_loaded;
    int32_t device_available;
    int32_t device_count;
    int32_t selected_device;
    int32_t driver_version;
    int32_t compute_major;
    int32_t compute_minor;
    int32_t sm_count;
    int32_t reserved;
    char name[256];
    char error_code[64];
} thb_device_info;

typedef struct thb_region thb_region;
typedef struct thb_pending thb_pending;

/* ---- backend identity (include/backend/v0/NativeGpu.hpp:96-102) ------ */

/* nativeGpuBackendBuilt() (NativeGpu.hpp:96). Always 1 for this library. */
int thb_backend_built(void);
/* ABI version of this header. */
uint32_t thb_abi_version(void);
/* probeNativeGpu(int) (NativeGpu.hpp:102). Never throws; fills `out`. */
int thb_probe(int device, thb_device_info* out);

/* ---- regions (include/backend/v0/NativeGpu.hpp:200-226) ------------- */

/* Verifies the region (TensorRegion.cpp:103-228 rules), builds the physical
 * plan (PhysicalPlan.cpp:366-482: fusion groups, slots), generates one CUDA
 * kernel per elementwise fusion group and compiles it for sm_100a through
 * NVRTC (cached by digest). Replaces buildPhysicalPlan + plannedPtx + the
 * per-call cuModuleLoadDataEx of submitNativeGpuAsync (NativeGpu.cpp:1524,
 * :590, :602). Failure: THB_STATUS_ABI with GPU-INVALID-REGION etc. */
int thb_region_compile(const thb_region_desc* region, thb_plan_options options, int device,
                       thb_region** out, char* failure, uint64_t failure_cap);
void thb_region_release(thb_region* region);

/* executeNativeGpu(region, inputs, device, options) (NativeGpu.hpp:219-222):
 * host inputs are uploaded, the plan runs on the region's stream, the result
 * (output_count elements of the output dtype) is downloaded and the call
 * synchronises. `evidence` may be NULL. */
int thb_region_execute(thb_region* region, const thb_abi_arg* args, uint64_t argc,
                       void* output, uint64_t output_count, thb_evidence* evidence,
                       char* failure, uint64_t failure_cap);

/* submitNativeGpuAsync (NativeGpu.hpp:200-203): preflight, upload and launch,
 * then return a pending handle without synchronising. The host input buffers
 * must stay unchanged until the handle is observed or released. */
int thb_region_submit(thb_region* region, const thb_abi_arg* args, uint64_t argc,
                      thb_pending** out, thb_evidence* evidence,
                      char* failure, uint64_t failure_cap);
/* PendingGpuExecution::state(): 0 pending, 1 complete. */
int thb_pending_state(const thb_pending* pending);
/* PendingGpuExecution::observe() (NativeGpu.hpp:122): waits (bounded by
 * `timeout_ms`, 0 = wait without limit), checks the error words, copies the
 * value out. May be called again; later calls return the same outcome. */
int thb_pending_observe(thb_pending* pending, void* output, uint64_t output_count,
                        uint64_t timeout_ms, thb_evidence* evidence,
                        char* failure, uint64_t failure_cap);
/* Dropping a PendingGpuExecution: an unobserved handle is drained and its
 * failure, if any, is queued for thb_take_unobserved_errors. */
void thb_pending_release(thb_pending* pending);
/* runtime::takeUnobservedAsyncErrors() (include/runtime/v0/Async.hpp:165):
 * writes the queued failure ids, newline separated, and clears the queue.
 * Returns the number of ids. */
uint64_t thb_take_unobserved_errors(char* buffer, uint64_t capacity);

/* Device-resident, stream-ordered launch: tensors in `args` and `output` are
 * device pointers on the region's device; nothing is copied and nothing
 * synchronises. Checked failures latch into the region's error words until
 * thb_region_check_errors reads and clears them. `stream` is a cudaStream_t
 * (NULL = legacy default stream). This is the hot path the benchmark times.
 * A scalar region output is written to a one-element device buffer. */
int thb_region_launch(thb_region* region, const thb_abi_arg* args, uint64_t argc,
                      void* output, uint64_t output_count, void* stream,
                      char* failure, uint64_t failure_cap);
/* Synchronises `stream`, reads and clears the latched error words; returns
 * THB_STATUS_SEMANTIC with the failure id of the first failing fusion group
 * in region order, else THB_STATUS_OK. */
int thb_region_check_errors(thb_region* region, void* stream, char* failure, uint64_t failure_cap);

/* emitNativeGpuPtx(region, options) (NativeGpu.hpp:101): the generated CUDA
 * source of all fusion groups (this engine's payload text). Writes up to
 * `capacity` bytes including the NUL; `needed` receives the full size. */
int thb_region_emit_source(const thb_region* region, char* buffer, uint64_t capacity, uint64_t* needed);
/* PhysicalPlan::dump() (include/backend/v0/PhysicalPlan.hpp:125). */
int thb_region_dump_plan(const thb_region* region, char* buffer, uint64_t capacity, uint64_t* needed);
/* Plan structure: number of fusion groups and how many of them fused >1 node. */
int thb_region_plan_counts(const thb_region* region, uint64_t* fusion_groups, uint64_t* fused_groups,
                           uint64_t* kernels);

/* Device-free planning, as emitNativeGpuPtx(region, options) is in the
 * reference (NativeGpu.hpp:101): verifies and plans the region without
 * touching the driver and writes `what` into `buffer`:
 *   THB_DESCRIBE_PLAN   region dump + physical plan dump,
 *   THB_DESCRIBE_SOURCE generated CUDA source,
 *   THB_DESCRIBE_CUBIN  compiles the source with NVRTC for sm_100a and writes
 *                       the cubin size in bytes as decimal text.
 * counts (optional, 3 entries): fusion groups, fused groups, kernel groups. */
enum { THB_DESCRIBE_PLAN = 0, THB_DESCRIBE_SOURCE = 1, THB_DESCRIBE_CUBIN = 2 };

/* ---- `.tha` artifacts (src/artifact/v0/NativeArtifacts.cpp) -------------
 * The reference's container ("THIRAN16" + little-endian manifest + serialized
 * TensorRegion + payload, NativeArtifacts.cpp:547-572) is read and written
 * byte-compatibly. Accepted: GPU artifacts with the reference's generated PTX
 * payload (payload kind 2; the region is verified and planned onto this
 * engine, the PTX is integrity-checked but never executed) and this engine's
 * own artifacts (payload kind 3, target "sm_100a", runtime requirement
 * "thiran-b200-runtime-abi=1;libcudart;sm_100a": the generated CUDA source
 * and its sm_100a cubin, so compiling one runs no NVRTC). CPU artifacts (ELF
 * payload) are refused with ARTIFACT-BACKEND. Failure ids follow
 * loadArtifactBytes / validateArtifact (NativeArtifacts.cpp:574-630,
 * 1100-1140): ARTIFACT-MAGIC, ARTIFACT-TRUNCATED, ARTIFACT-TRAILING-DATA,
 * ARTIFACT-FORMAT-VERSION, ARTIFACT-PAYLOAD-KIND, ARTIFACT-TARGET,
 * ARTIFACT-RUNTIME-REQUIREMENT, ARTIFACT-REGION-INTEGRITY, ARTIFACT-REGION,
 * ARTIFACT-SIGNATURE, ARTIFACT-PAYLOAD-INTEGRITY, ARTIFACT-PLAN-INTEGRITY,
 * ARTIFACT-PAYLOAD-MISMATCH, ... (status THB_STATUS_ABI). */
typedef struct thb_artifact thb_artifact;
/* loadArtifactBytes (NativeArtifacts.hpp:120): parse and validate; device-free. */
int thb_artifact_load(const void* bytes, uint64_t size, thb_artifact** out, char* failure, uint64_t failure_cap);
/* loadArtifact (NativeArtifacts.hpp:119). */
int thb_artifact_load_file(const char* path, thb_artifact** out, char* failure, uint64_t failure_cap);
void thb_artifact_release(thb_artifact* artifact);
/* inspectArtifact (NativeArtifacts.hpp:122) as JSON: manifest, region dump
 * and this engine's physical plan. */
int thb_artifact_inspect(const thb_artifact* artifact, char* buffer, uint64_t capacity, uint64_t* needed);
/* The compiled region of an artifact on `device`, used with
 * thb_region_execute / submit / launch like any compiled region
 * (executeArtifact / submitArtifactGpu, NativeArtifacts.hpp:125-136). */
int thb_artifact_compile(const thb_artifact* artifact, int device, thb_region** out, char* failure,
                         uint64_t failure_cap);
/* ---- software renderer (src/graphics/v0/Graphics.cpp, GraphicsGpu.cpp) --
 * renderGpu (include/graphics/v0/GraphicsGpu.hpp:76-86): positions [N][3] f32,
 * indices [T][3] i64, colors [N][4] f32 in [0, 1]; model / view / projection
 * 16 f32 row-major (column vectors, P*V*M); clear colour 4 f32 (NULL = 0).
 * Writes color [width*height][4] and depth [width*height] (host buffers) and
 * stats = {input triangles, post-clip triangles, shaded pixels, depth passes}
 * (RenderStatistics). Validation, transform and clipping run on the host as
 * the reference's shared prepareRender; rasterization runs on the GPU
 * bit-exactly with the reference's CPU rasterizer (f64 edge functions,
 * perspective-correct colour, strict-less depth test in submission order).
 * Failures: status 2 with the reference's TH019-* id. */
int thb_render(int device, const float* positions, uint64_t vertices, const int64_t* indices, uint64_t triangles,
               const float* colors, const float* model, const float* view, const float* projection, uint64_t width,
               uint64_t height, const float* clear, float* color, float* depth, uint64_t* stats,
               thb_evidence* evidence, char* failure, uint64_t failure_cap);

/* ---- `.thm` model bundles (src/model/v0/ModelBundle.cpp) ---------------
 * The reference's container ("THIRANMB", versions, FNV-1a 64 payload digest,
 * identity, entry, frozen parameters, public ABI, bindings, embedded
 * artifacts) is read byte-compatibly and validated with validateModelBundle's
 * MODEL-* ids (ModelBundle.cpp:242-326, 362-430). A compiled model uploads
 * its frozen parameters to HBM once and keeps them there; each
 * thb_model_execute uploads only the public inputs. (The reference's
 * submitModelGpu, ModelBundle.cpp:461-474, binds every parameter as a host
 * value and uploads it on every call.) Without an embedded GPU artifact
 * compilation fails with MODEL-BACKEND-UNAVAILABLE; there is no CPU
 * fallback. */
typedef struct thb_model thb_model;
typedef struct thb_model_session thb_model_session;
/* loadModelBundle(path, expectedModelIdentity) (ModelBundle.hpp:98-99);
 * `identity` may be NULL. */
int thb_model_load(const void* bytes, uint64_t size, const char* identity, thb_model** out, char* failure,
                   uint64_t failure_cap);
int thb_model_load_file(const char* path, const char* identity, thb_model** out, char* failure,
                        uint64_t failure_cap);
void thb_model_release(thb_model* model);
/* inspectModelBundle (ModelBundle.hpp:100) as JSON. */
int thb_model_inspect(const thb_model* model, char* buffer, uint64_t capacity, uint64_t* needed);
/* Compiles the embedded GPU artifact on `device` and uploads the frozen
 * parameters (evidence counts that upload). */
int thb_model_compile(const thb_model* model, int device, thb_model_session** out, thb_evidence* evidence,
                      char* failure, uint64_t failure_cap);
void thb_model_session_release(thb_model_session* session);
/* executeModel(bundle, Gpu, publicInputs) (ModelBundle.hpp:101-103): host
 * public inputs in bundle order (checked like validateRuntimeValue:
 * MODEL-PUBLIC-INPUT-COUNT / MODEL-PUBLIC-INPUT-ABI), host output; the
 * frozen parameters come from HBM. */
int thb_model_execute(thb_model_session* session, const thb_abi_arg* public_args, uint64_t argc, void* output,
                      uint64_t output_count, thb_evidence* evidence, char* failure, uint64_t failure_cap);

/* buildGpuAot (NativeArtifacts.hpp:117) for this engine: writes a payload
 * kind 3 artifact of `region` into `buffer` (device-free: NVRTC only).
 * `needed` receives the size; a NULL buffer only reports it. */
int thb_artifact_build(const thb_region_desc* region, thb_plan_options options, void* buffer, uint64_t capacity,
                       uint64_t* needed, char* failure, uint64_t failure_cap);

/* ---- tensor-core GEMM ----------------------------------------------------
 * Engine addition: the reference's only matmul is its Evaluator's sequential
 * f32 triple loop (src/semantic/v0/Evaluator.cpp:125-154), rejected by the
 * native extractor ("MatMul lowering deferred", TensorRegion.cpp:424).
 * C[M,N] = A[M,K] B[K,N], bf16 operands, f32 accumulation in tensor memory
 * (tcgen05). A is K-major (stored [M][K]) or MN-major (stored [K][M]); B is
 * K-major (stored [N][K]) or MN-major (stored [K][N]); leading dimensions in
 * elements, multiples of 8; operands 16-byte aligned. */
enum { THB_MAJOR_K = 0, THB_MAJOR_MN = 1 };
enum {
    THB_EPI_F32 = 0,       /* C f32  = acc */
    THB_EPI_BF16 = 1,      /* C bf16 = acc */
    THB_EPI_RELU_BF16 = 2, /* C bf16 = max(acc, 0) */
    THB_EPI_MASK_BF16 = 3  /* C bf16 = aux[i,j] > 0 ? acc : 0 (aux bf16 [M][N]) */
};
typedef struct thb_gemm_desc {
    uint64_t m, n, k;
    const void* a;
    uint32_t a_major;
    uint64_t lda;
    const void* b;
    uint32_t b_major;
    uint64_t ldb;
    void* c;
    uint64_t ldc;
    uint32_t epilogue;
    const void* aux;
    uint64_t ld_aux;
    void* c_f32_copy; /* optional f32 copy of a bf16 epilogue's values (ld = ldc) */
} thb_gemm_desc;

/* Stream-ordered launch on `device` (pointers are device memory there). A
 * bounded wait that expires inside the kernel latches GPU-KERNEL-TIMEOUT in
 * the device status word, read by thb_device_check_status. */
int thb_gemm_bf16(int device, const thb_gemm_desc* desc, void* stream, char* failure, uint64_t failure_cap);

/* Synchronises `stream`, reads and clears the device status word that
 * kernels outside a region (GEMM, MLP steps) latch. */
int thb_device_check_status(int device, void* stream, char* failure, uint64_t failure_cap);

/* ---- MLP training step -----------------------------------------------------
 * Replaces training::trainingStep (src/training/v0/Training.cpp:382-432) for
 * the two-layer MLP H = relu(X W1), Y = H W2, L = mean((Y - T)^2), whose
 * backward follows the reverse-AD rules of src/autodiff/v0/Autodiff.cpp
 * (matmul :216-227) and whose update is plain SGD (Training.cpp:368-371).
 * W1 is [in][hidden], W2 [hidden][out], f32 masters with bf16 GEMM copies.
 * `global_batch` is the batch summed over data-parallel ranks; dY is scaled
 * by 2 / (global_batch * out) so that summing rank gradients gives the
 * gradient of the global mean loss. All pointers are device memory. */
typedef struct thb_mlp thb_mlp;
enum {
    THB_MLP_W1 = 0, THB_MLP_W2 = 1, THB_MLP_DW1 = 2, THB_MLP_DW2 = 3,
    THB_MLP_Y = 4, THB_MLP_H = 5, THB_MLP_LOSS_SUM = 6,
    THB_MLP_B1 = 7, THB_MLP_B2 = 8, THB_MLP_DB1 = 9, THB_MLP_DB2 = 10
};
int thb_mlp_create(int device, uint64_t batch, uint64_t global_batch, uint64_t in, uint64_t hidden, uint64_t out,
                   thb_mlp** session, char* failure, uint64_t failure_cap);
void thb_mlp_release(thb_mlp* session);
/* Copies f32 W1, W2 (device) into the session and refreshes the bf16 copies. */
int thb_mlp_set_weights(thb_mlp* session, const float* w1, const float* w2, void* stream, char* failure,
                        uint64_t failure_cap);
/* Forward, loss and backward for x [batch][in], t [batch][out] (f32, 16-byte
 * aligned): fills Y, H, dW1, dW2 and the rank's loss sum. */
int thb_mlp_forward_backward(thb_mlp* session, const float* x, const float* t, void* stream, char* failure,
                             uint64_t failure_cap);
/* Optimizer update of every parameter (W1, W2 and, when enabled, b1, b2)
 * after any gradient all-reduce: p -= lr * g, or with momentum (thb_mlp_
 * set_momentum) v = mu * v + g; p -= lr * v (src/training/v0/Training.cpp:
 * 343-381, applyOptimizer). */
int thb_mlp_apply_sgd(thb_mlp* session, float lr, void* stream, char* failure, uint64_t failure_cap);
/* Enables the broadcast biases of the examples/mlp.th structure:
 * H = relu(X W1 + b1), Y = H W2 + b2, with b1 [hidden], b2 [out] copied from
 * device memory (both NULL: zeros). Their gradients THB_MLP_DB1 / DB2 are the
 * column sums of dH and dY (the reference's reduceToShape onto the bias,
 * Evaluator.cpp:258-277) and lie adjacent in memory (DB2 = DB1 + hidden), so
 * one all-reduce covers both. Re-setting resets their velocities. */
int thb_mlp_set_biases(thb_mlp* session, const float* b1, const float* b2, void* stream, char* failure,
                       uint64_t failure_cap);
/* Selects SGD (momentum 0) or SGD with momentum (0 < momentum < 1, the
 * reference's OPT05 / OPT06 bounds; otherwise status 2 with that id), and
 * zeroes every velocity (the reference initialises them ZeroLike). */
int thb_mlp_set_momentum(thb_mlp* session, float momentum, void* stream, char* failure, uint64_t failure_cap);
/* One full single-device training step (training::trainingStep,
 * src/training/v0/Training.cpp:382-432): forward, loss, backward and the
 * optimizer update. The weight updates run inside the weight-gradient GEMMs'
 * read-out, bit-identical to forward_backward + apply_sgd, so THB_MLP_DW1 /
 * DW2 are not written by this call (the bias gradients are). A session with
 * a bound gradient all-reduce is refused (GPU-MLP-ARGUMENT). */
int thb_mlp_step(thb_mlp* session, const float* x, const float* t, float lr, void* stream, char* failure,
                 uint64_t failure_cap);
/* Device pointer and element count of a session buffer (THB_MLP_*); Y, dW,
 * biases and their gradients are f32, H bf16, the loss sum one f64. Bias
 * buffers are NULL with 0 elements until thb_mlp_set_biases. */
int thb_mlp_buffer(thb_mlp* session, uint32_t which, void** device_pointer, uint64_t* elements);
/* Replaces a session buffer by caller-owned device memory of the same size
 * and type (for example a tensor a collective library reduces in place);
 * the caller keeps it alive while the session uses it. The previous
 * contents are not copied. */
int thb_mlp_bind(thb_mlp* session, uint32_t which, void* device_pointer);
/* Data-parallel gradient all-reduce fused into the weight-gradient GEMM
 * (THB_MLP_DW1 or THB_MLP_DW2) over NVLink. `peers[k]` is rank k's dW
 * buffer as mapped on this GPU (peer access or symmetric memory; peers[rank]
 * becomes the session's dW buffer) and `flag_peers[k]` rank k's
 * thb_mlp_reduction_flag_words() zeroed u32 signal words, for k < world <= 8.
 * Each finished dW tile is stored locally and announced to its owner rank,
 * whose reducer warps sum it over all ranks and write the total into every
 * rank's dW while later tiles still compute: with plain NVLink loads and
 * stores (summed in rank order) when `multicast` is NULL, or inside NVSwitch
 * (multimem.ld_reduce / multimem.st) through `multicast`, the NVLS multicast
 * address of the dW buffers. Waits on other ranks are bounded: on expiry the
 * status word gets bit 4 (thb_device_check_status) and the step's gradients
 * are incomplete. The caller synchronises the ranks after forward_backward
 * and before reading dW (apply_sgd); every rank binds the same way and runs
 * the same steps. NULL `peers` restores the local store: dW returns to the
 * session's own buffer, so the bound ones may be freed. Binding restarts the
 * step count the signal words are checked against, so they must be zero again
 * on every rank. */
int thb_mlp_bind_reduction(thb_mlp* session, uint32_t which, void* const* peers, void* multicast,
                           uint32_t* const* flag_peers, uint32_t rank, uint32_t world);
/* Gradient format of the fused all-reduce of `which` (THB_MLP_DW1 / DW2;
 * call after thb_mlp_bind_reduction, which resets it to THB_REDUCE_F32):
 *  - THB_REDUCE_F32: f32 tiles, the sum written to every rank (or, with the
 *    fused update, the new f32 parameters and bf16 copy written to every
 *    rank);
 *  - THB_REDUCE_BF16_SHARDED: each rank stores its tile as bf16 (the peers'
 *    dW buffers are then bf16 [rows][cols]); the tile's owner sums the
 *    ranks' tiles with f32 accumulation, applies the optimizer step to its
 *    own f32 parameters only and writes the bf16 copy to every rank. The f32
 *    parameters are sharded by tile owner (thb_mlp_gather_parameters
 *    assembles them); each element costs about 2 bytes of NVLink traffic per
 *    direction instead of 10. Needs thb_mlp_bind_update and
 *    thb_mlp_forward_backward_update. Engine addition: the reference has no
 *    multi-GPU training (src/distributed/PartitionPlanner.cpp:6-32). */
enum { THB_REDUCE_F32 = 0, THB_REDUCE_BF16_SHARDED = 1 };
int thb_mlp_set_reduction_format(thb_mlp* session, uint32_t which, uint32_t format);
/* With a THB_REDUCE_BF16_SHARDED reduction: copies every tile of weight
 * `which` (THB_MLP_W1 / W2) that this rank does not own from its owner's
 * f32 parameters (peer loads), so this rank holds them all. Every rank calls
 * it between steps, and no rank frees or rebinds its buffers until all have
 * finished (a barrier). */
int thb_mlp_gather_parameters(thb_mlp* session, uint32_t which, void* stream, char* failure, uint64_t failure_cap);
/* Signal words thb_mlp_bind_reduction needs for `which` (0 for an unknown
 * buffer or session). */
uint64_t thb_mlp_reduction_flag_words(thb_mlp* session, uint32_t which);
/* Lets the all-reduce of layer `which` (THB_MLP_W1 or THB_MLP_W2; bind its
 * reduction first) apply the optimizer step (applyOptimizer,
 * src/training/v0/Training.cpp:343-381):
 * - `param_peers[k]` is rank k's f32 parameter buffer as mapped on this GPU;
 * - `copy_peers[k]` is rank k's bf16 copy of it (16-byte aligned);
 * - param_peers[rank] and copy_peers[rank] become the session's buffers.
 *   Copy the weights in afterwards with thb_mlp_set_weights.
 * - With a multicast reduction, `param_multicast` and `copy_multicast` are
 *   their NVLS multicast addresses; otherwise both are NULL.
 * - NULL `param_peers` removes the binding, and so does rebinding the
 *   reduction. W and bf16 W then return to the session's own buffers, and the
 *   caller copies the weights in again with thb_mlp_set_weights. */
int thb_mlp_bind_update(thb_mlp* session, uint32_t which, float* const* param_peers, void* param_multicast,
                        void* const* copy_peers, void* copy_multicast);
/* thb_mlp_forward_backward with the weight updates done inside the
 * all-reduce (both layers bound with thb_mlp_bind_update, else status 1 with
 * GPU-MLP-ARGUMENT):
 * - The owner rank of each gradient tile applies SGD / momentum to the
 *   summed tile.
 * - It writes the new parameters and their bf16 copy to every rank.
 * - Results are bit-identical to forward_backward + apply_sgd in peer mode.
 * - dW is not written back to the ranks.
 * - Velocities of a tile live on its owner only.
 * After the ranks synchronise, thb_mlp_apply_sgd updates only the biases. */
int thb_mlp_forward_backward_update(thb_mlp* session, const float* x, const float* t, float lr, void* stream,
                                    char* failure, uint64_t failure_cap);
/* CUDA-event timing of the session's GEMM launches, recorded on the stream
 * they are launched on (up to 512 launches between reads). */
int thb_mlp_enable_timing(thb_mlp* session, int enabled);
/* Waits for the recorded events and returns the summed GEMM device time (ms)
 * and launch count since the previous read, then resets them. */
int thb_mlp_read_timing(thb_mlp* session, double* gemm_ms, uint64_t* gemm_launches);
int thb_region_describe(const thb_region_desc* region, thb_plan_options options, uint32_t what,
                        char* buffer, uint64_t capacity, uint64_t* needed, uint64_t* counts,
                        char* failure, uint64_t failure_cap);

/* ---- full-tensor sum without allocation --------------------------------
 * No counterpart in the reference. For callers that cannot allocate device
 * memory: hosts that own all device memory through their own allocator and
 * do not let a component call cudaMalloc / cudaFree (which can synchronise
 * the device and fragment the host's pool). The caller passes x (n f32
 * values on `device`) and at least one output (device pointers: *out_f32 the
 * f32 rounding, *out_f64 the f64 total). The block partials live in a fixed
 * scratch array inside the library — 4096 f64 values (32 KiB) that every GPU
 * loading the library holds until exit; a reduction needing more partials
 * than that is rejected with GPU-NOALLOC-SIZE (on a B200 the sum uses at most
 * 4 x 148 = 592). Nothing is allocated: the first call on a device resolves
 * the device addresses of the scratch and of a static status word once (make
 * that first call before any stream capture; a host that resets the device
 * with cudaDeviceReset after it must not call this entry point again). Every
 * call shares the one scratch array, and each call writes every partial it
 * later reads, so the partials need no clearing; the status word is cleared
 * by each call before its launches. The call waits for `stream` and reads the
 * status word before it returns: a bounded wait that ran out on the device
 * returns THB_STATUS_BACKEND with GPU-KERNEL-TIMEOUT (or
 * GPU-KERNEL-DRAIN-TIMEOUT) and the outputs are then invalid. Calls that
 * overlap on the GPU (different streams, or different host threads on one
 * device) race on the scratch and the status word and must be serialised by
 * the caller. Results are identical to the region Sum path (same kernels,
 * same grid). */
int thb_sum_all_f32_noalloc(int device, const float* x, uint64_t n, float* out_f32, double* out_f64,
                            void* stream, char* failure, uint64_t failure_cap);

#ifdef __cplusplus
}
#endif

#endif /* THIRAN_B200_H */
