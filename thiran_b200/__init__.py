"""Python binding of libthiran_b200.so, the B200-native TensorRegion engine.

Everything here is a thin ctypes layer over the C ABI in include/thiran_b200.h;
all planning, code generation and execution happens in the native library.
There is no CPU execution path: if the library is missing, importing the
binding raises, and without a CUDA device every execution call raises
GpuError("GPU-DRIVER-NOT-FOUND"), exactly like the reference's
`--backend gpu` (src/tooling/v0/Cli.cpp:150-156, no fallback).

The region builder mirrors the reference's TensorRegion
(include/backend/v0/TensorRegion.hpp:14-57): nodes are added in program order,
each gets a nonzero value id, and the region is compiled with
PhysicalPlanOptions(enable_reuse, enable_fusion)
(include/backend/v0/PhysicalPlan.hpp:37-41).
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field
from typing import Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY_PATH = os.path.join(_HERE, "libthiran_b200.so")

# ---- constants (include/thiran_b200.h) ------------------------------------------------
STATUS_OK, STATUS_ABI, STATUS_SEMANTIC, STATUS_BACKEND, STATUS_UNKNOWN = 0, 1, 2, 3, 4
I64, F32, BF16 = 1, 2, 3
KIND_SCALAR, KIND_TENSOR = 1, 2
(OP_INPUT, OP_INTEGER, OP_FLOAT, OP_TENSOR_LITERAL, OP_ALIAS, OP_COPY, OP_NEGATE, OP_ADD, OP_SUBTRACT,
 OP_ELEMENT_MULTIPLY, OP_EXTENSION, OP_INDEX, OP_UNSUPPORTED) = range(13)
OP_SUM, OP_ROW_MAX, OP_SOFTMAX, OP_RELU = 32, 33, 34, 35
(OP_EXTENSION_GRADIENT, OP_TRANSPOSE, OP_MATMUL, OP_BROADCAST_TO_SHAPE, OP_REDUCE_TO_SHAPE,
 OP_ZERO_LIKE) = range(36, 42)
(SCALAR_INPUT, SCALAR_CONSTANT_F32, SCALAR_ADD, SCALAR_SUBTRACT, SCALAR_MULTIPLY, SCALAR_DIVIDE,
 SCALAR_NEGATE) = range(1, 8)
EFFECT_PURE, EFFECT_MAY_TRAP = 0, 1
BACKEND_REFERENCE, BACKEND_CPU, BACKEND_GPU = 1, 2, 4
DESCRIBE_PLAN, DESCRIBE_SOURCE, DESCRIBE_CUBIN = 0, 1, 2

_NP = {I64: np.int64, F32: np.float32}


class ScalarNode(C.Structure):
    _fields_ = [("opcode", C.c_uint8), ("left", C.c_uint32), ("right", C.c_uint32), ("input", C.c_uint32),
                ("constant", C.c_float)]


class ScalarRecipe(C.Structure):
    _fields_ = [("nodes", C.POINTER(ScalarNode)), ("node_count", C.c_size_t), ("root", C.c_uint32),
                ("input_count", C.c_uint32)]


class Derivative(C.Structure):
    _fields_ = [("differentiable_inputs", C.c_uint64), ("saved_inputs", C.c_uint64), ("saves_output", C.c_uint8),
                ("gradients", C.POINTER(ScalarRecipe)), ("gradient_count", C.c_size_t)]


class OperationDesc(C.Structure):
    _fields_ = [("name", C.c_char_p), ("semantic_version", C.c_char_p), ("arity", C.c_uint32),
                ("minimum_rank", C.c_uint32), ("maximum_rank", C.c_uint32), ("result_like_input", C.c_uint32),
                ("same_shape", C.c_uint8), ("effect", C.c_uint8), ("backends", C.c_uint32), ("fusible", C.c_uint8),
                ("forward", ScalarRecipe), ("derivative", C.POINTER(Derivative))]


class RegionNode(C.Structure):
    _fields_ = [("id", C.c_uint32), ("op", C.c_uint32), ("dtype", C.c_uint32), ("rank", C.c_uint32),
                ("extent", C.c_int64 * 2), ("dependencies", C.POINTER(C.c_uint32)), ("dependency_count", C.c_uint32),
                ("indices", C.POINTER(C.c_uint32)), ("index_count", C.c_uint32), ("integer", C.c_int64),
                ("floating", C.c_float), ("axis", C.c_int32), ("extension", C.POINTER(OperationDesc))]


class RegionDesc(C.Structure):
    _fields_ = [("function", C.c_uint32), ("name", C.c_char_p), ("nodes", C.POINTER(RegionNode)),
                ("node_count", C.c_uint32), ("inputs", C.POINTER(C.c_uint32)), ("input_count", C.c_uint32),
                ("output", C.c_uint32)]


class PlanOptions(C.Structure):
    _fields_ = [("enable_reuse", C.c_uint32), ("enable_fusion", C.c_uint32)]


class AbiArg(C.Structure):
    _fields_ = [("kind", C.c_uint32), ("dtype", C.c_uint32), ("rank", C.c_uint32), ("reserved", C.c_uint32),
                ("shape", C.POINTER(C.c_uint64)), ("data", C.c_void_p), ("count", C.c_uint64)]


EVIDENCE_FIELDS = [
    "allocation_count", "allocation_bytes_requested", "host_to_device_copies", "host_to_device_bytes",
    "device_to_host_copies", "device_to_host_bytes", "device_to_device_copies", "device_to_device_bytes",
    "module_loads", "driver_jit_loads", "input_storage_uploads", "result_downloads", "kernel_launches",
    "synchronizations", "submitted_operations", "pending_operations", "active_read_reservations",
    "active_write_reservations", "stream_submissions", "event_records", "observations", "dropped_drains",
    "released_reservations", "logical_tensor_values", "logical_intermediates", "materialized_intermediates",
    "physical_slots", "physical_temporary_slots", "reused_slot_assignments", "fusion_groups", "fused_kernel_groups",
    "planner_owned_allocations", "retained_planner_allocations",
]


class Evidence(C.Structure):
    _fields_ = [(name, C.c_uint64) for name in EVIDENCE_FIELDS]

    def as_dict(self) -> dict:
        return {name: int(getattr(self, name)) for name in EVIDENCE_FIELDS}


class DeviceInfo(C.Structure):
    _fields_ = [("backend_built", C.c_int32), ("driver_loaded", C.c_int32), ("device_available", C.c_int32),
                ("device_count", C.c_int32), ("selected_device", C.c_int32), ("driver_version", C.c_int32),
                ("compute_major", C.c_int32), ("compute_minor", C.c_int32), ("sm_count", C.c_int32),
                ("reserved", C.c_int32), ("name", C.c_char * 256), ("error_code", C.c_char * 64)]


MAJOR_K, MAJOR_MN = 0, 1
MATMUL_TENSOR, MATMUL_EXACT = 0, 1  # f32 MatMul modes (node axis)
REDUCE_F32, REDUCE_BF16_SHARDED = 0, 1  # MLP gradient all-reduce formats
EPI_F32, EPI_BF16, EPI_RELU_BF16, EPI_MASK_BF16 = 0, 1, 2, 3


class GemmDesc(C.Structure):
    _fields_ = [("m", C.c_uint64), ("n", C.c_uint64), ("k", C.c_uint64), ("a", C.c_void_p), ("a_major", C.c_uint32),
                ("lda", C.c_uint64), ("b", C.c_void_p), ("b_major", C.c_uint32), ("ldb", C.c_uint64),
                ("c", C.c_void_p), ("ldc", C.c_uint64), ("epilogue", C.c_uint32), ("aux", C.c_void_p),
                ("ld_aux", C.c_uint64), ("c_f32_copy", C.c_void_p)]


# ---- library --------------------------------------------------------------------------

_lib = None

# Every symbol include/thiran_b200.h declares, with its ctypes signature.
SIGNATURES = {
    "thb_backend_built": (C.c_int, []),
    "thb_abi_version": (C.c_uint32, []),
    "thb_probe": (C.c_int, [C.c_int, C.POINTER(DeviceInfo)]),
    "thb_region_compile": (C.c_int, [C.POINTER(RegionDesc), PlanOptions, C.c_int, C.POINTER(C.c_void_p),
                                     C.c_char_p, C.c_uint64]),
    "thb_region_release": (None, [C.c_void_p]),
    "thb_region_execute": (C.c_int, [C.c_void_p, C.POINTER(AbiArg), C.c_uint64, C.c_void_p, C.c_uint64,
                                     C.POINTER(Evidence), C.c_char_p, C.c_uint64]),
    "thb_region_submit": (C.c_int, [C.c_void_p, C.POINTER(AbiArg), C.c_uint64, C.POINTER(C.c_void_p),
                                    C.POINTER(Evidence), C.c_char_p, C.c_uint64]),
    "thb_pending_state": (C.c_int, [C.c_void_p]),
    "thb_pending_observe": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint64, C.POINTER(Evidence),
                                      C.c_char_p, C.c_uint64]),
    "thb_pending_release": (None, [C.c_void_p]),
    "thb_take_unobserved_errors": (C.c_uint64, [C.c_char_p, C.c_uint64]),
    "thb_region_launch": (C.c_int, [C.c_void_p, C.POINTER(AbiArg), C.c_uint64, C.c_void_p, C.c_uint64,
                                    C.c_void_p, C.c_char_p, C.c_uint64]),
    "thb_region_check_errors": (C.c_int, [C.c_void_p, C.c_void_p, C.c_char_p, C.c_uint64]),
    "thb_region_emit_source": (C.c_int, [C.c_void_p, C.c_char_p, C.c_uint64, C.POINTER(C.c_uint64)]),
    "thb_region_dump_plan": (C.c_int, [C.c_void_p, C.c_char_p, C.c_uint64, C.POINTER(C.c_uint64)]),
    "thb_region_plan_counts": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64),
                                         C.POINTER(C.c_uint64)]),
    "thb_region_describe": (C.c_int, [C.POINTER(RegionDesc), PlanOptions, C.c_uint32, C.c_char_p, C.c_uint64,
                                      C.POINTER(C.c_uint64), C.POINTER(C.c_uint64), C.c_char_p, C.c_uint64]),
    "thb_artifact_load": (C.c_int, [C.c_void_p, C.c_uint64, C.POINTER(C.c_void_p), C.c_char_p, C.c_uint64]),
    "thb_artifact_load_file": (C.c_int, [C.c_char_p, C.POINTER(C.c_void_p), C.c_char_p, C.c_uint64]),
    "thb_artifact_release": (None, [C.c_void_p]),
    "thb_artifact_inspect": (C.c_int, [C.c_void_p, C.c_char_p, C.c_uint64, C.POINTER(C.c_uint64)]),
    "thb_artifact_compile": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_void_p), C.c_char_p, C.c_uint64]),
    "thb_artifact_build": (C.c_int, [C.POINTER(RegionDesc), PlanOptions, C.c_void_p, C.c_uint64,
                                     C.POINTER(C.c_uint64), C.c_char_p, C.c_uint64]),
    "thb_render": (C.c_int, [C.c_int, C.c_void_p, C.c_uint64, C.c_void_p, C.c_uint64, C.c_void_p, C.c_void_p,
                             C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint64, C.c_void_p, C.c_void_p, C.c_void_p,
                             C.c_void_p, C.POINTER(Evidence), C.c_char_p, C.c_uint64]),
    "thb_model_load": (C.c_int, [C.c_void_p, C.c_uint64, C.c_char_p, C.POINTER(C.c_void_p), C.c_char_p,
                                 C.c_uint64]),
    "thb_model_load_file": (C.c_int, [C.c_char_p, C.c_char_p, C.POINTER(C.c_void_p), C.c_char_p, C.c_uint64]),
    "thb_model_release": (None, [C.c_void_p]),
    "thb_model_inspect": (C.c_int, [C.c_void_p, C.c_char_p, C.c_uint64, C.POINTER(C.c_uint64)]),
    "thb_model_compile": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_void_p), C.POINTER(Evidence), C.c_char_p,
                                    C.c_uint64]),
    "thb_model_session_release": (None, [C.c_void_p]),
    "thb_model_execute": (C.c_int, [C.c_void_p, C.POINTER(AbiArg), C.c_uint64, C.c_void_p, C.c_uint64,
                                    C.POINTER(Evidence), C.c_char_p, C.c_uint64]),
    "thb_gemm_bf16": (C.c_int, [C.c_int, C.POINTER(GemmDesc), C.c_void_p, C.c_char_p, C.c_uint64]),
    "thb_device_check_status": (C.c_int, [C.c_int, C.c_void_p, C.c_char_p, C.c_uint64]),
    "thb_mlp_create": (C.c_int, [C.c_int, C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64,
                                 C.POINTER(C.c_void_p), C.c_char_p, C.c_uint64]),
    "thb_mlp_release": (None, [C.c_void_p]),
    "thb_mlp_set_weights": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_char_p, C.c_uint64]),
    "thb_mlp_forward_backward": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_char_p, C.c_uint64]),
    "thb_mlp_apply_sgd": (C.c_int, [C.c_void_p, C.c_float, C.c_void_p, C.c_char_p, C.c_uint64]),
    "thb_mlp_set_biases": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_char_p, C.c_uint64]),
    "thb_mlp_set_momentum": (C.c_int, [C.c_void_p, C.c_float, C.c_void_p, C.c_char_p, C.c_uint64]),
    "thb_mlp_step": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_float, C.c_void_p, C.c_char_p, C.c_uint64]),
    "thb_mlp_buffer": (C.c_int, [C.c_void_p, C.c_uint32, C.POINTER(C.c_void_p), C.POINTER(C.c_uint64)]),
    "thb_mlp_bind": (C.c_int, [C.c_void_p, C.c_uint32, C.c_void_p]),
    "thb_mlp_bind_reduction": (C.c_int, [C.c_void_p, C.c_uint32, C.POINTER(C.c_void_p), C.c_void_p,
                                         C.POINTER(C.c_void_p), C.c_uint32, C.c_uint32]),
    "thb_mlp_reduction_flag_words": (C.c_uint64, [C.c_void_p, C.c_uint32]),
    "thb_mlp_bind_update": (C.c_int, [C.c_void_p, C.c_uint32, C.POINTER(C.c_void_p), C.c_void_p,
                                      C.POINTER(C.c_void_p), C.c_void_p]),
    "thb_mlp_forward_backward_update": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_float, C.c_void_p,
                                                  C.c_char_p, C.c_uint64]),
    "thb_mlp_set_reduction_format": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32]),
    "thb_mlp_gather_parameters": (C.c_int, [C.c_void_p, C.c_uint32, C.c_void_p, C.c_char_p, C.c_uint64]),
    "thb_mlp_enable_timing": (C.c_int, [C.c_void_p, C.c_int]),
    "thb_mlp_read_timing": (C.c_int, [C.c_void_p, C.POINTER(C.c_double), C.POINTER(C.c_uint64)]),
    "thb_sum_all_f32_noalloc": (C.c_int, [C.c_int, C.c_void_p, C.c_uint64, C.c_void_p, C.c_void_p, C.c_void_p,
                                          C.c_char_p, C.c_uint64]),
}

MLP_W1, MLP_W2, MLP_DW1, MLP_DW2, MLP_Y, MLP_H, MLP_LOSS_SUM, MLP_B1, MLP_B2, MLP_DB1, MLP_DB2 = range(11)


class MlpSession:
    """Two-layer MLP training session (thb_mlp): H = relu(X W1 [+ b1]),
    Y = H W2 [+ b2], L = mean((Y - T)^2), SGD or SGD with momentum. Tensors
    are torch CUDA tensors."""

    def __init__(self, batch, d_in, hidden, d_out, global_batch=None, device=0):
        self.batch, self.d_in, self.hidden, self.d_out = batch, d_in, hidden, d_out
        self.global_batch = global_batch or batch
        self.device = device
        handle = C.c_void_p()
        fail = _failure()
        _raise(lib().thb_mlp_create(device, batch, self.global_batch, d_in, hidden, d_out, C.byref(handle), fail,
                                    len(fail)), fail)
        self.handle = handle

    def _call(self, name, *args):
        fail = _failure()
        _raise(getattr(lib(), name)(self.handle, *args, fail, len(fail)), fail)

    def set_weights(self, w1, w2, stream=0):
        self._call("thb_mlp_set_weights", w1.data_ptr(), w2.data_ptr(), C.c_void_p(stream))

    def set_weight_pointers(self, w1_ptr, w2_ptr, stream=0):
        """set_weights from raw device pointers (f32 [in][hidden], [hidden][out])."""
        self._call("thb_mlp_set_weights", C.c_void_p(w1_ptr), C.c_void_p(w2_ptr), C.c_void_p(stream))

    def forward_backward(self, x, t, stream=0):
        self._call("thb_mlp_forward_backward", x.data_ptr(), t.data_ptr(), C.c_void_p(stream))

    def apply_sgd(self, lr, stream=0):
        self._call("thb_mlp_apply_sgd", C.c_float(lr), C.c_void_p(stream))

    def set_biases(self, b1=None, b2=None, stream=0):
        """Enables the broadcast biases (zeros when not given)."""
        self._call("thb_mlp_set_biases", None if b1 is None else b1.data_ptr(),
                   None if b2 is None else b2.data_ptr(), C.c_void_p(stream))

    def set_momentum(self, momentum, stream=0):
        """SGD (0) or SGD with momentum; velocities restart at zero."""
        self._call("thb_mlp_set_momentum", C.c_float(momentum), C.c_void_p(stream))

    def step(self, x, t, lr, stream=0):
        """One single-device training step; the weight updates run in the dW
        GEMMs' read-out, so the DW1 / DW2 buffers are not written."""
        self._call("thb_mlp_step", x.data_ptr(), t.data_ptr(), C.c_float(lr), C.c_void_p(stream))

    def enable_timing(self, enabled=True):
        if lib().thb_mlp_enable_timing(self.handle, int(enabled)) != STATUS_OK:
            raise GpuError(STATUS_BACKEND, "GPU-RUNTIME: cannot create timing events")

    def read_timing(self):
        """(summed GEMM device ms, GEMM launches) since the previous read."""
        ms, n = C.c_double(), C.c_uint64()
        if lib().thb_mlp_read_timing(self.handle, C.byref(ms), C.byref(n)) != STATUS_OK:
            raise GpuError(STATUS_BACKEND, "GPU-RUNTIME: cannot read timing events")
        return ms.value, int(n.value)

    def bind_reduction(self, which, peer_ptrs, flag_peer_ptrs, rank, world, multicast_ptr=None):
        """Fuses the data-parallel all-reduce of dW1 / dW2 into its GEMM
        (thb_mlp_bind_reduction): `peer_ptrs[k]` / `flag_peer_ptrs[k]` are
        rank k's dW buffer and zeroed signal words as mapped on this GPU;
        `multicast_ptr` (NVLS address of the dW buffers) selects the in-switch
        reduction. `peer_ptrs=None` restores the local store."""
        peers = flags = None
        if peer_ptrs is not None:
            peers = (C.c_void_p * len(peer_ptrs))(*peer_ptrs)
            flags = (C.c_void_p * len(flag_peer_ptrs))(*flag_peer_ptrs)
        if lib().thb_mlp_bind_reduction(self.handle, which, peers, C.c_void_p(multicast_ptr), flags, rank,
                                        world) != STATUS_OK:
            raise GpuError(STATUS_ABI, "GPU-MLP-ARGUMENT: cannot bind the reduction target")

    def set_reduction_format(self, which, fmt):
        """THB_REDUCE_F32 or THB_REDUCE_BF16_SHARDED for the all-reduce of
        `which` (MLP_DW1 / MLP_DW2), after bind_reduction."""
        if lib().thb_mlp_set_reduction_format(self.handle, which, fmt) != STATUS_OK:
            raise GpuError(STATUS_ABI, "GPU-MLP-ARGUMENT: cannot set the reduction format")

    def gather_parameters(self, which, stream=0):
        """Assembles this rank's f32 weights `which` (MLP_W1 / MLP_W2) from
        their tile owners after bf16 sharded reductions."""
        self._call("thb_mlp_gather_parameters", which, C.c_void_p(stream))

    def reduction_flag_words(self, which):
        """Number of u32 signal words bind_reduction needs for `which`."""
        return int(lib().thb_mlp_reduction_flag_words(self.handle, which))

    def bind_update(self, which, param_ptrs, copy_ptrs, param_multicast=None, copy_multicast=None):
        """Lets the all-reduce of layer `which` (MLP_W1 / MLP_W2, reduction
        bound first) apply the optimizer step (thb_mlp_bind_update):
        `param_ptrs[k]` / `copy_ptrs[k]` are rank k's f32 parameters and their
        bf16 copy as mapped on this GPU. Copy the weights in afterwards with
        set_weights. `param_ptrs=None` removes the binding: W returns to the
        session's own buffers, into which set_weights copies them again."""
        params = copies = None
        if param_ptrs is not None:
            params = (C.c_void_p * len(param_ptrs))(*param_ptrs)
            copies = (C.c_void_p * len(copy_ptrs))(*copy_ptrs)
        if lib().thb_mlp_bind_update(self.handle, which, params, C.c_void_p(param_multicast), copies,
                                     C.c_void_p(copy_multicast)) != STATUS_OK:
            raise GpuError(STATUS_ABI, "GPU-MLP-ARGUMENT: cannot bind the fused update")

    def forward_backward_update(self, x, t, lr, stream=0):
        """forward_backward with the weight updates applied in the
        all-reduce; apply_sgd afterwards updates only the biases."""
        self._call("thb_mlp_forward_backward_update", x.data_ptr(), t.data_ptr(), C.c_float(lr), C.c_void_p(stream))

    def bind(self, which, tensor):
        """Makes the session use `tensor`'s device memory for buffer `which`."""
        if lib().thb_mlp_bind(self.handle, which, tensor.data_ptr()) != STATUS_OK:
            raise GpuError(STATUS_ABI, "GPU-MLP-ARGUMENT: cannot bind buffer")
        return tensor

    def buffer(self, which):
        """(device pointer, element count) of a session buffer."""
        ptr, count = C.c_void_p(), C.c_uint64()
        if lib().thb_mlp_buffer(self.handle, which, C.byref(ptr), C.byref(count)) != STATUS_OK:
            raise GpuError(STATUS_ABI, "GPU-MLP-ARGUMENT: unknown buffer")
        return ptr.value, int(count.value)

    def release(self):
        if self.handle:
            lib().thb_mlp_release(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


def gemm(a, b, c, m, n, k, a_major=MAJOR_K, b_major=MAJOR_K, epilogue=EPI_F32, aux=None, c_f32=None,
         device=0, stream=0, lda=None, ldb=None, ldc=None):
    """C = A B on the tensor cores; a, b, c, aux are CUDA tensors (torch)."""
    desc = GemmDesc(m, n, k, a.data_ptr(), a_major, lda or (m if a_major == MAJOR_MN else k), b.data_ptr(), b_major,
                    ldb or (n if b_major == MAJOR_MN else k), c.data_ptr(), ldc or n, epilogue,
                    aux.data_ptr() if aux is not None else None, n if aux is not None else 0,
                    c_f32.data_ptr() if c_f32 is not None else None)
    fail = _failure()
    _raise(lib().thb_gemm_bf16(device, C.byref(desc), C.c_void_p(stream), fail, len(fail)), fail)


def check_device_status(device=0, stream=0):
    fail = _failure()
    _raise(lib().thb_device_check_status(device, C.c_void_p(stream), fail, len(fail)), fail)


def lib() -> C.CDLL:
    """Loads libthiran_b200.so from this package directory (raises if absent)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIBRARY_PATH):
            raise ImportError(f"{LIBRARY_PATH} is missing: build it with `make -C thiran_b200` "
                              "(there is no fallback implementation)")
        handle = C.CDLL(LIBRARY_PATH)
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = handle
    return _lib


class GpuError(RuntimeError):
    """A failed engine call: `status` is the C-ABI status, `code` the failure id."""

    def __init__(self, status: int, text: str):
        code, _, message = text.partition(": ")
        super().__init__(text)
        self.status = status
        self.code = code
        self.message = message or code


def _failure():
    return C.create_string_buffer(1024)


def _raise(status: int, buf) -> None:
    if status != STATUS_OK:
        raise GpuError(status, buf.value.decode(errors="replace"))


def probe(device: int = 0) -> DeviceInfo:
    info = DeviceInfo()
    lib().thb_probe(device, C.byref(info))
    return info


def take_unobserved_errors() -> list[str]:
    buf = C.create_string_buffer(65536)
    count = lib().thb_take_unobserved_errors(buf, len(buf))
    text = buf.value.decode()
    return text.split("\n") if count else []


# ---- operations and regions ----------------------------------------------------------

@dataclass
class Operation:
    """An extension operation descriptor (OperationDescriptorV0,
    include/extension/v0/Extension.hpp:40-53) with its scalar forward recipe:
    a list of (opcode, left, right, input, constant) tuples."""
    name: str
    recipe: Sequence[tuple]
    root: int
    arity: int = 1
    semantic_version: str = "1.0.0"
    effect: int = EFFECT_PURE
    fusible: bool = True
    backends: int = BACKEND_REFERENCE | BACKEND_CPU | BACKEND_GPU
    minimum_rank: int = 1
    maximum_rank: int = 2
    # Reverse derivative (DerivativeV0): one gradient recipe (nodes, root) per
    # operand over (primals..., result, cotangent); None = not differentiable.
    gradients: Sequence = None
    saved_inputs: int = 0
    saves_output: bool = False
    _keep: list = field(default_factory=list, repr=False)

    def descriptor(self) -> OperationDesc:
        nodes = (ScalarNode * len(self.recipe))(*[ScalarNode(*t) for t in self.recipe])
        name = self.name.encode()
        version = self.semantic_version.encode()
        self._keep[:] = [nodes, name, version]
        derivative = None
        if self.gradients is not None:
            recipes = (ScalarRecipe * self.arity)()
            mask = 0
            for k, g in enumerate(self.gradients):
                if g is None:
                    continue
                g_nodes, g_root = g
                arr = (ScalarNode * len(g_nodes))(*[ScalarNode(*t) for t in g_nodes])
                self._keep.append(arr)
                recipes[k] = ScalarRecipe(arr, len(g_nodes), g_root, self.arity + 2)
                mask |= 1 << k
            d = Derivative(mask, self.saved_inputs or mask, 1 if self.saves_output else 0, recipes, self.arity)
            self._keep += [recipes, d]
            derivative = C.pointer(d)
        return OperationDesc(name, version, self.arity, self.minimum_rank, self.maximum_rank, 0, 1, self.effect,
                             self.backends, 1 if self.fusible else 0,
                             ScalarRecipe(nodes, len(self.recipe), self.root, self.arity), derivative)


def recipe_from_expression(ops: Sequence[tuple]) -> list[tuple]:
    """Builds a recipe from (opcode, a, b) / ('c', value) / ('x', input) steps."""
    out = []
    for step in ops:
        kind = step[0]
        if kind == "x":
            out.append((SCALAR_INPUT, 0, 0, step[1], 0.0))
        elif kind == "c":
            out.append((SCALAR_CONSTANT_F32, 0, 0, 0, float(step[1])))
        elif kind == SCALAR_NEGATE:
            out.append((SCALAR_NEGATE, step[1], 0, 0, 0.0))
        else:
            out.append((kind, step[1], step[2], 0, 0.0))
    return out


class RegionBuilder:
    """Builds a TensorRegion description node by node (ids start at 1)."""

    def __init__(self, name: str = "main", function: int = 1):
        self.name = name
        self.function = function
        self.nodes: list[dict] = []
        self.inputs: list[int] = []
        self.output = 0

    def _add(self, op, dtype, shape=(), deps=(), indices=(), integer=0, floating=0.0, axis=0, extension=None):
        node_id = len(self.nodes) + 1
        self.nodes.append(dict(id=node_id, op=op, dtype=dtype, shape=list(shape), deps=list(deps),
                               indices=list(indices), integer=integer, floating=floating, axis=axis,
                               extension=extension))
        return node_id

    def _like(self, v):
        n = self.nodes[v - 1]
        return n["dtype"], n["shape"]

    # reference RegionOps
    def input(self, dtype, shape=()):
        v = self._add(OP_INPUT, dtype, shape)
        self.inputs.append(v)
        return v

    def integer(self, value):
        return self._add(OP_INTEGER, I64, integer=int(value))

    def float(self, value):
        return self._add(OP_FLOAT, F32, floating=float(value))

    def literal(self, dtype, shape, elements):
        return self._add(OP_TENSOR_LITERAL, dtype, shape, deps=elements)

    def alias(self, a):
        return self._add(OP_ALIAS, *self._like(a), deps=[a])

    def copy(self, a):
        return self._add(OP_COPY, *self._like(a), deps=[a])

    def neg(self, a):
        return self._add(OP_NEGATE, *self._like(a), deps=[a])

    def _binary(self, a, b):
        """dtype and shape of an elementwise result: a scalar operand
        broadcasts, so the tensor operand decides the shape."""
        da, sa = self._like(a)
        return (da, sa) if sa or not self._like(b)[1] else self._like(b)

    def add(self, a, b):
        return self._add(OP_ADD, *self._binary(a, b), deps=[a, b])

    def sub(self, a, b):
        return self._add(OP_SUBTRACT, *self._binary(a, b), deps=[a, b])

    def mul(self, a, b):
        return self._add(OP_ELEMENT_MULTIPLY, *self._binary(a, b), deps=[a, b])

    def extension(self, operation: Operation, *args):
        return self._add(OP_EXTENSION, *self._like(args[0]), deps=list(args), extension=operation)

    def index(self, a, *coords):
        return self._add(OP_INDEX, self._like(a)[0], (), deps=[a], indices=list(coords))

    # engine additions
    def relu(self, a):
        return self._add(OP_RELU, *self._like(a), deps=[a])

    def softmax(self, a):
        dtype, shape = self._like(a)
        return self._add(OP_SOFTMAX, dtype, shape, deps=[a], axis=len(shape) - 1)

    def row_max(self, a):
        dtype, shape = self._like(a)
        return self._add(OP_ROW_MAX, dtype, [shape[0]], deps=[a], axis=1)

    def sum(self, a, axis):
        dtype, shape = self._like(a)
        kept = [e for i, e in enumerate(shape) if i != axis]
        return self._add(OP_SUM, dtype, kept, deps=[a], axis=axis)

    # reverse-AD operations (Autodiff.cpp emits them into backward functions)
    def extension_gradient(self, operation: Operation, operand: int, *args):
        """Gradient of `operation` w.r.t. operand `operand`; args = primal
        operands..., primal result, output cotangent."""
        return self._add(OP_EXTENSION_GRADIENT, *self._like(args[0]), deps=list(args), axis=operand,
                         extension=operation)

    def transpose(self, a):
        dtype, shape = self._like(a)
        return self._add(OP_TRANSPOSE, dtype, [shape[1], shape[0]], deps=[a])

    def matmul(self, a, b, exact=False):
        """C = A B. i64 operands: checked multiply and add. f32 operands:
        bf16 x bf16 -> f32 on the tensor cores, or with `exact` the
        reference Evaluator's sequential, separately rounded f32 sums."""
        dtype = self._like(a)[0]
        return self._add(OP_MATMUL, dtype, [self._like(a)[1][0], self._like(b)[1][1]], deps=[a, b],
                         axis=MATMUL_EXACT if exact else MATMUL_TENSOR)

    def broadcast_to_shape(self, value, reference, axis):
        return self._add(OP_BROADCAST_TO_SHAPE, *self._like(reference), deps=[value, reference], axis=axis)

    def reduce_to_shape(self, value, reference):
        return self._add(OP_REDUCE_TO_SHAPE, *self._like(reference), deps=[value, reference])

    def zero_like(self, reference):
        return self._add(OP_ZERO_LIKE, *self._like(reference), deps=[reference])

    def build(self, output: int) -> "RegionSpec":
        self.output = output
        return RegionSpec(self)


class RegionSpec:
    """A region description laid out in C structs (kept alive by this object)."""

    def __init__(self, builder: RegionBuilder):
        self._keep = []
        nodes = (RegionNode * len(builder.nodes))()
        for i, n in enumerate(builder.nodes):
            deps = (C.c_uint32 * max(1, len(n["deps"])))(*n["deps"])
            idx = (C.c_uint32 * max(1, len(n["indices"])))(*n["indices"])
            self._keep += [deps, idx]
            node = nodes[i]
            node.id, node.op, node.dtype, node.rank = n["id"], n["op"], n["dtype"], len(n["shape"])
            for a, e in enumerate(n["shape"]):
                node.extent[a] = -1 if e is None else int(e)
            for a in range(len(n["shape"]), 2):
                node.extent[a] = -1
            node.dependencies, node.dependency_count = deps, len(n["deps"])
            node.indices, node.index_count = idx, len(n["indices"])
            node.integer, node.floating, node.axis = n["integer"], n["floating"], n["axis"]
            if n["extension"] is not None:
                d = n["extension"].descriptor()
                self._keep += [d, n["extension"]]
                node.extension = C.pointer(d)
        inputs = (C.c_uint32 * max(1, len(builder.inputs)))(*builder.inputs)
        name = builder.name.encode()
        self._keep += [nodes, inputs, name]
        self.desc = RegionDesc(builder.function, name, nodes, len(builder.nodes), inputs, len(builder.inputs),
                               builder.output)
        self.input_types = [(builder.nodes[v - 1]["dtype"], builder.nodes[v - 1]["shape"]) for v in builder.inputs]
        out = builder.nodes[builder.output - 1] if 0 < builder.output <= len(builder.nodes) else None
        self.output_dtype = out["dtype"] if out else F32
        self.output_shape = out["shape"] if out else []
        self._nodes = builder.nodes
        self._inputs = builder.inputs
        self._output = builder.output

    def infer_output_shape(self, inputs) -> list:
        """Runtime output shape from the input shapes (for regions whose
        extents are unknown until execution)."""
        shapes = {}
        for v, value in zip(self._inputs, inputs):
            shapes[v] = list(np.shape(value)) if hasattr(value, "shape") else []
        for n in self._nodes:
            if n["id"] in shapes:
                continue
            deps = [shapes.get(d, []) for d in n["deps"]]
            op = n["op"]
            if op in (OP_INTEGER, OP_FLOAT, OP_INDEX):
                s = []
            elif op == OP_TENSOR_LITERAL:
                s = list(n["shape"])
            elif op == OP_SUM:
                s = [e for i, e in enumerate(deps[0]) if i != n["axis"]]
            elif op == OP_ROW_MAX:
                s = [deps[0][0]]
            elif op == OP_TRANSPOSE:
                s = [deps[0][1], deps[0][0]]
            elif op == OP_MATMUL:
                s = [deps[0][0], deps[1][1]]
            elif op in (OP_BROADCAST_TO_SHAPE, OP_REDUCE_TO_SHAPE):
                s = list(deps[1])
            else:  # elementwise and row ops: the first tensor operand's shape
                s = next((list(d) for d in deps if len(d)), list(n["shape"]) if not deps else [])
            shapes[n["id"]] = s
        return [int(e) for e in shapes[self._output]]

    def describe(self, what: int = DESCRIBE_PLAN, reuse=True, fusion=True) -> tuple[str, list[int]]:
        counts = (C.c_uint64 * 3)()
        needed = C.c_uint64(0)
        fail = _failure()
        status = lib().thb_region_describe(C.byref(self.desc), PlanOptions(int(reuse), int(fusion)), what, None, 0,
                                           C.byref(needed), counts, fail, len(fail))
        _raise(status, fail)
        buf = C.create_string_buffer(int(needed.value))
        status = lib().thb_region_describe(C.byref(self.desc), PlanOptions(int(reuse), int(fusion)), what, buf,
                                           len(buf), C.byref(needed), counts, fail, len(fail))
        _raise(status, fail)
        return buf.value.decode(), list(counts)

    def compile(self, device: int = 0, reuse=True, fusion=True) -> "CompiledRegion":
        handle = C.c_void_p()
        fail = _failure()
        status = lib().thb_region_compile(C.byref(self.desc), PlanOptions(int(reuse), int(fusion)), device,
                                          C.byref(handle), fail, len(fail))
        _raise(status, fail)
        return CompiledRegion(self, handle)


def _host_args(values) -> tuple:
    """Lays out host values (numpy arrays, python ints/floats) as AbiArg records."""
    keep = []
    args = (AbiArg * max(1, len(values)))()
    for i, v in enumerate(values):
        a = args[i]
        if isinstance(v, np.ndarray):
            dtype = I64 if v.dtype == np.int64 else F32 if v.dtype == np.float32 else 0
            shape = (C.c_uint64 * max(1, v.ndim))(*v.shape)
            keep.append(shape)
            a.kind, a.dtype, a.rank = KIND_TENSOR, dtype, v.ndim
            a.reserved = 0 if v.flags["C_CONTIGUOUS"] else 1
            a.shape, a.data, a.count = shape, v.ctypes.data if v.size else None, v.size
        else:
            is_int = isinstance(v, (int, np.integer)) and not isinstance(v, bool)
            scalar = C.c_int64(int(v)) if is_int else C.c_float(float(v))
            keep.append(scalar)
            a.kind, a.dtype, a.rank = KIND_SCALAR, I64 if is_int else F32, 0
            a.shape, a.data, a.count = None, C.cast(C.byref(scalar), C.c_void_p), 1
    return args, keep


def _device_args(tensors) -> tuple:
    """AbiArg records for device tensors (torch CUDA tensors) or host scalars."""
    keep = []
    args = (AbiArg * max(1, len(tensors)))()
    for i, t in enumerate(tensors):
        a = args[i]
        if hasattr(t, "data_ptr"):
            dtype = {"torch.int64": I64, "torch.float32": F32}.get(str(t.dtype), 0)
            shape = (C.c_uint64 * max(1, t.dim()))(*t.shape)
            keep.append(shape)
            a.kind, a.dtype, a.rank = KIND_TENSOR, dtype, t.dim()
            a.reserved = 0 if t.is_contiguous() else 1
            a.shape, a.data, a.count = shape, t.data_ptr() or None, t.numel()
        else:
            is_int = isinstance(t, (int, np.integer)) and not isinstance(t, bool)
            scalar = C.c_int64(int(t)) if is_int else C.c_float(float(t))
            keep.append(scalar)
            a.kind, a.dtype, a.rank = KIND_SCALAR, I64 if is_int else F32, 0
            a.shape, a.data, a.count = None, C.cast(C.byref(scalar), C.c_void_p), 1
    return args, keep


class Pending:
    """A submitted execution (PendingGpuExecution)."""

    def __init__(self, region: "CompiledRegion", handle: C.c_void_p, shape, dtype, evidence: dict):
        self.region, self.handle, self.shape, self.dtype = region, handle, shape, dtype
        self.submit_evidence = evidence
        self._value = None

    def state(self) -> int:
        return lib().thb_pending_state(self.handle)

    def observe(self, timeout_ms: int = 60000):
        out = np.empty(self.shape, dtype=_NP[self.dtype])
        ev = Evidence()
        fail = _failure()
        status = lib().thb_pending_observe(self.handle, out.ctypes.data if out.size else None, out.size,
                                           timeout_ms, C.byref(ev), fail, len(fail))
        self.evidence = ev.as_dict()
        _raise(status, fail)
        return out if self.shape != [] else out.reshape(()).item()

    def release(self):
        if self.handle:
            lib().thb_pending_release(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


class CompiledRegion:
    """A planned, code-generated, device-resident region (thb_region)."""

    def __init__(self, spec: RegionSpec, handle: C.c_void_p):
        self.spec, self.handle = spec, handle

    def execute(self, inputs, output_shape=None, out=None):
        """executeNativeGpu: host values in, host value out (numpy / scalar).
        `out` may supply a preallocated (for example pinned) host array."""
        args, keep = _host_args(inputs)
        shape = self.spec.infer_output_shape(inputs) if output_shape is None else list(output_shape)
        if out is None:
            out = np.empty([int(e) for e in shape], dtype=_NP[self.spec.output_dtype])
        ev = Evidence()
        fail = _failure()
        status = lib().thb_region_execute(self.handle, args, len(inputs), out.ctypes.data if out.size else None,
                                          out.size, C.byref(ev), fail, len(fail))
        self.evidence = ev.as_dict()
        _raise(status, fail)
        return out if len(shape) else out.reshape(()).item()

    def submit(self, inputs, output_shape=None) -> Pending:
        args, keep = _host_args(inputs)
        handle = C.c_void_p()
        ev = Evidence()
        fail = _failure()
        status = lib().thb_region_submit(self.handle, args, len(inputs), C.byref(handle), C.byref(ev), fail, len(fail))
        _raise(status, fail)
        shape = self.spec.infer_output_shape(inputs) if output_shape is None else list(output_shape)
        p = Pending(self, handle, [int(e) for e in shape], self.spec.output_dtype, ev.as_dict())
        p._inputs = inputs  # host buffers must outlive the submission
        return p

    def launch(self, tensors, output, stream=0) -> None:
        """Device-resident, stream-ordered launch (torch CUDA tensors)."""
        args, keep = _device_args(tensors)
        fail = _failure()
        status = lib().thb_region_launch(self.handle, args, len(tensors), output.data_ptr(), output.numel(),
                                         C.c_void_p(stream), fail, len(fail))
        _raise(status, fail)

    def check_errors(self, stream=0) -> None:
        fail = _failure()
        _raise(lib().thb_region_check_errors(self.handle, C.c_void_p(stream), fail, len(fail)), fail)

    def source(self) -> str:
        needed = C.c_uint64(0)
        lib().thb_region_emit_source(self.handle, None, 0, C.byref(needed))
        buf = C.create_string_buffer(int(needed.value))
        lib().thb_region_emit_source(self.handle, buf, len(buf), C.byref(needed))
        return buf.value.decode()

    def plan(self) -> str:
        needed = C.c_uint64(0)
        lib().thb_region_dump_plan(self.handle, None, 0, C.byref(needed))
        buf = C.create_string_buffer(int(needed.value))
        lib().thb_region_dump_plan(self.handle, buf, len(buf), C.byref(needed))
        return buf.value.decode()

    def release(self):
        if self.handle:
            lib().thb_region_release(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


class _ArtifactSpec:
    """Output dtype and shape rule of an artifact's region, from its entry
    signature (the manifest): a scalar result, the declared extents when all
    are known, else the first tensor parameter of the result's dtype and rank
    (specializeEntry, src/artifact/v0/NativeArtifacts.cpp:891-922)."""

    def __init__(self, manifest: dict):
        self.result = manifest["result"]
        self.parameters = manifest["parameters"]
        self.output_dtype = I64 if self.result["dtype"] == "i64" else F32

    def infer_output_shape(self, inputs):
        if self.result["kind"] == "scalar":
            return []
        if all(e is not None for e in self.result["extents"]):
            return list(self.result["extents"])
        for p, v in zip(self.parameters, inputs):
            if p["kind"] == "tensor" and p["dtype"] == self.result["dtype"] and p["rank"] == self.result["rank"]:
                return list(np.shape(v))
        raise GpuError(STATUS_ABI, "ARTIFACT-SIGNATURE: result extents are not known from the inputs")


class Artifact:
    """A loaded `.tha` artifact (thb_artifact): the reference's GPU artifacts
    (PTX payload, planned onto this engine) or this engine's own (cubin
    payload). `manifest` is the inspect JSON."""

    def __init__(self, handle: C.c_void_p):
        import json
        self.handle = handle
        needed = C.c_uint64(0)
        lib().thb_artifact_inspect(handle, None, 0, C.byref(needed))
        buf = C.create_string_buffer(int(needed.value))
        lib().thb_artifact_inspect(handle, buf, len(buf), C.byref(needed))
        self.manifest = json.loads(buf.value.decode())

    @classmethod
    def load(cls, source) -> "Artifact":
        """From a path or from bytes."""
        handle = C.c_void_p()
        fail = _failure()
        if isinstance(source, (bytes, bytearray)):
            data = bytes(source)
            status = lib().thb_artifact_load(data, len(data), C.byref(handle), fail, len(fail))
        else:
            status = lib().thb_artifact_load_file(os.fsencode(source), C.byref(handle), fail, len(fail))
        _raise(status, fail)
        return cls(handle)

    def compile(self, device: int = 0) -> CompiledRegion:
        handle = C.c_void_p()
        fail = _failure()
        _raise(lib().thb_artifact_compile(self.handle, device, C.byref(handle), fail, len(fail)), fail)
        return CompiledRegion(_ArtifactSpec(self.manifest), handle)

    def release(self):
        if self.handle:
            lib().thb_artifact_release(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


class ModelSession:
    """A compiled model (thb_model_session): frozen parameters resident in
    HBM, public inputs uploaded per call."""

    def __init__(self, model: "Model", handle: C.c_void_p, evidence: dict):
        self.model, self.handle, self.compile_evidence = model, handle, evidence
        self._spec = _ArtifactSpec({"result": model.result, "parameters": model.public_inputs})

    def execute(self, inputs, output_shape=None):
        args, keep = _host_args(inputs)
        shape = self._spec.infer_output_shape(inputs) if output_shape is None else list(output_shape)
        out = np.empty([int(e) for e in shape], dtype=_NP[self._spec.output_dtype])
        ev = Evidence()
        fail = _failure()
        status = lib().thb_model_execute(self.handle, args, len(inputs), out.ctypes.data if out.size else None,
                                         out.size, C.byref(ev), fail, len(fail))
        self.evidence = ev.as_dict()
        _raise(status, fail)
        return out if len(shape) else out.reshape(()).item()

    def release(self):
        if self.handle:
            lib().thb_model_session_release(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


class Model:
    """A loaded `.thm` model bundle (thb_model). `manifest` is the inspect
    JSON; `public_inputs` / `result` the public ABI of its GPU artifact."""

    def __init__(self, handle: C.c_void_p):
        import json
        self.handle = handle
        needed = C.c_uint64(0)
        lib().thb_model_inspect(handle, None, 0, C.byref(needed))
        buf = C.create_string_buffer(int(needed.value))
        lib().thb_model_inspect(handle, buf, len(buf), C.byref(needed))
        self.manifest = json.loads(buf.value.decode())
        self.public_inputs = self.manifest["public_abi"]
        self.result = self.manifest["result"]

    @classmethod
    def load(cls, source, identity=None) -> "Model":
        handle = C.c_void_p()
        fail = _failure()
        ident = identity.encode() if identity is not None else None
        if isinstance(source, (bytes, bytearray)):
            data = bytes(source)
            status = lib().thb_model_load(data, len(data), ident, C.byref(handle), fail, len(fail))
        else:
            status = lib().thb_model_load_file(os.fsencode(source), ident, C.byref(handle), fail, len(fail))
        _raise(status, fail)
        return cls(handle)

    def compile(self, device: int = 0) -> ModelSession:
        handle = C.c_void_p()
        ev = Evidence()
        fail = _failure()
        _raise(lib().thb_model_compile(self.handle, device, C.byref(handle), C.byref(ev), fail, len(fail)), fail)
        return ModelSession(self, handle, ev.as_dict())

    def release(self):
        if self.handle:
            lib().thb_model_release(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


def render(positions, indices, colors, model, view, projection, width, height, clear=(0, 0, 0, 0), device=0):
    """renderGpu (thb_render): returns (color [w*h, 4], depth [w*h], stats
    [input triangles, post-clip triangles, shaded pixels, depth passes]) and
    sets `render.evidence`."""
    pos = np.ascontiguousarray(positions, np.float32).reshape(-1, 3)
    col = np.ascontiguousarray(colors, np.float32).reshape(-1, 4)
    idx = np.ascontiguousarray(indices, np.int64).reshape(-1, 3)
    if pos.shape[0] != col.shape[0]:
        raise GpuError(STATUS_SEMANTIC, "TH019-GEOMETRY-COUNT")
    mats = [np.ascontiguousarray(m, np.float32).reshape(16) for m in (model, view, projection)]
    clr = np.ascontiguousarray(clear, np.float32).reshape(4)
    color = np.empty((width * height, 4), np.float32)
    depth = np.empty(width * height, np.float32)
    stats = np.zeros(4, np.uint64)
    ev = Evidence()
    fail = _failure()
    ptr = lambda a: a.ctypes.data if a.size else None
    status = lib().thb_render(device, ptr(pos), pos.shape[0], ptr(idx), idx.shape[0], ptr(col), mats[0].ctypes.data,
                              mats[1].ctypes.data, mats[2].ctypes.data, width, height, clr.ctypes.data, ptr(color),
                              ptr(depth), stats.ctypes.data, C.byref(ev), fail, len(fail))
    render.evidence = ev.as_dict()
    _raise(status, fail)
    return color, depth, stats


def build_artifact(spec: RegionSpec, reuse=True, fusion=True) -> bytes:
    """This engine's `.tha` artifact of `spec` (payload: generated source and
    sm_100a cubin; device-free)."""
    needed = C.c_uint64(0)
    fail = _failure()
    options = PlanOptions(int(reuse), int(fusion))
    buf = C.create_string_buffer(1 << 20)
    status = lib().thb_artifact_build(C.byref(spec.desc), options, buf, len(buf), C.byref(needed), fail, len(fail))
    if status != STATUS_OK and needed.value > len(buf):
        buf = C.create_string_buffer(int(needed.value))
        status = lib().thb_artifact_build(C.byref(spec.desc), options, buf, len(buf), C.byref(needed), fail, len(fail))
    _raise(status, fail)
    return buf.raw[:needed.value]
