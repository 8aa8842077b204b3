"""ctypes binding of the sm_100a runtime's C ABI.

The v1 half mirrors ArcQML's safe FFI facade ``arcqml-runtime-sys``
(``crates/arcqml-runtime-sys/src/lib.rs:123-336``): the same function names, argument meaning and
error behaviour (a non-zero status becomes ``RuntimeError`` carrying the runtime's thread-local
message, read as in ``last_error`` at ``lib.rs:330-336``). The v2 half drives device-resident
states held in torch CUDA tensors (``complex128``, ``[batch, 2^n]``).

There is no CPU fallback: importing this module loads ``libarcqml_runtime_private.so`` and fails
loudly if it is missing.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional, Sequence

import numpy as np

from .circuit import PlanOp

ABI_VERSION = 1
_HERE = os.path.dirname(os.path.abspath(__file__))
# ARCQML_RUNTIME_LIB may name another build of the same C ABI (e.g. an instrumented one).
LIB_PATH = os.environ.get("ARCQML_RUNTIME_LIB") or os.path.join(_HERE, "libarcqml_runtime_private.so")


class RuntimeError(Exception):  # noqa: A001 - mirrors arcqml_runtime_sys::RuntimeError
    """A failed runtime call; ``str(e)`` is the runtime's message."""

    def message(self) -> str:
        return str(self)


class C128(C.Structure):
    _fields_ = [("re", C.c_double), ("im", C.c_double)]


class GateDescriptor(C.Structure):
    _fields_ = [
        ("abi_version", C.c_uint32),
        ("opcode", C.c_uint32),
        ("arity", C.c_size_t),
        ("parameters", C.c_double * 3),
        ("matrix", C.c_void_p),
        ("matrix_len", C.c_size_t),
        ("name", C.c_void_p),
        ("name_len", C.c_size_t),
    ]


class DerivativeMatrixHandle(C.Structure):
    _fields_ = [("data", C.POINTER(C128)), ("len", C.c_size_t), ("capacity", C.c_size_t)]


class ParameterBindingDescriptor(C.Structure):
    _fields_ = [("parameter_slot", C.c_size_t), ("parent_index", C.c_size_t)]


class OperationDescriptor(C.Structure):
    _fields_ = [
        ("gate", GateDescriptor),
        ("qubits", C.POINTER(C.c_size_t)),
        ("qubits_len", C.c_size_t),
        ("parameters", C.POINTER(ParameterBindingDescriptor)),
        ("parameters_len", C.c_size_t),
    ]


class CircuitPlanHandle(C.Structure):
    _fields_ = [("opaque", C.c_void_p)]


class ObservableHandle(C.Structure):
    _fields_ = [("opaque", C.c_void_p)]


V1_SYMBOLS = (
    "arcqml_rt_abi_version", "arcqml_rt_v1_apply_gate", "arcqml_rt_v1_apply_adjoint_gate",
    "arcqml_rt_v1_parameter_derivative_into", "arcqml_rt_v1_derivative_matrix_create",
    "arcqml_rt_v1_derivative_matrix_apply", "arcqml_rt_v1_derivative_matrix_destroy",
    "arcqml_rt_v1_circuit_plan_create", "arcqml_rt_v1_circuit_plan_create_empty",
    "arcqml_rt_v1_circuit_plan_push", "arcqml_rt_v1_circuit_plan_apply",
    "arcqml_rt_v1_adjoint_backward", "arcqml_rt_v1_circuit_plan_destroy", "arcqml_rt_last_error",
)

_P, _S, _I32, _D = C.c_void_p, C.c_size_t, C.c_int32, C.c_double
# (result type, argument types) of every entry point the binding calls
SIGNATURES = {
    "arcqml_rt_abi_version": (C.c_uint32, []),
    "arcqml_rt_v1_apply_gate": (_I32, [_P, _S, _S, _P, _P, _S]),
    "arcqml_rt_v1_apply_adjoint_gate": (_I32, [_P, _S, _S, _P, _P, _S]),
    "arcqml_rt_v1_parameter_derivative_into": (_I32, [_P, _S, _P, _S, _P, _P, _S, _S]),
    "arcqml_rt_v1_derivative_matrix_create": (_I32, [_P, _S, _P]),
    "arcqml_rt_v1_derivative_matrix_apply": (_I32, [_P, _S, _P, _P, _S]),
    "arcqml_rt_v1_derivative_matrix_destroy": (None, [_P]),
    "arcqml_rt_v1_circuit_plan_create": (_I32, [_P, _S, _P]),
    "arcqml_rt_v1_circuit_plan_create_empty": (_I32, [_S, _P]),
    "arcqml_rt_v1_circuit_plan_push": (_I32, [_P, _P]),
    "arcqml_rt_v1_circuit_plan_apply": (_I32, [_P, _P, _S, _S]),
    "arcqml_rt_v1_adjoint_backward": (_I32, [_P, _P, _P, _S, _P, _S, _D, _P, _S, _P, _S]),
    "arcqml_rt_v1_circuit_plan_destroy": (None, [_P]),
    "arcqml_rt_last_error": (_S, [_P, _S]),
    "arcqml_rt_v2_observable_create": (_I32, [_S, _P, _P, _P, _S, _P]),
    "arcqml_rt_v2_observable_destroy": (None, [_P]),
    "arcqml_rt_v2_plan_apply": (_I32, [_P, _P, _S, _S, _P]),
    "arcqml_rt_v2_apply_gate": (_I32, [_P, _S, _S, _P, _P, _S, _I32, _P]),
    "arcqml_rt_v2_parameter_derivative": (_I32, [_P, _P, _S, _S, _P, _P, _S, _S, _P]),
    "arcqml_rt_v2_expectation": (_I32, [_P, _P, _S, _S, _P, _P]),
    "arcqml_rt_v2_observable_tile_passes": (_I32, [_P, _S, _P]),
    "arcqml_rt_v2_expectation_and_apply": (_I32, [_P, _P, _P, _S, _S, _P, _P]),
    "arcqml_rt_v2_expectation_and_accumulate": (_I32, [_P, _P, _P, _S, _S, _P, _P]),
    "arcqml_rt_v2_sample": (_I32, [_P, _S, C.c_uint64, C.c_uint64, _P, _P, _P]),
    "arcqml_rt_v2_shard_slices": (_I32, [_P, _S, _P, _S, C.c_uint64, C.c_uint64, C.c_uint64, _P,
                                        _I32, _P]),
    "arcqml_rt_v2_small_run": (_I32, [_P, _P, _P, _S, _P, _S, _P, _S, _P, _P, _P]),
    "arcqml_rt_v2_plan_emulate": (_I32, [_P, _P, _S, _I32, _P, _P, _S, _P, _S]),
    "arcqml_rt_v2_plan_schedule_export": (_I32, [_P, _S, _I32, _P, _S, _P, _S, _P]),
    "arcqml_rt_v2_probabilities": (_I32, [_P, _S, _S, _P, _P]),
    "arcqml_rt_v2_marginal_probabilities": (_I32, [_P, _S, _S, _P, _S, _P, _P]),
    "arcqml_rt_v2_bloch_vector": (_I32, [_P, _S, _S, _S, _P, _P]),
    "arcqml_rt_v2_overlap": (_I32, [_P, _P, _S, _S, _P, _P]),
    "arcqml_rt_v2_probability_cotangent": (_I32, [_P, _S, _S, _P, _S, _P, _P, _P]),
    "arcqml_rt_v2_scaled_copy": (_I32, [_P, _S, _S, _P, _P, _P]),
    "arcqml_rt_v2_small_adam": (_I32, [_P, _P, _P, _S, _P, _P, _S, _P, _P, C.c_uint64, _S, _D,
                                      _D, _D, _D, _D, _P, _P]),
    "arcqml_rt_v2_shard_slices_from": (_I32, [_P, _S, _P, _S, C.c_uint64, C.c_uint64, _P, _P]),
    "arcqml_rt_v2_shard_swap_nccl": (_I32, [_P, _S, _P, _P, _S, _P, _P, _S, _P]),
    "arcqml_rt_v2_peer_buffer_create": (_I32, [_S, _P, _P]),
    "arcqml_rt_v2_peer_buffer_open": (_I32, [_P, _P]),
    "arcqml_rt_v2_peer_buffer_close": (_I32, [_P]),
    "arcqml_rt_v2_peer_buffer_destroy": (_I32, [_P]),
    "arcqml_rt_v2_adjoint_backward": (_I32, [_P, _P, _P, _S, _S, _P, _P, _S, _P, _S, _P]),
    "arcqml_rt_v2_norms": (_I32, [_P, _S, _S, _P, _P]),
    "arcqml_rt_v2_norms_noalloc": (_I32, [_P, _S, _S, _P, _P]),
    "arcqml_rt_v2_set_basis_state": (_I32, [_P, _S, _S, C.c_uint64, _P]),
    "arcqml_rt_v2_plan_set_parameters": (_I32, [_P, _P, _S]),
    "arcqml_rt_v2_plan_len": (_S, [_P]),
    "arcqml_rt_v2_plan_schedule_stats": (_I32, [_P, _S, _I32, _P, _P, _P]),
    "arcqml_rt_v2_profile_enable": (None, [_I32]),
    "arcqml_rt_v2_profile_read": (_I32, [C.c_uint32, _P, _P, _P]),
    "arcqml_rt_v2_launch_count": (C.c_uint64, []),
    "arcqml_rt_v2_jit_info": (_S, [_P, _P, _P, _P, _S]),
    "arcqml_rt_v2_plan_jit_check": (_I32, [_P, _S, _I32, _P, _P, _P, _S]),
}

_lib = None


def load():
    """Loads the runtime library (once). Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m arcqml_b200.build` "
            "(the statevector path has no CPU fallback)")
    L = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    L = load()
    n = L.arcqml_rt_last_error(None, 0)
    buf = (C.c_uint8 * (n + 1))()
    L.arcqml_rt_last_error(buf, n + 1)
    return bytes(buf[:n]).decode("utf-8", errors="replace")


def _status(code: int) -> None:
    if code != 0:
        raise RuntimeError(last_error())


def ensure_compatible() -> None:
    actual = load().arcqml_rt_abi_version()
    if actual != ABI_VERSION:
        raise RuntimeError(f"ArcQML runtime ABI mismatch: expected {ABI_VERSION}, got {actual}")


# ------------------------------------------------------------------ descriptors


class _Keep:
    """Owns the ctypes buffers a descriptor points into."""

    def __init__(self):
        self.items = []

    def add(self, x):
        self.items.append(x)
        return x


def gate_descriptor(opcode: int, arity: int, params=(0.0, 0.0, 0.0), matrix=None,
                    name: str = "", keep: Optional[_Keep] = None,
                    abi_version: int = ABI_VERSION) -> GateDescriptor:
    keep = keep if keep is not None else _Keep()
    g = GateDescriptor()
    g.abi_version = abi_version
    g.opcode = opcode
    g.arity = arity
    p = list(params) + [0.0] * (3 - len(params))
    for i in range(3):
        g.parameters[i] = float(p[i])
    if matrix is not None:
        m = keep.add(np.ascontiguousarray(np.asarray(matrix, dtype=np.complex128).ravel()))
        g.matrix = m.ctypes.data
        g.matrix_len = m.size
    if name:
        nb = keep.add(C.create_string_buffer(name.encode()))
        g.name = C.addressof(nb)
        g.name_len = len(name.encode())
    return g


def _op_descriptor(op: PlanOp, keep: _Keep) -> OperationDescriptor:
    d = OperationDescriptor()
    d.gate = gate_descriptor(op.opcode, len(op.qubits), op.params, op.matrix, op.name, keep)
    q = keep.add((C.c_size_t * max(1, len(op.qubits)))(*op.qubits))
    d.qubits = C.cast(q, C.POINTER(C.c_size_t))
    d.qubits_len = len(op.qubits)
    b = keep.add((ParameterBindingDescriptor * 3)())
    for i, (slot, parent) in enumerate(op.bindings):
        b[i].parameter_slot = slot
        b[i].parent_index = parent
    d.parameters = C.cast(b, C.POINTER(ParameterBindingDescriptor))
    d.parameters_len = len(op.bindings)
    return d


def _state_ptr(a: np.ndarray):
    if a.dtype != np.complex128 or not a.flags.c_contiguous:
        raise TypeError("amplitudes must be a C-contiguous complex128 array")
    return a.ctypes.data


def _qubits(qubits: Sequence[int]):
    return (C.c_size_t * max(1, len(qubits)))(*[int(q) for q in qubits])


# ------------------------------------------------------------------ v1 (host buffers)


def apply_gate(amplitudes: np.ndarray, num_qubits: int, gate: GateDescriptor,
               qubits: Sequence[int]) -> None:
    """arcqml_runtime_sys::apply_gate (lib.rs:137-153): in place."""
    _status(load().arcqml_rt_v1_apply_gate(_state_ptr(amplitudes), amplitudes.size, num_qubits,
                                          C.byref(gate), _qubits(qubits), len(qubits)))


def apply_adjoint_gate(amplitudes: np.ndarray, num_qubits: int, gate: GateDescriptor,
                       qubits: Sequence[int]) -> None:
    """arcqml_runtime_sys::apply_adjoint_gate (lib.rs:155-171): in place."""
    _status(load().arcqml_rt_v1_apply_adjoint_gate(_state_ptr(amplitudes), amplitudes.size,
                                                  num_qubits, C.byref(gate), _qubits(qubits),
                                                  len(qubits)))


def parameter_derivative_into(inp: np.ndarray, out: np.ndarray, gate: GateDescriptor,
                              qubits: Sequence[int], parameter_slot: int) -> None:
    """arcqml_runtime_sys::parameter_derivative_into (lib.rs:173-192)."""
    _status(load().arcqml_rt_v1_parameter_derivative_into(
        _state_ptr(inp), inp.size, _state_ptr(out), out.size, C.byref(gate), _qubits(qubits),
        len(qubits), parameter_slot))


class DerivativeMatrix:
    """arcqml_runtime_sys::DerivativeMatrix (lib.rs:194-232)."""

    def __init__(self, gate: GateDescriptor, parameter_slot: int):
        self.raw = DerivativeMatrixHandle()
        _status(load().arcqml_rt_v1_derivative_matrix_create(C.byref(gate), parameter_slot,
                                                           C.byref(self.raw)))

    @classmethod
    def create(cls, gate: GateDescriptor, parameter_slot: int) -> "DerivativeMatrix":
        return cls(gate, parameter_slot)

    def matrix(self) -> np.ndarray:
        n = self.raw.len
        dim = int(round(np.sqrt(n)))
        flat = np.ctypeslib.as_array(C.cast(self.raw.data, C.POINTER(C.c_double)), shape=(2 * n,))
        return (flat[0::2] + 1j * flat[1::2]).reshape(dim, dim).copy()

    def apply(self, amplitudes: np.ndarray, qubits: Sequence[int]) -> None:
        _status(load().arcqml_rt_v1_derivative_matrix_apply(
            _state_ptr(amplitudes), amplitudes.size, C.byref(self.raw), _qubits(qubits),
            len(qubits)))

    def __del__(self):
        if _lib is not None and getattr(self, "raw", None) is not None:
            _lib.arcqml_rt_v1_derivative_matrix_destroy(C.byref(self.raw))


class CircuitPlan:
    """arcqml_runtime_sys::CircuitPlan (lib.rs:234-320)."""

    def __init__(self, raw: CircuitPlanHandle):
        self.raw = raw

    @classmethod
    def create(cls, operations: Sequence[PlanOp]) -> "CircuitPlan":
        ensure_compatible()
        keep = _Keep()
        arr = (OperationDescriptor * max(1, len(operations)))()
        for i, op in enumerate(operations):
            arr[i] = _op_descriptor(op, keep)
        raw = CircuitPlanHandle()
        _status(load().arcqml_rt_v1_circuit_plan_create(arr, len(operations), C.byref(raw)))
        return cls(raw)

    @classmethod
    def with_capacity(cls, operation_capacity: int) -> "CircuitPlan":
        ensure_compatible()
        raw = CircuitPlanHandle()
        _status(load().arcqml_rt_v1_circuit_plan_create_empty(operation_capacity, C.byref(raw)))
        return cls(raw)

    @classmethod
    def compile(cls, ops: Sequence[PlanOp]) -> "CircuitPlan":
        """RuntimeCircuitPlan::compile: one push per operation, descriptors from temporaries."""
        plan = cls.with_capacity(len(ops))
        for op in ops:
            plan.push(op)
        return plan

    def push(self, op: PlanOp) -> None:
        keep = _Keep()
        d = _op_descriptor(op, keep)
        _status(load().arcqml_rt_v1_circuit_plan_push(C.byref(self.raw), C.byref(d)))
        del keep  # the runtime deep-copied everything

    def apply(self, amplitudes: np.ndarray, num_qubits: int) -> None:
        _status(load().arcqml_rt_v1_circuit_plan_apply(C.byref(self.raw), _state_ptr(amplitudes),
                                                      amplitudes.size, num_qubits))

    def adjoint_backward(self, forward_state: np.ndarray, adjoint_state: np.ndarray,
                         derivative_state: np.ndarray, num_qubits: int, upstream: float,
                         parameter_requires_grad: np.ndarray, gradients: np.ndarray) -> None:
        if not (forward_state.size == adjoint_state.size == derivative_state.size):
            raise RuntimeError("adjoint buffers must have identical lengths")
        req = np.ascontiguousarray(parameter_requires_grad, dtype=np.uint8)
        if gradients.dtype != np.float64 or not gradients.flags.c_contiguous:
            raise TypeError("gradients must be a C-contiguous float64 array")
        _status(load().arcqml_rt_v1_adjoint_backward(
            C.byref(self.raw), _state_ptr(forward_state), _state_ptr(adjoint_state),
            forward_state.size, _state_ptr(derivative_state), num_qubits, float(upstream),
            req.ctypes.data, req.size, gradients.ctypes.data, gradients.size))

    # -- v2 extensions on the same plan -------------------------------------------
    def set_parameters(self, parent_values: np.ndarray) -> None:
        v = np.ascontiguousarray(parent_values, dtype=np.float64)
        _status(load().arcqml_rt_v2_plan_set_parameters(C.byref(self.raw), v.ctypes.data, v.size))

    def jit_check(self, num_qubits: int, adjoint: bool = False) -> dict:
        """Compiles the run-time kernels of this plan's fused passes (NVRTC only, no GPU):
        {compiled, eligible, message}."""
        c, e = C.c_uint64(), C.c_uint64()
        buf = C.create_string_buffer(4096)
        _status(load().arcqml_rt_v2_plan_jit_check(C.byref(self.raw), num_qubits, int(adjoint),
                                                   C.byref(c), C.byref(e), buf, 4096))
        return {"compiled": int(c.value), "eligible": int(e.value),
                "message": buf.value.decode("utf-8", errors="replace")}

    def __len__(self) -> int:
        return load().arcqml_rt_v2_plan_len(C.byref(self.raw))

    def schedule_stats(self, num_qubits: int, adjoint: bool = False) -> dict:
        """Fused-pass schedule size for an n-qubit state (host only)."""
        a, b, c = C.c_uint64(), C.c_uint64(), C.c_uint64()
        _status(load().arcqml_rt_v2_plan_schedule_stats(C.byref(self.raw), num_qubits,
                                                        int(adjoint), C.byref(a), C.byref(b),
                                                        C.byref(c)))
        return {"passes": a.value, "sub_blocks": b.value, "gates": c.value}

    def __del__(self):
        if _lib is not None and getattr(self, "raw", None) is not None:
            _lib.arcqml_rt_v1_circuit_plan_destroy(C.byref(self.raw))


# ------------------------------------------------------------------ v2 (device states)


def _stream_ptr(stream) -> Optional[int]:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return int(stream)


def _dev_ptr(t) -> int:
    import torch
    if not (isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.complex128
            and t.is_contiguous()):
        raise TypeError("device amplitudes must be a contiguous complex128 CUDA tensor")
    return t.data_ptr()


def _dev_ptr_f64(t) -> int:
    import torch
    if not (isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float64
            and t.is_contiguous()):
        raise TypeError("device values must be a contiguous float64 CUDA tensor")
    return t.data_ptr()


def _rows(t, num_qubits: int) -> int:
    dim = 1 << num_qubits
    if t.numel() % dim != 0 or t.numel() == 0:
        raise RuntimeError(f"device state of {t.numel()} amplitudes is not [batch, {dim}]")
    return t.numel() // dim


class Observable:
    """Compiled Pauli observable on the runtime (arcqml_rt_v2_observable_*)."""

    def __init__(self, num_qubits: int, coefficients, flip_masks, phase_masks):
        c = np.ascontiguousarray(coefficients, dtype=np.float64)
        f = np.ascontiguousarray(flip_masks, dtype=np.uint64)
        p = np.ascontiguousarray(phase_masks, dtype=np.uint64)
        if not (c.size == f.size == p.size):
            raise ValueError("term arrays differ in length")
        self.num_qubits = num_qubits
        self.raw = ObservableHandle()
        _status(load().arcqml_rt_v2_observable_create(num_qubits, c.ctypes.data, f.ctypes.data,
                                                      p.ctypes.data, c.size, C.byref(self.raw)))

    @classmethod
    def from_sparse_pauli_op(cls, op) -> "Observable":
        c, f, p = op.masks()
        return cls(op.num_qubits, c, f, p)

    def expectation(self, state, num_qubits: int, stream=None) -> np.ndarray:
        b = _rows(state, num_qubits)
        out = np.zeros(b, dtype=np.float64)
        _status(load().arcqml_rt_v2_expectation(C.byref(self.raw), _dev_ptr(state), b, num_qubits,
                                                out.ctypes.data, _stream_ptr(stream)))
        return out

    def expectation_and_apply(self, state, out_state, num_qubits: int, stream=None) -> np.ndarray:
        b = _rows(state, num_qubits)
        vals = np.zeros(b, dtype=np.float64)
        _status(load().arcqml_rt_v2_expectation_and_apply(
            C.byref(self.raw), _dev_ptr(state), _dev_ptr(out_state), b, num_qubits,
            vals.ctypes.data, _stream_ptr(stream)))
        return vals

    def tile_passes(self, num_qubits: int) -> int:
        """Passes over 12-qubit tiles this observable takes on a num_qubits state (0: the gather
        kernel evaluates it)."""
        v = C.c_uint32()
        _status(load().arcqml_rt_v2_observable_tile_passes(C.byref(self.raw), num_qubits,
                                                           C.byref(v)))
        return int(v.value)

    def expectation_and_accumulate(self, state, out_state, num_qubits: int,
                                   stream=None) -> np.ndarray:
        """out_state += H psi; returns <psi|H|psi> per row."""
        b = _rows(state, num_qubits)
        vals = np.zeros(b, dtype=np.float64)
        _status(load().arcqml_rt_v2_expectation_and_accumulate(
            C.byref(self.raw), _dev_ptr(state), _dev_ptr(out_state), b, num_qubits,
            vals.ctypes.data, _stream_ptr(stream)))
        return vals

    def __del__(self):
        if _lib is not None and getattr(self, "raw", None) is not None:
            _lib.arcqml_rt_v2_observable_destroy(C.byref(self.raw))


def plan_apply_device(plan: CircuitPlan, state, num_qubits: int, stream=None) -> None:
    b = _rows(state, num_qubits)
    _status(load().arcqml_rt_v2_plan_apply(C.byref(plan.raw), _dev_ptr(state), b, num_qubits,
                                           _stream_ptr(stream)))


def apply_gate_device(state, num_qubits: int, gate: GateDescriptor, qubits, adjoint=False,
                      stream=None) -> None:
    b = _rows(state, num_qubits)
    _status(load().arcqml_rt_v2_apply_gate(_dev_ptr(state), b, num_qubits, C.byref(gate),
                                           _qubits(qubits), len(qubits), int(adjoint),
                                           _stream_ptr(stream)))


def parameter_derivative_device(inp, out, num_qubits: int, gate: GateDescriptor, qubits, slot,
                                stream=None) -> None:
    b = _rows(inp, num_qubits)
    _status(load().arcqml_rt_v2_parameter_derivative(
        _dev_ptr(inp), _dev_ptr(out), b, num_qubits, C.byref(gate), _qubits(qubits), len(qubits),
        slot, _stream_ptr(stream)))


def adjoint_backward_device(plan: CircuitPlan, psi, lam, num_qubits: int, upstream,
                            requires_grad, num_gradients: int, stream=None) -> np.ndarray:
    b = _rows(psi, num_qubits)
    up = np.ascontiguousarray(np.broadcast_to(np.asarray(upstream, dtype=np.float64), (b,)))
    req = np.ascontiguousarray(requires_grad, dtype=np.uint8)
    grads = np.zeros(num_gradients, dtype=np.float64)
    _status(load().arcqml_rt_v2_adjoint_backward(
        C.byref(plan.raw), _dev_ptr(psi), _dev_ptr(lam), b, num_qubits, up.ctypes.data,
        req.ctypes.data, req.size, grads.ctypes.data, grads.size, _stream_ptr(stream)))
    return grads


SMALL_MAX_QUBITS = 10


def small_run_device(plan: CircuitPlan, observable: "Observable", initial_state, num_qubits: int,
                     requires_grad, num_gradients: int, lambda0=None, stream=None):
    """One-kernel forward + <H> + adjoint (upstream 1) of a small single state; returns
    (value, gradients). initial_state: device tensor or None for |0...0>; lambda0: optional
    device tensor receiving lambda at the start of the circuit."""
    req = np.ascontiguousarray(requires_grad, dtype=np.uint8)
    grads = np.zeros(num_gradients, dtype=np.float64)
    value = C.c_double()
    _status(load().arcqml_rt_v2_small_run(
        C.byref(plan.raw), C.byref(observable.raw),
        None if initial_state is None else _dev_ptr(initial_state), num_qubits,
        req.ctypes.data, req.size, grads.ctypes.data, grads.size, C.byref(value),
        None if lambda0 is None else _dev_ptr(lambda0), _stream_ptr(stream)))
    return float(value.value), grads


class AdamState:
    """Moments of the device optimizer loop (per parent index) and the steps taken so far."""

    def __init__(self, num_parameters: int):
        self.m = np.zeros(num_parameters, dtype=np.float64)
        self.v = np.zeros(num_parameters, dtype=np.float64)
        self.step = 0

    def update(self, values, grads, lr: float = 0.05, betas=(0.9, 0.999), eps: float = 1e-8,
               weight_decay: float = 0.0) -> np.ndarray:
        """One f64 Adam step on the host (crates/arcqml-optim/src/adam.rs:190-240: coupled L2
        weight decay, bias-corrected moments); advances the moments in place and returns the
        new values. The same update the device loop (`small_adam_device`) applies per step."""
        x = np.asarray(values, dtype=np.float64)
        g = np.asarray(grads, dtype=np.float64)
        if x.shape != self.m.shape or g.shape != self.m.shape:
            raise ValueError("values and grads must match the AdamState size")
        self.step += 1
        b1, b2 = float(betas[0]), float(betas[1])
        a = g + weight_decay * x
        self.m = b1 * self.m + (1.0 - b1) * a
        self.v = b2 * self.v + (1.0 - b2) * (a * a)
        m_hat = self.m / (1.0 - b1 ** self.step)
        v_hat = self.v / (1.0 - b2 ** self.step)
        return x - lr * m_hat / (np.sqrt(v_hat) + eps)


def small_adam_device(plan: CircuitPlan, observable: "Observable", num_qubits: int, parameters,
                      requires_grad, steps: int, lr: float = 0.05,
                      betas=(0.9, 0.999), eps: float = 1e-8, weight_decay: float = 0.0,
                      initial_state=None, state: "AdamState" = None, stream=None):
    """`steps` Adam steps of <H> in one launch (arcqml_rt_v2_small_adam): per step forward, <H>,
    adjoint gradient and the f64 Adam update on the device. parameters and requires_grad are
    indexed by parent (entry 0: the initial-state slot). Returns (energies before each update,
    parameters after the last one); `state` (AdamState) is advanced in place when given."""
    req = np.ascontiguousarray(requires_grad, dtype=np.uint8)
    params = np.array(parameters, dtype=np.float64, copy=True)
    if params.shape != req.shape:
        raise ValueError("parameters and requires_grad must have the same length")
    energies = np.zeros(max(int(steps), 0), dtype=np.float64)
    if state is not None and (state.m.size != params.size or state.v.size != params.size):
        raise ValueError("AdamState size does not match the parameters")
    _status(load().arcqml_rt_v2_small_adam(
        C.byref(plan.raw), C.byref(observable.raw),
        None if initial_state is None else _dev_ptr(initial_state), num_qubits,
        req.ctypes.data, params.ctypes.data, params.size,
        None if state is None else state.m.ctypes.data,
        None if state is None else state.v.ctypes.data,
        0 if state is None else int(state.step), int(steps), float(lr), float(betas[0]),
        float(betas[1]), float(eps), float(weight_decay),
        energies.ctypes.data if energies.size else None, _stream_ptr(stream)))
    if state is not None:
        state.step += int(steps)
    return energies, params


def norms_device(state, num_qubits: int, stream=None) -> np.ndarray:
    b = _rows(state, num_qubits)
    out = np.zeros(b, dtype=np.float64)
    _status(load().arcqml_rt_v2_norms(_dev_ptr(state), b, num_qubits, out.ctypes.data,
                                      _stream_ptr(stream)))
    return out


def norms_device_noalloc(state, num_qubits: int, stream=None) -> np.ndarray:
    """Row norms through the entry point that allocates no device memory (see its header)."""
    b = _rows(state, num_qubits)
    out = np.zeros(b, dtype=np.float64)
    _status(load().arcqml_rt_v2_norms_noalloc(_dev_ptr(state), b, num_qubits, out.ctypes.data,
                                              _stream_ptr(stream)))
    return out


def set_basis_state_device(state, num_qubits: int, index: int = 0, stream=None) -> None:
    b = _rows(state, num_qubits)
    _status(load().arcqml_rt_v2_set_basis_state(_dev_ptr(state), b, num_qubits, index,
                                                _stream_ptr(stream)))


# ------------------------------------------------------------------ kernel timing

PROFILE_CATEGORIES = ("gate", "fused_forward", "fused_adjoint", "adjoint_step", "observable",
                      "other", "shard_slices")


def sample_indices_device(state, num_qubits: int, shots: int, seed: int, stream=None):
    """Basis index of every shot (numpy uint64) and the state's norm squared; see
    arcqml_rt_v2_sample (bit-exact with the reference's sample_counts)."""
    out = np.zeros(max(int(shots), 1), dtype=np.uint64)
    norm = C.c_double()
    _status(load().arcqml_rt_v2_sample(_dev_ptr(state), num_qubits, int(shots),
                                       int(seed) & ((1 << 64) - 1), out.ctypes.data,
                                       C.byref(norm), _stream_ptr(stream)))
    return out[:int(shots)], float(norm.value)


def shard_slices(shard, num_local_qubits: int, positions: Sequence[int], chunk_begin: int,
                 chunk_len: int, skip_value: int, staging, unpack: bool, stream=None) -> None:
    """Moves slices of a shard to (unpack=False) or from (unpack=True) contiguous staging
    blocks, one block per slice value other than ``skip_value`` (see arcqml_rt_v2_shard_slices)."""
    pos = (C.c_uint32 * len(positions))(*positions)
    _status(load().arcqml_rt_v2_shard_slices(
        _dev_ptr(shard), num_local_qubits, pos, len(positions), chunk_begin, chunk_len,
        skip_value, _dev_ptr(staging), int(bool(unpack)), _stream_ptr(stream)))


def shard_slices_from(shard, num_local_qubits: int, positions: Sequence[int], chunk_begin: int,
                      chunk_len: int, sources: Sequence[Optional[int]], stream=None) -> None:
    """Gathers slice value y of a chunk from device address sources[y] (None: skip) into the
    shard (see arcqml_rt_v2_shard_slices_from)."""
    pos = (C.c_uint32 * len(positions))(*positions)
    src = (C.c_void_p * len(sources))(*[s if s else None for s in sources])
    _status(load().arcqml_rt_v2_shard_slices_from(
        _dev_ptr(shard), num_local_qubits, pos, len(positions), chunk_begin, chunk_len, src,
        _stream_ptr(stream)))


def shard_swap_nccl(shard, num_local_qubits: int, global_bits: Sequence[int],
                    local_positions: Sequence[int], nccl_comm: int, staging,
                    stream=None) -> None:
    """Swaps the global qubits at rank bits global_bits[i] with the shard's local positions
    local_positions[i] over a raw NCCL communicator (arcqml_rt_v2_shard_swap_nccl); staging is a
    complex128 CUDA tensor of scratch amplitudes."""
    gb = (C.c_uint32 * len(global_bits))(*global_bits)
    lp = (C.c_uint32 * len(local_positions))(*local_positions)
    _status(load().arcqml_rt_v2_shard_swap_nccl(
        _dev_ptr(shard), num_local_qubits, gb, lp, len(global_bits), C.c_void_p(nccl_comm),
        _dev_ptr(staging), staging.numel(), _stream_ptr(stream)))


def shard_slices_ptr(shard, num_local_qubits: int, positions: Sequence[int], chunk_begin: int,
                     chunk_len: int, skip_value: int, staging_address: int, unpack: bool,
                     stream=None) -> None:
    """shard_slices with the staging buffer given as a raw device address."""
    pos = (C.c_uint32 * len(positions))(*positions)
    _status(load().arcqml_rt_v2_shard_slices(
        _dev_ptr(shard), num_local_qubits, pos, len(positions), chunk_begin, chunk_len,
        skip_value, C.c_void_p(staging_address), int(bool(unpack)), _stream_ptr(stream)))


class PeerBuffer:
    """A device buffer other processes of the node can map (CUDA IPC)."""

    def __init__(self, nbytes: int):
        ptr = C.c_void_p()
        self.handle = (C.c_uint8 * 64)()
        _status(load().arcqml_rt_v2_peer_buffer_create(nbytes, C.byref(ptr), self.handle))
        self.address = int(ptr.value)
        self.nbytes = nbytes

    def handle_bytes(self) -> bytes:
        return bytes(self.handle)

    @staticmethod
    def open(handle: bytes) -> int:
        ptr = C.c_void_p()
        h = (C.c_uint8 * 64)(*handle)
        _status(load().arcqml_rt_v2_peer_buffer_open(h, C.byref(ptr)))
        return int(ptr.value)

    @staticmethod
    def close(address: int) -> None:
        _status(load().arcqml_rt_v2_peer_buffer_close(C.c_void_p(address)))

    def destroy(self) -> None:
        if self.address:
            _status(load().arcqml_rt_v2_peer_buffer_destroy(C.c_void_p(self.address)))
            self.address = 0


def profile_enable(on: bool = True) -> None:
    """Bracket the runtime's kernel launches with CUDA events (resets the totals)."""
    load().arcqml_rt_v2_profile_enable(int(on))


def profile_read() -> dict:
    """{category: (launches, total_ms, algorithmic_bytes)} since the last profile_enable."""
    out = {}
    for i, name in enumerate(PROFILE_CATEGORIES):
        n = C.c_uint64()
        ms = C.c_double()
        by = C.c_double()
        _status(load().arcqml_rt_v2_profile_read(i, C.byref(n), C.byref(ms), C.byref(by)))
        out[name] = (int(n.value), float(ms.value), float(by.value))
    return out


def launch_count() -> int:
    return int(load().arcqml_rt_v2_launch_count())


def jit_info() -> dict:
    """Run-time compiled pass kernels: {compiled, launches, fallbacks, last_error}."""
    c, l, f = C.c_uint64(), C.c_uint64(), C.c_uint64()
    buf = C.create_string_buffer(4096)
    load().arcqml_rt_v2_jit_info(C.byref(c), C.byref(l), C.byref(f), buf, 4096)
    return {"compiled": int(c.value), "launches": int(l.value), "fallbacks": int(f.value),
            "last_error": buf.value.decode("utf-8", errors="replace")}


def plan_emulate(plan: CircuitPlan, state, num_qubits: int, adjoint: bool = False, lam=None,
                 requires_grad=None, num_gradients: int = 0):
    """The engine's fused-pass schedule run on the CPU (arcqml_rt_v2_plan_emulate): returns the
    new state, or (psi, lambda, gradients) for the adjoint sweep. numpy complex128 inputs."""
    a = np.ascontiguousarray(state, dtype=np.complex128).copy()
    if not adjoint:
        _status(load().arcqml_rt_v2_plan_emulate(C.byref(plan.raw), a.ctypes.data, num_qubits, 0,
                                                 None, None, 0, None, 0))
        return a
    lm = np.ascontiguousarray(lam, dtype=np.complex128).copy()
    req = np.ascontiguousarray(requires_grad, dtype=np.uint8)
    grads = np.zeros(num_gradients, dtype=np.float64)
    _status(load().arcqml_rt_v2_plan_emulate(C.byref(plan.raw), a.ctypes.data, num_qubits, 1,
                                             lm.ctypes.data, req.ctypes.data, req.size,
                                             grads.ctypes.data, grads.size))
    return a, lm, grads


def plan_structure_key(ops: Sequence[PlanOp]) -> tuple:
    """What a plan holds besides its bound parameter values: per operation the opcode, qubits,
    parameter bindings, constant slot values and custom matrix. Plans with equal keys differ
    only in values that CircuitPlan.set_parameters replaces."""
    key = []
    for o in ops:
        bound = {slot for slot, _ in o.bindings}
        fixed = tuple(v for i, v in enumerate(o.params) if i not in bound)
        mat = None if o.matrix is None else np.asarray(o.matrix, dtype=np.complex128).tobytes()
        key.append((o.opcode, tuple(o.qubits), tuple(o.bindings), fixed, mat))
    return tuple(key)


def plan_bound_values(ops: Sequence[PlanOp]) -> Optional[np.ndarray]:
    """The parent values the operations' bindings carry (index = parent), for
    CircuitPlan.set_parameters; None when one parent carries two different values."""
    vals = {}
    for o in ops:
        for slot, parent in o.bindings:
            v = float(o.params[slot])
            if vals.setdefault(int(parent), v) != v:
                return None
    out = np.zeros(max(vals) + 1 if vals else 0)
    for p, v in vals.items():
        out[p] = v
    return out


def plan_schedule_export(plan: CircuitPlan, num_qubits: int, adjoint: bool = False,
                         requires_grad=None) -> bytes:
    """The engine's fused-pass schedule for the plan, serialised (arcqml_rt_v2_plan_schedule_export)."""
    req = np.ascontiguousarray([] if requires_grad is None else requires_grad, dtype=np.uint8)
    rp = req.ctypes.data if req.size else None
    size = C.c_size_t()
    _status(load().arcqml_rt_v2_plan_schedule_export(C.byref(plan.raw), num_qubits, int(adjoint),
                                                     rp, req.size, None, 0, C.byref(size)))
    buf = (C.c_uint8 * max(1, size.value))()
    _status(load().arcqml_rt_v2_plan_schedule_export(C.byref(plan.raw), num_qubits, int(adjoint),
                                                     rp, req.size, buf, size.value, C.byref(size)))
    return bytes(buf)[:size.value]


def plan_schedule_summary(plan: CircuitPlan, num_qubits: int, adjoint: bool = False,
                          requires_grad=None) -> dict:
    """Counts over the engine's fused-pass schedule (plan_schedule_export): passes, ops executed,
    rotation ops (one-qubit RX/RY forms and one-qubit phase diagonals, the ops whose FP64 work
    the scaled forms make one FMA per amplitude component), gradient rows and the further
    parameters that merged rotations add to a row. Layouts: arcqml_b200/csrc/fused.h."""
    blob = plan_schedule_export(plan, num_qubits, adjoint, requires_grad)
    off = 0

    def u32():
        nonlocal off
        v = int.from_bytes(blob[off:off + 4], "little")
        off += 4
        return v

    out = {"passes": 0, "ops": 0, "rotations": 0, "rows": 0, "aliases": 0, "custom": 0}
    for _ in range(u32()):
        if not u32():
            u32()
            out["custom"] += 1
            continue
        out["passes"] += 1
        off += 48                       # PassHeader
        nsub = u32()
        off += 24 * nsub                # SubBlocks
        nops = u32()
        for i in range(nops):           # FOp: kind at byte 0, code at byte 28
            kind, code = blob[off + 64 * i], blob[off + 64 * i + 28]
            if kind in (1, 2) or (kind == 3 and code in (4, 5)):
                out["rotations"] += 1
        out["ops"] += nops
        off += 64 * nops
        nmat = u32()
        off += 16 * nmat                # matrix entries
        rows = u32()
        out["rows"] += rows
        off += 8 * rows
        nal = u32()
        out["aliases"] += nal
        off += 16 * nal
        ncode = u32()
        off += ncode                    # compiled source
    if off != len(blob):
        raise RuntimeError("schedule export: unexpected length")
    return out


# ---------------------------------------------------------------- state analysis


def _selection(qubits):
    q = np.ascontiguousarray([int(x) for x in qubits], dtype=np.uintp)
    return q, (q.ctypes.data if q.size else None)


def probabilities_device(state, num_qubits: int, out=None, stream=None):
    """|psi_i|^2 of every row (arcqml_rt_v2_probabilities): a float64 CUDA tensor shaped like
    the state."""
    import torch
    b = _rows(state, num_qubits)
    if out is None:
        out = torch.empty(state.shape, dtype=torch.float64, device=state.device)
    _status(load().arcqml_rt_v2_probabilities(_dev_ptr(state), b, num_qubits, _dev_ptr_f64(out),
                                              _stream_ptr(stream)))
    return out


def marginal_probabilities_device(state, num_qubits: int, qubits, out=None, stream=None):
    """Marginal probabilities of the selected qubits (highest selected qubit as the most
    significant output bit) for every row: float64 CUDA tensor [2^k] or [batch, 2^k]."""
    import torch
    b = _rows(state, num_qubits)
    q, qp = _selection(qubits)
    if qp is None:  # empty selection: rejected by the runtime with the reference's message
        q = np.zeros(1, dtype=np.uintp)
        qp = q.ctypes.data
        q = q[:0]
    if out is None:
        shape = (1 << q.size,) if state.dim() == 1 else (b, 1 << q.size)
        out = torch.empty(shape, dtype=torch.float64, device=state.device)
    _status(load().arcqml_rt_v2_marginal_probabilities(
        _dev_ptr(state), b, num_qubits, qp, q.size, _dev_ptr_f64(out), _stream_ptr(stream)))
    return out


def bloch_vector_device(state, num_qubits: int, qubit: int, stream=None) -> np.ndarray:
    """(<X>, <Y>, <Z>) of one qubit per row: numpy [3] or [batch, 3]."""
    b = _rows(state, num_qubits)
    out = np.zeros((b, 3), dtype=np.float64)
    _status(load().arcqml_rt_v2_bloch_vector(_dev_ptr(state), b, num_qubits, int(qubit),
                                             out.ctypes.data, _stream_ptr(stream)))
    return out[0] if state.dim() == 1 else out


def overlap_device(lhs, rhs, num_qubits: int, stream=None):
    """<lhs|rhs> per row: a complex (1-D states) or a numpy complex array [batch]."""
    b = _rows(lhs, num_qubits)
    if rhs.shape != lhs.shape:
        raise RuntimeError("overlap of states with different shapes")
    out = np.zeros((b, 2), dtype=np.float64)
    _status(load().arcqml_rt_v2_overlap(_dev_ptr(lhs), _dev_ptr(rhs), b, num_qubits,
                                        out.ctypes.data, _stream_ptr(stream)))
    z = out[:, 0] + 1j * out[:, 1]
    return complex(z[0]) if lhs.dim() == 1 else z


def probability_cotangent_device(state, num_qubits: int, upstream, qubits=None, out=None,
                                 stream=None):
    """lambda_i = upstream[bin(i)] psi_i per row (arcqml_rt_v2_probability_cotangent): the
    adjoint sweep's lambda for an upstream gradient of the (marginal) probabilities; qubits=None
    for the full probability vector. upstream: float64 CUDA tensor [batch, 2^k] (or [2^k])."""
    import torch
    b = _rows(state, num_qubits)
    if qubits is None:
        q, qp, k = None, None, num_qubits
    else:
        # an explicit empty selection keeps a non-null pointer: the runtime rejects it
        q = np.ascontiguousarray([int(x) for x in qubits] or [0], dtype=np.uintp)
        qp, k = q.ctypes.data, len(list(qubits))
    if upstream.numel() != b << k:
        raise RuntimeError(f"upstream has {upstream.numel()} values, expected {b << k}")
    if out is None:
        out = torch.empty_like(state)
    _status(load().arcqml_rt_v2_probability_cotangent(
        _dev_ptr(state), b, num_qubits, qp, 0 if qubits is None else k, _dev_ptr_f64(upstream),
        _dev_ptr(out), _stream_ptr(stream)))
    return out


def scaled_copy_device(state, num_qubits: int, factors, out=None, stream=None):
    """out[row] = factors[row] * state[row] with complex factors (arcqml_rt_v2_scaled_copy)."""
    import torch
    b = _rows(state, num_qubits)
    f = np.asarray(factors, dtype=np.complex128).reshape(-1)
    if f.size == 1 and b > 1:
        f = np.full(b, f[0])
    if f.size != b:
        raise RuntimeError(f"{f.size} factors for {b} rows")
    fr = np.ascontiguousarray(np.stack([f.real, f.imag], axis=1).reshape(-1))
    if out is None:
        out = torch.empty_like(state)
    _status(load().arcqml_rt_v2_scaled_copy(_dev_ptr(state), b, num_qubits, fr.ctypes.data,
                                            _dev_ptr(out), _stream_ptr(stream)))
    return out
