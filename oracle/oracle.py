"""Python view of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU baseline / reference arm may
import this module. It loads ``oracle/liboracle.so`` (built by ``oracle/Makefile``), a plain-C f64
restatement of ArcQML's statevector path; see ``oracle/oracle.h`` for what it restates and how
it is pinned to the reference's known-answer tests.

Operations are duck-typed: any object with ``opcode``, ``qubits``, ``params`` (3 floats),
``matrix`` (complex128 array or None) and ``bindings`` (sequence of ``(slot, parent)``) works, so
the same operation lists feed the oracle and the runtime under test.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")


class _C128(C.Structure):
    _fields_ = [("re", C.c_double), ("im", C.c_double)]


class _Op(C.Structure):
    _fields_ = [
        ("opcode", C.c_uint32),
        ("arity", C.c_uint32),
        ("params", C.c_double * 3),
        ("matrix", C.c_void_p),
        ("qubits", C.POINTER(C.c_size_t)),
        ("num_bindings", C.c_uint32),
        ("slots", C.c_size_t * 3),
        ("parents", C.c_size_t * 3),
    ]


class _Term(C.Structure):
    _fields_ = [
        ("coefficient", C.c_double),
        ("flip_mask", C.c_uint64),
        ("phase_mask", C.c_uint64),
        ("y_count_mod_four", C.c_uint32),
    ]


def build() -> str:
    """Compile liboracle.so with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE, "liboracle.so"], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        P = C.c_void_p
        L.oracle_plan_apply.argtypes = [P, C.c_size_t, P, C.c_uint32]
        L.oracle_apply_gate.argtypes = [P, C.c_uint32, P, C.c_int]
        L.oracle_parameter_derivative.argtypes = [P, P, C.c_uint32, P, C.c_size_t]
        L.oracle_adjoint_backward.argtypes = [P, C.c_size_t, P, P, C.c_uint32, C.c_double, P,
                                              C.c_size_t, P, C.c_size_t]
        L.oracle_batch_plan_apply.argtypes = [P, C.c_size_t, P, C.c_size_t, C.c_uint32]
        L.oracle_batch_adjoint_backward.argtypes = [P, C.c_size_t, P, P, C.c_size_t, C.c_uint32,
                                                    P, P, C.c_size_t, P, C.c_size_t]
        L.oracle_expectation.argtypes = [P, C.c_size_t, P, C.c_uint32]
        L.oracle_expectation.restype = C.c_double
        L.oracle_expectation_and_apply.argtypes = [P, C.c_size_t, P, P, C.c_uint32]
        L.oracle_expectation_and_apply.restype = C.c_double
        L.oracle_apply_hamiltonian.argtypes = [P, C.c_size_t, P, P, C.c_uint32]
        L.oracle_gate_matrix.argtypes = [C.c_uint32, C.c_uint32, P, P, P]
        L.oracle_derivative_matrix.argtypes = [C.c_uint32, C.c_uint32, P, C.c_size_t, P]
        L.oracle_sample_indices.argtypes = [P, C.c_uint32, C.c_uint64, C.c_uint64, P]
        L.oracle_chacha_block.argtypes = [P, C.c_uint64, C.c_uint64, C.c_int, P]
        L.oracle_stdrng_key.argtypes = [C.c_uint64, P]
        L.oracle_stdrng_u64.argtypes = [C.c_uint64, C.c_uint64]
        L.oracle_stdrng_u64.restype = C.c_uint64
        L.oracle_probabilities.argtypes = [P, C.c_uint32, P]
        L.oracle_marginal_probabilities.argtypes = [P, C.c_uint32, P, C.c_size_t, P]
        L.oracle_bloch_vector.argtypes = [P, C.c_uint32, C.c_uint32, P]
        L.oracle_overlap_fidelity.argtypes = [P, P, C.c_uint32, P]
        L.oracle_num_threads.restype = C.c_int
        L.oracle_set_num_threads.argtypes = [C.c_int]
        _lib = L
    return _lib


def num_threads() -> int:
    return lib().oracle_num_threads()


def set_num_threads(n: int) -> None:
    lib().oracle_set_num_threads(int(n))


class _Packed:
    """Keeps the ctypes arrays of an operation list alive while the oracle runs."""

    def __init__(self, ops):
        ops = list(ops)
        self.n = len(ops)
        self.arr = (_Op * max(1, self.n))()
        self.keep = []
        for i, op in enumerate(ops):
            o = self.arr[i]
            o.opcode = int(op.opcode)
            o.arity = len(op.qubits)
            for j, p in enumerate(tuple(op.params)[:3]):
                o.params[j] = float(p)
            q = (C.c_size_t * len(op.qubits))(*[int(x) for x in op.qubits])
            self.keep.append(q)
            o.qubits = C.cast(q, C.POINTER(C.c_size_t))
            if op.matrix is not None:
                m = np.ascontiguousarray(np.asarray(op.matrix, dtype=np.complex128).ravel())
                self.keep.append(m)
                o.matrix = m.ctypes.data
            else:
                o.matrix = None
            b = list(op.bindings)
            o.num_bindings = len(b)
            for j, (slot, parent) in enumerate(b):
                o.slots[j] = int(slot)
                o.parents[j] = int(parent)

    @property
    def ptr(self):
        return C.addressof(self.arr)


def _terms(terms):
    """terms: iterable of (coefficient, flip_mask, phase_mask, y_count_mod_four)."""
    terms = list(terms)
    arr = (_Term * max(1, len(terms)))()
    for i, (c, f, p, y) in enumerate(terms):
        arr[i].coefficient = float(c)
        arr[i].flip_mask = int(f)
        arr[i].phase_mask = int(p)
        arr[i].y_count_mod_four = int(y) % 4
    return arr, len(terms)


def _state(a):
    a = np.ascontiguousarray(a, dtype=np.complex128)
    return a


def gate_matrix(opcode, arity, params=(0.0, 0.0, 0.0), custom=None):
    dim = 1 << arity
    out = np.zeros(dim * dim, dtype=np.complex128)
    p = (C.c_double * 3)(*[float(x) for x in tuple(params)[:3]] + [0.0] * (3 - len(tuple(params)[:3])))
    cm = None if custom is None else np.ascontiguousarray(np.asarray(custom, np.complex128).ravel())
    rc = lib().oracle_gate_matrix(opcode, arity, p, None if cm is None else cm.ctypes.data,
                                  out.ctypes.data)
    if rc != 0:
        raise ValueError(f"oracle: no matrix for opcode {opcode} arity {arity}")
    return out.reshape(dim, dim)


def derivative_matrix(opcode, arity, params, slot):
    dim = 1 << arity
    out = np.zeros(dim * dim, dtype=np.complex128)
    p = (C.c_double * 3)(*[float(x) for x in tuple(params)[:3]])
    if lib().oracle_derivative_matrix(opcode, arity, p, slot, out.ctypes.data) != 0:
        raise ValueError(f"oracle: opcode {opcode} has no parameter slot {slot}")
    return out.reshape(dim, dim)


def apply_gate(amps, num_qubits, op, adjoint=False):
    a = _state(amps).copy()
    pk = _Packed([op])
    if lib().oracle_apply_gate(a.ctypes.data, num_qubits, pk.ptr, int(adjoint)) != 0:
        raise ValueError("oracle: invalid gate")
    return a


def parameter_derivative(amps, num_qubits, op, slot):
    a = _state(amps)
    out = np.empty_like(a)
    pk = _Packed([op])
    if lib().oracle_parameter_derivative(a.ctypes.data, out.ctypes.data, num_qubits, pk.ptr, slot) != 0:
        raise ValueError("oracle: invalid derivative")
    return out


def plan_apply(ops, amps, num_qubits, batch=1):
    a = _state(amps).copy()
    pk = _Packed(ops)
    if batch == 1:
        rc = lib().oracle_plan_apply(pk.ptr, pk.n, a.ctypes.data, num_qubits)
    else:
        rc = lib().oracle_batch_plan_apply(pk.ptr, pk.n, a.ctypes.data, batch, num_qubits)
    if rc != 0:
        raise ValueError("oracle: invalid plan")
    return a


def adjoint_backward(ops, psi, lam, num_qubits, upstream, requires_grad, num_grads=None, batch=1):
    """Returns (psi_0, g*lambda_0, grads); grads summed over rows for batch > 1."""
    psi = _state(psi).copy()
    lam = _state(lam).copy()
    req = np.ascontiguousarray(np.asarray(requires_grad, dtype=np.uint8))
    ng = len(req) if num_grads is None else num_grads
    grads = np.zeros(ng, dtype=np.float64)
    pk = _Packed(ops)
    if batch == 1:
        rc = lib().oracle_adjoint_backward(pk.ptr, pk.n, psi.ctypes.data, lam.ctypes.data,
                                           num_qubits, float(upstream), req.ctypes.data, len(req),
                                           grads.ctypes.data, ng)
    else:
        up = np.ascontiguousarray(np.asarray(upstream, dtype=np.float64))
        rc = lib().oracle_batch_adjoint_backward(pk.ptr, pk.n, psi.ctypes.data, lam.ctypes.data,
                                                 batch, num_qubits, up.ctypes.data,
                                                 req.ctypes.data, len(req), grads.ctypes.data, ng)
    if rc != 0:
        raise ValueError("oracle: invalid adjoint call")
    return psi, lam, grads


def expectation(terms, amps, num_qubits):
    arr, nt = _terms(terms)
    a = _state(amps)
    return lib().oracle_expectation(C.addressof(arr), nt, a.ctypes.data, num_qubits)


def expectation_and_apply(terms, amps, num_qubits):
    arr, nt = _terms(terms)
    a = _state(amps)
    out = np.empty_like(a)
    v = lib().oracle_expectation_and_apply(C.addressof(arr), nt, a.ctypes.data, out.ctypes.data,
                                           num_qubits)
    return v, out


def apply_hamiltonian(terms, amps, num_qubits):
    arr, nt = _terms(terms)
    a = _state(amps)
    out = np.empty_like(a)
    lib().oracle_apply_hamiltonian(C.addressof(arr), nt, a.ctypes.data, out.ctypes.data, num_qubits)
    return out


def sample_indices(amps, num_qubits, shots, seed):
    """Basis index of every shot of sample_counts(shots, seed)
    (crates/arcqml-sim/src/statevector/api/measurement.rs:18-60)."""
    a = _state(amps)
    out = np.zeros(int(shots), dtype=np.uint64)
    if lib().oracle_sample_indices(a.ctypes.data, num_qubits, int(shots), int(seed),
                                   out.ctypes.data) != 0:
        raise ValueError("oracle: invalid sampling call")
    return out


def sample_counts(amps, num_qubits, shots, seed):
    """{bitstring q[n-1]..q0: count} sorted by bitstring, as the reference's BTreeMap."""
    idx = sample_indices(amps, num_qubits, shots, seed)
    vals, cnt = np.unique(idx, return_counts=True)
    d = {format(int(v), f"0{num_qubits}b"): int(c) for v, c in zip(vals, cnt)}
    return dict(sorted(d.items()))


def chacha_block(key, counter, stream=0, rounds=20):
    k = (C.c_uint32 * 8)(*key)
    out = (C.c_uint32 * 16)()
    lib().oracle_chacha_block(k, counter, stream, rounds, out)
    return list(out)


def stdrng_key(seed):
    k = (C.c_uint32 * 8)()
    lib().oracle_stdrng_key(seed, k)
    return list(k)


def stdrng_u64(seed, k):
    return int(lib().oracle_stdrng_u64(seed, k))


def adam_step(values, grads, state, lr=0.05, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0):
    """F64 Adam, crates/arcqml-optim/src/adam.rs:190-240 (coupled L2, bias-corrected)."""
    state["step"] = state.get("step", 0) + 1
    t = state["step"]
    first = state.setdefault("first", np.zeros_like(values))
    second = state.setdefault("second", np.zeros_like(values))
    b1c = 1.0 - beta1 ** t
    b2c = 1.0 - beta2 ** t
    out = values.copy()
    for i in range(len(values)):
        adjusted = grads[i] + weight_decay * out[i]
        first[i] = beta1 * first[i] + (1.0 - beta1) * adjusted
        second[i] = beta2 * second[i] + (1.0 - beta2) * adjusted * adjusted
        first_hat = first[i] / b1c
        second_hat = second[i] / b2c
        out[i] -= lr * first_hat / (np.sqrt(second_hat) + eps)
    return out


# ---------------------------------------------------------------- analysis
# crates/arcqml-analysis/src/statevector/{probabilities,marginal,bloch,fidelity}.rs


def probabilities(amps, num_qubits):
    """|psi_i|^2 as square(abs(psi_i)) (probabilities.rs:22-25)."""
    a = _state(amps)
    out = np.zeros(1 << num_qubits, dtype=np.float64)
    lib().oracle_probabilities(a.ctypes.data, num_qubits, out.ctypes.data)
    return out


def marginal_probabilities(amps, num_qubits, qubits):
    """Segment sums of the probabilities over the selected qubits, output bits in descending
    qubit order (marginal.rs:17-67); ValueError for an invalid selection."""
    a = _state(amps)
    q = np.ascontiguousarray(qubits, dtype=np.uint32)
    out = np.zeros(1 << max(len(q), 0), dtype=np.float64)
    rc = lib().oracle_marginal_probabilities(a.ctypes.data, num_qubits, q.ctypes.data, q.size,
                                            out.ctypes.data)
    if rc:
        raise ValueError("oracle: invalid qubit selection")
    return out


def bloch_vector(amps, num_qubits, qubit):
    """(<X>, <Y>, <Z>) of one qubit (bloch.rs:23-56)."""
    a = _state(amps)
    out = np.zeros(3, dtype=np.float64)
    if lib().oracle_bloch_vector(a.ctypes.data, num_qubits, int(qubit), out.ctypes.data):
        raise ValueError("oracle: qubit out of range")
    return out


def overlap_fidelity(lhs, rhs, num_qubits):
    """(<lhs|rhs>, |<lhs|rhs>|^2) (fidelity.rs:14-30)."""
    a, b = _state(lhs), _state(rhs)
    out = np.zeros(3, dtype=np.float64)
    lib().oracle_overlap_fidelity(a.ctypes.data, b.ctypes.data, num_qubits, out.ctypes.data)
    return complex(out[0], out[1]), float(out[2])
