"""Two interchangeable executors of the statevector path for the parity tests.

``OracleBackend`` runs the CPU oracle (oracle/liboracle.so); ``RuntimeBackend`` runs the sm_100a
runtime through its v1 C ABI with host buffers, exactly as ArcQML's ``arcqml-runtime-sys``
would call it. The reference test restatements in ``reference_cases.py`` take either one.
"""
from __future__ import annotations

import numpy as np

from arcqml_b200.circuit import PlanOp


def op(opcode, qubits, params=(0.0, 0.0, 0.0), matrix=None, bindings=()):
    p = tuple(params) + (0.0,) * (3 - len(tuple(params)))
    return PlanOp(opcode, tuple(qubits), p, matrix, tuple(bindings))


class OracleBackend:
    name = "oracle"

    def __init__(self, oracle_module):
        self.O = oracle_module

    def apply_gate(self, amps, n, o, adjoint=False):
        return self.O.apply_gate(amps, n, o, adjoint)

    def parameter_derivative(self, amps, n, o, slot):
        return self.O.parameter_derivative(amps, n, o, slot)

    def plan_apply(self, ops, amps, n):
        return self.O.plan_apply(ops, amps, n)

    def adjoint_backward(self, ops, psi, lam, n, upstream, req, num_grads):
        return self.O.adjoint_backward(ops, psi, lam, n, upstream, req, num_grads)

    def expectation_and_apply(self, terms, amps, n):
        return self.O.expectation_and_apply(terms, amps, n)


class RuntimeBackend:
    """v1 C ABI, host buffers (H2D -> sm_100a kernels -> D2H inside each call)."""

    name = "runtime-v1"

    def __init__(self, rt):
        self.rt = rt

    def _gate(self, o):
        return self.rt.gate_descriptor(o.opcode, len(o.qubits), o.params, o.matrix)

    def apply_gate(self, amps, n, o, adjoint=False):
        a = np.ascontiguousarray(amps, dtype=np.complex128).copy()
        g = self._gate(o)
        (self.rt.apply_adjoint_gate if adjoint else self.rt.apply_gate)(a, n, g, o.qubits)
        return a

    def parameter_derivative(self, amps, n, o, slot):
        a = np.ascontiguousarray(amps, dtype=np.complex128)
        out = np.full_like(a, 123.0 - 456.0j)
        self.rt.parameter_derivative_into(a, out, self._gate(o), o.qubits, slot)
        return out

    def plan_apply(self, ops, amps, n):
        a = np.ascontiguousarray(amps, dtype=np.complex128).copy()
        plan = self.rt.CircuitPlan.compile(ops)
        if a.ndim == 2:
            for row in a:
                r = np.ascontiguousarray(row)
                plan.apply(r, n)
                row[:] = r
        else:
            plan.apply(a, n)
        return a

    def adjoint_backward(self, ops, psi, lam, n, upstream, req, num_grads):
        psi = np.ascontiguousarray(psi, dtype=np.complex128).copy()
        lam = np.ascontiguousarray(lam, dtype=np.complex128).copy()
        scratch = np.zeros_like(psi)
        grads = np.zeros(num_grads, dtype=np.float64)
        plan = self.rt.CircuitPlan.compile(ops)
        plan.adjoint_backward(psi, lam, scratch, n, upstream, np.asarray(req, np.uint8), grads)
        return psi, lam, grads

    def expectation_and_apply(self, terms, amps, n):
        import torch
        c = np.array([t[0] for t in terms], np.float64)
        f = np.array([t[1] for t in terms], np.uint64)
        p = np.array([t[2] for t in terms], np.uint64)
        obs = self.rt.Observable(n, c, f, p)
        d = torch.from_numpy(np.ascontiguousarray(amps, dtype=np.complex128)).cuda()
        out = torch.empty_like(d)
        v = obs.expectation_and_apply(d, out, n)
        return float(v[0]), out.cpu().numpy()
