"""Device-resident statevector simulators over the sm_100a runtime.

Mirrors ArcQML's ``StateVectorSimulator`` / ``BatchStateVectorSimulator`` run path
(``crates/arcqml-sim/src/statevector/execution/adjoint/single.rs:29-163``, ``batch.rs:30-128``,
``row_major.rs:18-307``): ``run`` compiles the plan with parent offset 1 (the initial state is
parent 0), applies it, computes ``<H>`` and ``H|psi>`` in one pass, and returns a result whose
``backward(upstream)`` runs the adjoint reverse sweep. Parameter gradients follow the
reference's indexing (``gradients[1:]``); the initial-state gradient is ``2 * g * lambda_0``
(``adjoint/single.rs:138-146``). States live in HBM as torch ``complex128`` CUDA tensors; only
parameters, upstream factors, values and gradients cross PCIe.

Unlike the reference, ``backward`` consumes the saved psi/lambda buffers in place (a 32-qubit
state is 64 GiB; cloning them as the reference does would not fit). Pass ``retain=True`` to
keep the context for a second backward.
"""
from __future__ import annotations

import os
import weakref
from dataclasses import dataclass
from typing import Optional

import numpy as np

from . import runtime as rt
from .circuit import Circuit
from .observable import SparsePauliOp

NORM_TOLERANCE = 1e-10  # docs/ArcQML技术手册.md:206-213


class SimError(ValueError):
    pass


def _torch():
    import torch
    if not torch.cuda.is_available():
        raise SimError("the B200 statevector runtime needs a CUDA device")
    return torch


def _new_state(num_qubits: int, batch: Optional[int], device):
    torch = _torch()
    shape = (1 << num_qubits,) if batch is None else (batch, 1 << num_qubits)
    return torch.empty(shape, dtype=torch.complex128, device=device)


@dataclass(eq=False)  # identity hashing: plan pools hold contexts in weak sets
class _Context:
    num_qubits: int
    batch: Optional[int]
    psi: object
    lam: object
    plan: rt.CircuitPlan
    circuit: Circuit
    initial_requires_grad: bool


@dataclass
class _SmallContext:
    """Result of the one-kernel step: gradients for upstream 1 (the sweep is linear in it)."""
    grads: np.ndarray
    lam0: object
    circuit: Circuit
    initial_requires_grad: bool


def _small_enabled() -> bool:
    return os.environ.get("ARCQML_SMALL", "1") != "0"


def _pool(sim) -> "_PlanPool":
    return sim.__dict__.setdefault("_plan_pool", _PlanPool())


class _PlanPool:
    """Device plans by circuit structure. Creating a plan marshals every operation through the
    C ABI (milliseconds of host time for a hundred gates, more than a small batch's whole step);
    a run whose circuit has the structure of an earlier one takes a plan of that structure that
    no live result still holds and replaces its bound parameter values
    (arcqml_rt_v2_plan_set_parameters). A result keeps its plan until it is dropped, so its
    backward sweep always sees the values it ran with."""

    def __init__(self, limit: int = 64, per_key: int = 4):
        self._plans = {}
        self._limit, self._per_key = limit, per_key

    def get(self, circuit: Circuit, offset: int):
        """(plan, users): the caller adds the result context that holds the plan to users."""
        ops = circuit.compile_plan(offset)
        key = (offset, rt.plan_structure_key(ops))
        entries = self._plans.get(key)
        if entries is None:
            if len(self._plans) >= self._limit:
                self._plans.clear()
            entries = self._plans[key] = []
        for plan, users in entries:
            if len(users) == 0:
                plan.set_parameters(np.array([0.0] * offset + [p.f64() for p in circuit.parameters]))
                return plan, users
        plan, users = rt.CircuitPlan.create(ops), weakref.WeakSet()
        if len(entries) < self._per_key:
            entries.append((plan, users))
        return plan, users


class RunResult:
    """Output of ``run``: value(s) plus the adjoint context for ``backward``."""

    def __init__(self, values: np.ndarray, ctx: Optional[_Context]):
        self.values = values
        self._ctx = ctx
        self.initial_state_grad = None
        self.parameter_grads = None

    @property
    def value(self) -> float:
        return float(self.values[0])

    @property
    def requires_grad(self) -> bool:
        return self._ctx is not None

    def backward(self, upstream=1.0, retain: bool = False, stream=None):
        """Adjoint reverse sweep with upstream g (scalar, or [batch] for batch runs).

        Returns (parameter_grads, initial_state_grad). Parameter gradients are also
        accumulated into ``circuit.parameters[i].grad``.
        """
        if self._ctx is None:
            raise SimError("run was executed without gradient recording")
        c = self._ctx
        if isinstance(c, _SmallContext):
            g = float(np.asarray(upstream, dtype=np.float64).reshape(-1)[0])
            grads = g * c.grads
            lam = None if c.lam0 is None else g * c.lam0
        else:
            psi, lam = (c.psi.clone(), c.lam.clone()) if retain else (c.psi, c.lam)
            req = c.circuit.requires_grad_mask(True, c.initial_requires_grad)
            grads = rt.adjoint_backward_device(c.plan, psi, lam, c.num_qubits, upstream, req,
                                               len(req), stream)
        pgrads = grads[1:].copy()
        for p, g in zip(c.circuit.parameters, pgrads):
            if p.requires_grad:
                g = float(np.float32(g)) if p.dtype == "f32" else float(g)
                p.grad = g if getattr(p, "grad", None) is None else p.grad + g
        self.parameter_grads = pgrads
        self.initial_state_grad = (2.0 * lam) if c.initial_requires_grad else None
        if not retain:
            self._ctx = None
        return pgrads, self.initial_state_grad


class StateVectorSimulator:
    """Single state of ``num_qubits`` qubits, resident on a CUDA device.

    The simulator's own state buffer is created on first use: ``run`` on a fresh simulator
    starts its working copy from |0...0> directly, so a 32-qubit run holds only psi and
    lambda (2 x 64 GiB) in HBM.
    """

    def __init__(self, num_qubits: int, device=None):
        if num_qubits < 0 or num_qubits >= 40:
            raise SimError(f"state dimension overflow for {num_qubits} qubits")
        self.num_qubits = num_qubits
        self.device = device if device is not None else _torch().device("cuda", _torch().cuda.current_device())
        self._state = None  # None means |0...0>, not materialised
        self.initial_requires_grad = False

    @property
    def state(self):
        if self._state is None:
            self._state = _new_state(self.num_qubits, None, self.device)
            rt.set_basis_state_device(self._state, self.num_qubits, 0)
        return self._state

    @classmethod
    def from_amplitudes(cls, num_qubits: int, amplitudes, requires_grad: bool = False):
        a = np.ascontiguousarray(amplitudes, dtype=np.complex128)
        if a.shape != (1 << num_qubits,):
            raise SimError(f"state must have shape [{1 << num_qubits}], got {list(a.shape)}")
        norm = float(np.vdot(a, a).real)
        if abs(norm - 1.0) > NORM_TOLERANCE:
            raise SimError(f"state is not normalized: squared norm {norm}")
        sim = cls(num_qubits)
        sim.state.copy_(_torch().from_numpy(a))
        sim.initial_requires_grad = requires_grad
        return sim

    def reset(self) -> None:
        self._state = None

    def amplitudes(self) -> np.ndarray:
        return self.state.cpu().numpy()

    def apply_circuit(self, circuit: Circuit) -> None:
        self._check(circuit)
        plan = rt.CircuitPlan.create(circuit.compile_plan(0))
        rt.plan_apply_device(plan, self.state, self.num_qubits)

    def expectation(self, observable: SparsePauliOp) -> float:
        obs = rt.Observable.from_sparse_pauli_op(observable)
        return float(obs.expectation(self.state, self.num_qubits)[0])

    def gradient(self, circuit: Circuit, cotangent, stream=None):
        """Parameter gradients of a loss of this simulator's state, given the loss's cotangent
        (the lambda of ``arcqml_b200.analysis``'s ``*_cotangent`` helpers, a complex128 CUDA
        tensor): the adjoint sweep of ``circuit`` adds 2 Re<lambda| dU/dp |psi> per bound slot.
        The state must be ``circuit`` applied to this simulator's initial state; it is copied
        (the sweep runs it back to the start), so the simulator keeps it. Returns the gradients
        indexed like ``circuit.parameters`` and accumulates them into each parameter's
        ``grad``, as ``RunResult.backward`` does."""
        self._check(circuit)
        plan = rt.CircuitPlan.create(circuit.compile_plan(1))
        psi = self.state.clone()
        lam = cotangent.clone()
        req = circuit.requires_grad_mask(True, False)
        grads = rt.adjoint_backward_device(plan, psi, lam, self.num_qubits, 1.0, req, len(req),
                                           stream)
        pgrads = grads[1:].copy()
        for p, g in zip(circuit.parameters, pgrads):
            if p.requires_grad:
                g = float(np.float32(g)) if p.dtype == "f32" else float(g)
                p.grad = g if getattr(p, "grad", None) is None else p.grad + g
        return pgrads

    def norm(self) -> float:
        return float(rt.norms_device(self.state, self.num_qubits)[0])

    def sample_counts(self, shots: int, seed: Optional[int] = None) -> dict:
        """Counts of ``shots`` full-register measurements of the current state, keyed by the
        bitstring q[n-1]..q0 and sorted by it; the state is not collapsed. The same seed gives
        the reference's counts bit for bit (StdRng::seed_from_u64, sequential running sum;
        ``crates/arcqml-sim/src/statevector/api/measurement.rs:18-60``); ``None`` draws a seed."""
        if shots <= 0:
            raise SimError("invalid shot count: shots must be greater than zero")
        if seed is None:
            seed = int.from_bytes(os.urandom(8), "little")
        try:
            idx, _ = rt.sample_indices_device(self.state, self.num_qubits, shots, seed)
        except rt.RuntimeError as e:
            raise SimError(str(e)) from None
        vals, cnt = np.unique(idx, return_counts=True)
        n = self.num_qubits
        return dict(sorted((format(int(v), f"0{n}b"), int(c)) for v, c in zip(vals, cnt)))

    def run(self, circuit: Circuit, observable: SparsePauliOp, grad: bool = True,
            initial_state=None) -> RunResult:
        """Expectation of ``observable`` after ``circuit``; ``backward`` gives the gradients.

        ``initial_state`` (optional, a CPU torch tensor or numpy array of 2^n complex128,
        ideally pinned) replaces the simulator's state as the input of this run; it is copied
        to the device on the current stream.
        """
        self._check(circuit)
        if observable.num_qubits != self.num_qubits:
            raise SimError("observable and state qubit counts differ")
        torch = _torch()
        records = grad and (self.initial_requires_grad or any(p.requires_grad for p in circuit.parameters))
        if records and self.num_qubits <= rt.SMALL_MAX_QUBITS and _small_enabled():
            return self._run_small(circuit, observable, initial_state)
        psi = _new_state(self.num_qubits, None, self.device)
        if initial_state is not None:
            src = initial_state if isinstance(initial_state, torch.Tensor) else torch.from_numpy(
                np.ascontiguousarray(initial_state, dtype=np.complex128))
            if src.shape != psi.shape or src.dtype != torch.complex128:
                raise SimError(f"initial state must be complex128 of shape [{1 << self.num_qubits}]")
            psi.copy_(src, non_blocking=True)
        elif self._state is None:
            rt.set_basis_state_device(psi, self.num_qubits, 0)
        else:
            psi.copy_(self._state)
        plan, users = _pool(self).get(circuit, 1 if records else 0)
        rt.plan_apply_device(plan, psi, self.num_qubits)
        obs = rt.Observable.from_sparse_pauli_op(observable)
        if not records:
            return RunResult(obs.expectation(psi, self.num_qubits), None)
        lam = torch.empty_like(psi)
        vals = obs.expectation_and_apply(psi, lam, self.num_qubits)
        ctx = _Context(self.num_qubits, None, psi, lam, plan, circuit, self.initial_requires_grad)
        users.add(ctx)
        return RunResult(vals, ctx)

    # -- small states: one kernel for forward, <H> and the adjoint sweep ----------------------
    def _small_plan(self, circuit: Circuit):
        """A plan for the circuit's structure, reused across runs with its bound parameter
        values replaced (plan creation costs more host time than the step itself; the one-kernel
        step uses the plan at once, so no result holds it)."""
        ops = circuit.compile_plan(1)
        key = rt.plan_structure_key(ops)
        plans = self.__dict__.setdefault("_plans", {})
        plan = plans.get(key)
        if plan is None:
            if len(plans) > 64:
                plans.clear()
            plan = rt.CircuitPlan.create(ops)
            plans[key] = plan
        else:
            plan.set_parameters(np.array([0.0] + [p.f64() for p in circuit.parameters]))
        return plan

    def _small_observable(self, observable: SparsePauliOp):
        key = tuple(observable.terms)
        cache = self.__dict__.setdefault("_observables", {})
        obs = cache.get(key)
        if obs is None:
            if len(cache) > 16:
                cache.clear()
            obs = rt.Observable.from_sparse_pauli_op(observable)
            cache[key] = obs
        return obs

    def _run_small(self, circuit: Circuit, observable: SparsePauliOp, initial_state) -> RunResult:
        torch = _torch()
        init = None
        if initial_state is not None:
            src = initial_state if isinstance(initial_state, torch.Tensor) else torch.from_numpy(
                np.ascontiguousarray(initial_state, dtype=np.complex128))
            if src.numel() != (1 << self.num_qubits) or src.dtype != torch.complex128:
                raise SimError(f"initial state must be complex128 of shape [{1 << self.num_qubits}]")
            init = src.reshape(-1).to(self.device, non_blocking=True)
        elif self._state is not None:
            init = self._state
        lam0 = torch.empty(1 << self.num_qubits, dtype=torch.complex128, device=self.device) \
            if self.initial_requires_grad else None
        req = circuit.requires_grad_mask(True, self.initial_requires_grad)
        value, grads = rt.small_run_device(self._small_plan(circuit),
                                           self._small_observable(observable), init,
                                           self.num_qubits, req, len(req), lam0)
        return RunResult(np.array([value]), _SmallContext(grads, lam0, circuit,
                                                          self.initial_requires_grad))

    def _check(self, circuit: Circuit):
        if circuit.num_qubits != self.num_qubits:
            raise SimError(f"circuit has {circuit.num_qubits} qubits, simulator has {self.num_qubits}")


class BatchStateVectorSimulator:
    """[batch, 2^n] independent states sharing one circuit and observable."""

    def __init__(self, num_qubits: int, batch_size: int, device=None):
        if batch_size <= 0:
            raise SimError("batch size must be non-zero")
        self.num_qubits = num_qubits
        self.batch_size = batch_size
        self.device = device if device is not None else _torch().device("cuda", _torch().cuda.current_device())
        self.state = _new_state(num_qubits, batch_size, self.device)
        self.initial_requires_grad = False
        rt.set_basis_state_device(self.state, num_qubits, 0)

    @classmethod
    def from_amplitudes(cls, num_qubits: int, amplitudes, requires_grad: bool = False):
        a = np.ascontiguousarray(amplitudes, dtype=np.complex128)
        if a.ndim != 2 or a.shape[1] != (1 << num_qubits) or a.shape[0] == 0:
            raise SimError(f"batch state must have shape [B, {1 << num_qubits}]")
        norms = np.einsum("ij,ij->i", a.conj(), a).real
        bad = np.nonzero(np.abs(norms - 1.0) > NORM_TOLERANCE)[0]
        if bad.size:
            raise SimError(f"batch row {int(bad[0])} is not normalized")
        sim = cls(num_qubits, a.shape[0])
        sim.state.copy_(_torch().from_numpy(a))
        sim.initial_requires_grad = requires_grad
        return sim

    @classmethod
    def from_device_state(cls, num_qubits: int, state, requires_grad: bool = False):
        sim = cls.__new__(cls)
        sim.num_qubits = num_qubits
        sim.batch_size = state.shape[0]
        sim.device = state.device
        sim.state = state
        sim.initial_requires_grad = requires_grad
        return sim

    def amplitudes(self) -> np.ndarray:
        return self.state.cpu().numpy()

    def apply_circuit(self, circuit: Circuit) -> None:
        plan = rt.CircuitPlan.create(circuit.compile_plan(0))
        rt.plan_apply_device(plan, self.state, self.num_qubits)

    def expectation(self, observable: SparsePauliOp) -> np.ndarray:
        return rt.Observable.from_sparse_pauli_op(observable).expectation(self.state, self.num_qubits)

    def run(self, circuit: Circuit, observable: SparsePauliOp, grad: bool = True) -> RunResult:
        if circuit.num_qubits != self.num_qubits or observable.num_qubits != self.num_qubits:
            raise SimError("circuit, observable and state qubit counts differ")
        records = grad and (self.initial_requires_grad or any(p.requires_grad for p in circuit.parameters))
        psi = self.state.clone()
        plan, users = _pool(self).get(circuit, 1 if records else 0)
        rt.plan_apply_device(plan, psi, self.num_qubits)
        obs = rt.Observable.from_sparse_pauli_op(observable)
        if not records:
            return RunResult(obs.expectation(psi, self.num_qubits), None)
        lam = _torch().empty_like(psi)
        vals = obs.expectation_and_apply(psi, lam, self.num_qubits)
        ctx = _Context(self.num_qubits, self.batch_size, psi, lam, plan, circuit,
                       self.initial_requires_grad)
        users.add(ctx)
        return RunResult(vals, ctx)
