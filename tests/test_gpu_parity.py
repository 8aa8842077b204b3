"""sm_100a runtime vs the CPU oracle, through the C ABI (needs a B200).

Tolerances: amplitudes and matrices 1e-12 absolute on normalized states (the kernels use FMA,
the oracle does not); expectations and gradients 1e-10 relative, the bar the reference's
row_major_batch_tests.rs sets.
"""
import math

import numpy as np
import pytest

import reference_cases as rc
from backends import OracleBackend, RuntimeBackend, op
from plans import random_plan, random_state, random_terms, random_unitary
from arcqml_b200 import circuit as cm

pytestmark = pytest.mark.gpu

RTOL = 1e-10


def rel_close(a, b, tol=RTOL):
    a, b = np.asarray(a), np.asarray(b)
    scale = max(1.0, float(np.max(np.abs(b))) if b.size else 1.0)
    assert float(np.max(np.abs(a - b))) <= tol * scale, (a, b)


@pytest.fixture(scope="module")
def be(runtime):
    return RuntimeBackend(runtime)


@pytest.mark.parametrize("case", rc.ALL_CASES, ids=lambda f: f.__name__)
def test_runtime_reference_case(be, case):
    case(be)


def test_runtime_h2_vqe_trajectory(be, oracle):
    rc.case_h2_vqe_trajectory(be, oracle.adam_step)


def all_gate_ops(g, n):
    """One op per opcode (and several MCX / custom arities) on random distinct qubits."""
    ops = []
    for code in range(37):
        arity = 1 if code <= 15 else (2 if code <= 34 else 3)
        if arity > n:
            continue
        q = [int(x) for x in g.choice(n, size=arity, replace=False)]
        p = tuple(float(x) for x in g.uniform(-math.pi, math.pi, size=3))
        ops.append(op(code, q, p))
    for k in range(2, min(n, 6) + 1):
        ops.append(op(cm.MCX, [int(x) for x in g.choice(n, size=k, replace=False)]))
    for k in range(1, min(n, 4) + 1):
        ops.append(op(cm.CUSTOM_UNITARY, [int(x) for x in g.choice(n, size=k, replace=False)],
                      matrix=random_unitary(g, k)))
    return ops


@pytest.mark.parametrize("n", [1, 2, 3, 5, 9, 13])
def test_every_gate_forward_and_adjoint_matches_oracle(be, oracle, n):
    g = np.random.Generator(np.random.PCG64(100 + n))
    ob = OracleBackend(oracle)
    for o in all_gate_ops(g, n):
        a = random_state(g, n)
        for adj in (False, True):
            got = be.apply_gate(a, n, o, adjoint=adj)
            want = ob.apply_gate(a, n, o, adjoint=adj)
            assert np.max(np.abs(got - want)) < 1e-12, (o.opcode, o.qubits, adj)


@pytest.mark.parametrize("n", [2, 4, 11])
def test_every_parameter_derivative_matches_oracle(be, oracle, n):
    g = np.random.Generator(np.random.PCG64(200 + n))
    ob = OracleBackend(oracle)
    for code in range(35):
        slots = cm.slot_count(code)
        arity = 1 if code <= 15 else 2
        for slot in range(slots):
            q = [int(x) for x in g.choice(n, size=arity, replace=False)]
            o = op(code, q, tuple(float(x) for x in g.uniform(-3, 3, size=3)))
            a = random_state(g, n)
            got = be.parameter_derivative(a, n, o, slot)
            want = ob.parameter_derivative(a, n, o, slot)
            assert np.max(np.abs(got - want)) < 1e-12, (code, slot, q)


def test_derivative_matrix_apply_matches_oracle(runtime, oracle):
    g = np.random.Generator(np.random.PCG64(7))
    n = 6
    for code, arity in [(11, 1), (15, 1), (24, 2), (34, 2), (30, 2)]:
        for slot in range(cm.slot_count(code)):
            p = tuple(float(x) for x in g.uniform(-3, 3, size=3))
            q = [int(x) for x in g.choice(n, size=arity, replace=False)]
            dm = runtime.DerivativeMatrix.create(runtime.gate_descriptor(code, arity, p), slot)
            a = random_state(g, n)
            got = a.copy()
            dm.apply(got, q)
            want = oracle.parameter_derivative(a, n, op(code, q, p), slot)
            assert np.max(np.abs(got - want)) < 1e-12


@pytest.mark.parametrize("n,num_ops", [(3, 40), (8, 120), (12, 200), (16, 120)])
def test_run_and_adjoint_match_oracle(be, oracle, n, num_ops):
    g = np.random.Generator(np.random.PCG64(300 + n))
    ob = OracleBackend(oracle)
    npar = 12
    ops = random_plan(g, n, num_ops, npar)
    terms = random_terms(g, n, 25)
    init = random_state(g, n)
    req = [1] + [int(x) for x in (g.uniform(size=npar) < 0.8)]
    up = float(g.normal())
    results = []
    for b in (be, ob):
        psi = b.plan_apply(ops, init, n)
        v, lam = b.expectation_and_apply(terms, psi, n)
        psi0, lam0, grads = b.adjoint_backward(ops, psi, lam, n, up, req, npar + 1)
        results.append((psi, v, lam, psi0, lam0, grads))
    (p1, v1, l1, a1, b1, g1), (p2, v2, l2, a2, b2, g2) = results
    assert np.max(np.abs(p1 - p2)) < 1e-12
    rel_close(v1, v2)
    rel_close(l1, l2)
    assert np.max(np.abs(a1 - init)) < 1e-10
    rel_close(b1, b2)
    rel_close(g1, g2)
    assert g1[0] == 0.0  # the initial-state slot is never written


def test_device_batch_api_matches_oracle(runtime, oracle):
    import torch

    g = np.random.Generator(np.random.PCG64(11))
    n, batch, npar = 7, 6, 9
    ops = random_plan(g, n, 80, npar)
    terms = random_terms(g, n, 17)
    init = random_state(g, n, batch)
    up = g.normal(size=batch)
    req = np.array([0] + [1] * npar, np.uint8)
    plan = runtime.CircuitPlan.compile(ops)
    psi = torch.from_numpy(init.copy()).cuda()
    runtime.plan_apply_device(plan, psi, n)
    c = np.array([t[0] for t in terms]); f = np.array([t[1] for t in terms], np.uint64)
    p = np.array([t[2] for t in terms], np.uint64)
    obs = runtime.Observable(n, c, f, p)
    lam = torch.empty_like(psi)
    vals = obs.expectation_and_apply(psi, lam, n)
    vals2 = obs.expectation(psi, n)
    grads = runtime.adjoint_backward_device(plan, psi, lam, n, up, req, npar + 1)
    ref_psi = oracle.plan_apply(ops, init, n, batch=batch)
    ref_vals = [oracle.expectation_and_apply(terms, r, n)[0] for r in ref_psi]
    ref_lam = np.stack([oracle.expectation_and_apply(terms, r, n)[1] for r in ref_psi])
    _, ref_lam0, ref_grads = oracle.adjoint_backward(ops, ref_psi, ref_lam, n, up, req,
                                                    npar + 1, batch=batch)
    rel_close(vals, ref_vals)
    rel_close(vals2, ref_vals)
    rel_close(grads, ref_grads)
    rel_close(lam.cpu().numpy(), ref_lam0)
    assert np.max(np.abs(psi.cpu().numpy() - init)) < 1e-10
    norms = runtime.norms_device(psi, n)
    assert np.max(np.abs(norms - 1.0)) < 1e-12


def test_basis_state_and_errors(runtime):
    import torch

    s = torch.empty((3, 16), dtype=torch.complex128, device="cuda")
    runtime.set_basis_state_device(s, 4, 5)
    want = np.zeros((3, 16), np.complex128); want[:, 5] = 1
    assert np.array_equal(s.cpu().numpy(), want)
    with pytest.raises(runtime.RuntimeError, match="basis index out of range"):
        runtime.set_basis_state_device(s, 4, 16)
    plan = runtime.CircuitPlan.compile([op(16, [0, 5])])
    with pytest.raises(runtime.RuntimeError, match="out of range for 4 qubits"):
        runtime.plan_apply_device(plan, s, 4)


def test_brickwork_20q_matches_oracle(runtime, oracle):
    """A brickwork circuit and 200-term observable of the benchmark generators at 20 qubits."""
    import torch
    from arcqml_b200 import workloads

    n = 20
    c = workloads.brickwork(n, 6, seed=5)
    obs = workloads.random_pauli_sum(n, 60, seed=6)
    ops = c.compile_plan(1)
    init = np.zeros(1 << n, np.complex128); init[0] = 1
    plan = runtime.CircuitPlan.compile(ops)
    psi = torch.from_numpy(init.copy()).cuda()
    runtime.plan_apply_device(plan, psi, n)
    robs = runtime.Observable.from_sparse_pauli_op(obs)
    lam = torch.empty_like(psi)
    v = robs.expectation_and_apply(psi, lam, n)[0]
    req = c.requires_grad_mask(True)
    grads = runtime.adjoint_backward_device(plan, psi, lam, n, 1.0, req, len(req))
    ref_psi = oracle.plan_apply(ops, init, n)
    rv, rlam = oracle.expectation_and_apply(obs.compiled_terms(), ref_psi, n)
    _, _, rgrads = oracle.adjoint_backward(ops, ref_psi, rlam, n, 1.0, req, len(req))
    rel_close(v, rv)
    rel_close(grads, rgrads)


def with_bindings(g, ops, num_params):
    """Binds every parameter slot of the parameterized ops to random parents 1..num_params."""
    out = []
    for o in ops:
        slots = cm.slot_count(o.opcode)
        binds = tuple((s, int(g.integers(1, num_params + 1))) for s in range(slots))
        out.append(op(o.opcode, o.qubits, o.params, o.matrix, binds))
    return out


@pytest.mark.parametrize("n", [11, 12, 14])
def test_fused_passes_with_every_gate_match_oracle(be, oracle, n):
    """Every opcode, MCX and custom unitaries (3-4 qubit ones run between fused passes) on
    random qubits, forward and adjoint, at sizes that take the fused-pass path."""
    g = np.random.Generator(np.random.PCG64(400 + n))
    ob = OracleBackend(oracle)
    ops = all_gate_ops(g, n) + all_gate_ops(g, n)
    g.shuffle(ops)
    npar = 6
    ops = with_bindings(g, ops, npar)
    terms = random_terms(g, n, 30)
    init = random_state(g, n)
    req = [0] + [1] * npar
    res = []
    for b in (be, ob):
        psi = b.plan_apply(ops, init, n)
        v, lam = b.expectation_and_apply(terms, psi, n)
        psi0, lam0, grads = b.adjoint_backward(ops, psi, lam, n, 0.7, req, npar + 1)
        res.append((psi, v, lam0, psi0, grads))
    (p1, v1, l1, a1, g1), (p2, v2, l2, a2, g2) = res
    assert np.max(np.abs(p1 - p2)) < 1e-12
    rel_close(v1, v2)
    rel_close(l1, l2)
    assert np.max(np.abs(a1 - init)) < 1e-10
    rel_close(g1, g2)


def test_fused_batch_rows_match_oracle(runtime, oracle):
    """[batch, 2^n] rows through the fused forward and adjoint passes."""
    import torch

    g = np.random.Generator(np.random.PCG64(12))
    n, batch, npar = 12, 3, 8
    ops = random_plan(g, n, 150, npar)
    terms = random_terms(g, n, 12)
    init = random_state(g, n, batch)
    up = g.normal(size=batch)
    req = np.array([0] + [1] * npar, np.uint8)
    plan = runtime.CircuitPlan.compile(ops)
    psi = torch.from_numpy(init.copy()).cuda()
    runtime.plan_apply_device(plan, psi, n)
    c = np.array([t[0] for t in terms]); f = np.array([t[1] for t in terms], np.uint64)
    p = np.array([t[2] for t in terms], np.uint64)
    obs = runtime.Observable(n, c, f, p)
    lam = torch.empty_like(psi)
    vals = obs.expectation_and_apply(psi, lam, n)
    grads = runtime.adjoint_backward_device(plan, psi, lam, n, up, req, npar + 1)
    ref_psi = oracle.plan_apply(ops, init, n, batch=batch)
    ref = [oracle.expectation_and_apply(terms, r, n) for r in ref_psi]
    ref_lam = np.stack([x[1] for x in ref])
    _, ref_lam0, ref_grads = oracle.adjoint_backward(ops, ref_psi, ref_lam, n, up, req, npar + 1,
                                                    batch=batch)
    rel_close(vals, [x[0] for x in ref])
    rel_close(grads, ref_grads)
    rel_close(lam.cpu().numpy(), ref_lam0)
    assert np.max(np.abs(psi.cpu().numpy() - init)) < 1e-10


@pytest.mark.parametrize("n", [22, 24])
def test_observable_coset_traversal_matches_oracle(runtime, oracle, n):
    """States above 21 qubits are visited coset by coset (2^21 amplitudes, qubits chosen from
    the flip masks): <H>, H psi and the accumulate mode against the oracle."""
    import torch
    from arcqml_b200.workloads import random_pauli_sum
    g = np.random.Generator(np.random.PCG64(n))
    psi = random_state(g, n)
    obs = random_pauli_sum(n, 60, seed=n + 3)
    terms = obs.compiled_terms()
    v_ref, h_ref = oracle.expectation_and_apply(terms, psi, n)
    dev = torch.from_numpy(psi).cuda()
    ob = runtime.Observable.from_sparse_pauli_op(obs)
    out = torch.empty_like(dev)
    vals = ob.expectation_and_apply(dev, out, n)
    rel_close(vals[0], v_ref)
    assert float(np.max(np.abs(out.cpu().numpy() - h_ref))) <= 1e-12 * max(1.0, np.abs(h_ref).max())
    base = torch.from_numpy(g.normal(size=1 << n) + 0j).cuda()
    acc = base.clone()
    vals2 = ob.expectation_and_accumulate(dev, acc, n)
    rel_close(vals2[0], v_ref)
    got = acc.cpu().numpy() - base.cpu().numpy()
    assert float(np.max(np.abs(got - h_ref))) <= 1e-11 * max(1.0, np.abs(h_ref).max())


def test_compiled_pass_kernels_run_and_match_oracle(runtime, oracle):
    """Brickwork passes run as run-time compiled kernels (no fallback) and match the oracle."""
    import torch
    from arcqml_b200.workloads import brickwork, random_pauli_sum
    n = 14
    c = brickwork(n, 5, seed=77)
    obs = random_pauli_sum(n, 30, seed=78)
    before = runtime.jit_info()
    ops = c.compile_plan(1)
    req = c.requires_grad_mask(True)
    plan = runtime.CircuitPlan.create(ops)
    psi = torch.zeros(1 << n, dtype=torch.complex128, device="cuda")
    runtime.set_basis_state_device(psi, n, 0)
    runtime.plan_apply_device(plan, psi, n)
    lam = torch.empty_like(psi)
    ro = runtime.Observable.from_sparse_pauli_op(obs)
    value = ro.expectation_and_apply(psi, lam, n)[0]
    grads = runtime.adjoint_backward_device(plan, psi, lam, n, 0.5, req, len(req))
    after = runtime.jit_info()
    assert after["launches"] > before["launches"], after
    assert after["fallbacks"] == before["fallbacks"], after["last_error"]
    init = np.zeros(1 << n, np.complex128)
    init[0] = 1
    ref_psi = oracle.plan_apply(ops, init, n)
    ref_v, ref_lam = oracle.expectation_and_apply(obs.compiled_terms(), ref_psi, n)
    _, _, ref_g = oracle.adjoint_backward(ops, ref_psi, ref_lam, n, 0.5, req, len(req))
    rel_close(value, ref_v)
    rel_close(grads, ref_g)


EDGE_ANGLES = (math.pi, -math.pi, math.pi * (1 - 1e-9), 3 * math.pi, math.pi / 2, 0.0, 1e-300,
               -2.9999, 2.9999)


def test_scaled_passes_with_edge_angles_match_oracle(runtime, oracle):
    """Compiled passes carry a per-pass factor for rotations in unit-diagonal form: angles at
    and near pi (forms refused, cos(theta/2) ~ 1e-17), long runs of near-pi rotations (the
    2^300 growth cap), same-axis pairs merged in forward passes, fixed phase gates (S, T, Z)
    and rotation-diagonal products, forward and adjoint against the oracle."""
    import torch
    n = 14
    g = np.random.Generator(np.random.PCG64(31))
    c = cm.Circuit(n)
    for layer in range(12):
        for q in range(n):
            for _ in range(2):
                axis = ("rx", "ry", "rz")[int(g.integers(0, 3))]
                a = EDGE_ANGLES[int(g.integers(0, len(EDGE_ANGLES)))] if g.uniform() < 0.6 \
                    else float(g.uniform(-math.pi, math.pi))
                c.rot(axis, a, q)
            if g.uniform() < 0.3:
                c.append(("s", "t", "z", "sdg")[int(g.integers(0, 4))], (q,))
            if g.uniform() < 0.2:
                c.append("phase", (q,), float(EDGE_ANGLES[int(g.integers(0, len(EDGE_ANGLES)))]))
        for a in range(layer % 2, n - 1, 2):
            c.append("cz", (a, a + 1))
    # a long run of rotations on one qubit at pi (1 - 1e-9): growth ~30 bits each
    for _ in range(40):
        c.rot("ry", math.pi * (1 - 1e-9), 3)
    obs = cm_random_sum(n, 25, seed=32)
    ops = c.compile_plan(1)
    req = c.requires_grad_mask(True)
    init = random_state(g, n)
    before = runtime.jit_info()
    plan = runtime.CircuitPlan.create(ops)
    psi = torch.from_numpy(init.copy()).cuda()
    runtime.plan_apply_device(plan, psi, n)
    lam = torch.empty_like(psi)
    ro = runtime.Observable.from_sparse_pauli_op(obs)
    value = ro.expectation_and_apply(psi, lam, n)[0]
    fwd = psi.cpu().numpy()
    grads = runtime.adjoint_backward_device(plan, psi, lam, n, -1.5, req, len(req))
    after = runtime.jit_info()
    assert after["launches"] > before["launches"], after
    ref_psi = oracle.plan_apply(ops, init, n)
    ref_v, ref_lam = oracle.expectation_and_apply(obs.compiled_terms(), ref_psi, n)
    ref_psi0, ref_lam0, ref_g = oracle.adjoint_backward(ops, ref_psi, ref_lam, n, -1.5, req,
                                                        len(req))
    assert float(np.max(np.abs(fwd - ref_psi))) < 1e-12
    rel_close(value, ref_v)
    rel_close(grads, ref_g)
    rel_close(lam.cpu().numpy(), ref_lam0)
    assert float(np.max(np.abs(psi.cpu().numpy() - init))) < 1e-10


def cm_random_sum(n, terms, seed):
    from arcqml_b200.workloads import random_pauli_sum
    return random_pauli_sum(n, terms, seed=seed)


def test_precompiled_pass_kernels_match_oracle_without_jit(runtime):
    """With ARCQML_JIT=0 every pass runs the precompiled table-driven kernel (subprocess)."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = (
        "import sys; sys.path[:0]=[%r, %r]\n"
        "import numpy as np, torch, oracle as O\n"
        "from arcqml_b200 import runtime as rt, workloads as W\n"
        "n=14; c=W.brickwork(n,5,seed=77); obs=W.random_pauli_sum(n,30,seed=78)\n"
        "ops=c.compile_plan(1); req=c.requires_grad_mask(True); plan=rt.CircuitPlan.create(ops)\n"
        "psi=torch.zeros(1<<n,dtype=torch.complex128,device='cuda'); rt.set_basis_state_device(psi,n,0)\n"
        "rt.plan_apply_device(plan,psi,n); lam=torch.empty_like(psi)\n"
        "v=rt.Observable.from_sparse_pauli_op(obs).expectation_and_apply(psi,lam,n)[0]\n"
        "g=rt.adjoint_backward_device(plan,psi,lam,n,0.5,req,len(req))\n"
        "init=np.zeros(1<<n,np.complex128); init[0]=1; rp=O.plan_apply(ops,init,n)\n"
        "rv,rl=O.expectation_and_apply(obs.compiled_terms(),rp,n)\n"
        "_,_,rg=O.adjoint_backward(ops,rp,rl,n,0.5,req,len(req))\n"
        "assert abs(v-rv)<=1e-10*max(1,abs(rv)), (v,rv)\n"
        "assert np.max(np.abs(g-rg))<=1e-10*max(1,np.max(np.abs(rg)))\n"
        "assert rt.jit_info()['launches']==0\n"
        "print('aot-ok')\n") % (root, os.path.join(root, "oracle"))
    env = dict(os.environ, ARCQML_JIT="0")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env,
                       timeout=600)
    assert r.returncode == 0 and "aot-ok" in r.stdout, r.stdout + r.stderr


@pytest.mark.parametrize("n", [2, 3, 6, 10])
def test_one_kernel_small_step_matches_oracle(runtime, oracle, n):
    """arcqml_rt_v2_small_run (forward, <H>, adjoint in one launch) against the oracle, with an
    initial state, controlled and custom gates, shared parameters and lambda_0."""
    import torch
    g = np.random.Generator(np.random.PCG64(4000 + n))
    npar = 7
    ops = random_plan(g, n, 60, npar)
    if n >= 3:
        ops.append(op(38, (0, 2, 1), matrix=random_unitary(g, 3)))
    if n >= 6:
        ops.append(op(38, (5, 1, 3, 0), matrix=random_unitary(g, 4)))
    terms_obj = __import__("arcqml_b200.workloads", fromlist=["x"]).random_pauli_sum(
        n, 12, seed=n + 40)
    init = random_state(g, n)
    req = [1] + [int(x) for x in (g.uniform(size=npar) < 0.8)]
    plan = runtime.CircuitPlan.create(ops)
    obs = runtime.Observable.from_sparse_pauli_op(terms_obj)
    dev = torch.from_numpy(init).cuda()
    lam0 = torch.empty_like(dev)
    value, grads = runtime.small_run_device(plan, obs, dev, n, req, len(req), lam0)
    ref_psi = oracle.plan_apply(ops, init, n)
    ref_v, ref_lam = oracle.expectation_and_apply(terms_obj.compiled_terms(), ref_psi, n)
    _, ref_lam0, ref_g = oracle.adjoint_backward(ops, ref_psi, ref_lam, n, 1.0, req, len(req))
    rel_close(value, ref_v)
    rel_close(grads, ref_g)
    rel_close(lam0.cpu().numpy(), ref_lam0)
    # |0...0> when no initial state is given
    v0, _ = runtime.small_run_device(plan, obs, None, n, req, len(req))
    z = np.zeros(1 << n, np.complex128)
    z[0] = 1
    rel_close(v0, oracle.expectation(terms_obj.compiled_terms(), oracle.plan_apply(ops, z, n), n))
