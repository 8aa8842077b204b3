"""The device optimizer loop (arcqml_rt_v2_small_adam) against the oracle (needs a B200).

Each step of the oracle loop: the plan at the current parameters, psi = plan |init>,
(<H>, H psi), the adjoint gradient with upstream 1, then the f64 Adam step
(crates/arcqml-optim/src/adam.rs:190-240) on the trained parameters. Energies before every update
and the final parameters at 1e-10.
"""
import math

import numpy as np
import pytest

from arcqml_b200 import circuit as cm

pytestmark = pytest.mark.gpu


def rel_err(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return float(np.max(np.abs(a - b))) / max(1.0, float(np.max(np.abs(b))))


def oracle_loop(oracle, c, terms, n, init, steps, lr, betas, eps, wd):
    req = c.requires_grad_mask(True)
    trained = np.flatnonzero(req[1:])
    theta = c.parameter_values().astype(np.float64)
    st, energies = {}, []
    for _ in range(steps):
        c.set_parameter_values(theta)
        ops = c.compile_plan(1)
        psi = oracle.plan_apply(ops, init, n)
        e, lam = oracle.expectation_and_apply(terms, psi, n)
        _, _, g = oracle.adjoint_backward(ops, psi, lam, n, 1.0, req, len(req))
        energies.append(e)
        sub = oracle.adam_step(theta[trained], g[1:][trained], st, lr=lr, beta1=betas[0],
                               beta2=betas[1], eps=eps, weight_decay=wd)
        theta = theta.copy()
        theta[trained] = sub
    return np.array(energies), theta


def device_loop(runtime, c, obs, n, steps, lr, betas, eps, wd, init=None, state=None):
    plan = runtime.CircuitPlan.create(c.compile_plan(1))
    ro = runtime.Observable.from_sparse_pauli_op(obs)
    params = np.concatenate([[0.0], c.parameter_values()])
    return runtime.small_adam_device(plan, ro, n, params, c.requires_grad_mask(True), steps,
                                     lr=lr, betas=betas, eps=eps, weight_decay=wd,
                                     initial_state=init, state=state)


def test_vqe4_hundred_steps_in_one_launch_match_oracle(runtime, oracle):
    from arcqml_b200.workloads import vqe4
    c, obs = vqe4(seed=1)
    init = np.zeros(16, np.complex128)
    init[0] = 1
    before = runtime.launch_count()
    energies, params = device_loop(runtime, c, obs, 4, 100, 0.05, (0.9, 0.999), 1e-8, 0.0)
    assert runtime.launch_count() - before == 1
    c2, _ = vqe4(seed=1)
    ref_e, ref_theta = oracle_loop(oracle, c2, obs.compiled_terms(), 4, init, 100, 0.05,
                                   (0.9, 0.999), 1e-8, 0.0)
    assert rel_err(energies, ref_e) <= 1e-10
    assert rel_err(params[1:], ref_theta) <= 1e-10
    assert ref_e[-1] < ref_e[0]


def mixed_circuit(seed):
    """Every gate family the loop rebuilds, fixed gates between them, a shared parameter used by
    two gates, an untrained parameter and edge angles."""
    g = np.random.Generator(np.random.PCG64(seed))
    n = 6
    c = cm.Circuit(n)
    shared = c.add_parameter(0.4)
    frozen = c.add_parameter(1.1, requires_grad=False)
    one = ("rx", "ry", "rz", "phase")
    two = ("crx", "cry", "crz", "rxx", "ryy", "rzz", "rzx", "cphase")
    for layer in range(3):
        for q in range(n):
            c.append("h" if (q + layer) % 3 == 0 else "sx", (q,))
            name = one[int(g.integers(0, len(one)))]
            v = float(g.uniform(-math.pi, math.pi)) if q != 2 else math.pi
            c.append(name, (q,), c.add_parameter(v))
        for a in range(layer % 2, n - 1, 2):
            name = two[int(g.integers(0, len(two)))]
            c.append(name, (a, a + 1), c.add_parameter(float(g.uniform(-3, 3))))
            c.append("cnot", (a + 1, a))
        c.append("ry", (layer,), shared)
        c.append("rz", (layer + 1,), frozen)
    c.append("cz", (0, n - 1))
    return c, n


def test_every_rebuilt_gate_family_matches_oracle(runtime, oracle):
    import torch
    from arcqml_b200.workloads import random_pauli_sum
    c, n = mixed_circuit(5)
    obs = random_pauli_sum(n, 20, seed=6)
    g = np.random.Generator(np.random.PCG64(7))
    init = g.normal(size=1 << n) + 1j * g.normal(size=1 << n)
    init /= np.linalg.norm(init)
    dev_init = torch.from_numpy(init.copy()).cuda()
    args = (0.03, (0.8, 0.99), 1e-7, 0.01)
    energies, params = device_loop(runtime, c, obs, n, 25, *args, init=dev_init)
    c2, _ = mixed_circuit(5)
    ref_e, ref_theta = oracle_loop(oracle, c2, obs.compiled_terms(), n, init, 25, *args)
    assert rel_err(energies, ref_e) <= 1e-10
    assert rel_err(params[1:], ref_theta) <= 1e-10
    assert params[2] == 1.1  # the frozen parameter is not updated


def test_resumed_loop_equals_one_long_loop(runtime):
    from arcqml_b200.workloads import vqe4
    c, obs = vqe4(seed=3)
    st = runtime.AdamState(c.num_parameters() + 1)
    e_all, p_all = device_loop(runtime, c, obs, 4, 20, 0.05, (0.9, 0.999), 1e-8, 0.0, state=st)
    assert st.step == 20
    st2 = runtime.AdamState(c.num_parameters() + 1)
    e1, p1 = device_loop(runtime, c, obs, 4, 10, 0.05, (0.9, 0.999), 1e-8, 0.0, state=st2)
    c.set_parameter_values(p1[1:])
    e2, p2 = device_loop(runtime, c, obs, 4, 10, 0.05, (0.9, 0.999), 1e-8, 0.0, state=st2)
    assert np.array_equal(np.concatenate([e1, e2]), e_all)
    assert np.array_equal(p2, p_all)
    assert np.array_equal(st2.m, st.m) and np.array_equal(st2.v, st.v)
