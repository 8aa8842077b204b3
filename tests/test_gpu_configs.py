"""The benchmark configurations end to end on the GPU against the oracle (needs a B200).

* 4-qubit VQE: 100 steps of run -> backward -> Adam (lr 0.05) through StateVectorSimulator,
  every energy and the final parameters at 1e-10;
* batched QNN: 1024 rows of 10 qubits, 80 parameters, half-MSE upstream, values and the
  row-summed gradient at 1e-10 through BatchStateVectorSimulator;
* 28 qubits: the fused forward pass against the per-gate kernels on the full-size state (two
  independent GPU paths), plus norm preservation and <H> against the same state.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def rel_err(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return float(np.max(np.abs(a - b))) / max(1.0, float(np.max(np.abs(b))))


def test_config1_vqe4_adam_trajectory_matches_oracle(runtime, oracle):
    from arcqml_b200.simulator import StateVectorSimulator
    from arcqml_b200.workloads import vqe4
    c, obs = vqe4(seed=1)
    terms = obs.compiled_terms()
    sim = StateVectorSimulator(4)
    theta = c.parameter_values().astype(np.float64)
    ref_theta = theta.copy()
    st_gpu, st_ref = {}, {}
    init = np.zeros(16, np.complex128)
    init[0] = 1
    for step in range(100):
        c.set_parameter_values(theta)
        res = sim.run(c, obs)
        grads, _ = res.backward(1.0)
        energy = res.value
        theta = oracle.adam_step(theta, np.asarray(grads), st_gpu, lr=0.05)

        c.set_parameter_values(ref_theta)
        ops = c.compile_plan(1)
        psi = oracle.plan_apply(ops, init, 4)
        e_ref, lam = oracle.expectation_and_apply(terms, psi, 4)
        req = c.requires_grad_mask(True)
        _, _, g_ref = oracle.adjoint_backward(ops, psi, lam, 4, 1.0, req, len(req))
        ref_theta = oracle.adam_step(ref_theta, g_ref[1:], st_ref, lr=0.05)
        assert abs(energy - e_ref) <= 1e-10 * max(1.0, abs(e_ref)), (step, energy, e_ref)
    assert rel_err(theta, ref_theta) <= 1e-10


def test_config2_batched_qnn_matches_oracle(runtime, oracle):
    from arcqml_b200.simulator import BatchStateVectorSimulator
    from arcqml_b200.workloads import half_mse_upstream, qnn
    n, b = 10, 1024
    c, obs, init, labels = qnn(n, b, 4, seed=7)
    sim = BatchStateVectorSimulator.from_amplitudes(n, init)
    res = sim.run(c, obs)
    loss, up = half_mse_upstream(res.values, labels)
    grads, _ = res.backward(up)

    ops = c.compile_plan(1)
    psi = oracle.plan_apply(ops, init.reshape(-1), n, b).reshape(b, -1)
    terms = obs.compiled_terms()
    vals = np.array([oracle.expectation(terms, psi[i], n) for i in range(b)])
    lam = np.stack([oracle.expectation_and_apply(terms, psi[i], n)[1] for i in range(b)])
    loss_ref, up_ref = half_mse_upstream(vals, labels)
    req = c.requires_grad_mask(True, False)
    _, _, g = oracle.adjoint_backward(ops, psi.reshape(-1), lam.reshape(-1), n, up_ref, req,
                                      len(req), b)
    assert rel_err(res.values, vals) <= 1e-10
    assert abs(loss - loss_ref) <= 1e-10
    assert rel_err(grads, g[1:]) <= 1e-10


def test_config3_28q_fused_pass_equals_per_gate_kernels(runtime):
    import torch
    from arcqml_b200.workloads import brickwork, random_pauli_sum
    n = 28
    c = brickwork(n, 4, seed=1234)
    ops = c.compile_plan(0)
    a = torch.zeros(1 << n, dtype=torch.complex128, device="cuda")
    runtime.set_basis_state_device(a, n, 0)
    runtime.plan_apply_device(runtime.CircuitPlan.create(ops), a, n)
    b = torch.zeros_like(a)
    runtime.set_basis_state_device(b, n, 0)
    for o in ops:
        g = runtime.gate_descriptor(o.opcode, len(o.qubits), o.params, o.matrix)
        runtime.apply_gate_device(b, n, g, o.qubits)
    diff = float((a - b).abs().max().item())
    scale = float(b.abs().max().item())
    assert diff <= 1e-12 * max(scale, 1e-300) + 1e-15, (diff, scale)
    del b
    torch.cuda.empty_cache()
    norm = float(runtime.norms_device(a, n)[0])
    assert abs(norm - 1.0) <= 1e-10
    obs = runtime.Observable.from_sparse_pauli_op(random_pauli_sum(n, 200, seed=1235))
    v1 = obs.expectation(a, n)[0]
    out = torch.empty_like(a)
    v2 = obs.expectation_and_apply(a, out, n)[0]
    assert abs(v1 - v2) <= 1e-12
    assert abs(v1) <= 200 * 4.0
