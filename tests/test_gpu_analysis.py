"""State analysis on the device against the oracle (needs a B200): probabilities, marginal
probabilities (both kernel shapes: one thread per bin, and chunked bins), Bloch vectors and
overlaps on random states and batch rows, the reference's analysis tests
(crates/arcqml-analysis/tests/statevector_analysis.rs) through the simulator, and gradients of
analysis losses through the cotangents and the adjoint sweep."""
import math

import numpy as np
import pytest

from arcqml_b200 import circuit as cm
from plans import random_state

pytestmark = pytest.mark.gpu


def rel_close(a, b, tol=1e-12):
    a, b = np.asarray(a), np.asarray(b)
    scale = max(1.0, float(np.max(np.abs(b))) if b.size else 1.0)
    assert float(np.max(np.abs(a - b))) <= tol * scale, (a, b)


SELECTIONS = {1: [[0]], 3: [[0], [2, 0], [0, 1, 2]], 10: [[0], [9, 4, 1], [3, 5, 7, 8, 9, 0, 1],
                                                          list(range(10))],
              20: [[0], [19], [19, 0], [2, 5, 11, 17, 3, 8, 13, 14], list(range(12))],
              24: [[23, 22, 21], [0, 12]]}


@pytest.mark.parametrize("n", [1, 3, 10, 20, 24])
def test_analysis_matches_oracle_on_random_states(runtime, oracle, n):
    import torch
    g = np.random.Generator(np.random.PCG64(700 + n))
    a, b = random_state(g, n), random_state(g, n)
    da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    rel_close(runtime.probabilities_device(da, n).cpu().numpy(), oracle.probabilities(a, n))
    for qs in SELECTIONS[n]:
        got = runtime.marginal_probabilities_device(da, n, qs).cpu().numpy()
        rel_close(got, oracle.marginal_probabilities(a, n, qs))
    for q in sorted({0, n // 2, n - 1}):
        rel_close(runtime.bloch_vector_device(da, n, q), oracle.bloch_vector(a, n, q))
    s = runtime.overlap_device(da, db, n)
    rs, _ = oracle.overlap_fidelity(a, b, n)
    rel_close([s.real, s.imag], [rs.real, rs.imag])


def test_analysis_of_batch_rows(runtime, oracle):
    import torch
    g = np.random.Generator(np.random.PCG64(71))
    n, rows = 9, 3
    a, b = random_state(g, n, rows), random_state(g, n, rows)
    da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    p = runtime.probabilities_device(da, n).cpu().numpy()
    m = runtime.marginal_probabilities_device(da, n, [8, 1]).cpu().numpy()
    xyz = runtime.bloch_vector_device(da, n, 4)
    s = runtime.overlap_device(da, db, n)
    assert p.shape == (rows, 512) and m.shape == (rows, 4) and xyz.shape == (rows, 3)
    for r in range(rows):
        rel_close(p[r], oracle.probabilities(a[r], n))
        rel_close(m[r], oracle.marginal_probabilities(a[r], n, [8, 1]))
        rel_close(xyz[r], oracle.bloch_vector(a[r], n, 4))
        rs, _ = oracle.overlap_fidelity(a[r], b[r], n)
        rel_close([s[r].real, s[r].imag], [rs.real, rs.imag])


def test_reference_analysis_cases_through_the_simulator(runtime):
    from arcqml_b200 import analysis
    from arcqml_b200.simulator import StateVectorSimulator
    bell = StateVectorSimulator(2)
    bell.apply_circuit(cm.Circuit(2).append("h", (0,)).append("cnot", (0, 1)))
    rel_close(analysis.probabilities(bell), [0.5, 0, 0, 0.5])
    rel_close(analysis.marginal_probabilities(bell, [0]), [0.5, 0.5])
    rel_close(analysis.marginal_probabilities(bell, [0, 1]), [0.5, 0, 0, 0.5])
    zero = StateVectorSimulator(2)
    assert abs(analysis.fidelity(bell, bell) - 1.0) < 1e-12
    assert abs(analysis.fidelity(bell, zero) - 0.5) < 1e-12
    plus = StateVectorSimulator(1)
    plus.apply_circuit(cm.Circuit(1).append("h", (0,)))
    rel_close(list(analysis.bloch_vector(plus, 0)), [1.0, 0.0, 0.0])
    for qs, msg in (([], "at least one qubit must be selected"),
                    ([0, 0], "duplicate qubit in selection: 0"),
                    ([2], "qubit index out of range: simulator has 2 qubits, got 2")):
        with pytest.raises(analysis.AnalysisError, match=msg):
            analysis.marginal_probabilities(bell, qs)


def ry_sim(theta, entangle=False):
    from arcqml_b200.simulator import StateVectorSimulator
    c = cm.Circuit(2 if entangle else 1)
    c.rot("ry", theta, 0)
    if entangle:
        c.append("cnot", (0, 1))
    sim = StateVectorSimulator(c.num_qubits)
    sim.apply_circuit(c)
    return sim, c


def test_reference_gradient_cases_through_cotangents(runtime):
    # statevector_analysis.rs:109-181
    from arcqml_b200 import analysis
    from arcqml_b200.simulator import StateVectorSimulator
    t = 0.4
    sim, c = ry_sim(t)
    g = sim.gradient(c, analysis.amplitudes_cotangent(sim, np.array([0, 1], np.complex128)))
    assert abs(g[0] - 0.5 * math.cos(t / 2)) < 1e-12
    g = sim.gradient(c, analysis.probabilities_cotangent(sim, [0.0, 1.0]))
    assert abs(g[0] - 0.5 * math.sin(t)) < 1e-12
    sim, c = ry_sim(t, entangle=True)
    g = sim.gradient(c, analysis.probabilities_cotangent(sim, [0.0, 1.0], qubits=[1]))
    assert abs(g[0] - 0.5 * math.sin(t)) < 1e-12
    t, phi = 0.2, 0.8
    sim, c = ry_sim(t)
    target = StateVectorSimulator.from_amplitudes(
        1, np.array([math.cos(phi / 2), math.sin(phi / 2)], np.complex128))
    assert abs(analysis.fidelity(sim, target) - math.cos((t - phi) / 2) ** 2) < 1e-12
    g = sim.gradient(c, analysis.fidelity_cotangent(sim, target))
    assert abs(g[0] + 0.5 * math.sin(t - phi)) < 1e-12
    # the simulator keeps its state through gradient()
    assert abs(analysis.fidelity(sim, target) - math.cos((t - phi) / 2) ** 2) < 1e-12


def test_marginal_loss_gradient_matches_oracle_adjoint(runtime, oracle):
    import torch
    from arcqml_b200 import analysis, workloads
    from arcqml_b200.simulator import StateVectorSimulator
    n = 12
    c = workloads.brickwork(n, 4, seed=9)
    sim = StateVectorSimulator(n)
    sim.apply_circuit(c)
    qs = [3, 11, 7]
    g = np.random.Generator(np.random.PCG64(5)).normal(size=8)
    grads = sim.gradient(c, analysis.probabilities_cotangent(sim, g, qubits=qs))
    ops = c.compile_plan(1)
    init = np.zeros(1 << n, np.complex128)
    init[0] = 1.0
    psi = oracle.plan_apply(ops, init, n)
    disp = sorted(qs, reverse=True)
    bins = np.zeros(1 << n, np.int64)
    for j, q in enumerate(disp):
        bins |= ((np.arange(1 << n) >> q) & 1) << (len(disp) - 1 - j)
    lam = g[bins] * psi
    req = c.requires_grad_mask(True)
    _, _, ref = oracle.adjoint_backward(ops, psi, lam, n, 1.0, req, len(req))
    rel_close(grads, ref[1:], tol=1e-10)
    dev = torch.from_numpy(psi).cuda()
    lam_dev = runtime.probability_cotangent_device(dev, n, torch.from_numpy(g).cuda(), qubits=qs)
    rel_close(lam_dev.cpu().numpy(), lam)
