"""Edge cases of the device path against the oracle (needs a B200): empty plans on the per-gate
and the fused sizes, observables with no terms or only the identity, flip masks over every
qubit (coset traversal), the one-kernel step with nothing in it, sampling of basis states at
both ends of the index range, and the optimizer loop with nothing to train."""
import numpy as np
import pytest

from plans import random_state

pytestmark = pytest.mark.gpu


def rel_close(a, b, tol=1e-10):
    a, b = np.asarray(a), np.asarray(b)
    scale = max(1.0, float(np.max(np.abs(b))) if b.size else 1.0)
    assert float(np.max(np.abs(a - b))) <= tol * scale, (a, b)


@pytest.mark.parametrize("n", [1, 9, 12])
def test_empty_plan_keeps_state_and_adjoint_only_scales_lambda(runtime, n):
    import torch
    g = np.random.Generator(np.random.PCG64(n))
    psi, lam = random_state(g, n), random_state(g, n)
    plan = runtime.CircuitPlan.compile([])
    d = torch.from_numpy(psi.copy()).cuda()
    runtime.plan_apply_device(plan, d, n)
    assert np.array_equal(d.cpu().numpy(), psi)
    dl = torch.from_numpy(lam.copy()).cuda()
    grads = runtime.adjoint_backward_device(plan, d, dl, n, -0.25, np.ones(1, np.uint8), 1)
    assert np.array_equal(d.cpu().numpy(), psi)
    assert np.array_equal(dl.cpu().numpy(), -0.25 * lam)
    assert np.array_equal(grads, [0.0])


def observable(runtime, n, terms):
    c = np.array([t[0] for t in terms], np.float64)
    f = np.array([t[1] for t in terms], np.uint64)
    p = np.array([t[2] for t in terms], np.uint64)
    return runtime.Observable(n, c, f, p)


@pytest.mark.parametrize("n", [5, 12, 22])
def test_observables_without_terms_identity_only_and_full_flips(runtime, oracle, n):
    import torch
    g = np.random.Generator(np.random.PCG64(100 + n))
    psi = random_state(g, n)
    d = torch.from_numpy(psi).cuda()
    out = torch.full_like(d, 7.0)
    v = observable(runtime, n, []).expectation_and_apply(d, out, n)
    assert v[0] == 0.0 and not out.abs().max().item()
    full = (1 << n) - 1
    top = 1 << (n - 1)

    def term(c, f, p):  # (coefficient, flip, phase, Y count mod 4) as the oracle takes them
        return (c, f, p, bin(f & p).count("1") % 4)
    cases = [[term(1.75, 0, 0)],
             [term(0.7, full, 0), term(-1.2, full, full), term(0.3, top, top),
              term(2.0, 0, full), term(0.4, 1, 0)]]
    for terms in cases:
        v = observable(runtime, n, terms).expectation_and_apply(d, out, n)
        rv, rh = oracle.expectation_and_apply(terms, psi, n)
        rel_close(v[0], rv)
        assert float(np.max(np.abs(out.cpu().numpy() - rh))) <= 1e-12 * max(1.0, np.abs(rh).max())
    rel_close(observable(runtime, n, cases[0]).expectation(d, n)[0], 1.75)


def test_one_kernel_step_with_nothing_in_it(runtime):
    plan = runtime.CircuitPlan.compile([])
    obs = observable(runtime, 3, [])
    value, grads = runtime.small_run_device(plan, obs, None, 3, np.zeros(1, np.uint8), 1)
    assert value == 0.0 and np.array_equal(grads, [0.0])
    obs = observable(runtime, 3, [(0.5, 0, 1, 0)])  # Z0 on |000>
    value, _ = runtime.small_run_device(plan, obs, None, 3, np.zeros(1, np.uint8), 1)
    assert value == 0.5


@pytest.mark.parametrize("index", [0, 127])
def test_sampling_basis_states_at_both_ends(runtime, oracle, index):
    import torch
    n = 7
    a = np.zeros(1 << n, np.complex128)
    a[index] = 1.0
    got, total = runtime.sample_indices_device(torch.from_numpy(a).cuda(), n, 500, 9)
    assert total == 1.0
    assert np.array_equal(got, np.full(500, index, np.uint64))
    assert np.array_equal(got, oracle.sample_indices(a, n, 500, 9))


def test_optimizer_loop_with_nothing_to_train_and_one_step(runtime):
    from arcqml_b200.workloads import vqe4
    c, obs = vqe4(seed=2)
    plan = runtime.CircuitPlan.create(c.compile_plan(1))
    ro = runtime.Observable.from_sparse_pauli_op(obs)
    p0 = np.concatenate([[0.0], c.parameter_values()])
    frozen = np.zeros(p0.size, np.uint8)
    e, p = runtime.small_adam_device(plan, ro, 4, p0, frozen, 6)
    assert np.array_equal(p, p0)
    assert np.all(e == e[0])
    value, _ = runtime.small_run_device(plan, ro, None, 4, frozen, p0.size)
    rel_close(e[0], value)
    e1, p1 = runtime.small_adam_device(plan, ro, 4, p0, c.requires_grad_mask(True), 1)
    rel_close(e1[0], value)
    assert not np.array_equal(p1, p0)
