"""Argument checks of the device optimizer loop (arcqml_rt_v2_small_adam) on CPU: every
rejected call fails with its message before any CUDA call, so no GPU is needed."""
import math

import numpy as np
import pytest

from arcqml_b200 import circuit as cm
from arcqml_b200.workloads import random_pauli_sum, vqe4


def call(runtime, c, obs, n, steps=5, **kw):
    plan = runtime.CircuitPlan.create(c.compile_plan(1))
    ro = runtime.Observable.from_sparse_pauli_op(obs)
    params = kw.pop("params", None)
    if params is None:
        params = np.concatenate([[0.0], c.parameter_values()])
    req = kw.pop("req", None)
    if req is None:
        req = c.requires_grad_mask(True)
    kw.setdefault("stream", 0)  # the legacy default stream: no torch CUDA call on CPU
    return runtime.small_adam_device(plan, ro, n, params, req, steps, **kw)


def test_rejects_states_above_ten_qubits(runtime):
    c = cm.Circuit(11)
    c.rot("ry", 0.3, 0)
    with pytest.raises(runtime.RuntimeError, match="at most 10 qubits"):
        call(runtime, c, random_pauli_sum(11, 3, seed=1), 11)


def test_rejects_trained_gates_it_cannot_rebuild(runtime):
    c = cm.Circuit(3)
    c.append("u3", (0,), c.add_parameter(0.1), 0.2, 0.3)
    with pytest.raises(runtime.RuntimeError, match="opcode 15 has a trained parameter"):
        call(runtime, c, random_pauli_sum(3, 3, seed=1), 3)
    # the same gate with its parameter frozen is fine for the checks (it is never rebuilt)
    c2 = cm.Circuit(3)
    c2.append("u3", (0,), c2.add_parameter(0.1, requires_grad=False), 0.2, 0.3)
    c2.rot("ry", 0.5, 1)
    with pytest.raises(runtime.RuntimeError, match="step count"):
        call(runtime, c2, random_pauli_sum(3, 3, seed=1), 3, steps=0)


@pytest.mark.parametrize("kw,msg", [
    (dict(steps=0), "step count"),
    (dict(betas=(1.0, 0.999)), "invalid Adam hyperparameters"),
    (dict(betas=(0.9, -0.1)), "invalid Adam hyperparameters"),
    (dict(lr=math.inf), "invalid Adam hyperparameters"),
    (dict(eps=-1.0), "invalid Adam hyperparameters"),
])
def test_rejects_bad_loop_arguments(runtime, kw, msg):
    c, obs = vqe4(seed=1)
    with pytest.raises(runtime.RuntimeError, match=msg):
        call(runtime, c, obs, 4, **kw)


def test_rejects_bad_parameter_arrays(runtime):
    c, obs = vqe4(seed=1)
    p = np.concatenate([[0.0], c.parameter_values()])
    p[3] = math.nan
    with pytest.raises(runtime.RuntimeError, match="must be finite"):
        call(runtime, c, obs, 4, params=p)
    with pytest.raises(ValueError, match="same length"):
        call(runtime, c, obs, 4, params=p[:-1])
    with pytest.raises(runtime.RuntimeError, match="out of range"):
        call(runtime, c, obs, 4, params=p[:4], req=np.ones(4, np.uint8))
    with pytest.raises(runtime.RuntimeError, match="observable acts on 4 qubits"):
        c5 = cm.Circuit(5)
        c5.rot("ry", 0.2, 0)
        call(runtime, c5, obs, 5)


def test_host_adam_update_matches_oracle(oracle):
    """AdamState.update (the host loop's optimizer) against the oracle's f64 Adam over 50
    steps, with and without weight decay."""
    from arcqml_b200.runtime import AdamState
    rng = np.random.default_rng(5)
    for wd in (0.0, 0.01):
        x = rng.uniform(-np.pi, np.pi, 9)
        y, st, ost = x.copy(), AdamState(9), {}
        for _ in range(50):
            g = rng.normal(size=9)
            x = st.update(x, g, lr=0.05, weight_decay=wd)
            y = oracle.adam_step(y, g, ost, lr=0.05, weight_decay=wd)
            np.testing.assert_allclose(x, y, rtol=1e-14, atol=1e-15)
        assert st.step == 50
    with pytest.raises(ValueError):
        AdamState(3).update(np.zeros(4), np.zeros(4))
