"""Run-time compiled pass kernels on CPU: the generated sources of a forward and an adjoint
schedule compile for sm_100a with NVRTC (no GPU needed)."""
import pytest

from arcqml_b200 import workloads


def test_generated_pass_kernels_compile(runtime):
    c = workloads.brickwork(10, 3, seed=5)
    plan = runtime.CircuitPlan.create(c.compile_plan(1))
    for adjoint in (False, True):
        r = plan.jit_check(10, adjoint)
        if r["eligible"] == 0 and "not found" in r["message"]:
            pytest.skip("NVRTC is not available: " + r["message"])
        assert r["eligible"] >= 1
        assert r["compiled"] == r["eligible"], r["message"]


def test_jit_check_rejects_small_states(runtime):
    c = workloads.brickwork(4, 1, seed=5)
    plan = runtime.CircuitPlan.create(c.compile_plan(1))
    with pytest.raises(runtime.RuntimeError, match="below 8 qubits"):
        plan.jit_check(4, False)
