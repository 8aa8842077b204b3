"""Argument checks of the state-analysis entry points on CPU: every rejected call fails with the
reference's AnalysisError message (crates/arcqml-analysis/src/error.rs) before any CUDA call,
so no GPU is needed. The amplitude pointers are placeholders that the runtime never reads."""
import ctypes as C

import numpy as np
import pytest

FAKE = C.c_void_p(4096)


def sel(qubits):
    a = np.ascontiguousarray(list(qubits) or [0], dtype=np.uintp)
    return a, a.ctypes.data, len(list(qubits))


@pytest.mark.parametrize("qubits,msg", [
    ([], "at least one qubit must be selected"),
    ([0, 0], "duplicate qubit in selection: 0"),
    ([2], "qubit index out of range: simulator has 2 qubits, got 2"),
    ([1, 0, 1], "duplicate qubit in selection: 1"),
])
def test_marginal_and_cotangent_reject_bad_selections(runtime, qubits, msg):
    L = runtime.load()
    keep, qp, k = sel(qubits)
    with pytest.raises(runtime.RuntimeError, match=msg):
        runtime._status(L.arcqml_rt_v2_marginal_probabilities(FAKE, 1, 2, qp, k, FAKE, None))
    if qubits:  # the cotangent takes an empty selection only as NULL (every qubit)
        with pytest.raises(runtime.RuntimeError, match=msg):
            runtime._status(L.arcqml_rt_v2_probability_cotangent(FAKE, 1, 2, qp, k, FAKE, FAKE,
                                                                 None))


def test_bloch_overlap_and_copy_argument_errors(runtime):
    L = runtime.load()
    with pytest.raises(runtime.RuntimeError, match="simulator has 3 qubits, got 3"):
        runtime._status(L.arcqml_rt_v2_bloch_vector(FAKE, 1, 3, 3, FAKE, None))
    with pytest.raises(runtime.RuntimeError, match="amplitude buffer is null"):
        runtime._status(L.arcqml_rt_v2_overlap(FAKE, None, 1, 3, FAKE, None))
    with pytest.raises(runtime.RuntimeError, match="overlap buffer is null"):
        runtime._status(L.arcqml_rt_v2_overlap(FAKE, FAKE, 1, 3, None, None))
    with pytest.raises(runtime.RuntimeError, match="probability buffer is null"):
        runtime._status(L.arcqml_rt_v2_probabilities(FAKE, 1, 3, None, None))
    with pytest.raises(runtime.RuntimeError, match="batch size must be non-zero"):
        runtime._status(L.arcqml_rt_v2_probabilities(FAKE, 0, 3, FAKE, None))
    f = np.array([1.0, np.nan])
    with pytest.raises(runtime.RuntimeError, match="factors must be finite"):
        runtime._status(L.arcqml_rt_v2_scaled_copy(FAKE, 1, 3, f.ctypes.data, FAKE, None))
    with pytest.raises(runtime.RuntimeError, match="upstream buffer is null"):
        runtime._status(L.arcqml_rt_v2_probability_cotangent(FAKE, 1, 3, None, 0, None, FAKE,
                                                             None))


def test_fidelity_rejects_different_qubit_counts():
    from arcqml_b200 import analysis

    class Fake:
        def __init__(self, n):
            self.num_qubits = n
    with pytest.raises(analysis.AnalysisError,
                       match="cannot compare states with different qubit counts: 2 and 3"):
        analysis.fidelity(Fake(2), Fake(3))
