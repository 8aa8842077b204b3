"""Device sampling (arcqml_rt_v2_sample) against the oracle: shot indices and the running
total bit for bit (needs a B200)."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def rand_state(rng, n, zero_frac=0.2):
    a = rng.normal(size=1 << n) + 1j * rng.normal(size=1 << n)
    a[rng.uniform(size=a.size) < zero_frac] = 0
    return a / np.linalg.norm(a)


@pytest.mark.parametrize("n,shots,seed", [(1, 100, 0), (3, 1000, 42), (10, 20000, 7),
                                          (16, 50000, 2 ** 64 - 1), (22, 4096, 31337)])
def test_sample_indices_match_oracle_bit_for_bit(runtime, oracle, n, shots, seed):
    import torch
    rng = np.random.Generator(np.random.PCG64(n * 1000 + shots))
    a = rand_state(rng, n)
    dev = torch.from_numpy(a).cuda()
    got, total = runtime.sample_indices_device(dev, n, shots, seed)
    ref = oracle.sample_indices(a, n, shots, seed)
    assert np.array_equal(got, ref)
    run = 0.0
    for p in (a.real * a.real + a.imag * a.imag):  # sequential, no FMA
        run += float(p)
    assert total == run


def test_bell_state_sample_counts_through_simulator(runtime, oracle):
    from arcqml_b200.circuit import Circuit
    from arcqml_b200.simulator import StateVectorSimulator
    c = Circuit(2)
    c.append("h", (0,)).append("cnot", (0, 1))
    sim = StateVectorSimulator(2)
    sim.apply_circuit(c)
    counts = sim.sample_counts(1000, seed=42)
    assert sum(counts.values()) == 1000 and set(counts) <= {"00", "11"}
    assert counts == oracle.sample_counts(sim.amplitudes(), 2, 1000, 42)


def test_sampling_errors(runtime):
    import torch
    from arcqml_b200.simulator import SimError, StateVectorSimulator
    sim = StateVectorSimulator(3)
    with pytest.raises(SimError, match="shots must be greater than zero"):
        sim.sample_counts(0, seed=1)
    bad = torch.full((8,), 0.5, dtype=torch.complex128, device="cuda")
    with pytest.raises(runtime.RuntimeError, match="not normalized"):
        runtime.sample_indices_device(bad, 3, 10, 1)
