"""Analysis of a sharded state through the device backend (needs a B200): marginals, Bloch
vectors, overlaps and fidelities after a random plan on 4 and 8 ranks emulated as threads on
one GPU, against the oracle on the full state (1e-10)."""
import pytest

from test_sharded_analysis_host import analysis_world

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("size,n", [(4, 9), (8, 10)])
def test_sharded_analysis_on_device_matches_oracle(runtime, size, n):
    from arcqml_b200.sharded import RuntimeBackend, ShardedStateVectorSimulator

    def sim_for(n, comm):
        return ShardedStateVectorSimulator(n, comm=comm, backend=RuntimeBackend(),
                                           chunk_amplitudes=1 << 6, transport="p2p")

    analysis_world(size, n, sim_for, tol=1e-10)
