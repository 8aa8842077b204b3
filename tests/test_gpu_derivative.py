"""The device-resident parameter derivative (arcqml_rt_v2_parameter_derivative: out <- dU/dp_slot
psi on every row of a [batch, 2^n] state) against the oracle for every parametrised gate and
slot, controls and targets anywhere (needs a B200). The host-buffer twin (v1) is covered by the
reference cases in test_gpu_parity.py."""
import numpy as np
import pytest

from backends import op
from plans import random_state

pytestmark = pytest.mark.gpu

SLOTS = {11: 1, 12: 1, 13: 1, 14: 1, 15: 3, 22: 1, 23: 1, 24: 1, 25: 1, 30: 1, 31: 1, 32: 1,
         33: 1, 34: 2}


@pytest.mark.parametrize("n,batch", [(3, 4), (9, 3)])
def test_device_parameter_derivative_matches_oracle(runtime, oracle, n, batch):
    import torch
    g = np.random.Generator(np.random.PCG64(31 + n))
    states = random_state(g, n, batch).reshape(batch, -1)
    for opcode, slots in SLOTS.items():
        arity = 1 if opcode <= 15 else 2
        qubits = [int(x) for x in g.choice(n, size=arity, replace=False)]
        o = op(opcode, qubits, [float(x) for x in g.uniform(-3, 3, 3)])
        gate = runtime.gate_descriptor(o.opcode, arity, o.params)
        for slot in range(slots):
            inp = torch.from_numpy(states.copy()).cuda()
            out = torch.full_like(inp, 7.0)
            runtime.parameter_derivative_device(inp, out, n, gate, qubits, slot)
            got = out.cpu().numpy()
            for b in range(batch):
                want = oracle.parameter_derivative(states[b], n, o, slot)
                assert float(np.max(np.abs(got[b] - want))) <= 1e-12, (opcode, slot, b)
            assert np.array_equal(inp.cpu().numpy(), states)  # the input is not written
