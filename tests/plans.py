"""Seeded random inputs shared by the parity tests: states, unitaries, plans, Pauli sums."""
import math

import numpy as np

from arcqml_b200 import circuit as cm
from backends import op


def random_state(g, n, batch=None):
    shape = (1 << n,) if batch is None else (batch, 1 << n)
    a = g.normal(size=shape) + 1j * g.normal(size=shape)
    a /= np.linalg.norm(a, axis=-1, keepdims=True)
    return np.ascontiguousarray(a)


def random_unitary(g, k):
    dim = 1 << k
    z = g.normal(size=(dim, dim)) + 1j * g.normal(size=(dim, dim))
    q, r = np.linalg.qr(z)
    return q * (np.diag(r) / np.abs(np.diag(r)))


def random_plan(g, n, num_ops, num_params):
    """Random circuit over every parameterized opcode plus fixed gates; shared parameters."""
    param_codes = [11, 12, 13, 14, 15, 22, 23, 24, 25, 30, 31, 32, 33, 34]
    fixed_codes = [1, 2, 3, 4, 5, 9, 16, 18, 19, 26, 27, 28, 29, 35, 36]
    values = g.uniform(-math.pi, math.pi, size=num_params)
    ops = []
    for _ in range(num_ops):
        if g.uniform() < 0.65:
            code = int(g.choice(param_codes))
            arity = 1 if code <= 15 else 2
            q = [int(x) for x in g.choice(n, size=arity, replace=False)]
            slots = cm.slot_count(code)
            params, binds = [0.0, 0.0, 0.0], []
            for s in range(slots):
                if g.uniform() < 0.8:
                    pid = int(g.integers(0, num_params))
                    params[s] = values[pid]
                    binds.append((s, pid + 1))
                else:
                    params[s] = float(g.uniform(-3, 3))
            ops.append(op(code, q, params, bindings=binds))
        else:
            code = int(g.choice(fixed_codes))
            arity = 1 if code <= 15 else (2 if code <= 34 else 3)
            if arity > n:
                continue
            ops.append(op(code, [int(x) for x in g.choice(n, size=arity, replace=False)]))
    return ops


def random_terms(g, n, count):
    from arcqml_b200.workloads import random_pauli_sum
    return random_pauli_sum(n, count, seed=int(g.integers(1 << 30))).compiled_terms()
