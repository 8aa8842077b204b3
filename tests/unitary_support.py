"""A CPU backend for arcqml_b200.unitary over the oracle (test infrastructure): the same
operations as the device backend on numpy [D, D] batches."""
import numpy as np


class OracleUnitaryBackend:
    def __init__(self, oracle):
        self.O = oracle

    def basis_batch(self, n):
        return np.eye(1 << n, dtype=np.complex128)

    def apply(self, plan_ops, batch, n):
        out = self.O.plan_apply(plan_ops, batch.reshape(-1), n, batch=batch.shape[0])
        batch[...] = out.reshape(batch.shape)

    def rows_of(self, target):
        return np.ascontiguousarray(target.matrix().T)

    def trace_overlap(self, rows, batch, n):
        # fit/loss.rs:5-19: inputs outer, outputs inner
        s = 0j
        for i in range(rows.shape[0]):
            for o in range(rows.shape[1]):
                s += np.conj(rows[i, o]) * batch[i, o]
        return complex(s)

    def scaled(self, rows, factor, n):
        return factor * rows

    def adjoint(self, plan_ops, batch, lam, n, requires_grad):
        b = batch.shape[0]
        _, _, g = self.O.adjoint_backward(plan_ops, batch.reshape(-1), lam.reshape(-1), n,
                                          np.ones(b), requires_grad, len(requires_grad), batch=b)
        return g

    def to_host(self, batch):
        return batch
