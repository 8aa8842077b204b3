"""SparsePauliOp on CPU: the reference's JSON form and validation (observable_tests.rs) and the
compiled (coefficient, flip, phase, y mod 4) terms the runtime receives."""
import json

import pytest

from arcqml_b200.observable import ObservableError, SparsePauliOp


def test_from_json_constructs_operator():
    # crates/arcqml-observable/tests/observable_tests.rs:303-341
    op = SparsePauliOp.from_json(json.dumps({"num_qubits": 3, "terms": [
        {"coefficient": -0.5, "paulis": [{"qubit": 2, "pauli": "X"}, {"qubit": 0, "pauli": "Z"}]},
        {"coefficient": 0.25, "paulis": []}]}))
    assert op.num_qubits == 3 and len(op) == 2
    assert op.compiled_terms() == [(-0.5, 0b100, 0b001, 0), (0.25, 0, 0, 0)]
    assert SparsePauliOp.from_json(op.to_json()) == op


def test_from_json_rejects_unknown_pauli_and_bad_documents():
    # observable_tests.rs:343-358 ("I" is not a JSON Pauli name)
    with pytest.raises(ObservableError, match="must be X, Y or Z, got I"):
        SparsePauliOp.from_json('{"num_qubits": 1, "terms": [{"coefficient": 1.0, '
                                '"paulis": [{"qubit": 0, "pauli": "I"}]}]}')
    for bad in ('{"num_qubits": 1}', '[1, 2]', '{"num_qubits": 1, "terms": [{"paulis": []}]}',
                'not json'):
        with pytest.raises(ObservableError, match="invalid observable JSON"):
            SparsePauliOp.from_json(bad)


def test_constant_and_validation():
    # observable_tests.rs:203-212 and :251-276
    c = SparsePauliOp.constant(2, -0.75)
    assert c.compiled_terms() == [(-0.75, 0, 0, 0)]
    with pytest.raises(ObservableError, match="at least one qubit"):
        SparsePauliOp(0)
    op = SparsePauliOp(2)
    with pytest.raises(ObservableError, match="finite"):
        op.add_term(float("nan"), [(0, "Z")])
    with pytest.raises(ObservableError, match="out of range"):
        op.add_term(1.0, [(2, "Z")])
    with pytest.raises(ObservableError, match="duplicate qubit"):
        op.add_term(1.0, [(1, "X"), (1, "Y")])


def test_compiled_masks_count_y_factors():
    op = SparsePauliOp(4).add_term(0.3, [(0, "Y"), (1, "X"), (3, "Y"), (2, "Z")])
    op.add_term(-1.0, [(1, "Y")]).add_term(2.0, [(0, "Y"), (1, "Y"), (2, "Y")])
    assert op.compiled_terms() == [(0.3, 0b1011, 0b1101, 2), (-1.0, 0b0010, 0b0010, 1),
                                   (2.0, 0b0111, 0b0111, 3)]
    c, f, p = op.masks()
    assert list(c) == [0.3, -1.0, 2.0] and list(f) == [11, 2, 7] and list(p) == [13, 2, 7]


def test_add_scale_and_simplify():
    # observable_tests.rs:213-249
    op = SparsePauliOp(2).add_term(1.0, [(0, "Z")]).add_term(2.0, [(0, "Z")])
    assert len(op) == 2
    s = op.simplify(1e-12)
    assert len(s) == 1 and s.terms[0][0] == 3.0
    assert s.scale(0.5).terms[0][0] == 1.5
    assert len(SparsePauliOp(2).add_term(1e-13, [(0, "Z")]).simplify(1e-12)) == 0
    mixed = SparsePauliOp(3).add_term(0.5, [(2, "X"), (0, "Y")]).add_term(0.25, [(0, "Y"), (2, "X")])
    mixed.add_term(-1.0, [(1, "I"), (0, "Z")]).add_term(1.0, [(0, "Z")])
    t = mixed.simplify()
    assert t.compiled_terms() == [(0.75, 0b101, 0b001, 1)]
    with pytest.raises(ObservableError, match="tolerance"):
        op.simplify(-1.0)
    with pytest.raises(ObservableError, match="finite"):
        op.scale(float("inf"))
