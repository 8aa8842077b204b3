"""Pins the CPU oracle to the reference's own known-answer tests (no GPU needed)."""
import pytest

import reference_cases as rc
from backends import OracleBackend


@pytest.mark.parametrize("case", rc.ALL_CASES, ids=lambda f: f.__name__)
def test_oracle_reference_case(oracle, case):
    case(OracleBackend(oracle))


def test_oracle_h2_vqe_trajectory(oracle):
    rc.case_h2_vqe_trajectory(OracleBackend(oracle), oracle.adam_step)
