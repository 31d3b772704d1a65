"""Test-only CPU oracle for the DenseGPA core (see ``oracle/dense_gpa.py``).

Never imported by the product package ``gpa_b200``.
"""
from .dense_gpa import (OracleConfig, OracleState, edges_of, forward, gdn_scan,
                        init_parameters, initial_state, tensors_of, unit)

__all__ = ["OracleConfig", "OracleState", "edges_of", "forward", "gdn_scan",
           "init_parameters", "initial_state", "tensors_of", "unit"]
