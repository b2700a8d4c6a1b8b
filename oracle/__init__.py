"""CPU oracle for the decode hot path -- test infrastructure only (see oracle.py)."""
