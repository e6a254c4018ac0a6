"""CPU oracle for the scan path (test infrastructure only; see oracle.py)."""
