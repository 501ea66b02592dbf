"""CPU oracle (test infrastructure only; see oracle/eager.py)."""
