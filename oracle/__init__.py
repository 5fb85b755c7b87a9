"""CPU checker for the W13 hot path (test infrastructure only; see oracle.py)."""
