"""CPU checker for the tests (test infrastructure only; see oracle.py)."""
