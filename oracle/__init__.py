"""CPU checkers for the hot path -- test infrastructure only (see oracle.py)."""
