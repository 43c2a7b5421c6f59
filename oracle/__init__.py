"""CPU checkers for the MoE FFN path -- test infrastructure only (see oracle.py)."""
