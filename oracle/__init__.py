"""CPU oracle of the routed-MoE chain (test infrastructure only; see oracle.py)."""
