"""CPU oracle of the Chronos MoE layer — test infrastructure only (see moe_oracle.py)."""
