"""CPU oracle (test infrastructure only; see stepquant_oracle.py)."""
