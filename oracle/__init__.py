"""CPU oracle (test infrastructure only; see icsa_oracle.py)."""
