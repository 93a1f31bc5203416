"""CPU oracle of the π0.5 M1 hot path — test infrastructure only (see pi0_oracle.py)."""
