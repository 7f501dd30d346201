"""CPU oracle of the S6 decode path (test infrastructure only; see s6_oracle.py)."""
