"""CPU oracle for the SBDA hot path (test infrastructure only; see sbda_oracle)."""
