"""CPU oracle package (test infrastructure only; see tierkv_oracle.py)."""
