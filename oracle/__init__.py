"""CPU oracle (test infrastructure only; see fd_oracle.py)."""
