"""CPU oracle (test infrastructure only): see ``oracle/ring_oracle.py``."""
