"""CPU oracle (test infrastructure only; see ``oracle/w8a8_oracle.py``)."""
