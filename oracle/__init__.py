"""CPU oracle (test infrastructure only; see oracle/mx_oracle.h)."""
