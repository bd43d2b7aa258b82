"""CPU oracle for the LCSA hot path — test infrastructure only (see oracle/oracle.py)."""
