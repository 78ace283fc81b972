"""CPU oracle of the serving path — test infrastructure only (see oracle/oracle.py)."""
