"""CPU oracle for the `weft` path -- test infrastructure only (see oracle/oracle.py)."""
