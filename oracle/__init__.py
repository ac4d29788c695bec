"""CPU oracle for the NVFP4 path — test infrastructure only (see oracle/oracle.py)."""
