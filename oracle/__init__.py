"""ORACLE — test infrastructure only (see oracle/oracle.py); never imported by the product."""
