"""ORACLE — test infrastructure only (see oracle/eager.py).  Never imported by the
product package."""
