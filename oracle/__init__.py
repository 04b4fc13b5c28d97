"""Test infrastructure: the CPU oracle (see oracle/oracle.py). Not part of the product."""
