"""CPU oracle and reference comparators: TEST INFRASTRUCTURE ONLY (see oracle.py)."""
