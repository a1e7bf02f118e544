"""TEST INFRASTRUCTURE ONLY: CPU oracle and reference comparators for the h3q parity tests."""
