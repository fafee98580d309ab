"""Test infrastructure: CPU oracle and reference-library bindings (see oracle.py)."""
