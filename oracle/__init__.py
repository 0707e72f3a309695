"""Parity checker (test infrastructure only; see oracle.py)."""
