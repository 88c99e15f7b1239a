"""Parity checkers (test infrastructure only; see oracle.py)."""
