"""Test infrastructure: CPU checkers for the Envision dense-linear path (never product code)."""
