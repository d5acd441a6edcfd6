"""Test oracles for the fixed-mode codec (test infrastructure only; never
imported by the product package)."""
