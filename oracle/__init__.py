"""Parity oracle and CPU baseline: test infrastructure only, never the product path."""
