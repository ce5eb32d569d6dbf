"""Test infrastructure: CPU oracle for the attention hot path (never shipped or measured)."""
