"""CPU oracle (test infrastructure only)."""
