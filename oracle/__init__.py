"""CPU oracle for the attention hot path (test infrastructure only)."""
