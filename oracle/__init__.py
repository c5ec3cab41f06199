"""CPU oracle for the INT4 KV-cache hot path (test infrastructure only)."""
