"""CPU oracle for the Walsh forward hot path (test infrastructure only)."""
