"""CPU oracle of the reference's KV swap semantics (test infrastructure only)."""
