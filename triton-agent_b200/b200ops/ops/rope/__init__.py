"""rope operator family."""
