"""rmsnorm operator family."""
