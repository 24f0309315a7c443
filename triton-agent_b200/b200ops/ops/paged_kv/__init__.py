"""paged_kv operator family."""
