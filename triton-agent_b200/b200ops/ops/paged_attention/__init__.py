"""paged_attention operator family."""
