"""rope_kv_append_paged operator family."""
