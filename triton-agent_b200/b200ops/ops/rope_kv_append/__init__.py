"""rope_kv_append operator family."""
