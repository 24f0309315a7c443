"""kv_append operator family."""
