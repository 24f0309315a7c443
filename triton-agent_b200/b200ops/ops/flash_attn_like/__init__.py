"""flash_attn_like operator family."""
