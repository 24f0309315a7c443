"""quant_matmul operator family."""
