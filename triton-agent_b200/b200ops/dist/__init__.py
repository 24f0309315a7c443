"""Multi-GPU partitioning of the hot path (one process per GPU)."""
