"""Bandit / policy-gradient search over CUDA launch and tile parameters."""
