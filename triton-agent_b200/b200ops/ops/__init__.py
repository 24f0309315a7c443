"""Operator families: one directory per op with contract.yaml,
reference.py (PyTorch reference + generate_test_inputs), templates/cuda_v*.py
(the CUDA variants), verify.py and benchmark.py -- the five-file layout of
the reference project's triton_agent/ops."""

from pathlib import Path

OPS_DIR = Path(__file__).resolve().parent
