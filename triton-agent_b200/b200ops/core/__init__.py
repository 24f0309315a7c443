"""Operator contracts, registry, action/state/result types, and the
compile -> verify -> profile -> reward pipeline pieces."""
