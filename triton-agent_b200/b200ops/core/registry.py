"""Registry of operator contracts (API of triton_agent/core/registry.py:13-63)."""

from __future__ import annotations

from pathlib import Path

from .contract import OpContract


class RegistryError(Exception):
    """Lookup of an operator that was never registered."""


class OpRegistry:
    def __init__(self) -> None:
        self._ops: dict[str, OpContract] = {}

    def register(self, contract: OpContract) -> None:
        self._ops[contract.op] = contract

    def get(self, op_name: str) -> OpContract:
        try:
            return self._ops[op_name]
        except KeyError:
            raise RegistryError(f"Operator '{op_name}' not registered") from None

    def list(self) -> list[str]:
        return sorted(self._ops)

    def has(self, op_name: str) -> bool:
        return op_name in self._ops

    def load_from_dir(self, ops_dir: str | Path) -> int:
        """Registers every */contract.yaml under ops_dir that parses; returns the count."""
        n = 0
        for path in sorted(Path(ops_dir).rglob("contract.yaml")):
            try:
                self.register(OpContract.from_yaml(path))
            except Exception:
                continue
            n += 1
        return n


_REGISTRY: OpRegistry | None = None


def get_registry() -> OpRegistry:
    global _REGISTRY
    if _REGISTRY is None:
        _REGISTRY = OpRegistry()
    return _REGISTRY
