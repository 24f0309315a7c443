"""b200ops -- sm_100a CUDA backend for the Triton-Agent operator library.

The package mirrors the reference's triton_agent layout (core/, agent/,
microrl/, ops/<op>/...) so an operator registered from its contract.yaml
gets a CUDA variant that the correctness gate and the tuner drive exactly
like the reference's Triton templates.  Kernels live in libb200ops.so
(csrc/, built by build.py) and are reached through runtime.lib (ctypes).
There is no CPU or Triton fallback: if the library or a GPU is missing the
ops raise.
"""

__version__ = "0.1.0"
