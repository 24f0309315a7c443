"""CPU oracle for the Triton-Agent operator hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the algorithms of the reference project's
PyTorch operator references (triton_agent/ops/<op>/reference.py).  It is the
parity oracle for the CUDA library: only tests/, __graft_entry__.smoke() and the
cpu_baseline leg of bench.py may import it.  Nothing in the product package
(triton-agent_b200/b200ops) imports or calls it, and the product never falls
back to it.

Parity pinning: the reference ships no golden vectors or known-answer tests
for these operators.  The restatements are pinned against fixtures produced
by running the reference's own functions in this container
(tests/golden/make_golden.py writes tests/golden/*.pt; tests/test_oracle_golden.py
checks them).  paged_attention's reference raises at reference.py:50, so its
restatement is pinned through the reference's flash_attn_like SDPA applied to
the gathered pages, which is the same softmax(q K^T * scale) V the paged
reference intends.
"""

from . import ops  # noqa: F401
