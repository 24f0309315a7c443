"""The drop-in boundary through the reference's own loader (CPU).

INTEGRATION.md tells a maintainer to register each CUDA variant inside a
Triton-Agent checkout with a one-line shim file, ops/<op>/templates/
triton_v9.py, that imports this package's factory `sm100`.  This test runs
the reference's unmodified discovery (`_load_templates`, triton_agent/
cli.py:321-360) and compile-argument builder (`_build_compile_args`,
cli.py:281-293), and its compile step (`compile_kernel`, core/compiler.py:37,
46-52; with the default its CompileResult lacks, see the fixture) over such
shim files written into a temporary ops tree, and checks
that `sm100` is discovered, called with the reference's compile_args, and
returns a kernel_fn whose launch configuration maps NUM_WARPS/NUM_STAGES
onto the CUDA launch fields.  Calling it on CPU tensors raises (no CPU
fallback), which the reference pipeline records in compile_log
(cli.py:253-258).  Skipped where no reference checkout is available
(TRITON_AGENT_REF names one)."""

import os
import sys
from pathlib import Path

import pytest
import torch

REF = Path(os.environ.get("TRITON_AGENT_REF", "/root/reference"))
pytestmark = pytest.mark.skipif(not (REF / "triton_agent" / "cli.py").exists(), reason="no reference checkout")

# op -> (shim line, whether the variant takes a CTA size)
OPS = {
    "rmsnorm": True,
    "rope": True,
    "kv_append": True,
    "paged_kv": True,
    "rope_kv_append": True,
    "paged_attention": False,
    "quant_matmul": False,
    "flash_attn_like": False,
    "matmul_epilogue": False,
}


@pytest.fixture(scope="module")
def ref():
    sys.path.insert(0, str(REF))
    try:
        import triton_agent.cli as cli
        import triton_agent.core.compiler as comp
        from triton_agent.core.spec import OpAction, OpState
    finally:
        sys.path.remove(str(REF))
    # The reference's TritonCompiler.compile builds `CompileResult()` before
    # calling the template (core/compiler.py:34), but CompileResult's
    # `success` field has no default (:9-13), so as shipped every
    # compile_kernel call raises TypeError before any template runs.
    with pytest.raises(TypeError):
        comp.compile_kernel(lambda **kw: None, {})
    # With that one default supplied (in memory only), the rest of its
    # compile path is the reference's own.
    import dataclasses

    fixed = dataclasses.make_dataclass("CompileResult", [("success", bool, dataclasses.field(default=False))],
                                       bases=(comp.CompileResult,))
    orig = comp.CompileResult
    comp.CompileResult = fixed
    yield cli, comp.compile_kernel, OpAction, OpState
    comp.CompileResult = orig


@pytest.mark.parametrize("op", sorted(OPS))
def test_reference_loader_discovers_and_compiles_the_shim(op, ref, tmp_path):
    cli, compile_kernel, OpAction, OpState = ref
    tdir = tmp_path / "ops" / op / "templates"
    tdir.mkdir(parents=True)
    (tdir / "triton_v9.py").write_text(
        f"from b200ops.ops.{op}.templates.cuda_v1 import sm100  # noqa: F401  (factory: sm100(**compile_args))\n")
    templates = cli._load_templates(op, tmp_path / "ops")
    assert "sm100" in templates and callable(templates["sm100"]), templates
    state = OpState(op_name=op, B=2, T=64, D=128, dtype="bf16", device="cuda")
    action = OpAction(template_id="sm100", block_d=128, num_warps=4, num_stages=3)
    args = cli._build_compile_args(state, action, op)
    res = compile_kernel(templates["sm100"], args)
    assert res.success, res.error_log
    cfg = res.kernel_fn.launch_cfg
    assert cfg["stages"] == 3
    assert cfg.get("threads") == (128 if OPS[op] else None)


def test_shim_kernel_has_no_cpu_fallback(ref, tmp_path):
    cli, compile_kernel, OpAction, OpState = ref
    from b200ops.runtime import lib as L

    tdir = tmp_path / "ops" / "rmsnorm" / "templates"
    tdir.mkdir(parents=True)
    (tdir / "triton_v9.py").write_text("from b200ops.ops.rmsnorm.templates.cuda_v1 import sm100  # noqa: F401\n")
    fn = compile_kernel(cli._load_templates("rmsnorm", tmp_path / "ops")["sm100"], {"B": 1, "T": 4, "D": 64}).kernel_fn
    with pytest.raises(L.B200OpsError):
        fn(torch.randn(1, 4, 64), torch.ones(64))
