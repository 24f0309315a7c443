"""Drop-in boundary on the host: every hot-path op has a contract, a
reference, and a CUDA variant discovered by the reference's rule, and the
factory follows the template(**compile_args) -> kernel_fn(*inputs) convention."""

from click.testing import CliRunner

from b200ops import cli
from b200ops.core.spec import OpAction, OpState
from b200ops.ops._variant import launch_cfg_from_args

HOT_OPS = ["rmsnorm", "rope", "kv_append", "paged_kv", "rope_kv_append", "rope_kv_append_paged", "paged_attention",
           "quant_matmul", "flash_attn_like", "rmsnorm_quant", "matmul_epilogue"]


def test_discovery_per_op():
    for op in HOT_OPS:
        t = cli.load_templates(op)
        assert list(t) == ["cuda_v1.sm100"], (op, list(t))
        ref, gen = cli.load_reference(op)
        assert callable(ref) and callable(gen)


def test_compile_args_carry_launch_cfg():
    st = OpState("paged_attention", 64, 1, 128, "bf16", "cuda")
    args = cli.build_compile_args(st, OpAction("cuda_v1.sm100", num_warps=4, num_stages=3, split=32), "paged_attention")
    assert args["split"] == 32 and args["NUM_STAGES"] == 3 and args["B"] == 64
    assert launch_cfg_from_args(args) == {"split": 32, "stages": 3, "threads": 128}
    fac = cli.load_templates("paged_attention")["cuda_v1.sm100"]
    fn = fac(**args)
    assert callable(fn) and fn.launch_cfg["split"] == 32 and "threads" not in fn.launch_cfg


def test_cli_list_runs():
    res = CliRunner().invoke(cli.main, ["list"])
    assert res.exit_code == 0
    for op in HOT_OPS:
        assert op in res.output


def test_shape_parsing():
    assert cli.parse_shape("B=8, T=2048,D=4096") == {"B": 8, "T": 2048, "D": 4096}
