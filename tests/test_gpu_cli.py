"""The drop-in path end to end on the GPU: the correctness gate
(verify-correctness) passes every CUDA variant against its PyTorch reference
through the same discovery / compile / check_numerical pipeline as the
reference's CLI, and the tuner (optimize) evaluates CUDA launch
configurations and records a verified best."""

import json

import pytest
from click.testing import CliRunner

from b200ops import cli

pytestmark = pytest.mark.gpu

CASES = [
    ("rmsnorm", "B=2,T=64,D=4096", "bf16"),
    ("rmsnorm", "B=2,T=33,D=1000", "fp32"),
    ("rope", "B=2,H=4,T=64,D=128", "bf16"),
    ("kv_append", "B=3,H=4,L=256,T_new=5,D=128", "bf16"),
    ("paged_kv", "B=4,H=8,num_blocks=64,block_size=16,T_new=2,D=128", "fp16"),
    ("rope_kv_append", "B=2,H=4,L=64,T_new=3,D=64", "fp16"),
    ("rope_kv_append_paged", "T=16,Hq=32,Hkv=8,D=128,num_blocks=512,block_size=16", "bf16"),
    ("paged_attention", "B=4,H=32,D=128,num_blocks=256,block_size=16,max_blocks=32,ctx_len=500,H_kv=8", "bf16"),
    ("paged_attention", "B=2,H=8,D=128,num_blocks=64,block_size=16,max_blocks=8,ctx_len=100", "fp16"),
    ("quant_matmul", "B=2,M=64,K=512,N=384", "fp16"),
    ("quant_matmul", "B=1,M=300,K=1024,N=512", "fp32"),
    ("flash_attn_like", "B=1,H=4,T=256,S=256,D=64", "bf16"),
    ("flash_attn_like", "B=1,H=2,T=384,S=384,D=128", "fp16"),
    ("rmsnorm_quant", "B=2,T=64,D=4096", "bf16"),
    ("rmsnorm_quant", "B=3,T=5,D=1024", "fp32"),
    ("matmul_epilogue", "B=2,M=256,K=1024,N=768", "fp16"),
    ("matmul_epilogue", "B=1,M=300,K=512,N=264", "bf16"),
]


@pytest.mark.parametrize("op,shape,dtype", CASES)
def test_verify_correctness_passes(op, shape, dtype, tmp_path):
    out = tmp_path / "r.json"
    res = CliRunner().invoke(cli.main, ["verify-correctness", op, "--shape", shape, "--dtype", dtype,
                                        "--json-out", str(out)])
    rows = json.loads(out.read_text()) if out.exists() else []
    assert res.exit_code == 0, (res.output, rows)
    assert rows and all(r["verify"] for r in rows), rows


@pytest.mark.parametrize("strategy", ["grid", "ucb"])
def test_optimize_records_a_verified_best(strategy, tmp_path):
    res = CliRunner().invoke(cli.main, ["optimize", "rmsnorm", "--shape", "B=4,T=256,D=4096", "--dtype", "bf16",
                                        "--strategy", strategy, "--max-candidates", "4", "--out", str(tmp_path)])
    assert res.exit_code == 0, res.output
    eps = list((tmp_path / "rmsnorm").glob("*/record.json"))
    assert len(eps) == 1
    rec = json.loads(eps[0].read_text())
    assert rec["result"]["verify_pass"] and rec["result"]["latency_us_p50"] > 0
    assert len(rec["extra"]["candidates"]) == 4
    assert {c["action"]["threads"] for c in rec["extra"]["candidates"]} <= {0, 128, 256, 512, 1024}
    assert (tmp_path / "leaderboard.sqlite").exists()
    # a second run warm-starts from the leaderboard's best and evaluates it first
    res = CliRunner().invoke(cli.main, ["optimize", "rmsnorm", "--shape", "B=4,T=256,D=4096", "--dtype", "bf16",
                                        "--strategy", strategy, "--max-candidates", "1", "--out", str(tmp_path)])
    assert res.exit_code == 0, res.output
    recs = sorted((tmp_path / "rmsnorm").glob("*/record.json"))
    second = json.loads(recs[-1].read_text())
    assert second["extra"]["warm_start"] and second["extra"]["candidates"][0]["action"] == \
        second["extra"]["warm_start"][0]


def test_bad_launch_config_becomes_a_failed_candidate():
    """A launch parameter the kernel rejects is caught into compile_log, as in
    the reference pipeline, instead of aborting the run."""
    from b200ops.core.contract import OpContract
    from b200ops.core.spec import OpAction, OpState
    from b200ops.ops import OPS_DIR

    contract = OpContract.from_yaml(OPS_DIR / "rmsnorm" / "contract.yaml")
    ref_fn, gen_fn = cli.load_reference("rmsnorm")
    inputs = gen_fn(B=1, T=4, D=256, dtype=__import__("torch").float32, device="cuda")
    factory = cli.load_templates("rmsnorm")["cuda_v1.sm100"]
    st = OpState("rmsnorm", 1, 4, 256, "fp32", "cuda")
    r = cli.evaluate("rmsnorm", contract, factory, OpAction("cuda_v1.sm100", threads=48), st, inputs,
                     ref_fn(*inputs))
    assert r.compile_pass and not r.verify_pass and "bad argument" in r.compile_log


# The hot kernels' real launch parameters: the persistent decode (kv heads per
# CTA, ring depth, grid, claimed chunks), the INT8 GEMM at a CTA-pair size and
# at a streaming size, and the flash prefill (head groups, FMA-pipe
# exponentials, persistent kernel).
TUNE = [
    ("paged_attention", "B=32,H=32,H_kv=8,D=128,num_blocks=4096,block_size=16,max_blocks=128,ctx_len=1800", "bf16"),
    ("quant_matmul", "B=1,M=512,K=1024,N=2048", "fp16"),
    ("quant_matmul", "B=1,M=16,K=4096,N=4096", "fp16"),
    ("flash_attn_like", "B=1,H=8,T=1024,S=1024,D=128", "bf16"),
]


@pytest.mark.parametrize("op,shape,dtype", TUNE)
def test_optimize_tunes_the_hot_kernels_launch_parameters(op, shape, dtype, tmp_path):
    """optimize --strategy ucb measures the kernel's all-default launch and
    other configurations of the parameters b200_query_config_space says the
    selected kernel reads; every candidate passes the correctness gate and
    the episode records the default beside the best."""
    from b200ops.core.spec import CUDA_FIELDS

    res = CliRunner().invoke(cli.main, ["optimize", op, "--shape", shape, "--dtype", dtype, "--strategy", "ucb",
                                        "--max-candidates", "6", "--out", str(tmp_path)])
    assert res.exit_code == 0, res.output
    rec = json.loads(next((tmp_path / op).glob("*/record.json")).read_text())
    extra = rec["extra"]
    space = extra["config_space"]
    assert space and space["op"] == op
    reads = set(space["fields"])
    cands = extra["candidates"]
    assert len(cands) == 6 and all(c["result"]["verify_pass"] for c in cands), cands
    cfgs = set()
    for c in cands:
        a = c["action"]
        knobs = {f: a[f] for f in CUDA_FIELDS if a[f]}
        if a["num_stages"]:
            knobs["stages"] = a["num_stages"]
        assert set(knobs) <= reads, (knobs, reads)  # no dead knob is ever timed
        cfgs.add(tuple(sorted(knobs.items())))
    assert len(cfgs) == 6  # six different launches
    assert () in cfgs  # the kernel's defaults
    d = extra["default"][0]["result"]
    assert d["verify_pass"] and d["latency_us_p50"] > 0
    assert rec["result"]["latency_us_p50"] > 0
