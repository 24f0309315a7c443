"""API conformance of the kept reference interface: contract schema,
registry, OpState/OpAction/CandidateResult, verifier, reward, compile step."""

import json
from pathlib import Path

import pytest
import torch

from b200ops.core.compiler import compile_kernel
from b200ops.core.contract import ContractError, OpContract, SearchSpace
from b200ops.core.registry import OpRegistry, RegistryError, get_registry
from b200ops.core.reward import compute_score
from b200ops.core.spec import CandidateResult, OpAction, OpState
from b200ops.core.verifier import check_numerical
from b200ops.ops import OPS_DIR

HOT_OPS = ["rmsnorm", "rope", "kv_append", "paged_kv", "rope_kv_append", "rope_kv_append_paged", "paged_attention",
           "quant_matmul", "flash_attn_like", "rmsnorm_quant", "matmul_epilogue"]


def minimal(**over):
    d = {"op": "x", "inputs": {"a": ["N"]}, "outputs": {"b": ["N"]},
         "tolerance": {"max_abs_error": 1e-3, "mean_abs_error": 1e-4}}
    d.update(over)
    return d


def test_every_op_contract_loads_and_round_trips():
    for op in HOT_OPS:
        c = OpContract.from_yaml(OPS_DIR / op / "contract.yaml")
        assert c.op == op
        assert OpContract.from_dict(c.to_dict()).to_dict() == c.to_dict()


def test_missing_fields_and_bad_files_raise():
    with pytest.raises(ContractError):
        OpContract.from_dict({"op": "x"})
    with pytest.raises(ContractError):
        OpContract.from_yaml("/nonexistent/contract.yaml")


def test_defaults_match_reference_schema():
    c = OpContract.from_dict(minimal())
    assert c.search_space.BLOCK_D == [64, 128, 256, 512]
    assert c.search_space.num_warps == [1, 2, 4, 8]
    assert c.benchmark.warmup == 20 and c.benchmark.repeat == 100
    assert c.promotion.min_speedup == 1.05 and c.promotion.max_variance == 0.10
    assert c.tolerance.max_rel_error is None and c.tolerance.exact is False


def test_search_space_keeps_cuda_axes():
    ss = SearchSpace.from_raw({"split": [8, 16], "stages": [2, 3], "BLOCK_D": [128]})
    assert ss.cuda == {"split": [8, 16], "stages": [2, 3]}
    assert ss.BLOCK_D == [128]
    assert ss.to_dict()["split"] == [8, 16]


def test_registry():
    r = OpRegistry()
    assert r.load_from_dir(OPS_DIR) >= len(HOT_OPS)
    assert set(HOT_OPS) <= set(r.list())
    with pytest.raises(RegistryError):
        r.get("nope")
    assert get_registry() is get_registry()


def test_spec_round_trips_and_legacy_records():
    s = OpState("rmsnorm", 8, 2048, 4096, "bf16", "cuda")
    assert OpState.from_dict(s.to_dict()) == s
    a = OpAction("cuda_v1.sm100", block_d=256, num_warps=8, num_stages=4, split=16, tile_n=256)
    assert OpAction.from_dict(a.to_dict()) == a
    legacy = {"template_id": "v1", "block_d": 64, "num_warps": 2, "num_stages": 3, "vectorize": True, "fusion": False}
    b = OpAction.from_dict(legacy)
    assert b.split == 0 and b.threads == 0
    assert b.launch_cfg()["threads"] == 64 and b.launch_cfg()["stages"] == 3
    r = CandidateResult(compile_pass=True, latency_us_p50=23.4, roofline_fraction=0.8)
    assert CandidateResult.from_dict(r.to_dict()) == r
    assert CandidateResult.from_dict({"compile_pass": True}).verify_pass is False


def test_verifier_tolerances():
    c = OpContract.from_dict(minimal())
    ref = torch.ones(4, 4)
    assert check_numerical(ref + 5e-5, ref, c).verify_pass
    assert not check_numerical(ref + 1e-2, ref, c).verify_pass
    assert not check_numerical(ref.half(), ref, c).verify_pass            # dtype must match
    assert not check_numerical(torch.ones(4, 5), ref, c).verify_pass      # shape must match
    bad = ref.clone()
    bad[0, 0] = float("nan")
    r = check_numerical(bad, ref, c)
    assert not r.verify_pass and json.loads(r.verify_log)["has_nan"]
    rel = OpContract.from_dict(minimal(tolerance={"max_abs_error": 1e-3, "mean_abs_error": 1.0,
                                                  "max_rel_error": 1e-2}))
    big = torch.full((8,), 100.0)
    assert check_numerical(big * 1.005, big, rel).verify_pass
    assert not check_numerical(big * 1.02, big, rel).verify_pass
    ex = OpContract.from_dict(minimal(tolerance={"max_abs_error": 0, "mean_abs_error": 0, "exact": True}))
    assert check_numerical((ref, ref.clone()), (ref, ref), ex).verify_pass
    assert not check_numerical((ref, ref + 1e-7), (ref, ref), ex).verify_pass


def test_reward_rules():
    r = CandidateResult(compile_pass=True, verify_pass=True)
    assert compute_score(r) == pytest.approx(0.8)
    r = CandidateResult(compile_pass=True, verify_pass=True, speedup=1.3)
    assert compute_score(r) == pytest.approx(1.1)
    r = CandidateResult(compile_pass=True, verify_pass=True, speedup=3.0, variance=0.2)
    assert compute_score(r) == pytest.approx(1.1)
    r = CandidateResult(compile_pass=True, verify_pass=False, verify_log=json.dumps({"has_nan": True}))
    assert compute_score(r) == pytest.approx(-1.8)
    r = CandidateResult(compile_pass=True, verify_pass=True, memory_peak_mb=200)
    assert compute_score(r, baseline_memory_mb=100) == pytest.approx(0.6)


def test_compile_step_captures_errors():
    def factory(**kw):
        if kw.get("split", 0) < 0:
            raise ValueError("bad split")
        return lambda *a: a

    ok = compile_kernel(factory, {"split": 4})
    assert ok.success and callable(ok.kernel_fn)
    bad = compile_kernel(factory, {"split": -1})
    assert not bad.success and "bad split" in bad.error_log
