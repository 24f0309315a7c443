"""Tuner: candidate generation over CUDA axes, planner, selector, promoter,
repairer, and the bandit / policy-gradient policies on synthetic rewards."""

import random

import pytest

from b200ops.agent.generator import generate_best_of_n, generate_grid
from b200ops.agent.planner import plan
from b200ops.agent.promoter import should_promote
from b200ops.agent.repairer import repair_action, should_retry
from b200ops.agent.selector import select_best
from b200ops.core.contract import OpContract
from b200ops.core.spec import CandidateResult, OpAction, OpState
from b200ops.microrl.bandit import EpsilonGreedyPolicy, ThompsonSamplingPolicy, UCBPolicy
from b200ops.microrl.grpo_lite import GRPOLite
from b200ops.microrl.reinforce_lite import REINFORCELite, softmax
from b200ops.microrl.trainer import ALL_STRATEGIES, Trainer
from b200ops.ops import OPS_DIR

STATE = OpState("paged_attention", 64, 1, 128, "bf16", "cuda")


def contract(op="paged_attention"):
    return OpContract.from_yaml(OPS_DIR / op / "contract.yaml")


def test_grid_spans_cuda_axes():
    c = contract()
    grid = generate_grid(c, STATE, {"cuda_v1.sm100": None})
    assert {a.rows_per_cta for _, a in grid} == {0, 4} and {a.num_stages for _, a in grid} == {0, 3}
    assert {a.tile_m for _, a in grid} == {0, 296} and {a.tile_k for _, a in grid} == {0, 10}
    assert len(grid) == len({a.arm_key() for _, a in grid})  # no duplicate launches


ROWS = (0, 16, 100, 4096, 16384)


@pytest.mark.parametrize("op", sorted(d.name for d in OPS_DIR.iterdir() if (d / "contract.yaml").exists()))
def test_contract_axes_are_parameters_the_kernels_read(op):
    """Every CUDA axis a contract searches is a b200_launch_cfg field that the
    kernel the op selects (for some size) reads, and every value the contract
    lists is one that kernel accepts -- the tuner never times a dead knob."""
    from b200ops.runtime import lib as L

    spaces = [L.config_space(op, r) for r in ROWS]
    assert all(sp is not None and sp["op"] == op and sp["kernel"] for sp in spaces)
    fields = {}
    for sp in spaces:
        for k, v in sp["fields"].items():
            fields.setdefault(k, set()).update(v["values"])
    for key, values in contract(op).search_space.cuda.items():
        assert key in fields, (op, key, sorted(fields))
        assert set(values) <= fields[key], (op, key, values, fields[key])
        assert 0 in values, (op, key)  # the kernel's default is always an arm


def test_axes_are_pruned_to_the_selected_kernel():
    from b200ops.agent.generator import _axes, default_action, library_axes
    from b200ops.runtime import lib as L

    big = dict(_axes(contract("quant_matmul"), L.config_space("quant_matmul", 4096)))
    assert big["tile_k"] == [0] and big["flags"] == [0, 2, 8] and big["num_stages"] == [0, 4, 6, 8]
    small = dict(_axes(contract("quant_matmul"), L.config_space("quant_matmul", 16)))
    assert small["flags"] == [0] and small["tile_n"] == [0] and small["tile_k"] == [0, 256, 1024]
    assert small["num_stages"] == [0, 4, 6, 8, 12] and small["num_warps"] == [0]
    dec = dict(_axes(contract("paged_attention"), L.config_space("paged_attention", 64)))
    assert dec.get("split", [0]) == [0] and dec["rows_per_cta"] == [0, 4] and dec["tile_m"] == [0, 296]
    fl = dict(_axes(contract("flash_attn_like"), L.config_space("flash_attn_like", 0)))
    assert fl["num_stages"] == [0] and fl["split"] == [0, 4, 16] and fl["flags"] == [0, 16]
    # the default arm launches with an empty b200_launch_cfg
    axes = _axes(contract("paged_attention"), L.config_space("paged_attention", 64))
    d = default_action("cuda_v1.sm100", axes)
    assert not any(d.launch_cfg().values())
    assert d.arm_key() in {a.arm_key() for _, a in generate_grid(contract(), STATE, {"cuda_v1.sm100": None},
                                                                   axes=axes)}
    lib = dict(library_axes(L.config_space("flash_attn_like", 0)))
    assert lib["tile_k"] == [0, 1, 2, 3, 4] and lib["num_stages"] == [0] and lib["num_warps"] == [0]
    assert L.config_space("no_such_op") is None


def test_best_of_n_is_seeded_and_planner_threshold():
    c = contract("quant_matmul")
    a = generate_best_of_n(c, STATE, {"t": None}, n=10, seed=3)
    b = generate_best_of_n(c, STATE, {"t": None}, n=10, seed=3)
    assert [x.to_dict() for _, x in a] == [x.to_dict() for _, x in b]
    def space(**axes):
        return OpContract.from_dict({"op": "x", "inputs": {"a": ["N"]}, "outputs": {"b": ["N"]},
                                     "tolerance": {"max_abs_error": 1, "mean_abs_error": 1}, "search_space": axes})
    # up to 64 points: the whole grid; above: 64 seeded samples
    assert plan(space(split=list(range(16)), stages=list(range(4))), STATE) == {"strategy": "grid", "candidates": 64}
    assert plan(space(split=list(range(20)), stages=list(range(5))), STATE)["strategy"] == "best_of_n"


def test_selector_and_promoter():
    rs = [CandidateResult(reward=1.0, latency_us_p50=50), CandidateResult(reward=1.2, latency_us_p50=80),
          CandidateResult(reward=1.2, latency_us_p50=60)]
    assert select_best([0, 1, 2], rs)[0] == 2
    c = contract()
    good = CandidateResult(compile_pass=True, verify_pass=True, speedup=2.0, variance=0.01)
    assert should_promote(good, c)
    assert not should_promote(CandidateResult(compile_pass=True, verify_pass=True, speedup=1.01), c)
    assert not should_promote(CandidateResult(compile_pass=True, verify_pass=False, speedup=9), c)


def test_repairer_moves_the_failing_parameter():
    a = OpAction("t", num_stages=4, tile_n=256, split=16)
    r = CandidateResult(compile_pass=False, compile_log="int8_gemm: unsupported dtype or shape (status -2)")
    fixed = repair_action(a, r)
    assert fixed.num_stages == 3 and fixed.tile_n == 128 and should_retry(fixed, a, r)
    ws = repair_action(a, CandidateResult(compile_pass=False, compile_log="workspace missing (status -5)"))
    assert ws.split == 0
    assert repair_action(a, CandidateResult(compile_pass=True, verify_pass=True)) is None
    assert not should_retry(a, a, r)


def _arms():
    return [("t", OpAction("t", split=s, num_stages=st)) for s in (8, 16, 32) for st in (2, 3)]


def _reward(a):
    return 1.0 if (a.split == 16 and a.num_stages == 3) else 0.2


@pytest.mark.parametrize("policy", [UCBPolicy(), EpsilonGreedyPolicy(seed=0), ThompsonSamplingPolicy(seed=0)])
def test_bandits_find_the_best_arm(policy):
    arms = _arms()
    acts = [a for _, a in arms]
    for _ in range(150):
        i = policy.select(acts, STATE)
        policy.update(acts[i], STATE, _reward(acts[i]))
    i, _ = policy.best_action(acts, STATE)
    assert acts[i].split == 16 and acts[i].num_stages == 3


def test_reinforce_and_grpo_converge():
    random.seed(0)
    arms = _arms()
    pg = REINFORCELite(learning_rate=0.5, seed=0)
    for _ in range(300):
        i = pg.select(arms, STATE)
        pg.update(arms[i][1], STATE, _reward(arms[i][1]), arms)
    assert _reward(arms[pg.best_action(arms, STATE)][1]) == 1.0
    gr = GRPOLite(learning_rate=0.5, group_size=4, seed=0)
    for _ in range(100):
        idx = gr.select_group(arms, STATE)
        gr.update_group([arms[i][1] for i in idx], [_reward(arms[i][1]) for i in idx], STATE, arms)
    assert _reward(arms[gr.best_action(arms, STATE)][1]) == 1.0
    p = softmax([1.0, 2.0, 3.0])
    assert abs(sum(p) - 1) < 1e-9 and p[2] > p[1] > p[0]


def test_trainer_all_strategies(tmp_path):
    arms = _arms()
    for name in ALL_STRATEGIES:
        tr = Trainer(name, store_path=tmp_path / f"{name}.json")
        for _ in range(5):
            i = tr.select(arms, STATE)
            res = CandidateResult(compile_pass=True, verify_pass=True, reward=_reward(arms[i][1]))
            tr.update(arms[i][1], STATE, res, arms)  # policy-gradient updates get the candidates
    tr = Trainer("ucb", store_path=tmp_path / "best.json")
    res = CandidateResult(compile_pass=True, verify_pass=True, reward=1.0, promoted=True, latency_us_p50=10)
    tr.update(arms[0][1], STATE, res, arms)
    again = Trainer("ucb", store_path=tmp_path / "best.json")
    assert again.get_best_config(STATE)["action"]["split"] == arms[0][1].split
