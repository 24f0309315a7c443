"""Episode / leaderboard persistence and the tuner's warm start, on CPU.

Mirrors the reference's storage tests (test/test_core_modules.py:39-117: save,
list and load episodes; leaderboard upsert on the same key; best config;
empty leaderboard) and adds the roofline and CUDA launch columns plus a warm
start: a second `optimize` search evaluates the stored best configuration
first.  Candidate evaluation is a deterministic stand-in for the GPU
measurement, so the search, record and warm-start logic run without a GPU."""

import json

from b200ops import cli
from b200ops.core.contract import OpContract
from b200ops.core.reward import compute_score
from b200ops.core.spec import CandidateResult, OpAction, OpState
from b200ops.core.storage import EpisodeStore, LeaderboardStore
from b200ops.microrl.bandit import context_key
from b200ops.microrl.trainer import ShapeConfigStore
from b200ops.ops import OPS_DIR

TEMPLATES = {"cuda_v1.sm100": None}


def _state(shape="B=64,Hq=32,D=128"):
    return OpState("paged_attention", 64, 1, 128, "bf16", "cuda", shape=shape)


def test_episode_store_round_trip(tmp_path):
    store = EpisodeStore(tmp_path)
    state = _state()
    action = OpAction(template_id="cuda_v1.sm100", split=32, num_stages=3)
    result = CandidateResult(compile_pass=True, verify_pass=True, latency_us_p50=12.5, speedup=1.3,
                             achieved_GBps=6100.0, roofline_fraction=0.84)
    d = store.save("paged_attention", "ep001", state, action, result, extra={"strategy": "grid"})
    assert (d / "record.json").exists()
    store.save("paged_attention", "ep002", state, action, result)
    assert store.list_episodes("paged_attention") == ["ep001", "ep002"]
    assert store.list_episodes("other") == []
    rec = store.load("paged_attention", "ep001")
    assert rec["episode_id"] == "ep001" and rec["extra"]["strategy"] == "grid"
    assert OpAction.from_dict(rec["action"]) == action
    assert CandidateResult.from_dict(rec["result"]).roofline_fraction == 0.84
    assert OpState.from_dict(rec["state"]).shape == "B=64,Hq=32,D=128"
    assert store.load("paged_attention", "missing") is None


def test_leaderboard_upsert_query_best(tmp_path):
    store = LeaderboardStore(tmp_path / "lb.sqlite")
    a = OpAction(template_id="v1", block_d=256, num_warps=4, threads=256, split=16, tile_m=128, tile_n=256,
                 tile_k=128, num_stages=7)
    r = CandidateResult(compile_pass=True, verify_pass=True, latency_us_p50=23.4, speedup=1.18, reward=0.88,
                        promoted=True, achieved_TOPS=3000.0, roofline_fraction=0.9)
    store.upsert("rmsnorm", "B=8,T=2048,D=4096", "fp16", "cuda", a, r, "ep_001")
    store.upsert("rmsnorm", "B=8,T=2048,D=4096", "fp16", "cuda", a, r, "ep_002")
    rows = store.query("rmsnorm")
    assert len(rows) == 1 and rows[0]["template_id"] == "v1" and rows[0]["speedup"] == 1.18
    assert rows[0]["episode_id"] == "ep_002"  # the newer record of the same key wins
    assert rows[0]["roofline_fraction"] == 0.9 and rows[0]["achieved_TOPS"] == 3000.0
    assert LeaderboardStore.action_of(rows[0]) == a
    store.upsert("rmsnorm", "B=8,T=2048,D=4096", "fp16", "cuda", OpAction(template_id="v2"),
                 CandidateResult(speedup=1.5, reward=0.9, promoted=True), "ep_003")
    store.upsert("rmsnorm", "B=1,T=1,D=4096", "fp16", "cuda", a, CandidateResult(speedup=9.0), "ep_004")
    best = store.best_config("rmsnorm", "B=8,T=2048,D=4096", "fp16")
    assert best["template_id"] == "v2"
    assert [r["episode_id"] for r in store.query("rmsnorm")] == ["ep_004", "ep_003", "ep_002"]
    assert len(store.query("rmsnorm", shape="B=8,T=2048,D=4096", dtype="fp16")) == 2
    assert store.query("nonexistent") == [] and store.best_config("nonexistent", "s", "fp16") is None


def test_state_shape_keys_the_config_store(tmp_path):
    a, b = _state("B=64,Hq=32,D=128"), _state("B=64,Hq=64,D=128")
    assert context_key(a) != context_key(b)
    assert context_key(OpState("x", 1, 2, 3, "bf16", "cuda")) == "x|1|2|3|bf16|cuda"
    store = ShapeConfigStore(tmp_path / "best.json")
    store.set_best(a, OpAction(template_id="t", split=64), CandidateResult(speedup=2.0, roofline_fraction=0.8))
    again = ShapeConfigStore(tmp_path / "best.json")
    assert again.get_historical_best(a)["split"] == 64 and a.historical_best_config["split"] == 64
    assert again.get_historical_best(b) is None
    assert json.loads((tmp_path / "best.json").read_text())[context_key(a)]["roofline_fraction"] == 0.8


def _fake_eval(log):
    """Deterministic stand-in for compile -> verify -> profile: split 64 with
    3 stages is the fastest configuration."""
    def ev(tid, action):
        log.append(action)
        # best arm: 4 kv heads per CTA, two CTAs per SM, ring depth 3, no claimed chunks
        lat = (10.0 + (0 if action.rows_per_cta == 4 else 2) + (0 if action.tile_m == 296 else 1)
               + (0 if action.num_stages == 3 else 0.5) + action.tile_k / 10)
        r = CandidateResult(compile_pass=True, verify_pass=True, latency_us_p50=lat, speedup=12.0 / lat,
                            roofline_fraction=8.0 / lat)
        compute_score(r)
        return r
    return ev


def _run(tmp_path, strategy, max_candidates, warm_start=True):
    from b200ops.agent.promoter import should_promote
    from b200ops.agent.selector import select_best

    contract = OpContract.from_yaml(OPS_DIR / "paged_attention" / "contract.yaml")
    state = _state()
    warm = cli.warm_start_actions(state, TEMPLATES, ShapeConfigStore(tmp_path / "best_configs.json"),
                                  LeaderboardStore(tmp_path / "leaderboard.sqlite")) if warm_start else []
    log = []
    cands, results = cli.search(contract, state, TEMPLATES, _fake_eval(log), strategy, max_candidates, 1,
                                tmp_path / "best_configs.json", warm)
    best_i, best = select_best(cands, results)
    best.promoted = should_promote(best, contract)
    path, ep = cli.record_outcome(state, cands, results, best_i, tmp_path, {"strategy": strategy})
    return log, cands[best_i][1], best, path, ep


def test_optimize_records_and_warm_starts(tmp_path):
    best_key = (4, 296, 3, 0)
    key = lambda a: (a.rows_per_cta, a.tile_m, a.num_stages, a.tile_k)  # noqa: E731
    log, action, best, path, ep = _run(tmp_path, "grid", 32)
    assert len(log) == 16 and key(action) == best_key and best.promoted
    rec = json.loads((path / "record.json").read_text())
    assert len(rec["extra"]["candidates"]) == 16 and rec["result"]["latency_us_p50"] == best.latency_us_p50
    row = LeaderboardStore(tmp_path / "leaderboard.sqlite").best_config("paged_attention", "B=64,Hq=32,D=128", "bf16")
    assert row["episode_id"] == ep and row["rows_per_cta"] == 4 and abs(row["roofline_fraction"] - 0.8) < 1e-9

    # one candidate only: without a warm start the grid's first point (every default)
    log, action, _, _, _ = _run(tmp_path / "cold", "grid", 1, warm_start=False)
    assert key(action) == (0, 0, 0, 0)
    # with it, the stored best is evaluated first and stays the best
    for strategy in ("grid", "best_of_n", "ucb", "reinforce", "grpo"):
        log, action, _, _, _ = _run(tmp_path, strategy, 1)
        assert key(log[0]) == best_key, strategy
        assert key(action) == best_key, strategy
    assert len(EpisodeStore(tmp_path).list_episodes("paged_attention")) == 6


def test_leaderboard_and_replay_commands(tmp_path):
    from click.testing import CliRunner

    _, _, _, _, ep = _run(tmp_path, "grid", 4)
    res = CliRunner().invoke(cli.main, ["leaderboard", "paged_attention", "--out", str(tmp_path)])
    assert res.exit_code == 0 and "rows_per_cta=0 tile=296x0x0 flags=0 stages=0" in res.output and ep in res.output, \
        res.output
    res = CliRunner().invoke(cli.main, ["replay", "paged_attention", ep, "--out", str(tmp_path)])
    assert res.exit_code == 0 and json.loads(res.output)["episode_id"] == ep
    res = CliRunner().invoke(cli.main, ["replay", "paged_attention", "nope", "--out", str(tmp_path)])
    assert res.exit_code != 0


def test_leaderboard_gains_columns_added_after_it_was_written(tmp_path):
    """A leaderboard written before the flags column existed is migrated in
    place: old rows read back with flags NULL -> 0, new rows store it."""
    import sqlite3

    db = tmp_path / "lb.sqlite"
    conn = sqlite3.connect(str(db))
    conn.execute("CREATE TABLE leaderboard (id INTEGER PRIMARY KEY AUTOINCREMENT, op_name TEXT NOT NULL, "
                 "shape TEXT NOT NULL, dtype TEXT NOT NULL, device TEXT NOT NULL, template_id TEXT, block_d INTEGER, "
                 "num_warps INTEGER, num_stages INTEGER, vectorize INTEGER, threads INTEGER, rows_per_cta INTEGER, "
                 "split INTEGER, tile_m INTEGER, tile_n INTEGER, tile_k INTEGER, latency_us_p50 REAL, speedup REAL, "
                 "reward REAL, promoted INTEGER, achieved_GBps REAL, achieved_TOPS REAL, roofline_fraction REAL, "
                 "num_gpus INTEGER, episode_id TEXT, timestamp REAL, "
                 "UNIQUE(op_name, shape, dtype, device, template_id))")
    conn.execute("INSERT INTO leaderboard (op_name, shape, dtype, device, template_id, block_d, num_warps, "
                 "num_stages, vectorize, threads, rows_per_cta, split, tile_m, tile_n, tile_k, speedup) "
                 "VALUES ('gemm', 'M=16', 'fp16', 'cuda', 'old', 128, 4, 3, 0, 0, 0, 0, 0, 0, 256, 1.0)")
    conn.commit()
    conn.close()
    lb = LeaderboardStore(db)
    assert lb.action_of(lb.best_config("gemm", "M=16", "fp16")).flags == 0
    lb.upsert("gemm", "M=4096", "fp16", "cuda", OpAction("new", flags=2),
              CandidateResult(compile_pass=True, verify_pass=True, speedup=2.0), "e1")
    assert lb.action_of(lb.best_config("gemm", "M=4096", "fp16")).flags == 2
