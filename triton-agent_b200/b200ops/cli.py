"""Command line: the correctness gate and the tuner over the CUDA variants.

    python -m b200ops.cli list
    python -m b200ops.cli verify-correctness OP [--shape K=V,...] [--dtype bf16]
    python -m b200ops.cli optimize OP [--shape ...] [--strategy grid|best_of_n|ucb|thompson|epsilon|reinforce|grpo]
    python -m b200ops.cli leaderboard OP [--shape ...] [--dtype ...]
    python -m b200ops.cli replay OP EPISODE_ID

Pipeline glue follows the reference's triton_agent/cli.py: contracts are
registered from ops/<op>/contract.yaml (:408-416), variants are discovered
from ops/<op>/templates (:321-360, here cuda_v*.py), the reference function
and input generator come from ops/<op>/reference.py (:363-390), and each
candidate goes compile -> run -> check_numerical -> profile -> reward
(:193-278, :705-769).  Failures are caught into compile_log/verify_log, so a
bad launch configuration costs a candidate, not the run.
"""

from __future__ import annotations

import importlib.util
import json
import sys
import time
from pathlib import Path
from typing import Any

import click

from .core.compiler import compile_kernel
from .core.contract import OpContract
from .core.registry import get_registry
from .core.reward import compute_score
from .core.spec import CandidateResult, OpAction, OpState
from .core.verifier import check_numerical
from .ops import OPS_DIR

DTYPES = {"fp16": "float16", "bf16": "bfloat16", "fp32": "float32"}


def ensure_registered(op: str, ops_dir: Path = OPS_DIR) -> None:
    reg = get_registry()
    if not reg.has(op):
        path = ops_dir / op / "contract.yaml"
        if path.exists():
            reg.register(OpContract.from_yaml(path))


def _import_path(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(name, str(path))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_templates(op: str, ops_dir: Path = OPS_DIR) -> dict[str, Any]:
    """template_id -> factory, for every public callable of
    ops/<op>/templates/cuda_v*.py whose name neither starts with the op name
    nor ends with `_kernel` (the reference's discovery rule)."""
    out: dict[str, Any] = {}
    tdir = ops_dir / op / "templates"
    for path in sorted(tdir.glob("cuda_v*.py")):
        mod = _import_path(f"b200ops.ops.{op}.templates.{path.stem}", path)
        for name in dir(mod):
            if name.startswith("_") or name.startswith(op) or name.endswith("_kernel"):
                continue
            obj = getattr(mod, name)
            if callable(obj) and not isinstance(obj, type):
                out[f"{path.stem}.{name}"] = obj
    return out


def load_reference(op: str, ops_dir: Path = OPS_DIR):
    path = ops_dir / op / "reference.py"
    if not path.exists():
        return None, None
    mod = _import_path(f"b200ops.ops.{op}.reference", path)
    return getattr(mod, op, None), getattr(mod, "generate_test_inputs", None)


def build_compile_args(state: Any, action: OpAction, op: str) -> dict[str, Any]:
    args = {"B": state.B, "T": state.T, "D": state.D, "BLOCK_SIZE": action.block_d,
            "NUM_WARPS": action.num_warps, "NUM_STAGES": action.num_stages}
    if "rope" in op:
        args["H"] = getattr(state, "H", 32)
    args.update({k: v for k, v in action.launch_cfg().items() if v})
    return args


def parse_shape(shape: str) -> dict[str, int]:
    out = {}
    for kv in filter(None, (s.strip() for s in shape.split(","))):
        k, v = kv.split("=")
        out[k.strip()] = int(v)
    return out


def _torch_dtype(name: str):
    import torch

    return getattr(torch, DTYPES.get(name, name))


def _clone_inputs(inputs):
    import torch

    return tuple(x.clone() if isinstance(x, torch.Tensor) else x for x in inputs)


def evaluate(op: str, contract: OpContract, factory, action: OpAction, state, inputs, ref_out,
             baseline_us: float = 0.0, profile: bool = True) -> CandidateResult:
    """compile -> run -> verify -> profile -> reward for one candidate."""
    from .core.profiler import profile_kernel

    comp = compile_kernel(factory, build_compile_args(state, action, op))
    if not comp.success:
        r = CandidateResult(compile_pass=False, compile_log=comp.error_log)
        compute_score(r)
        return r
    run_inputs = _clone_inputs(inputs)  # in-place variants must not see earlier writes
    try:
        out = comp.kernel_fn(*run_inputs)
    except Exception as e:
        r = CandidateResult(compile_pass=True, verify_pass=False, compile_log=str(e))
        compute_score(r)
        return r
    r = check_numerical(out, ref_out, contract)
    if r.verify_pass and profile:
        p = profile_kernel(comp.kernel_fn, run_inputs, warmup=contract.benchmark.warmup,
                           repeat=contract.benchmark.repeat, baseline_latency_us=baseline_us)
        p.verify_log = r.verify_log
        r = p
    compute_score(r)
    return r


@click.group()
def main() -> None:
    """sm_100a operator backend: correctness gate and tuner."""


@main.command("list")
def list_ops() -> None:
    """Operators with a contract and a CUDA variant."""
    for d in sorted(OPS_DIR.iterdir()):
        if (d / "contract.yaml").exists():
            click.echo(f"{d.name}: {', '.join(load_templates(d.name)) or '(no variants)'}")


@main.command("verify-correctness")
@click.argument("op")
@click.option("--shape", default="", help="generate_test_inputs keyword arguments, e.g. B=8,T=2048,D=4096")
@click.option("--dtype", default="fp16")
@click.option("--json-out", default=None, help="write the per-variant results as JSON")
def verify_correctness(op: str, shape: str, dtype: str, json_out: str | None) -> None:
    """Checks every CUDA variant of OP against its PyTorch reference."""
    ensure_registered(op)
    if not get_registry().has(op):
        raise click.ClickException(f"Operator '{op}' not found.")
    contract = get_registry().get(op)
    ref_fn, gen_fn = load_reference(op)
    inputs = gen_fn(**parse_shape(shape), dtype=_torch_dtype(dtype), device="cuda")
    ref_out = ref_fn(*_clone_inputs(inputs))
    parsed = parse_shape(shape)
    state = OpState(op, parsed.get("B", 8), parsed.get("T", 2048), parsed.get("D", 4096), dtype, "cuda")
    rows = []
    ok_all = True
    for tid, factory in sorted(load_templates(op).items()):
        action = OpAction(template_id=tid, block_d=256, num_warps=4, num_stages=3)
        r = evaluate(op, contract, factory, action, state, inputs, ref_out, profile=False)
        ok_all &= r.verify_pass
        log = json.loads(r.verify_log) if r.verify_log.startswith("{") else {}
        rows.append({"template": tid, "compile": r.compile_pass, "verify": r.verify_pass,
                     "max_abs_error": log.get("max_abs_error"), "mean_abs_error": log.get("mean_abs_error"),
                     "nan_inf": bool(log.get("has_nan") or log.get("has_inf")),
                     "error": (r.compile_log or ("" if r.verify_pass else r.verify_log))[:200]})
    try:
        from rich.console import Console
        from rich.table import Table

        t = Table(title=f"Correctness: {op} ({shape or 'defaults'}, {dtype})")
        for col in ("Template", "Compile", "Max AE", "Mean AE", "NaN/Inf", "Verdict"):
            t.add_column(col)
        for r in rows:
            fmt = lambda v: "—" if v is None else f"{v:.1e}"  # noqa: E731
            t.add_row(r["template"], "OK" if r["compile"] else "FAIL", fmt(r["max_abs_error"]),
                      fmt(r["mean_abs_error"]), "YES" if r["nan_inf"] else "no", "PASS" if r["verify"] else "FAIL")
        Console().print(t)
    except ImportError:
        for r in rows:
            click.echo(json.dumps(r))
    if json_out:
        Path(json_out).write_text(json.dumps(rows, indent=2))
    if not ok_all:
        sys.exit(1)


def shape_key(parsed: dict[str, int]) -> str:
    """Leaderboard and config-store key of a --shape: its K=V pairs in key
    order (the reference keys by "B=..,T=..,D=.." at cli.py:177; these
    operators also have M/N/K, heads and cache axes)."""
    return ",".join(f"{k}={parsed[k]}" for k in sorted(parsed)) or "default"


def warm_start_actions(state: OpState, templates: dict[str, Any], config_store, leaderboard) -> list[tuple[str, OpAction]]:
    """Historical best configurations for this (op, shape, dtype): the tuner's
    ShapeConfigStore entry (microrl/trainer.py:41-80) and the leaderboard's
    best row (core/storage.py:150-165), for variants that still exist,
    without duplicates.  They are evaluated first, so a later search starts
    from the best known launch configuration."""
    found = []
    hist = config_store.get_historical_best(state)
    if hist:
        found.append(OpAction.from_dict(hist))
    row = leaderboard.best_config(state.op_name, state.shape, state.dtype)
    if row:
        found.append(leaderboard.action_of(row))
    out, seen = [], set()
    for a in found:
        if a.template_id in templates and a.arm_key() not in seen:
            seen.add(a.arm_key())
            out.append((a.template_id, a))
    return out


def space_rows(op: str, parsed: dict[str, int], gen_fn=None) -> int:
    """The row count b200_query_config_space selects an op's kernel by: GEMM
    rows (B*M), new tokens of the paged append, sequences of the decode;
    unspecified sizes take the input generator's defaults."""
    import inspect

    dflt = {}
    if gen_fn is not None:
        dflt = {k: p.default for k, p in inspect.signature(gen_fn).parameters.items()
                if isinstance(p.default, int) and not isinstance(p.default, bool)}
    get = lambda k, d=0: int(parsed.get(k, dflt.get(k, d)))  # noqa: E731
    if op in ("quant_matmul", "matmul_epilogue"):
        return get("B", 1) * get("M", 0)
    if op == "rope_kv_append_paged":
        return get("T", 0)
    if op == "paged_attention":
        return get("B", 0)
    return 0


def search(contract: OpContract, state: OpState, templates: dict[str, Any], eval_fn, strategy: str,
           max_candidates: int, retry: int, store_path: Path, warm=(), axes=None) -> tuple[list, list[CandidateResult]]:
    """Candidate search of `optimize` (reference cli.py:57-160): grid or
    best-of-n lists, or a bandit / policy-gradient / GRPO trainer choosing
    one candidate per step, with repair-and-retry of failed candidates.
    `warm` candidates are evaluated first.  `axes` (OpAction field, values)
    replaces the contract's search space when given.  eval_fn(template_id,
    action) returns the CandidateResult."""
    from .agent.generator import generate_best_of_n, generate_grid
    from .agent.repairer import repair_action, should_retry
    from .microrl.trainer import Trainer

    warm = list(warm)
    warm_keys = {a.arm_key() for _, a in warm}
    if strategy in ("grid", "best_of_n"):
        gen = generate_grid(contract, state, templates, axes=axes) if strategy == "grid" else \
            generate_best_of_n(contract, state, templates, n=max_candidates, seed=0, axes=axes)
        cands = (warm + [c for c in gen if c[1].arm_key() not in warm_keys])[:max_candidates]
        return cands, [eval_fn(t, a) for t, a in cands]
    all_c = warm + [c for c in generate_grid(contract, state, templates, axes=axes)
                    if c[1].arm_key() not in warm_keys]
    trainer = Trainer(strategy=strategy, store_path=store_path)
    cands, results = [], []
    for step in range(max_candidates):
        i = step if step < len(warm) else trainer.select(all_c, state)
        tid, action = all_c[i]
        r = eval_fn(tid, action)
        for _ in range(retry):
            if r.compile_pass and r.verify_pass:
                break
            fixed = repair_action(action, r)
            if not should_retry(fixed, action, r):
                break
            action = fixed
            if all(a.arm_key() != action.arm_key() for _, a in all_c):
                all_c.append((tid, action))
            r = eval_fn(tid, action)
        trainer.update(action, state, r, all_c)
        cands.append((tid, action))
        results.append(r)
    return cands, results


def record_outcome(state: OpState, cands: list, results: list[CandidateResult], best_i: int, out: Path,
                   extra: dict[str, Any] | None = None) -> tuple[Path, str]:
    """Saves the episode (core/storage.py:13-65 layout), upserts the best into
    the leaderboard (storage.py:102-137, cli.py:171-181) and, when promoted,
    into the ShapeConfigStore the next run warm-starts from."""
    from .core.storage import EpisodeStore, LeaderboardStore
    from .microrl.trainer import ShapeConfigStore

    tid, action = cands[best_i]
    best = results[best_i]
    episode_id = f"{int(time.time() * 1000)}_{tid}"
    rec_extra = dict(extra or {})
    rec_extra["candidates"] = [{"action": a.to_dict(), "result": r.to_dict()} for (_, a), r in zip(cands, results)]
    path = EpisodeStore(out).save(state.op_name, episode_id, state, action, best, extra=rec_extra)
    LeaderboardStore(out / "leaderboard.sqlite").upsert(state.op_name, state.shape, state.dtype, state.device,
                                                        action, best, episode_id)
    if best.promoted:
        ShapeConfigStore(out / "best_configs.json").set_best(state, action, best)
    return path, episode_id


@main.command()
@click.argument("op")
@click.option("--shape", default="")
@click.option("--dtype", default="fp16")
@click.option("--strategy", default="grid",
              type=click.Choice(["grid", "best_of_n", "ucb", "thompson", "epsilon", "reinforce", "grpo"]))
@click.option("--max-candidates", default=16, type=int)
@click.option("--retry", default=1, type=int)
@click.option("--out", default="episodes", help="directory for episodes, leaderboard.sqlite and best_configs.json")
@click.option("--warm-start/--no-warm-start", default=True, help="evaluate the stored best configuration first")
@click.option("--space", "space_mode", default="contract", type=click.Choice(["contract", "library"]),
              help="contract: the contract's search space pruned to the parameters the selected kernel reads; "
                   "library: every value b200_query_config_space lists")
def optimize(op: str, shape: str, dtype: str, strategy: str, max_candidates: int, retry: int, out: str,
             warm_start: bool, space_mode: str) -> None:
    """Searches the CUDA launch/tile space of OP and promotes the best variant.

    The kernel's all-default launch (after any stored best) is always among
    the candidates, and the episode records it, so a promoted configuration
    is measured against the default on the same inputs."""
    from .agent.generator import _axes, default_action, library_axes
    from .agent.promoter import should_promote
    from .agent.selector import select_best
    from .core.profiler import time_device
    from .core.storage import LeaderboardStore
    from .microrl.trainer import ShapeConfigStore
    from .runtime import lib as L

    ensure_registered(op)
    contract = get_registry().get(op)
    parsed = parse_shape(shape)
    state = OpState(op, parsed.get("B", 8), parsed.get("T", 2048), parsed.get("D", 4096), dtype, "cuda",
                    shape=shape_key(parsed))
    templates = load_templates(op)
    ref_fn, gen_fn = load_reference(op)
    inputs = gen_fn(**parsed, dtype=_torch_dtype(dtype), device="cuda")
    ref_out = ref_fn(*_clone_inputs(inputs))
    base_inputs = _clone_inputs(inputs)
    lat = sorted(time_device(lambda: ref_fn(*base_inputs), warmup=3, repeat=10))
    baseline_us = lat[len(lat) // 2]
    state.baseline_latency_us = baseline_us

    outdir = Path(out)
    space = L.config_space(op, space_rows(op, parsed, gen_fn))
    axes = library_axes(space) if (space_mode == "library" and space) else _axes(contract, space)
    warm = warm_start_actions(state, templates, ShapeConfigStore(outdir / "best_configs.json"),
                              LeaderboardStore(outdir / "leaderboard.sqlite")) if warm_start else []
    stored = [a.to_dict() for _, a in warm]
    keys = {a.arm_key() for _, a in warm}
    defaults = [(t, default_action(t, axes)) for t in sorted(templates)]
    warm += [(t, a) for t, a in defaults if a.arm_key() not in keys]
    cands, results = search(contract, state, templates,
                            lambda t, a: evaluate(op, contract, templates[t], a, state, inputs, ref_out, baseline_us),
                            strategy, max_candidates, retry, outdir / "best_configs.json", warm, axes=axes)
    best_i, best = select_best(cands, results)
    best.promoted = should_promote(best, contract)
    dkeys = {a.arm_key(): t for t, a in defaults}
    default_res = [{"template": t, "action": a.to_dict(), "result": r.to_dict()}
                   for (t, a), r in zip(cands, results) if a.arm_key() in dkeys]
    path, _ = record_outcome(state, cands, results, best_i, outdir,
                             {"strategy": strategy, "shape": parsed, "baseline_latency_us": baseline_us,
                              "warm_start": stored, "config_space": space, "space_mode": space_mode,
                              "axes": {a: v for a, v in axes}, "default": default_res})
    vs = ""
    if default_res and default_res[0]["result"]["latency_us_p50"] > 0:
        vs = f" default_p50={default_res[0]['result']['latency_us_p50']:.1f}us"
    click.echo(f"best {cands[best_i][0]} {cands[best_i][1].launch_cfg()} p50={best.latency_us_p50:.1f}us{vs} "
               f"speedup={best.speedup:.2f}x reward={best.reward:.2f} promoted={best.promoted} -> {path}")


@main.command("leaderboard")
@click.argument("op")
@click.option("--shape", default="", help="only this shape (K=V,... as given to optimize)")
@click.option("--dtype", default="")
@click.option("--out", default="episodes")
@click.option("--limit", default=20, type=int)
def leaderboard(op: str, shape: str, dtype: str, out: str, limit: int) -> None:
    """Best recorded configurations of OP (reference cli.py:419-467)."""
    from .core.storage import LeaderboardStore

    key = shape_key(parse_shape(shape)) if shape else None
    rows = LeaderboardStore(Path(out) / "leaderboard.sqlite").query(op, shape=key, dtype=dtype or None, limit=limit)
    if not rows:
        click.echo(f"no entries for {op}")
        return
    for r in rows:
        click.echo(f"{r['shape']} {r['dtype']} {r['template_id']} threads={r['threads']} split={r['split']} "
                   f"rows_per_cta={r['rows_per_cta']} tile={r['tile_m']}x{r['tile_n']}x{r['tile_k']} "
                   f"flags={r.get('flags') or 0} stages={r['num_stages']} "
                   f"p50={r['latency_us_p50']:.1f}us speedup={r['speedup']:.2f}x "
                   f"roofline={r['roofline_fraction']:.2f} promoted={bool(r['promoted'])} ep={r['episode_id']}")


@main.command("replay")
@click.argument("op")
@click.argument("episode_id")
@click.option("--out", default="episodes")
def replay(op: str, episode_id: str, out: str) -> None:
    """Prints a stored episode record (reference cli.py:470-490)."""
    from .core.storage import EpisodeStore

    rec = EpisodeStore(out).load(op, episode_id)
    if rec is None:
        raise click.ClickException(f"episode {op}/{episode_id} not found")
    click.echo(json.dumps({k: rec[k] for k in ("episode_id", "state", "action", "result")}, indent=2))


if __name__ == "__main__":
    main()
