"""Tuner orchestration (triton_agent/microrl/trainer.py:41-165).

Trainer(strategy) wraps one policy behind select / update / select_group /
update_group; ShapeConfigStore persists the best promoted configuration per
(op, shape, dtype, device) so a later run starts from it.  Unlike the
reference (trainer.py:139-140, which drops the candidate list and makes
REINFORCE-lite raise), update always forwards the candidates to
policy-gradient strategies.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any

from ..core.spec import CandidateResult, OpAction, OpState
from .bandit import EpsilonGreedyPolicy, ThompsonSamplingPolicy, UCBPolicy, context_key
from .grpo_lite import GRPOLite
from .reinforce_lite import REINFORCELite

BANDIT_MAP = {"ucb": UCBPolicy, "thompson": ThompsonSamplingPolicy, "epsilon_greedy": EpsilonGreedyPolicy,
              "epsilon": EpsilonGreedyPolicy}
PG_MAP = {"reinforce": REINFORCELite, "reinforce_lite": REINFORCELite}
GRPO_MAP = {"grpo": GRPOLite, "grpo_lite": GRPOLite}
ALL_STRATEGIES = {**BANDIT_MAP, **PG_MAP, **GRPO_MAP}


class ShapeConfigStore:
    def __init__(self, path: str | Path = "leaderboard/best_configs.json") -> None:
        self.path = Path(path)
        self._data: dict[str, Any] = json.loads(self.path.read_text()) if self.path.exists() else {}

    def save(self) -> None:
        self.path.parent.mkdir(parents=True, exist_ok=True)
        self.path.write_text(json.dumps(self._data, indent=2))

    def get_best(self, state: OpState) -> dict | None:
        return self._data.get(context_key(state))

    def set_best(self, state: OpState, action: OpAction, result: CandidateResult) -> None:
        self._data[context_key(state)] = {"action": action.to_dict(), "speedup": result.speedup,
                                          "latency_us_p50": result.latency_us_p50, "reward": result.reward,
                                          "roofline_fraction": result.roofline_fraction}
        self.save()

    def get_historical_best(self, state: OpState) -> dict | None:
        e = self.get_best(state)
        if e:
            state.historical_best_config = e["action"]
            return e["action"]
        return None


class Trainer:
    def __init__(self, strategy: str = "ucb", store_path: str | Path | None = None, **policy_kwargs) -> None:
        self.strategy = strategy
        if strategy in PG_MAP:
            self.kind = "pg"
        elif strategy in GRPO_MAP:
            self.kind = "grpo"
        else:
            self.kind = "bandit"
        self.policy = ALL_STRATEGIES.get(strategy, UCBPolicy)(**policy_kwargs)
        self.config_store = ShapeConfigStore(store_path or "leaderboard/best_configs.json")

    def select(self, candidates: list[tuple[str, OpAction]], state: OpState) -> int:
        if self.kind == "bandit":
            return self.policy.select([a for _, a in candidates], state)
        return self.policy.select(candidates, state)

    def select_group(self, candidates: list[tuple[str, OpAction]], state: OpState) -> list[int]:
        if hasattr(self.policy, "select_group"):
            return self.policy.select_group(candidates, state)
        return [self.select(candidates, state)]

    def update(self, action: OpAction, state: OpState, result: CandidateResult,
               candidates: list[tuple[str, OpAction]] | None = None) -> None:
        if self.kind == "bandit":
            self.policy.update(action, state, result.reward)
        elif self.kind == "pg":
            if candidates is None:
                raise ValueError("policy-gradient strategies need the candidate list")
            self.policy.update(action, state, result.reward, candidates)
        else:
            if candidates is not None:
                self.policy.update_group([action], [result.reward], state, candidates)
        if result.promoted:
            self.config_store.set_best(state, action, result)

    def update_group(self, actions: list[OpAction], rewards: list[float], state: OpState,
                     candidates: list[tuple[str, OpAction]]) -> None:
        if hasattr(self.policy, "update_group"):
            self.policy.update_group(actions, rewards, state, candidates)

    def get_best_config(self, state: OpState) -> dict | None:
        return self.config_store.get_best(state)
