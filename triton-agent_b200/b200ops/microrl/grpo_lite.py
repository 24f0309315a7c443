"""GRPO-lite (algorithm of triton_agent/microrl/grpo_lite.py:30-147).

Evaluates a group of G distinct arms, normalises their rewards by the group
mean and standard deviation, and applies the REINFORCE-lite logit update
with those advantages.  Until G groups have been seen, single selections are
uniform.
"""

from __future__ import annotations

import math

from ..core.spec import OpAction, OpState
from .reinforce_lite import _SoftmaxPolicy, sample


class GRPOLite(_SoftmaxPolicy):
    def __init__(self, learning_rate: float = 0.1, temperature: float = 1.0, group_size: int = 4,
                 seed: int | None = None):
        super().__init__(learning_rate, temperature, seed)
        self.group_size = group_size
        self._steps = 0

    def select(self, candidates: list[tuple[str, OpAction]], state: OpState) -> int:
        probs = self.probs(candidates, state)
        if self._rng.random() < 0.05 or self._steps < self.group_size:
            return self._rng.randrange(len(candidates))
        return sample(probs, self._rng)

    def select_group(self, candidates: list[tuple[str, OpAction]], state: OpState) -> list[int]:
        probs = self.probs(candidates, state)
        k = min(self.group_size, len(candidates))
        chosen: list[int] = []
        for idx in self._rng.choices(range(len(candidates)), weights=probs, k=k):
            if idx not in chosen:
                chosen.append(idx)
        rest = [i for i in range(len(candidates)) if i not in chosen]
        self._rng.shuffle(rest)
        chosen.extend(rest[: k - len(chosen)])
        return chosen

    def update_group(self, actions: list[OpAction], rewards: list[float], state: OpState,
                     candidates: list[tuple[str, OpAction]]) -> None:
        self._steps += 1
        if not rewards:
            return
        mu = sum(rewards) / len(rewards)
        sigma = math.sqrt(sum((r - mu) ** 2 for r in rewards) / len(rewards)) + 1e-6
        # advantages against one snapshot of the policy, as a group update
        probs_snapshot = self.probs(candidates, state)
        keys = self._keys(candidates, state)
        for action, r in zip(actions, rewards):
            adv = (r - mu) / sigma
            sel = next(i for i, (_, a) in enumerate(candidates) if a.arm_key() == action.arm_key())
            for i, key in enumerate(keys):
                self._policy.update(key, self.lr * adv * ((1.0 if i == sel else 0.0) - probs_snapshot[i]))

    def update(self, action: OpAction, state: OpState, reward: float,
               candidates: list[tuple[str, OpAction]] | None = None) -> None:
        """Single results are folded in through update_group by the caller."""
