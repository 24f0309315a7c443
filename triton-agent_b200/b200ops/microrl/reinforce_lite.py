"""REINFORCE-lite over configurations (algorithm of
triton_agent/microrl/reinforce_lite.py:59-132).

A softmax policy over per-arm logits; after each evaluated arm, every logit
moves by lr * advantage * (1[selected] - prob), with the advantage taken
against an exponentially smoothed reward baseline.  5% of selections are
uniform exploration.
"""

from __future__ import annotations

import math
import random
from collections import defaultdict
from dataclasses import dataclass, field

from ..core.spec import OpAction, OpState
from .bandit import arm_key, context_key


@dataclass
class PolicyWeights:
    weights: dict[str, float] = field(default_factory=dict)

    def get_logit(self, key: str) -> float:
        return self.weights.get(key, 0.0)

    def update(self, key: str, delta: float) -> None:
        self.weights[key] = self.weights.get(key, 0.0) + delta


def softmax(logits: list[float], temperature: float = 1.0) -> list[float]:
    t = temperature if temperature > 0 else 1e-6
    z = [x / t for x in logits]
    mx = max(z)
    e = [math.exp(x - mx) for x in z]
    s = sum(e)
    return [x / s for x in e]


def sample(probs: list[float], rng: random.Random | None = None) -> int:
    r = (rng or random).random()
    acc = 0.0
    for i, p in enumerate(probs):
        acc += p
        if r <= acc:
            return i
    return len(probs) - 1


class _SoftmaxPolicy:
    def __init__(self, learning_rate: float, temperature: float, seed: int | None):
        self.lr = learning_rate
        self.temperature = temperature
        self._policy = PolicyWeights()
        self._rng = random.Random(seed)

    def _keys(self, candidates, state) -> list[str]:
        ctx = context_key(state)
        return [f"{ctx}|{arm_key(a)}" for _, a in candidates]

    def probs(self, candidates, state) -> list[float]:
        return softmax([self._policy.get_logit(k) for k in self._keys(candidates, state)], self.temperature)

    def _gradient_step(self, candidates, state, action: OpAction, advantage: float) -> None:
        keys = self._keys(candidates, state)
        probs = softmax([self._policy.get_logit(k) for k in keys], self.temperature)
        sel = next(i for i, (_, a) in enumerate(candidates) if arm_key(a) == arm_key(action))
        for i, k in enumerate(keys):
            self._policy.update(k, self.lr * advantage * ((1.0 if i == sel else 0.0) - probs[i]))

    def best_action(self, candidates, state) -> int:
        keys = self._keys(candidates, state)
        logits = [self._policy.get_logit(k) for k in keys]
        return max(range(len(logits)), key=lambda i: (logits[i], -i))

    @property
    def arm_count(self) -> int:
        return len(self._policy.weights)


class REINFORCELite(_SoftmaxPolicy):
    def __init__(self, learning_rate: float = 0.1, temperature: float = 1.0, baseline_smoothing: float = 0.9,
                 seed: int | None = None):
        super().__init__(learning_rate, temperature, seed)
        self.baseline_smoothing = baseline_smoothing
        self._baseline: dict[str, float] = defaultdict(float)
        self._steps = 0

    def select(self, candidates: list[tuple[str, OpAction]], state: OpState) -> int:
        probs = self.probs(candidates, state)
        if self._rng.random() < 0.05:
            return self._rng.randrange(len(candidates))
        return sample(probs, self._rng)

    def update(self, action: OpAction, state: OpState, reward: float,
               candidates: list[tuple[str, OpAction]]) -> None:
        self._steps += 1
        bk = context_key(state)
        self._baseline[bk] = self.baseline_smoothing * self._baseline[bk] + (1 - self.baseline_smoothing) * reward
        self._gradient_step(candidates, state, action, reward - self._baseline[bk])
