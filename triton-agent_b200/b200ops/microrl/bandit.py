"""Bandit policies over configurations (algorithms of
triton_agent/microrl/bandit.py:17-222, kept so tuning behaves the same).

Each arm is one OpAction (all of its launch/tile fields) in a context of
(op, shape, dtype, device):
  UCBPolicy             mean + c * sqrt(ln(total) / count); unseen arms first
  ThompsonSamplingPolicy Beta(alpha, beta) per arm, reward clipped to [0, 1]
  EpsilonGreedyPolicy   explore with eps = max(eps_min, eps0 / sqrt(1 + n*decay)),
                        unseen arms valued 0.5 when exploiting
"""

from __future__ import annotations

import math
import random
from collections import defaultdict
from dataclasses import dataclass

from ..core.spec import OpAction, OpState


def context_key(state: OpState) -> str:
    """(op, shape, dtype, device) key of bandit arms and stored best configs
    (microrl/trainer.py:59-60); the full generator shape when the state has one."""
    if state.shape:
        return f"{state.op_name}|{state.shape}|{state.dtype}|{state.device}"
    return f"{state.op_name}|{state.B}|{state.T}|{state.D}|{state.dtype}|{state.device}"


def arm_key(action: OpAction) -> str:
    return action.arm_key()


@dataclass
class ArmStats:
    count: int = 0
    mean_reward: float = 0.0
    variance: float = 0.0
    sum_rewards: float = 0.0
    sum_sq_rewards: float = 0.0

    def update(self, reward: float) -> None:
        self.count += 1
        self.sum_rewards += reward
        self.sum_sq_rewards += reward * reward
        self.mean_reward = self.sum_rewards / self.count
        if self.count > 1:
            v = (self.sum_sq_rewards - self.sum_rewards ** 2 / self.count) / (self.count - 1)
            self.variance = max(0.0, v)


class _ArmTable:
    def __init__(self):
        self._arms: dict[str, ArmStats] = defaultdict(ArmStats)

    def stats(self, state: OpState, action: OpAction) -> ArmStats:
        return self._arms[f"{context_key(state)}|{arm_key(action)}"]

    def best(self, actions: list[OpAction], state: OpState) -> tuple[int, float]:
        means = [self.stats(state, a).mean_reward for a in actions]
        i = max(range(len(actions)), key=lambda k: (means[k], -k))
        return i, means[i]

    @property
    def arm_count(self) -> int:
        return len(self._arms)


class UCBPolicy(_ArmTable):
    def __init__(self, c: float = 2.0):
        super().__init__()
        self.c = c
        self._total = 0

    def select(self, candidate_actions: list[OpAction], state: OpState) -> int:
        self._total += 1
        best_i, best_v = 0, -math.inf
        for i, a in enumerate(candidate_actions):
            st = self.stats(state, a)
            v = math.inf if st.count == 0 else st.mean_reward + self.c * math.sqrt(math.log(self._total) / st.count)
            if v > best_v:
                best_i, best_v = i, v
        return best_i

    def update(self, action: OpAction, state: OpState, reward: float) -> None:
        self.stats(state, action).update(reward)

    def best_action(self, candidate_actions, state):
        return self.best(candidate_actions, state)


class ThompsonSamplingPolicy:
    def __init__(self, seed: int | None = None):
        self._ab: dict[str, tuple[float, float]] = defaultdict(lambda: (1.0, 1.0))
        self._rng = random.Random(seed)

    def _key(self, state, action):
        return f"{context_key(state)}|{arm_key(action)}"

    def select(self, candidate_actions: list[OpAction], state: OpState) -> int:
        draws = [self._rng.betavariate(*self._ab[self._key(state, a)]) for a in candidate_actions]
        return max(range(len(draws)), key=lambda i: (draws[i], -i))

    def update(self, action: OpAction, state: OpState, reward: float) -> None:
        k = self._key(state, action)
        a, b = self._ab[k]
        r = min(1.0, max(0.0, reward))
        self._ab[k] = (a + r, b + 1.0 - r)

    def best_action(self, candidate_actions, state):
        means = []
        for a in candidate_actions:
            al, be = self._ab[self._key(state, a)]
            means.append(al / (al + be))
        i = max(range(len(means)), key=lambda k: (means[k], -k))
        return i, means[i]

    @property
    def arm_count(self) -> int:
        return len(self._ab)


class EpsilonGreedyPolicy(_ArmTable):
    def __init__(self, epsilon_init: float = 0.3, epsilon_min: float = 0.05, decay_rate: float = 0.01,
                 seed: int | None = None):
        super().__init__()
        self.epsilon_init, self.epsilon_min, self.decay_rate = epsilon_init, epsilon_min, decay_rate
        self._total = 0
        self._rng = random.Random(seed)

    def epsilon(self) -> float:
        return max(self.epsilon_min, self.epsilon_init / math.sqrt(1 + self._total * self.decay_rate))

    def select(self, candidate_actions: list[OpAction], state: OpState) -> int:
        self._total += 1
        if self._rng.random() < self.epsilon():
            return self._rng.randrange(len(candidate_actions))
        vals = []
        for a in candidate_actions:
            st = self.stats(state, a)
            vals.append(0.5 if st.count == 0 else st.mean_reward)
        return max(range(len(vals)), key=lambda i: (vals[i], -i))

    def update(self, action: OpAction, state: OpState, reward: float) -> None:
        self.stats(state, action).update(reward)

    def best_action(self, candidate_actions, state):
        return self.best(candidate_actions, state)
