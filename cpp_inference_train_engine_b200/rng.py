"""The reference engine's Rng (include/mini_mla/rng.hpp:7-35): splitmix64 with the same
uniform/bounded draws, used to build the synthetic GRPO workloads with the seeds the
benchmark plan fixes (prompt ids Rng(2), rollout seeds Rng(1), rewards Rng(3),
teacher-forced ids Rng(4), normal rewards Rng(5))."""
from __future__ import annotations

import numpy as np

_MASK = (1 << 64) - 1
_GAMMA = 0x9E3779B97F4A7C15


class Rng:
    def __init__(self, seed: int):
        self.state = seed & _MASK

    def next(self) -> int:
        self.state = (self.state + _GAMMA) & _MASK
        z = self.state
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _MASK
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _MASK
        return z ^ (z >> 31)

    def uniform(self) -> float:
        return float((np.float32(self.next() >> 40) + np.float32(0.5)) / np.float32(16777216.0))

    def bounded(self, bound: int) -> int:
        if bound == 0:
            return 0
        threshold = ((1 << 64) - bound) % bound
        while True:
            r = self.next()
            if r >= threshold:
                return r % bound

    def normal(self) -> float:
        u1 = np.float32(self.uniform())
        u2 = np.float32(self.uniform())
        return float(np.sqrt(np.float32(-2.0) * np.log(u1)) *
                     np.cos(np.float32(2.0 * np.pi) * u2))


def grpo_workload(n_prompts: int, group: int, prompt_len: int, vocab: int, p_reward):
    """Synthetic GRPO inputs: prompts [n_prompts*group, prompt_len] (each prompt repeated for
    its group), per-rollout seeds, Bernoulli(p_reward) rewards (N(0, 1) when p_reward is
    None)."""
    pr = Rng(2)
    base = np.array([[pr.bounded(vocab) for _ in range(prompt_len)] for _ in range(n_prompts)],
                    np.uint16)
    prompts = np.repeat(base, group, axis=0)
    sr = Rng(1)
    seeds = np.array([sr.next() for _ in range(n_prompts * group)], np.uint64)
    rr = Rng(3)
    if p_reward is None:
        rewards = np.array([rr.normal() for _ in range(n_prompts * group)], np.float32)
    else:
        rewards = np.array([1.0 if rr.uniform() < p_reward else 0.0
                            for _ in range(n_prompts * group)], np.float32)
    return prompts, seeds, rewards
