"""Draft-shape policies (python/woodcock/policies.py; src/core/spec.cpp:35-45). Host logic:
they decide the round's shape before it is launched.

StaticPolicy drafts a fixed chain (width 1) or a top-k tree keeping `budget` nodes.
CostAwareChain picks the chain length before each round, maximising the expected
tokens per unit time E(k)/T(k) with E(k) = (1 - a^(k+1)) / (1 - a) (Leviathan et al.,
arXiv:2211.17192 Eq. 1) and T(k) = t_verify(k+1) + k * t_step + (t_step - t_head)
from measured latencies; a is estimated from the last `window` rounds.
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass


@dataclass
class Plan:
    max_depth: int
    width: int
    budget: int
    _remaining: int = 0

    def __post_init__(self):
        self._remaining = self.budget

    def children_for(self, phat: float, depth: int) -> int:
        """Children to draw for one node, fixed before drawing (stochastic trees)."""
        m = min(self.width, self._remaining)
        self._remaining -= m
        return max(m, 0)


class Policy:
    def reset(self):
        pass

    def plan(self, context_len: int, stochastic: bool) -> Plan:
        raise NotImplementedError

    def continue_drafting(self, depth: int, gain: float, context_len: int, num_nodes: int) -> bool:
        return True

    def select_frontier(self, level_nodes, nodes, width):
        return sorted(level_nodes, key=lambda v: (-nodes[v].phat, nodes[v].depth))[:width]

    def select_verify(self, nodes, context_len: int, stochastic: bool) -> list[int]:
        raise NotImplementedError

    def observe(self, accepted, verified, depth, t_draft, t_verify):
        pass


class StaticPolicy(Policy):
    def __init__(self, depth: int, width: int = 1, budget: int | None = None):
        self.depth, self.width = depth, width
        self.budget = budget if budget is not None else (depth if width == 1 else 4 * depth)

    def plan(self, context_len, stochastic):
        return Plan(self.depth, self.width, self.budget)

    def select_verify(self, nodes, context_len, stochastic):
        if stochastic or len(nodes) - 1 <= self.budget:
            return list(range(len(nodes)))
        ranked = sorted(range(1, len(nodes)), key=lambda v: (-nodes[v].phat, nodes[v].depth, v))[: self.budget]
        return [0] + sorted(ranked)


class CostAwareChain(StaticPolicy):
    def __init__(self, step_ms: float, head_ms: float, verify_ms: dict[int, float], k_max: int = 8,
                 alpha0: float = 0.6, prior: float = 4.0, window: int = 16):
        k_max = min(k_max, max(verify_ms) - 1)
        super().__init__(depth=1)
        self.k_max, self.alpha0, self.prior = k_max, alpha0, prior
        self.cost = [None] + [verify_ms[k + 1] + k * step_ms + (step_ms - head_ms) for k in range(1, k_max + 1)]
        self.hist: deque[tuple[int, int]] = deque(maxlen=window)
        self.chosen: list[int] = []

    @classmethod
    def from_costs(cls, costs: dict, head: str, **kw) -> "CostAwareChain":
        d = costs["drafter"][head]
        return cls(d["step_ms"], d["head_ms"], {int(n): v for n, v in costs["verify_ms"].items()}, **kw)

    def reset(self):
        self.hist.clear()

    def alpha(self) -> float:
        s = sum(a for a, _ in self.hist)
        f = sum(a < k for a, k in self.hist)
        return min(0.99, max(0.01, (s + self.prior * self.alpha0) / (s + f + self.prior)))

    def best_depth(self, alpha: float) -> int:
        def rate(k):
            return (1 - alpha ** (k + 1)) / (1 - alpha) / self.cost[k]

        return max(range(1, self.k_max + 1), key=lambda k: (rate(k), -k))

    def plan(self, context_len, stochastic):
        self.depth = self.budget = self.best_depth(self.alpha())
        self.chosen.append(self.depth)
        return Plan(self.depth, 1, self.depth)

    def observe(self, accepted, verified, depth, t_draft, t_verify):
        self.hist.append((accepted, depth))
