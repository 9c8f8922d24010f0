"""Draft-shape policies: the interface of python/woodcock/policies.py (class and method names,
argument meaning) with implementations written for this package.

A policy fixes a round's shape before the round is launched: the device round needs its chain
length (or tree depth, width and verify budget) at graph-selection time, so everything here is
host logic on small integers.

* StaticPolicy(depth, width=1, budget=None): a chain of `depth` drafts, or a top-`width` tree
  whose verified part is the `budget` nodes of largest path probability (EAGLE-2,
  arXiv:2406.16858 section 4; the reference default budget is 4 * depth for trees).
* CostAwareChain: the chain length that maximises expected emitted tokens per unit of round
  time, re-chosen every round from a running estimate of the per-draft acceptance rate.
"""

from __future__ import annotations

import heapq
import math


class Plan:
    """One round's shape: depth, width and verify budget. For sampled trees `children_for`
    hands out the budget to nodes in drafting order before their children are drawn (the
    count must not depend on the draws, or the output law is biased)."""

    __slots__ = ("max_depth", "width", "budget", "_left")

    def __init__(self, max_depth: int, width: int, budget: int):
        self.max_depth, self.width, self.budget = int(max_depth), int(width), int(budget)
        self._left = self.budget

    def children_for(self, phat: float, depth: int) -> int:
        take = max(0, min(self.width, self._left))
        self._left -= take
        return take

    def __repr__(self) -> str:
        return f"Plan(max_depth={self.max_depth}, width={self.width}, budget={self.budget})"


class Policy:
    """Base interface. plan() once per round; continue_drafting / select_frontier after each
    drafted level of a tree; select_verify before verification; observe() after the round."""

    def reset(self) -> None:
        return None

    def plan(self, context_len: int, stochastic: bool) -> Plan:
        raise NotImplementedError

    def continue_drafting(self, depth: int, gain: float, context_len: int, num_nodes: int) -> bool:
        return True

    def select_frontier(self, level_nodes, nodes, width):
        """The `width` nodes of the new level to expand next: largest path probability first,
        shallower first on equal probability, then in drafting order."""
        return heapq.nsmallest(width, level_nodes, key=lambda v: (-nodes[v].phat, nodes[v].depth, v))

    def select_verify(self, nodes, context_len: int, stochastic: bool) -> list[int]:
        raise NotImplementedError

    def observe(self, accepted, verified, depth, t_draft, t_verify) -> None:
        return None


class StaticPolicy(Policy):
    """Fixed depth / width / budget; width 1 is a plain chain of `depth` drafts."""

    def __init__(self, depth: int, width: int = 1, budget: int | None = None):
        if depth < 1 or width < 1:
            raise ValueError("depth and width must be >= 1")
        self.depth, self.width = int(depth), int(width)
        self.budget = int(budget) if budget is not None else self.depth * (1 if self.width == 1 else 4)

    def plan(self, context_len, stochastic):
        return Plan(self.depth, self.width, self.budget)

    def select_verify(self, nodes, context_len, stochastic):
        """All drafted nodes when they fit the budget (or when sampling, where pruning a drawn
        node would bias the output); otherwise the root plus the `budget` nodes of largest path
        probability (ties: shallower, then earlier), in node order. Keeping the best nodes by a
        product of probabilities along the path keeps every kept node's ancestors too, since a
        child's product never exceeds its parent's."""
        n = len(nodes) - 1
        if stochastic or n <= self.budget:
            return list(range(len(nodes)))
        best = heapq.nsmallest(self.budget, range(1, len(nodes)), key=lambda v: (-nodes[v].phat, nodes[v].depth, v))
        return [0] + sorted(best)


class CostAwareChain(StaticPolicy):
    """Chain length chosen before each round from measured costs.

    For a per-draft acceptance probability a (drafts accepted independently, the model of
    Leviathan et al., arXiv:2211.17192, Eq. 1), a chain of k drafts emits on average
    E(k) = 1 + a + ... + a^k = (1 - a^(k+1)) / (1 - a) tokens. With T(k) the round time of a
    chain of k, the policy picks k* = argmax E(k) / T(k) over 1..k_max; equal rates (to 1e-12
    relative) go to the shorter chain.

    T(k) comes from a cost table: either measured whole-round times `round_ms[k]` (this
    package's device round, written by `bench.py --workload costs`), or the reference's
    per-part timings (scripts/time_draft_step.py: head_ms, step_ms = head + one drafter layer,
    verify_ms[n]) combined as the round does its work: k heads, k - 1 drafter layers, a verify
    of k + 1 rows and the drafter update (one more layer pass):
    T(k) = verify_ms[k+1] + k * head_ms + k * (step_ms - head_ms).

    Acceptance estimate: a chain round with a accepted out of k drafts shows a successes and,
    when a < k, one failure (drafts after the first rejection are never tested). Successes and
    failures are accumulated with exponential forgetting, weight (1 - 1/window) per round, on
    top of a prior of `prior` pseudo-observations at rate `alpha0`; a = S / (S + F), clamped to
    [0.01, 0.99].
    """

    def __init__(self, step_ms: float | None = None, head_ms: float | None = None,
                 verify_ms: dict[int, float] | None = None, k_max: int = 8, alpha0: float = 0.6,
                 prior: float = 4.0, window: int = 16, round_ms: dict[int, float] | None = None):
        super().__init__(depth=1)
        if round_ms:
            times = {int(k): float(v) for k, v in round_ms.items() if int(k) >= 1}
        else:
            if verify_ms is None or step_ms is None or head_ms is None:
                raise ValueError("give round_ms, or step_ms, head_ms and verify_ms")
            layer = float(step_ms) - float(head_ms)
            times = {k: float(verify_ms[k + 1]) + k * float(head_ms) + k * layer
                     for k in range(1, max(int(n) for n in verify_ms)) if (k + 1) in {int(n) for n in verify_ms}}
        ks = [k for k in sorted(times) if k <= k_max]
        if not ks or any(times[k] <= 0 for k in ks):
            raise ValueError("cost table has no usable chain lengths")
        self.k_max = ks[-1]
        self.times = {k: times[k] for k in ks}
        self.alpha0, self.prior = float(alpha0), float(prior)
        self.decay = 1.0 - 1.0 / max(1, int(window))
        self.chosen: list[int] = []
        self.reset()

    @classmethod
    def from_costs(cls, costs: dict, head: str, **kw) -> "CostAwareChain":
        """costs: the JSON of scripts/time_draft_step.py ({"drafter": {head: {"head_ms", "step_ms"}},
        "verify_ms": {n: ms}}), optionally with this package's measured "round_ms": {head: {k: ms}}."""
        rm = (costs.get("round_ms") or {}).get(head)
        if rm:
            return cls(round_ms={int(k): v for k, v in rm.items()}, **kw)
        d = costs["drafter"][head]
        return cls(d["step_ms"], d["head_ms"], {int(n): v for n, v in costs["verify_ms"].items()}, **kw)

    def reset(self) -> None:
        self.succ = self.alpha0 * self.prior
        self.fail = (1.0 - self.alpha0) * self.prior

    def alpha(self) -> float:
        a = self.succ / (self.succ + self.fail)
        return min(0.99, max(0.01, a))

    @staticmethod
    def expected_tokens(a: float, k: int) -> float:
        return k + 1.0 if a == 1.0 else (1.0 - a ** (k + 1)) / (1.0 - a)

    def best_depth(self, alpha: float) -> int:
        best_k, best_rate = None, -math.inf
        for k in sorted(self.times):
            rate = self.expected_tokens(alpha, k) / self.times[k]
            if rate > best_rate * (1.0 + 1e-12):
                best_k, best_rate = k, rate
        return best_k

    def plan(self, context_len, stochastic):
        k = self.best_depth(self.alpha())
        self.depth = self.budget = k
        self.chosen.append(k)
        return Plan(k, 1, k)

    def observe(self, accepted, verified, depth, t_draft, t_verify):
        self.succ = self.decay * self.succ + float(accepted)
        self.fail = self.decay * self.fail + (1.0 if accepted < depth else 0.0)
