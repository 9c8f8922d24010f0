"""Acceptance rules on the device (python/woodcock/sampling.py; src/sampling/sampling.cpp).

* greedy chain / tree: longest draft path matching the target's argmax, plus the
  target's argmax at the first mismatch (one single-thread kernel walk);
* stochastic chain / tree: recursive rejection sampling, accept child x when
  u < min(1, p(x)/q(x)); after a rejection p <- norm(max(0, p - q)), q[x] <- 0 and
  renormalised; the final draw is an inverse-CDF sample (fp64) from p.

Uniforms come from a counter-based Philox4x32-10 stream (``PhiloxStream``), so
the device and any host checker read the same numbers in the same order: one per
tested child with q(x) > 0, one for the final draw.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np
import torch

from ._lib import lib
from .context import Context, device_ints, ptr


@dataclass(frozen=True)
class SamplingParams:
    temperature: float = 0.0  # 0 => greedy
    top_k: int = 0
    top_p: float = 1.0
    seed: int = 0

    @property
    def greedy(self) -> bool:
        return self.temperature <= 0.0


@dataclass
class DraftTree:
    """Flattened draft tree, node 0 = root; children in draw order (sampling.py:88-115)."""

    tokens: list[int]
    parents: list[int]
    depth: list[int]
    children: list[list[int]] = field(default_factory=list)

    def __post_init__(self):
        if not self.children:
            self.children = [[] for _ in self.tokens]
            for v, p in enumerate(self.parents):
                if p >= 0:
                    self.children[p].append(v)

    def __len__(self):
        return len(self.tokens)

    def path_to(self, v: int) -> list[int]:
        out = []
        while v > 0:
            out.append(v)
            v = self.parents[v]
        return out[::-1]

    def is_chain(self) -> bool:
        return all(p == i - 1 for i, p in enumerate(self.parents))


class PhiloxStream:
    """Sequential reader of the Philox4x32-10 uniform stream (seed, counter offset)."""

    def __init__(self, seed: int, offset: int = 0, device=0):
        self.seed, self.pos = int(seed), int(offset)
        self.ctx = Context.get(device)

    def random(self, size=None):
        n = 1 if size is None else int(np.prod(size))
        out = torch.empty((max(n, 1),), dtype=torch.float64, device=self.ctx.device)
        with self.ctx.enter(out):
            self.ctx.check(lib().wc_philox_uniforms(self.ctx.h, self.seed, self.pos, n, ptr(out)))
        self.pos += n
        u = out[:n].cpu().numpy()
        return float(u[0]) if size is None else u.reshape(size)


def tree_attention_mask(tree: DraftTree, prefix_len: int) -> np.ndarray:
    """(N, prefix + N) bool: every node sees the prefix and its ancestors, itself included
    (sampling.py:118-128). Host-side: it is input description, not compute."""
    N = len(tree)
    m = np.zeros((N, prefix_len + N), dtype=bool)
    m[:, :prefix_len] = True
    for v in range(N):
        u = v
        while u >= 0:
            m[v, prefix_len + u] = True
            u = tree.parents[u]
    return m


def _tree_args(tree: DraftTree, dev):
    """Device copies of a flattened tree, after checking it: node 0 is the root (parent -1) and
    every other node's parent precedes it."""
    par = list(tree.parents)
    if not par or par[0] != -1 or any(not 0 <= p < v for v, p in enumerate(par) if v > 0) or \
            len(tree.tokens) != len(par):
        raise ValueError("malformed draft tree: node 0 must be the root and parents must precede their nodes")
    return device_ints(tree.tokens, dev), device_ints(par, dev)


def verify_tree_greedy(target_argmax, tree: DraftTree, device=0) -> tuple[list[int], int]:
    """sampling.py:131-140 on the device."""
    ctx = Context.get(device)
    dev = ctx.device
    am = device_ints(target_argmax, dev)
    tok, par = _tree_args(tree, dev)
    N = len(tree)
    out = torch.zeros((N + 2,), dtype=torch.int32, device=dev)
    with ctx.enter(am, tok, par, out):
        ctx.check(lib().wc_accept_greedy(ctx.h, ptr(am), ptr(tok), ptr(par), N, ptr(out[2:]), ptr(out[0:1]),
                                         ptr(out[1:2])))
    o = out.cpu().tolist()
    return o[2 : 2 + o[0]], o[1]


def verify_chain_greedy(target_logits: torch.Tensor, draft_tokens: list[int]) -> tuple[int, int]:
    """sampling.py:60-66: (n accepted, next token) from (K+1, V) logits."""
    from .ops import argmax

    am = argmax(target_logits.reshape(-1, target_logits.shape[-1]))
    K = len(draft_tokens)
    tree = DraftTree([0] + list(draft_tokens), [-1] + list(range(K)), list(range(K + 1)))
    path, nxt = verify_tree_greedy(am, tree, device=target_logits.device.index or 0)
    return len(path), nxt


def _as_rows(x, N: int, V: int, dev) -> torch.Tensor:
    if isinstance(x, dict):
        out = torch.zeros((N, V), dtype=torch.float64, device=dev)
        for v, row in x.items():
            out[int(v)] = torch.as_tensor(np.asarray(row, dtype=np.float64), device=dev)
        return out
    return torch.as_tensor(np.asarray(x.cpu() if isinstance(x, torch.Tensor) else x, dtype=np.float64),
                           device=dev).reshape(N, V).contiguous()


def verify_tree_stochastic(p, q, tree: DraftTree, rng: PhiloxStream) -> tuple[list[int], int]:
    """sampling.py:143-177 on the device. p: {node: target probs} or [N][V]; q: {node: draft probs
    its children were drawn from} or [N][V]. Consumes uniforms from `rng`."""
    ctx = rng.ctx
    dev = ctx.device
    N = len(tree)
    V = len(next(iter(p.values()))) if isinstance(p, dict) else np.asarray(p).shape[-1]
    P = _as_rows(p, N, V, dev)
    Q = _as_rows(q, N, V, dev)
    tok, par = _tree_args(tree, dev)
    out = torch.zeros((N + 3,), dtype=torch.int32, device=dev)
    with ctx.enter(P, Q, tok, par, out):
        ctx.check(lib().wc_accept_stochastic(ctx.h, ptr(P), ptr(Q), V, ptr(tok), ptr(par), N, rng.seed, rng.pos,
                                             ptr(out[3:]), ptr(out[0:1]), ptr(out[1:2]), ptr(out[2:3])))
    o = out.cpu().tolist()
    rng.pos += o[2]
    return o[3 : 3 + o[0]], o[1]


def verify_chain_stochastic(p, q, draft_tokens: list[int], rng: PhiloxStream) -> tuple[int, int]:
    """sampling.py:69-82: p (K+1, V), q (K, V). Equal to the tree rule on a chain."""
    K = len(draft_tokens)
    p = np.asarray(p.cpu() if isinstance(p, torch.Tensor) else p, dtype=np.float64)
    q = np.asarray(q.cpu() if isinstance(q, torch.Tensor) else q, dtype=np.float64)
    qq = np.zeros_like(p)
    qq[:K] = q
    tree = DraftTree([0] + list(draft_tokens), [-1] + list(range(K)), list(range(K + 1)))
    path, nxt = verify_tree_stochastic(p, qq, tree, rng)
    return len(path), nxt


def probs_from_logits(logits: torch.Tensor, sp: SamplingParams) -> torch.Tensor:
    """sampling.py:39-55 on the device: temperature, top-k, top-p (wc_probs_from_logits)."""
    ctx = Context.get(logits.device)
    V = logits.shape[-1]
    x = logits.float().reshape(-1, V).contiguous()
    out = torch.empty_like(x)
    with ctx.enter(x, out):
        ctx.check(lib().wc_probs_from_logits(ctx.h, ptr(x), x.shape[0], V, float(sp.temperature), int(sp.top_k),
                                             float(sp.top_p), ptr(out)))
    return out.reshape(logits.shape)
