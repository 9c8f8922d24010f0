"""Sampled draft trees, and policies whose hooks must run between drafted levels, as rounds
driven from the host over the device API. Greedy StaticPolicy trees and chains do not come
here: they run as device rounds (wc_decoder_round / wc_decoder_tree_round).

Semantics kept from the reference (python/woodcock/spec.py:216-329, src/core/spec.cpp:86-233):

* a drafter entry at depth t of the tree sits at position n - 1 + t and sees the committed
  entries, its drafted ancestors and itself;
* each expanded node draws its children from q = softmax(z / T) of its drafter head (scattered
  to token ids), as many as Plan.children_for grants before the draw, without replacement by
  Gumbel-top-k (Vieira 2014; Kool, van Hoof & Welling 2019) with one uniform per nonzero entry
  of q in token order, so a shared uniform stream gives the same draws as the reference;
* the policy chooses which new nodes to expand (select_frontier), when to stop
  (continue_drafting) and which nodes to verify (select_verify); the kept nodes are verified in
  one target pass with the tree mask and positions n + depth, by the recursive rejection rule
  (wc_accept_stochastic; greedy: wc_accept_greedy); the target cache keeps the accepted path and
  the drafter is updated on the accepted rows.

Every forward, head, softmax, acceptance and compaction is a device call; the host holds the
tree (tens of nodes) and synchronises once per drafted level.
"""

from __future__ import annotations

import time
from dataclasses import dataclass

import numpy as np
import torch

from .ops import argmax, softmax
from .sampling import DraftTree, PhiloxStream, SamplingParams, probs_from_logits, tree_attention_mask, \
    verify_tree_greedy, verify_tree_stochastic


@dataclass
class TreeNode:
    """One drafted node as policies see it (token, parent, depth, path probability)."""

    token: int
    parent: int
    depth: int
    phat: float


def gumbel_top_k(q: np.ndarray, k: int, rng: PhiloxStream) -> list[int]:
    """k distinct ids drawn from q without replacement: the k largest log q_i + G_i over the
    nonzero entries, G_i = -log(-log u_i), one uniform per nonzero entry in id order (drawn even
    when k is 0, so the stream position does not depend on k)."""
    ids = np.nonzero(q > 0)[0]
    if ids.size == 0:
        return []
    u = np.asarray(rng.random(ids.size), dtype=np.float64).reshape(-1)
    keys = np.log(q[ids]) - np.log(-np.log(u))
    order = np.argsort(-keys, kind="stable")
    return [int(ids[i]) for i in order[: min(k, ids.size)]]


def inverse_cdf_draw(p: np.ndarray, rng: PhiloxStream) -> int:
    """One id from p by the inverse CDF of its fp64 running sum."""
    c = np.cumsum(np.asarray(p, dtype=np.float64))
    return int(min(np.searchsorted(c, rng.random() * c[-1], side="right"), c.size - 1))


class SyncedRounds:
    """One request decoded by host-driven rounds: both caches and the chain root (the drafter
    output and feature after the last committed token)."""

    def __init__(self, target, drafter, policy, capacity: int):
        self.t, self.d, self.policy, self.capacity = target, drafter, policy, capacity
        ids = drafter.vocab_ids
        self.head_ids = ids.cpu().numpy() if ids is not None else None

    # ---------------------------------------------------------------- prefill
    def prefill(self, prompt: list[int], sp: SamplingParams, rng: PhiloxStream) -> int:
        dev = self.t.ctx.device
        self.tc = self.t.make_cache(self.capacity)
        o = self.t(torch.tensor(prompt, dtype=torch.int32, device=dev), self.tc, logits_from=len(prompt) - 1)
        first = self._pick(o.logits[0, -1:], sp, rng)
        self.dc = self.d.make_cache(self.capacity)
        hid, out = self.d(list(prompt[1:]) + [first], self.d.fuse(o.features), self.dc)
        self._set_root(hid[:, -1:], out[:, -1:])
        return first

    def _set_root(self, hid, out):
        self.root = (out, self.d.feedback(hid, out))

    def _pick(self, logits, sp, rng) -> int:
        if sp.greedy:
            return int(argmax(logits.reshape(1, -1))[0])
        p = probs_from_logits(logits.reshape(1, -1), sp)[0].double().cpu().numpy()
        return inverse_cdf_draw(p / p.sum(), rng)

    # ---------------------------------------------------------------- drafting
    def _head_probs(self, outs: torch.Tensor, sp: SamplingParams) -> np.ndarray:
        """[rows][vocab] fp64 draft distributions of drafter output rows, scattered to token ids."""
        z = self.d.logits(outs)
        q = softmax(z.float()) if sp.greedy else probs_from_logits(z, SamplingParams(temperature=sp.temperature))
        q = q.double().cpu().numpy()
        full = np.zeros((q.shape[0], self.t.cfg.vocab))
        if self.head_ids is None:
            full[:, : q.shape[1]] = q
        else:
            full[:, self.head_ids] = q
        return full / full.sum(axis=1, keepdims=True)

    def _children(self, q: np.ndarray, sp: SamplingParams, plan, parent: TreeNode, rng) -> list[tuple[int, float]]:
        """(token, q) of a node's children: top-width ids by q when greedy (ties: lower id), else
        Gumbel-top-k draws of the count the plan grants."""
        if sp.greedy:
            ids = np.argsort(-q, kind="stable")[: plan.width]
        else:
            ids = gumbel_top_k(q, plan.children_for(parent.phat, parent.depth + 1), rng)
        return [(int(x), float(q[x])) for x in ids]

    def draft(self, root_token: int, n: int, sp: SamplingParams, rng: PhiloxStream):
        plan = self.policy.plan(context_len=n, stochastic=not sp.greedy)
        nodes = [TreeNode(root_token, -1, 0, 1.0)]
        state = {0: self.root}        # node -> (out row, feature row) of its drafter entry
        slot = {0: n - 1}              # node -> drafter cache row
        qdist: dict[int, np.ndarray] = {}
        base = self.dc.size()
        expand = [0]
        for depth in range(1, plan.max_depth + 1):
            q = self._head_probs(torch.cat([state[v][0].reshape(1, -1) for v in expand]), sp)
            level = []
            for r, v in enumerate(expand):
                if not sp.greedy:
                    qdist[v] = q[r]
                for tok, qx in self._children(q[r], sp, plan, nodes[v], rng):
                    nodes.append(TreeNode(tok, v, depth, nodes[v].phat * qx))
                    level.append(len(nodes) - 1)
            gain = sum(nodes[v].phat for v in level)
            if depth == plan.max_depth or not level or \
                    not self.policy.continue_drafting(depth, gain, n, len(nodes) - 1):
                break
            expand = self.policy.select_frontier(level, nodes, plan.width)
            if not expand:
                break
            self._forward_level(nodes, expand, state, slot, base, n)
        self.dc.trim_to(base)  # the drafting entries are discarded
        keep = self.policy.select_verify(nodes, n, stochastic=not sp.greedy)
        row = {v: i for i, v in enumerate(keep)}
        tree = DraftTree([nodes[v].token for v in keep], [row.get(nodes[v].parent, -1) for v in keep],
                         [nodes[v].depth for v in keep])
        q_rows = {row[v]: qdist[v] for v in keep if v in qdist}
        return tree, q_rows

    def _forward_level(self, nodes, expand, state, slot, base, n) -> None:
        """One drafter pass over the nodes to expand: positions n - 1 + depth, each row seeing the
        committed entries (within the window), its drafted ancestors and itself."""
        first = self.dc.size()
        m = len(expand)
        vis = np.zeros((m, first + m), dtype=bool)
        win = int(self.d.cfg.window)
        for r, v in enumerate(expand):
            lo = max(0, base - 1 + nodes[v].depth - win + 1) if win else 0
            vis[r, lo:base] = True
            u = nodes[v].parent
            while u > 0:
                vis[r, slot[u]] = True
                u = nodes[u].parent
            vis[r, first + r] = True
        feats = torch.cat([state[nodes[v].parent][1].reshape(1, 1, -1) for v in expand], dim=1)
        hid, out = self.d([nodes[v].token for v in expand], feats, self.dc,
                          positions=[n - 1 + nodes[v].depth for v in expand], mask=vis)
        fb = self.d.feedback(hid, out)
        for r, v in enumerate(expand):
            state[v] = (out[:, r : r + 1], fb[:, r : r + 1])
            slot[v] = first + r

    # ---------------------------------------------------------------- verification + update
    def verify(self, tree: DraftTree, q_rows, n: int, sp: SamplingParams, rng: PhiloxStream):
        toks = torch.tensor(tree.tokens, dtype=torch.int32, device=self.t.ctx.device)
        if tree.is_chain():
            o = self.t(toks, self.tc)
        else:
            o = self.t(toks, self.tc, positions=[n + x for x in tree.depth], mask=tree_attention_mask(tree, n))
        z = o.logits[0]
        if sp.greedy:
            path, nxt = verify_tree_greedy(argmax(z), tree, device=self.t.ctx.device.index or 0)
        else:
            p = probs_from_logits(z, sp).double().cpu().numpy()
            path, nxt = verify_tree_stochastic({v: p[v] for v in range(len(tree))}, q_rows, tree, rng)
        keep = [0] + list(path)
        self.tc.compact(n, keep)
        idx = torch.tensor(keep, dtype=torch.long, device=z.device)
        return list(path), int(nxt), [f[:, idx] for f in o.features]

    def update(self, accepted: list[int], feats) -> None:
        hid, out = self.d(accepted, self.d.fuse(feats), self.dc)
        self._set_root(hid[:, -1:], out[:, -1:])

    def round(self, x_n: int, n: int, sp: SamplingParams, rng: PhiloxStream, st) -> list[int]:
        t0 = time.perf_counter()
        tree, q_rows = self.draft(x_n, n, sp, rng)
        t1 = time.perf_counter()
        path, nxt, feats = self.verify(tree, q_rows, n, sp, rng)
        t2 = time.perf_counter()
        acc = [tree.tokens[v] for v in path] + [nxt]
        self.update(acc, feats)
        t3 = time.perf_counter()
        st.t_draft += t1 - t0
        st.t_verify += t2 - t1
        st.t_update += t3 - t2
        st.rounds += 1
        st.accepted.append(len(path))
        st.drafted.append(len(tree) - 1)
        st.depths.append(max(tree.depth))
        self.policy.observe(len(path), len(tree) - 1, max(tree.depth), t1 - t0, t3 - t1)
        return acc
