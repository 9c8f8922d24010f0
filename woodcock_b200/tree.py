"""Draft trees, and the synced (non-fused) path, as host-driven rounds over the device API
(python/woodcock/spec.py:129-147, 216-329, 366-374; src/core/spec.cpp:86-233).

Each round drafts level by level: the drafter's distribution at every frontier node
(softmax of its head, with the temperature when sampling), children by top-w (greedy) or
drawn without replacement (sampling, count fixed before drawing), the policy choosing the
next frontier and the nodes to verify (EAGLE-2 path probabilities). The target verifies the
tree in one forward with the tree mask and depth positions, the greedy or recursive
rejection rule picks the path, the target cache is compacted to it and the drafter is
updated on the accepted rows. Every forward, head, softmax, acceptance and compaction is a
device call; the host holds the tree (tens of nodes) and synchronises once per level, as
the reference's synced path does.
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
class _Node:
    token: int
    parent: int
    depth: int
    phat: float  # product of draft probabilities along the path
    out: torch.Tensor | None = None  # (1, 1, d) drafter output at this node
    fb: torch.Tensor | None = None   # (1, 1, d) feature for its children's drafter pass
    cache_idx: int = -1
    q: np.ndarray | None = None      # sampling: the distribution its children were drawn from


def _sample(p: np.ndarray, rng: PhiloxStream) -> int:
    """sampling.py:190-193: inverse CDF on the fp64 cumulative sum."""
    c = np.cumsum(np.asarray(p, dtype=np.float64))
    return int(min(np.searchsorted(c, rng.random() * c[-1], side="right"), len(c) - 1))


def _sample_without_replacement(q: np.ndarray, k: int, rng: PhiloxStream) -> list[int]:
    """sampling.py:196-203: Gumbel-top-k over the nonzero entries, one uniform each in id order
    (drawn even when k is 0, as the reference does, so the stream stays aligned)."""
    nz = np.flatnonzero(q > 0)
    k = min(k, len(nz))
    if len(nz) == 0:
        return []
    with np.errstate(divide="ignore"):
        g = np.log(q[nz]) - np.log(-np.log(rng.random(len(nz))))
    return [int(nz[i]) for i in np.argsort(-g, kind="stable")[:k]]


class HostRounds:
    """State of one request decoded through host-driven rounds: target and drafter caches,
    the chain root (drafter output and feature after the last committed token)."""

    def __init__(self, target, drafter, policy, capacity: int):
        self.t, self.d, self.policy, self.capacity = target, drafter, policy, capacity

    # ------------------------------------------------------------------ prefill (spec.py:129-147)
    def prefill(self, prompt: list[int], sp: SamplingParams, rng: PhiloxStream) -> int:
        self.tc = self.t.make_cache(self.capacity)
        n = len(prompt)
        o = self.t(torch.tensor(prompt, dtype=torch.int32, device=self.t.ctx.device), self.tc, logits_from=n - 1)
        first = self._sample_target(o.logits[0, -1:], sp, rng)
        self.dc = self.d.make_cache(self.capacity)
        g = self.d.fuse(o.features)
        hid, out = self.d(list(prompt[1:]) + [first], g, self.dc)
        self.root_out = out[:, -1:]
        self.root_fb = self.d.feedback(hid[:, -1:], out[:, -1:])
        return first

    def _sample_target(self, logits: torch.Tensor, sp: SamplingParams, rng: PhiloxStream) -> int:
        if sp.greedy:
            return int(argmax(logits.reshape(1, -1))[0])
        p = probs_from_logits(logits.reshape(1, -1), sp)[0].double().cpu().numpy()
        return _sample(p / p.sum(), rng)

    # ------------------------------------------------------------------ drafting (spec.py:216-294)
    def _draft_dist(self, outs: torch.Tensor, sp: SamplingParams) -> torch.Tensor:
        z = self.d.logits(outs)  # (m, head rows)
        if sp.greedy:
            return softmax(z.float())
        return probs_from_logits(z, SamplingParams(temperature=sp.temperature))

    def draft(self, root_token: int, n: int, sp: SamplingParams, rng: PhiloxStream):
        pol = self.policy
        plan = pol.plan(context_len=n, stochastic=not sp.greedy)
        nodes = [_Node(root_token, -1, 0, 1.0, out=self.root_out, fb=self.root_fb, cache_idx=n - 1)]
        base = self.dc.size()
        frontier, tree_cache = [0], 0
        ids = self.d.vocab_ids
        ids_np = ids.cpu().numpy() if ids is not None else None
        V = self.t.cfg.vocab
        for depth in range(1, plan.max_depth + 1):
            outs = torch.cat([nodes[v].out.reshape(1, -1) for v in frontier], dim=0)
            q = self._draft_dist(outs, sp)
            new = []
            if sp.greedy:
                w = plan.width
                # top-w rows of each frontier node, largest first, ties by row index
                order = torch.sort(-q, dim=-1, stable=True).indices[:, :w].cpu().numpy()
                qv = torch.gather(q, 1, torch.as_tensor(order, device=q.device)).double().cpu().numpy()
                for r_, v in enumerate(frontier):
                    for c, qc in zip(order[r_], qv[r_]):
                        tok = int(c) if ids_np is None else int(ids_np[c])
                        new.append(_Node(tok, v, depth, nodes[v].phat * float(qc)))
            else:
                qn = q.double().cpu().numpy()
                for r_, v in enumerate(frontier):
                    full = np.zeros(V)
                    if ids_np is None:
                        full[: qn.shape[1]] = qn[r_]
                    else:
                        full[ids_np] = qn[r_]
                    full /= full.sum()
                    nodes[v].q = full
                    m = plan.children_for(nodes[v].phat, depth)
                    for x in _sample_without_replacement(full, m, rng):
                        new.append(_Node(int(x), v, depth, nodes[v].phat * float(full[x])))
            nodes.extend(new)
            level = list(range(len(nodes) - len(new), len(nodes)))
            gain = sum(nodes[v].phat for v in level)
            if depth == plan.max_depth or not pol.continue_drafting(depth, gain, n, len(nodes) - 1):
                break
            frontier = pol.select_frontier(level, nodes, plan.width)
            if not frontier:
                break
            toks = [nodes[v].token for v in frontier]
            fb = torch.cat([nodes[nodes[v].parent].fb.reshape(1, 1, -1) for v in frontier], dim=1)
            pos = [n - 1 + nodes[v].depth for v in frontier]
            mask = self._draft_mask(nodes, frontier, base, tree_cache)
            hid, out = self.d(toks, fb, self.dc, positions=pos, mask=mask)
            fbk = self.d.feedback(hid, out)
            for r_, v in enumerate(frontier):
                nodes[v].out = out[:, r_ : r_ + 1]
                nodes[v].fb = fbk[:, r_ : r_ + 1]
                nodes[v].cache_idx = base + tree_cache + r_
            tree_cache += len(frontier)
        self.dc.trim_to(base)  # the speculative drafter entries are discarded
        keep = pol.select_verify(nodes, n, stochastic=not sp.greedy)
        remap = {v: i for i, v in enumerate(keep)}
        tree = DraftTree([nodes[v].token for v in keep], [remap.get(nodes[v].parent, -1) for v in keep],
                         [nodes[v].depth for v in keep])
        return tree, [nodes[v] for v in keep]

    def _draft_mask(self, nodes, frontier, base, tree_cache) -> np.ndarray:
        """Committed entries (within the window) + the node's drafted ancestors + itself."""
        m = len(frontier)
        mask = np.zeros((m, base + tree_cache + m), dtype=bool)
        w = int(self.d.cfg.window)
        for r_, v in enumerate(frontier):
            pos = base - 1 + nodes[v].depth
            lo = 0 if not w else max(0, pos - w + 1)
            mask[r_, lo:base] = True
            u = nodes[v].parent
            while u > 0:
                mask[r_, nodes[u].cache_idx] = True
                u = nodes[u].parent
            mask[r_, base + tree_cache + r_] = True
        return mask

    # ------------------------------------------------------------------ verification (spec.py:296-329)
    def verify(self, tree: DraftTree, kept: list[_Node], n: int, sp: SamplingParams, rng: PhiloxStream):
        toks = torch.tensor(tree.tokens, dtype=torch.int32, device=self.t.ctx.device)
        if tree.is_chain():
            o = self.t(toks, self.tc)
        else:
            o = self.t(toks, self.tc, positions=[n + d for d in tree.depth], mask=tree_attention_mask(tree, n))
        logits = o.logits[0]
        if sp.greedy:
            path, nxt = verify_tree_greedy(argmax(logits), tree, device=self.t.ctx.device.index or 0)
        else:
            p_all = probs_from_logits(logits, sp).double()
            p = {v: p_all[v].cpu().numpy() for v in range(len(tree))}
            q = {v: kept[v].q for v in range(len(tree)) if kept[v].q is not None}
            path, nxt = verify_tree_stochastic(p, q, tree, rng)
        keep = [0] + list(path)
        self.tc.compact(n, keep)
        idx = torch.tensor(keep, dtype=torch.long, device=logits.device)
        return list(path), int(nxt), [f[:, idx] for f in o.features]

    # ------------------------------------------------------------------ drafter update (spec.py:366-374)
    def update(self, acc_tokens: list[int], feats) -> None:
        g = self.d.fuse(feats)
        hid, out = self.d(acc_tokens, g, self.dc)
        self.root_out = out[:, -1:]
        self.root_fb = self.d.feedback(hid[:, -1:], out[:, -1:])

    def round(self, x_n: int, n: int, sp: SamplingParams, rng: PhiloxStream, st) -> list[int]:
        ta = time.perf_counter()
        tree, nodes = self.draft(x_n, n, sp, rng)
        tb = time.perf_counter()
        path, nxt, feats = self.verify(tree, nodes, n, sp, rng)
        tc = time.perf_counter()
        acc = [tree.tokens[v] for v in path] + [nxt]
        self.update(acc, feats)
        td = time.perf_counter()
        st.t_draft += tb - ta
        st.t_verify += tc - tb
        st.t_update += td - tc
        st.rounds += 1
        st.accepted.append(len(path))
        st.drafted.append(len(tree) - 1)
        st.depths.append(max(tree.depth))
        self.policy.observe(len(path), len(tree) - 1, max(tree.depth), tb - ta, td - tb)
        return acc
