"""Batched tree verification: many independent requests verify their
draft token trees in one pass over the target, then compact the accepted paths in place.

The reference decodes one request at a time; its per-request semantics are kept: node 0
is the request's newest committed token, positions are lens[r] + depth, each node attends
to the committed prefix and to its tree ancestors (sampling.py:118-128), the greedy rule
picks the path (sampling.py:131-140) and the accepted rows move down in the cache
(src/cache/kv_cache.cpp:21-31). At 2048 verify rows the projections run as tcgen05 GEMMs
(wc_batch_* / wc_gemm_bf16 in the C ABI).
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ._lib import int_array, lib
from .cache import KVCache
from .context import ptr
from .target import Target


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


class BatchVerifier:
    def __init__(self, target: Target, max_requests: int, max_nodes: int, capacity: int,
                 drafter_cache: tuple[int, int, int] | None = None):
        """drafter_cache = (layers, kv_heads, head_dim) of a drafter arena compacted alongside."""
        self.t, self.ctx = target, target.ctx
        self.max_requests, self.max_nodes, self.capacity = max_requests, max_nodes, capacity
        dl, dh, dd = drafter_cache or (0, 0, 0)
        h = C.c_void_p()
        self.ctx.check(lib().wc_batch_create(target.h, max_requests, max_nodes, capacity, dl, dh, dd, C.byref(h)))
        self.h = h

    def __del__(self):
        if getattr(self, "h", None):
            lib().wc_batch_destroy(self.h)
            self.h = None

    def set_prefix(self, r: int, cache: KVCache, n: int) -> None:
        self.ctx.check(lib().wc_batch_set_prefix(self.h, r, cache.h, n))

    def fill_synthetic(self, nreq: int, n: int, seed: int = 0) -> None:
        self.ctx.check(lib().wc_batch_fill_synthetic(self.h, nreq, n, seed))

    def verify(self, tokens, parents, logits: bool = False):
        """tokens, parents: [nreq][nodes]. Returns the target argmax per node [nreq][nodes]
        (and the logits [nreq][nodes][V] when asked)."""
        tok, par = _i32(tokens), _i32(parents)
        nreq, nodes = tok.shape
        am = np.empty((nreq, nodes), dtype=np.int32)
        lg = np.empty((nreq, nodes, self.t.cfg.vocab), dtype=np.float32) if logits else None
        self.ctx.check(lib().wc_batch_verify(self.h, nreq, nodes, tok.ctypes.data, par.ctypes.data, am.ctypes.data,
                                             lg.ctypes.data if logits else None))
        return (am, lg) if logits else am

    PROFILE_KINDS = ("qkv_gemm", "tree_attention", "o_gemm", "gate_up_gemm", "down_gemm", "head_gemm")

    def verify_profiled(self, tokens, parents):
        """verify with CUDA events around kernel classes: (argmax, {kind: {mean_ms, launches}})."""
        tok, par = _i32(tokens), _i32(parents)
        nreq, nodes = tok.shape
        am = np.empty((nreq, nodes), dtype=np.int32)
        ms = (C.c_float * 16)()
        cnt = (C.c_int * 16)()
        self.ctx.check(lib().wc_batch_verify_profiled(self.h, nreq, nodes, tok.ctypes.data, par.ctypes.data,
                                                      am.ctypes.data, ms, cnt))
        return am, {k: {"total_ms": float(ms[i]), "launches": int(cnt[i])} for i, k in enumerate(self.PROFILE_KINDS)}

    def commit(self, keeps: list[list[int]]) -> None:
        """keeps[r] = [0] + accepted path (increasing node indices)."""
        nreq = len(keeps)
        mk = max(len(k) for k in keeps)
        arr = np.zeros((nreq, mk), dtype=np.int32)
        for r, k in enumerate(keeps):
            arr[r, : len(k)] = k
        nk = _i32([len(k) for k in keeps])
        self.ctx.check(lib().wc_batch_commit(self.h, nreq, arr.ctypes.data, nk.ctypes.data, mk))

    def lens(self, nreq: int) -> list[int]:
        out = np.empty(nreq, dtype=np.int32)
        self.ctx.check(lib().wc_batch_lens(self.h, nreq, out.ctypes.data))
        return out.tolist()

    def read_kv(self, r: int, layer: int, n: int) -> tuple[np.ndarray, np.ndarray]:
        """Rows [0, n) of request r at `layer` as float32 [n][kv_heads][head_dim]."""
        c = self.t.cfg
        k = np.empty((n, c.kv_heads, c.head_dim), dtype=np.uint16)
        v = np.empty_like(k)
        self.ctx.check(lib().wc_batch_read_kv(self.h, r, layer, n, k.ctypes.data, v.ctypes.data))
        f = lambda x: (x.astype(np.uint32) << 16).view(np.float32)
        return f(k), f(v)


def greedy_keep(argmax_row, tokens_row, parents_row) -> list[int]:
    """verify_tree_greedy (sampling.py:131-140) on one request: [0] + the accepted node path."""
    children = [[] for _ in tokens_row]
    for v, p in enumerate(parents_row):
        if p >= 0:
            children[p].append(v)
    v, keep = 0, [0]
    while True:
        want = int(argmax_row[v])
        nxt = next((c for c in children[v] if int(tokens_row[c]) == want), None)
        if nxt is None:
            return keep
        keep.append(nxt)
        v = nxt


def gemm_bf16(A: torch.Tensor, B: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
    """A [M][K] . B[N][K]^T (+ residual) on the tensor cores; bf16 in, fp32 out."""
    from .context import Context

    ctx = Context.get(A.device)
    A = A.to(torch.bfloat16).contiguous()
    B = B.to(torch.bfloat16).contiguous()
    M, K = A.shape
    N = B.shape[0]
    out = residual.clone().float().contiguous() if residual is not None else \
        torch.empty((M, N), dtype=torch.float32, device=A.device)
    with ctx.enter(A, B, out):
        ctx.check(lib().wc_gemm_bf16(ctx.h, ptr(A), ptr(B), ptr(out), M, N, K, ptr(out) if residual is not None
                                     else None))
    return out
