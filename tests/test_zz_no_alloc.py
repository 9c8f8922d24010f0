"""wc_accept_stochastic_noalloc (scratch compiled into the library, no device allocation in the
call) against wc_accept_stochastic, both through the C ABI on the same device inputs: the
accepted path, the next token and the number of uniforms consumed are integers and must be
identical, on two calls in a row. The file name sorts last so that the test also runs after the
rest of the suite in one process; it passes alone in a fresh process as well."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_V = 163840  # WC_ACCEPT_NOALLOC_MAX_V in include/woodcock_b200.h


def _run(fn_name, ctx, P, Q, tok, par, seed, offset):
    from woodcock_b200._lib import lib
    from woodcock_b200.context import ptr

    N, V = P.shape
    out = torch.full((N + 3,), -7, dtype=torch.int32, device=ctx.device)
    with ctx.enter(P, Q, tok, par, out):
        ctx.check(getattr(lib(), fn_name)(ctx.h, ptr(P), ptr(Q), V, ptr(tok), ptr(par), N, seed, offset,
                                          ptr(out[3:]), ptr(out[0:1]), ptr(out[1:2]), ptr(out[2:3])))
    o = out.cpu().tolist()
    return o[3 : 3 + o[0]], o[1], o[2]


def _case(rng, V, K, dev):
    p = rng.dirichlet(np.full(V, 0.05), size=K + 1)
    q = np.zeros((K + 1, V))
    q[:K] = rng.dirichlet(np.full(V, 0.05), size=K)
    toks = [0] + [int(rng.choice(V, p=q[j])) for j in range(K)]
    par = [-1] + list(range(K))
    P = torch.tensor(p, dtype=torch.float64, device=dev)
    Q = torch.tensor(q, dtype=torch.float64, device=dev)
    return P, Q, torch.tensor(toks, dtype=torch.int32, device=dev), torch.tensor(par, dtype=torch.int32, device=dev)


def test_noalloc_matches_allocating_entry_twice_in_a_row():
    from woodcock_b200.context import Context

    ctx = Context.get(0)
    torch.cuda.set_device(ctx.device)
    rng = np.random.default_rng(2024)
    for V, K, seed in ((151936, 4, 11), (4096, 3, 12)):
        P, Q, tok, par = _case(rng, V, K, ctx.device)
        ref = _run("wc_accept_stochastic", ctx, P, Q, tok, par, seed, 5)
        first = _run("wc_accept_stochastic_noalloc", ctx, P, Q, tok, par, seed, 5)
        second = _run("wc_accept_stochastic_noalloc", ctx, P, Q, tok, par, seed, 5)
        assert first == ref
        assert second == ref
        assert ref[2] >= 1 and 0 <= ref[1] < V


def test_noalloc_rejects_vocabulary_above_its_scratch():
    from woodcock_b200._lib import WC_ERR_CAPACITY, lib
    from woodcock_b200.context import Context, ptr

    ctx = Context.get(0)
    torch.cuda.set_device(ctx.device)
    V = MAX_V + 1
    P = torch.zeros((1, V), dtype=torch.float64, device=ctx.device)
    tok = torch.zeros((1,), dtype=torch.int32, device=ctx.device)
    par = torch.full((1,), -1, dtype=torch.int32, device=ctx.device)
    out = torch.zeros((4,), dtype=torch.int32, device=ctx.device)
    st = lib().wc_accept_stochastic_noalloc(ctx.h, ptr(P), ptr(P), V, ptr(tok), ptr(par), 1, 1, 0, ptr(out[3:]),
                                            ptr(out[0:1]), ptr(out[1:2]), ptr(out[2:3]))
    assert st == WC_ERR_CAPACITY
    assert b"WC_ACCEPT_NOALLOC_MAX_V" in lib().wc_last_error(ctx.h)


def test_noalloc_call_records_into_a_global_mode_capture():
    """The property the entry point exists for: after one warm call, a second call records into
    a CUDA graph captured in global mode, which refuses cudaMalloc, cudaFree and any device or
    stream synchronisation made during the capture. Replays give the eager result."""
    from woodcock_b200._lib import lib
    from woodcock_b200.context import Context, ptr

    ctx = Context.get(0)
    torch.cuda.set_device(ctx.device)
    rng = np.random.default_rng(77)
    P, Q, tok, par = _case(rng, 32000, 4, ctx.device)
    N, V = P.shape
    ref = _run("wc_accept_stochastic", ctx, P, Q, tok, par, 31, 9)
    assert _run("wc_accept_stochastic_noalloc", ctx, P, Q, tok, par, 31, 9) == ref  # warm call
    out = torch.full((N + 3,), -7, dtype=torch.int32, device=ctx.device)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=ctx.stream, capture_error_mode="global"):
        st = lib().wc_accept_stochastic_noalloc(ctx.h, ptr(P), ptr(Q), V, ptr(tok), ptr(par), N, 31, 9,
                                                ptr(out[3:]), ptr(out[0:1]), ptr(out[1:2]), ptr(out[2:3]))
    assert st == 0, lib().wc_last_error(ctx.h)
    for _ in range(2):
        out.fill_(-7)
        g.replay()
        torch.cuda.synchronize()
        o = out.cpu().tolist()
        assert (o[3 : 3 + o[0]], o[1], o[2]) == ref
    del g
