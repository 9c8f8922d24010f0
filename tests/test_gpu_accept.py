"""Acceptance kernels against the reference's own decisions (tests/golden/sampling.json, made
by python/woodcock/sampling.py with the same Philox uniform tape): accept/reject paths,
next tokens and uniforms consumed are bit-exact. KV compaction against the reference's
known answer and the oracle's sequential memmove, aliasing included."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import wc_oracle as O

pytestmark = pytest.mark.gpu


def test_philox_stream_matches_oracle():
    from woodcock_b200.sampling import PhiloxStream

    s = PhiloxStream(1234, 99)
    u = s.random(1000)
    np.testing.assert_array_equal(u, O.philox_uniforms(1234, 99, 1000))
    assert s.pos == 1099


def test_greedy_tree_known_answer_and_fixtures(golden):
    from woodcock_b200.sampling import DraftTree, verify_tree_greedy

    tree = DraftTree([0, 1, 2, 4], [-1, 0, 0, 2], [0, 1, 1, 2])
    assert verify_tree_greedy([2, 9, 4, 3], tree) == ([2, 3], 3)  # tests/cpp/test_main.cpp:32-40
    for c in golden("sampling")["greedy_tree"]:
        t = DraftTree(c["tokens"], c["parents"], c["depth"])
        assert verify_tree_greedy(c["argmax"], t) == (c["path"], c["next"])


def test_chain_stochastic_bit_exact_with_reference(golden):
    from woodcock_b200.sampling import PhiloxStream, verify_chain_stochastic

    for c in golden("sampling")["chain"]:
        rng = PhiloxStream(c["seed"])
        n, nxt = verify_chain_stochastic(np.array(c["p"]), np.array(c["q"]), c["tokens"], rng)
        assert (n, nxt, rng.pos) == (c["accepted"], c["next"], c["uniforms_used"])


def test_tree_stochastic_bit_exact_with_reference(golden):
    from woodcock_b200.sampling import DraftTree, PhiloxStream, verify_tree_stochastic

    for c in golden("sampling")["tree"]:
        tree = DraftTree(c["tokens"], c["parents"], c["depth"])
        p = {v: np.array(r) for v, r in enumerate(c["p"])}
        q = {int(k): np.array(v) for k, v in c["q"].items()}
        # uniforms the reference drew before verification (children drawn w/o replacement)
        probe = O.Tape(c["seed"])
        for start in range(c["uniforms_used"] + 1):
            probe = O.Tape(c["seed"], start)
            pp, nn = O.verify_tree_stochastic(p, q, tree, probe)
            if probe.pos == c["uniforms_used"] and (pp, nn) == (c["path"], c["next"]):
                break
        rng = PhiloxStream(c["seed"], start)
        path, nxt = verify_tree_stochastic(p, q, tree, rng)
        assert (path, nxt, rng.pos) == (c["path"], c["next"], c["uniforms_used"])


def test_stochastic_large_vocab_matches_oracle():
    """151,936-entry distributions: parallel fp64 residual / scan vs the oracle's sequential one."""
    from woodcock_b200.sampling import DraftTree, PhiloxStream, verify_tree_stochastic

    rng = np.random.default_rng(7)
    V = 151936
    mism = 0
    for i in range(12):
        K = int(rng.integers(1, 5))
        p = rng.dirichlet(np.full(V, 0.05), size=K + 1)
        q = np.zeros((K + 1, V))
        q[:K] = rng.dirichlet(np.full(V, 0.05), size=K)
        toks = [int(rng.choice(V, p=q[j])) for j in range(K)]
        tree = DraftTree([0] + toks, [-1] + list(range(K)), list(range(K + 1)))
        a = verify_tree_stochastic(p, q, tree, PhiloxStream(77 + i))
        tape = O.Tape(77 + i)
        b = O.verify_tree_stochastic({v: p[v] for v in range(K + 1)}, {v: q[v] for v in range(K)}, tree, tape)
        mism += a != b
    assert mism == 0


def test_kv_compact_known_answer_and_aliasing():
    from woodcock_b200.cache import KVCache

    kv = KVCache.create(1, 1, 2, 8, dtype=0)
    k = torch.tensor([[0, 0], [1, 1], [2, 2], [3, 3], [4, 4]], dtype=torch.float32, device="cuda")[:, None, :]
    kv.append(0, k, k)
    kv.commit(5)
    kv.compact(1, [0, 2, 3])  # tests/cpp/test_main.cpp:42-50
    assert kv.size() == 4
    assert kv.read(0)[0][:, 0, 0].cpu().tolist() == [0, 1, 3, 4]

    rng = np.random.default_rng(4)
    for dt in (0, 1):
        L, Hk, D, n0 = 3, 2, 64, 11
        kv = KVCache.create(L, Hk, D, 64, dtype=dt)
        oc = O.KVCache(L, Hk, D)
        for layer in range(L):
            kk = rng.standard_normal((n0 + 9, Hk, D)).astype(np.float32)
            vv = rng.standard_normal((n0 + 9, Hk, D)).astype(np.float32)
            if dt == 1:
                kk = torch.tensor(kk).to(torch.bfloat16).float().numpy()
                vv = torch.tensor(vv).to(torch.bfloat16).float().numpy()
            kv.append(layer, torch.tensor(kk, device="cuda"), torch.tensor(vv, device="cuda"))
            oc.append(layer, kk, vv)
        kv.commit(n0 + 9)
        oc.commit(n0 + 9)
        keep = [0, 1, 4, 5, 8]  # overlapping source / destination rows
        kv.compact(n0, keep)
        oc.compact(n0, keep)
        assert kv.size() == oc.size() == n0 + 5
        for layer in range(L):
            K, Vv = kv.read(layer)
            np.testing.assert_array_equal(K.cpu().numpy(), oc.keys(layer, oc.size()))
            np.testing.assert_array_equal(Vv.cpu().numpy(), oc.values(layer, oc.size()))
