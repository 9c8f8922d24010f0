"""The oracle (oracle/wc_oracle.py) pinned against the reference itself: golden fixtures
made by the reference's C++ core and Python sampling functions (tests/golden/), the
known answers of the reference's own tests, and the distribution-preservation
chi-square tests of tests/test_sampling.py restated on the oracle's functions."""

from __future__ import annotations

import itertools

import numpy as np
import pytest
from scipy.stats import chisquare

import wc_oracle as O
from conftest import weights_checksum


# ------------------------------------------------------------------ model path vs the reference C++ core

@pytest.mark.parametrize("name", ["c1", "c1u"])
def test_oracle_matches_reference_cpp_core(name, golden, tiny_models, prompt64):
    g = golden(name)
    td, dd, tw, dw = tiny_models[name]
    assert g["prompt"] == prompt64
    assert weights_checksum(tw) == pytest.approx(g["weights_checksum"], rel=1e-9)
    t = O.Qwen3.load(td, taps=g["taps"])
    d = O.Drafter.load(dd)
    z, taps = t.forward(prompt64, t.make_cache(), logits_from=len(prompt64) - 1)
    np.testing.assert_allclose(z[-1], np.array(g["last_logits"], np.float32), rtol=0, atol=2e-5)
    assert O.argmax(z[-1]) == g["argmax"]
    for f in range(3):
        np.testing.assert_allclose(taps[f][-1][:8], g["taps_last_head8"][f], rtol=0, atol=1e-5)
    ar = O.generate_autoregressive(t, prompt64, 128)
    assert ar == g["ar_tokens"]
    for pol, P in (("chain:4", O.StaticPolicy(4)), ("tree:3,3,8", O.StaticPolicy(3, 3, 8))):
        sd, st = O.SpeculativeDecoder(t, d, P).generate(prompt64, 128)
        assert sd == g[f"spec_{pol}"]["tokens"] == ar
        assert sum(st.accepted) == g[f"spec_{pol}"]["accepted"]


def forced_from_ar(ar, corrupt_every=4, vocab=4096):
    """forced(round, k, emitted): the next k autoregressive tokens; every `corrupt_every`-th round
    the third draft is replaced by a different token, so acceptance varies between rounds."""

    def forced(r, k, emitted):
        toks = [ar[min(emitted + j, len(ar) - 1)] for j in range(k)]
        if corrupt_every and r % corrupt_every == corrupt_every - 1 and k > 2:
            toks[2] = (toks[2] + 1) % vocab
        return toks

    return forced


def test_oracle_forced_drafts_accept_and_stay_exact(tiny_models, prompt64):
    """Oracle-drafter mode: drafts from the known continuation, corrupted every 4th round,
    are partially accepted and the output still equals autoregressive greedy."""
    td, dd, _, _ = tiny_models["c1u"]
    t, d = O.Qwen3.load(td, taps=[1, 2, 3]), O.Drafter.load(dd)
    ar = O.generate_autoregressive(t, prompt64, 48)
    out, st = O.SpeculativeDecoder(t, d, O.StaticPolicy(4)).generate(prompt64, 48, forced=forced_from_ar(ar))
    assert out == ar
    assert sum(st.accepted) > 20 and min(st.accepted) < 4


# ------------------------------------------------------------------ acceptance vs the reference's Python functions

@pytest.mark.parametrize("name", ["chain4", "chain6", "tree"])
def test_oracle_forced_rounds_match_reference(name, golden, tiny_models, prompt64):
    """tests/golden/c1u_forced.json was made by the reference's C++ core in oracle-drafter mode
    (drafts forced from its own greedy continuation, partially accepted; trees with branching
    accepted paths). The oracle restatement reproduces every round: tree, accepted path, next
    token, the drafter's own proposals and their logits, and both cache lengths."""
    g = golden("c1u_forced")
    ref = g[name]
    assert g["prompt"] == prompt64
    td, dd, _, _ = tiny_models["c1u"]
    t, d = O.Qwen3.load(td, taps=g["taps"]), O.Drafter.load(dd)
    r = O.forced_tree_run(t, d, prompt64, g["max_new"], ref["templates"])
    assert r["tokens"] == ref["tokens"] == ref["ar"][: g["max_new"]]
    assert r["accepted"] == ref["accepted"] and ref["accepted"] >= 50
    assert len(r["rounds"]) == len(ref["rounds"])
    for a, b in zip(r["rounds"], ref["rounds"]):
        for key in ("tokens", "parents", "path", "next", "proposals", "n", "drafter_len"):
            assert a[key] == b[key], key
        np.testing.assert_allclose(a["proposal_logits"], b["proposal_logits"], rtol=0, atol=2e-5)
    assert any(len(x["path"]) not in (0, len(x["tokens"]) - 1) for x in ref["rounds"])  # partial acceptance


def test_oracle_chain_stochastic_matches_reference(golden):
    for c in golden("sampling")["chain"]:
        tape = O.Tape(c["seed"])
        n, nxt = O.verify_chain_stochastic(np.array(c["p"]), np.array(c["q"]), c["tokens"], tape)
        assert (n, nxt, tape.pos) == (c["accepted"], c["next"], c["uniforms_used"])


def test_oracle_tree_stochastic_matches_reference(golden):
    for c in golden("sampling")["tree"]:
        tree = O.DraftTree(c["tokens"], c["parents"], c["depth"])
        p = {v: np.array(row) for v, row in enumerate(c["p"])}
        q = {int(k): np.array(v) for k, v in c["q"].items()}
        tape = O.Tape(c["seed"])
        # the fixture's tape was also used to draw the children: replay from after those draws
        tape.pos = c["uniforms_used"] - _uniforms_in_verify(tree, p, q, c)
        path, nxt = O.verify_tree_stochastic(p, q, tree, tape)
        assert (path, nxt) == (c["path"], c["next"])
        assert tape.pos == c["uniforms_used"]


def _uniforms_in_verify(tree, p, q, c):
    """Count uniforms consumed by verify_tree_stochastic for this case (replay on a probe tape)."""
    for start in range(0, c["uniforms_used"] + 1):
        t = O.Tape(c["seed"], start)
        path, nxt = O.verify_tree_stochastic(p, q, tree, t)
        if t.pos == c["uniforms_used"] and (path, nxt) == (c["path"], c["next"]):
            return c["uniforms_used"] - start
    raise AssertionError("no consistent replay")


def test_oracle_greedy_tree_and_mask_match_reference(golden):
    s = golden("sampling")
    for c in s["greedy_tree"]:
        tree = O.DraftTree(c["tokens"], c["parents"], c["depth"])
        assert O.verify_tree_greedy(c["argmax"], tree) == (c["path"], c["next"])
    for c in s["mask"]:
        tree = O.DraftTree(c["tokens"], c["parents"], c["depth"])
        assert O.tree_attention_mask(tree, c["prefix"]).astype(int).tolist() == c["mask"]


def test_oracle_gumbel_topk_matches_reference(golden):
    for c in golden("sampling")["gumbel"]:
        tape = O.Tape(c["seed"])
        assert O.sample_without_replacement(np.array(c["q"]), c["k"], tape) == c["out"]
        assert tape.pos == c["uniforms_used"]


# ------------------------------------------------------------------ known answers of the reference's tests

def test_known_answer_greedy_tree_and_mask():
    """tests/cpp/test_main.cpp:32-40 and tests/test_sampling.py:185-205."""
    tree = O.DraftTree([0, 1, 2, 4], [-1, 0, 0, 2], [0, 1, 1, 2])
    assert O.verify_tree_greedy([2, 9, 4, 3], tree) == ([2, 3], 3)
    m = O.tree_attention_mask(tree, 2)
    assert m.shape == (4, 6) and m[:, :2].all()
    assert list(m[3, 2:]) == [True, False, True, True]
    assert list(m[1, 2:]) == [True, True, False, False]


def test_known_answer_kv_compact():
    """tests/cpp/test_main.cpp:42-50: keep rows 1, 3, 4 of 5."""
    c = O.KVCache(1, 1, 2)
    k = np.array([[0, 0], [1, 1], [2, 2], [3, 3], [4, 4]], np.float32)
    c.append(0, k, k)
    c.commit(5)
    c.compact(1, [0, 2, 3])
    assert c.size() == 4
    assert c.k[0][:4, 0].tolist() == [0, 1, 3, 4]


def test_known_answer_probs_warping():
    """tests/test_sampling.py:208-216."""
    z = np.array([[2.0, 1.0, 0.0, -1.0]], np.float32)
    p = O.probs_from_logits(z, O.SamplingParams(temperature=1.0, top_k=2))
    assert p[0, 2] == 0 and p[0, 3] == 0 and abs(p.sum() - 1) < 1e-6
    p = O.probs_from_logits(z, O.SamplingParams(temperature=1.0, top_p=0.5))
    assert (p[0] > 0).sum() == 1
    p = O.probs_from_logits(z, O.SamplingParams(temperature=0.5))
    ref = np.exp(np.array([2, 1, 0, -1.0]) / 0.5)
    np.testing.assert_allclose(p[0], ref / ref.sum(), rtol=1e-5)


def test_philox_known_vector():
    """Philox4x32-10 known answer (Random123 kat_vectors: counter 0, key 0)."""
    r = O.philox4x32_10(np.array([0], np.uint32), np.array([0], np.uint32), 0)
    assert [int(x[0]) for x in r] == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]


# ------------------------------------------------------------------ chi-square distribution tests (test_sampling.py)

V, N_EMIT, TRIALS = 5, 3, 20000


def _markov(seed, sharp):
    return np.random.default_rng(seed).dirichlet(np.full(V, sharp), size=V)


P = _markov(1, 0.7)
Q = 0.5 * _markov(2, 0.7) + 0.5 * P
Q_TRUNC = Q * (np.arange(V) < 3)
Q_TRUNC /= Q_TRUNC.sum(-1, keepdims=True)


def _exact_law(root=0):
    law = np.zeros((V,) * N_EMIT)
    for seq in itertools.product(range(V), repeat=N_EMIT):
        pr, prev = 1.0, root
        for t in seq:
            pr *= P[prev, t]
            prev = t
        law[seq] = pr
    return law.ravel()


def _run(gen_round, trials=TRIALS, seed=0):
    rng = np.random.default_rng(seed)
    counts = np.zeros(V ** N_EMIT)
    for _ in range(trials):
        out = []
        while len(out) < N_EMIT:
            out.extend(gen_round(out[-1] if out else 0, rng))
        counts[np.ravel_multi_index(tuple(out[:N_EMIT]), (V,) * N_EMIT)] += 1
    return counts


def _pvalue(counts):
    exp = _exact_law() * counts.sum()
    keep = exp > 0
    return chisquare(counts[keep], exp[keep] * counts[keep].sum() / exp[keep].sum()).pvalue


def _chain_round(K, Qm=Q):
    def gen(prev, rng):
        toks, qs, ps, cur = [], [], [P[prev]], prev
        for _ in range(K):
            x = int(rng.choice(V, p=Qm[cur]))
            qs.append(Qm[cur])
            toks.append(x)
            cur = x
            ps.append(P[cur])
        n, nxt = O.verify_chain_stochastic(np.array(ps), np.array(qs), toks, rng)
        return toks[:n] + [nxt]

    return gen


def _tree_round(depth, width, draw_wor=True, Qm=Q):
    def gen(prev, rng):
        tokens, parents, depths, frontier = [prev], [-1], [0], [0]
        for dd in range(1, depth + 1):
            nxt = []
            for v in frontier:
                kids = O.sample_without_replacement(Qm[tokens[v]], width, rng) if draw_wor else \
                    list(np.argsort(-Qm[tokens[v]])[:width])
                for x in kids:
                    tokens.append(int(x)); parents.append(v); depths.append(dd); nxt.append(len(tokens) - 1)
            frontier = nxt
        tree = O.DraftTree(tokens, parents, depths)
        path, nxt = O.verify_tree_stochastic({v: P[t] for v, t in enumerate(tokens)},
                                             {v: Qm[t] for v, t in enumerate(tokens)}, tree, rng)
        return [tree.tokens[v] for v in path] + [nxt]

    return gen


@pytest.mark.parametrize("K", [1, 3])
def test_chain_stochastic_preserves_target(K):
    assert _pvalue(_run(_chain_round(K))) > 1e-3


def test_chain_stochastic_truncated_draft_vocab_preserves_target():
    assert _pvalue(_run(_chain_round(3, Q_TRUNC))) > 1e-3


@pytest.mark.parametrize("depth,width", [(1, 2), (2, 3)])
def test_tree_stochastic_preserves_target(depth, width):
    assert _pvalue(_run(_tree_round(depth, width))) > 1e-3


def test_negative_control_topk_children_is_biased():
    assert _pvalue(_run(_tree_round(1, 2, draw_wor=False))) < 1e-6


def test_negative_control_skipping_the_residual_is_biased():
    """Resampling from p instead of norm(max(0, p - q)) after a rejection must fail."""
    def gen(prev, rng):
        x = int(rng.choice(V, p=Q[prev]))
        if rng.random() < min(1.0, P[prev, x] / Q[prev, x]):
            return [x, int(rng.choice(V, p=P[x]))]
        return [int(rng.choice(V, p=P[prev]))]

    assert _pvalue(_run(gen)) < 1e-6


# ------------------------------------------------------------------ the device's sampled-round protocol

def _device_chain_round(K, Qm=Q, skip_residual=False):
    """One sampled chain round as the CUDA path draws it (Gumbel-max drafts from Philox
    stream i, acceptance uniforms and residual noise from their streams), on log-probabilities
    as logits at T = 1; each round takes the next counter block."""
    state = {"base": 0}

    def gen(prev, rng):
        base = state["base"]
        state["base"] += O.RNG_ROUND_STRIDE
        with np.errstate(divide="ignore"):
            toks, zd, zt, cur = [prev], [], [np.log(P[prev])], prev
            for i in range(K):
                z = np.log(Qm[cur]).astype(np.float32)
                cur = O.gumbel_draw(z, 1.0, 77, base, i)
                toks.append(cur)
                zd.append(z)
                zt.append(np.log(P[cur]))
        a, nxt = O.sampled_chain_accept(np.array(zt, np.float32), np.array(zd, np.float32), toks, 1.0, 77, base,
                                        skip_residual=skip_residual)
        return toks[1:a + 1] + [nxt]

    return gen


DEVICE_TRIALS = 5000  # numpy Philox per draw is slow; the planted mistake is still caught by far


def test_device_protocol_preserves_target():
    assert _pvalue(_run(_device_chain_round(3, Q_TRUNC), trials=DEVICE_TRIALS)) > 1e-3


def test_device_protocol_negative_control_skipping_the_residual_is_biased():
    assert _pvalue(_run(_device_chain_round(3, Q_TRUNC, skip_residual=True), trials=DEVICE_TRIALS)) < 1e-6


def test_device_protocol_decisions_equal_the_reference_rule_on_its_uniforms():
    """The accept count of sampled_chain_accept equals verify_chain_stochastic (pinned to the
    reference above) fed the acceptance stream as its uniform tape."""
    rng = np.random.default_rng(5)
    Vs, K = 64, 4
    for trial in range(200):
        zt = rng.normal(0, 1.5, (K + 1, Vs)).astype(np.float32)
        zd = rng.normal(0, 1.5, (K, Vs)).astype(np.float32)
        toks = [0] + [int(x) for x in rng.integers(0, Vs, K)]
        base = trial * O.RNG_ROUND_STRIDE
        a, _ = O.sampled_chain_accept(zt, zd, toks, 0.7, 9, base)
        sm = lambda z: (lambda e: e / e.sum())(np.exp((z / np.float32(0.7)).astype(np.float64) -
                                                      (z / np.float32(0.7)).max()))
        p = np.array([sm(r) for r in zt])
        q = np.array([sm(r) for r in zd])
        ref_a, _ = O.verify_chain_stochastic(p, q, toks[1:], O.Tape(9, base + O.RNG_ACCEPT_STREAM * O.RNG_STREAM_LEN))
        assert a == ref_a, trial


def test_device_warping_threshold_equals_reference_warping():
    """The device's threshold form of top-k / top-p equals probs_from_logits (pinned to
    sampling.py:39-55) on untied logits."""
    rng = np.random.default_rng(21)
    for trial in range(60):
        V = int(rng.integers(20, 3000))
        z = rng.normal(0, rng.uniform(0.5, 4.0), V).astype(np.float32)
        T = float(rng.uniform(0.3, 1.5))
        top_k = int(rng.integers(0, V)) if trial % 3 else 0
        top_p = float(rng.uniform(0.05, 1.0)) if trial % 2 else 1.0
        ref = O.probs_from_logits(z, O.SamplingParams(temperature=T, top_k=top_k, top_p=top_p))
        got = O.warped_probs(z, T, top_k, top_p)
        assert ((ref > 0) == (got > 0)).all(), trial
        np.testing.assert_allclose(got, ref, rtol=2e-5, atol=1e-9)
