"""Draft trees (spec.py:216-374; src/core/spec.cpp:86-233).

(a) Greedy top-k trees (StaticPolicy(3, 3, 8)) on C1 fp32, as device tree rounds: tokens equal
    the reference C++ core's tree:3,3,8 run and autoregressive decoding, and the accepted total
    equals the reference's (tests/golden/c1*.json).
(b) fused=False on a chain (a width-1 device tree round): the autoregressive tokens.
(c) Forced trees with branching accepted paths (tests/golden/c1u_forced.json, made by the
    reference C++ core in oracle-drafter mode): every round's accepted path and next token,
    the drafter's own proposals and logits at the root and every drafted node (these depend on
    the tree-masked drafter passes and on the previous round's multi-row update), and both
    cache lengths equal the reference's.
(d) Sampled trees: the same Philox stream drives the oracle's restatement of the reference
    (wc_oracle.SpeculativeDecoder with Tape(seed)) and this path; the token streams agree.
"""

from __future__ import annotations

import pytest

import wc_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def c1_models(tiny_models):
    from woodcock_b200 import Drafter, Target

    return {name: (Target.load(td, feature_layers=[1, 2, 3], dtype="fp32"), Drafter.load(dd, dtype="fp32"))
            for name, (td, dd, _, _) in tiny_models.items()}


@pytest.mark.parametrize("name", ["c1", "c1u"])
def test_greedy_tree_matches_reference(name, golden, c1_models, prompt64):
    from woodcock_b200 import SpeculativeDecoder, StaticPolicy

    g = golden(name)
    t, d = c1_models[name]
    out, st = SpeculativeDecoder(t, d, StaticPolicy(3, 3, 8), max_context=512).generate(prompt64, 128)
    assert out == g["spec_tree:3,3,8"]["tokens"] == g["ar_tokens"]
    assert sum(st.accepted) == g["spec_tree:3,3,8"]["accepted"]
    assert st.fused and st.rounds == len(st.accepted) and max(st.depths) <= 3


def test_synced_chain_equals_autoregressive(golden, c1_models, prompt64):
    from woodcock_b200 import SpeculativeDecoder, StaticPolicy

    t, d = c1_models["c1u"]
    out, st = SpeculativeDecoder(t, d, StaticPolicy(4), fused=False, max_context=512).generate(prompt64, 64)
    assert out == golden("c1u")["ar_tokens"][:64]


def test_forced_tree_rounds_match_reference(golden, c1_models, prompt64):
    import numpy as np

    from woodcock_b200 import SpeculativeDecoder, StaticPolicy

    g = golden("c1u_forced")
    ref = g["tree"]
    t, d = c1_models["c1u"]
    V, A = t.cfg.vocab, ref["ar"]
    templates = [O.parse_template(x) for x in ref["templates"]]
    dec = SpeculativeDecoder(t, d, StaticPolicy(4, 2, 8), max_context=512)
    emitted = [dec.prefill(prompt64)]
    assert emitted[0] == ref["first"]
    branched = 0
    for r, rr in enumerate(ref["rounds"]):
        e = len(emitted)
        tpl = templates[r % len(templates)]
        toks = [emitted[-1]] + [(A[e + o] + dl) % V for _, o, dl in tpl]
        pars = [-1] + [p for p, _, _ in tpl]
        assert toks == rr["tokens"] and pars == rr["parents"]
        dec.set_forced_tree(toks, pars)
        acc = dec.tree_round(4, 2, 8)
        assert acc[:-1] == [rr["tokens"][v] for v in rr["path"]], r
        assert acc[-1] == rr["next"], r
        nodes = dec.tree_nodes()
        assert nodes["tokens"][1:] == toks[1:] and nodes["parents"] == pars
        assert nodes["proposals"] == rr["proposals"], r
        drafted = [i for i, x in enumerate(rr["proposals"]) if x >= 0]
        np.testing.assert_allclose([nodes["proposal_logits"][i] for i in drafted],
                                   [rr["proposal_logits"][i] for i in drafted], rtol=0, atol=1e-4)
        assert dec.state() == (rr["n"], rr["drafter_len"]), r
        branched += any(p not in (-1, i - 1) for i, p in enumerate(rr["parents"])) and len(rr["path"]) > 1
        emitted.extend(acc[: g["max_new"] - len(emitted)])
    dec.set_forced_tree(None)
    assert emitted == ref["tokens"]
    assert branched >= 4


def test_sampled_tree_follows_the_oracle_on_one_philox_stream(tiny_models, c1_models, prompt64):
    from woodcock_b200 import SamplingParams, SpeculativeDecoder, StaticPolicy

    td, dd, _, _ = tiny_models["c1u"]
    t, d = c1_models["c1u"]
    sp = SamplingParams(temperature=0.8, seed=5)
    out, st = SpeculativeDecoder(t, d, StaticPolicy(2, 2, 4), max_context=512).generate(prompt64, 24, sp,
                                                                                         stop_on_eos=False)
    to = O.Qwen3.load(td, taps=[1, 2, 3])
    do = O.Drafter.load(dd)
    ref, rst = O.SpeculativeDecoder(to, do, O.StaticPolicy(2, 2, 4)).generate(
        prompt64, 24, O.SamplingParams(temperature=0.8, seed=5), stop_on_eos=False, rng=O.Tape(5))
    assert out == ref
    assert st.accepted == rst.accepted


def test_policy_with_host_hooks_runs_synced_rounds(golden, c1_models, prompt64):
    """A policy that is not a StaticPolicy (its hooks may need the host between levels) takes the
    host-driven rounds; with the static tree:3,3,8 rules it reproduces the reference's run."""
    from woodcock_b200 import Policy, SpeculativeDecoder, StaticPolicy

    class HookedTree(Policy):
        def __init__(self):
            self.inner = StaticPolicy(3, 3, 8)
            self.seen = 0

        def plan(self, context_len, stochastic):
            return self.inner.plan(context_len, stochastic)

        def select_verify(self, nodes, context_len, stochastic):
            self.seen += 1
            return self.inner.select_verify(nodes, context_len, stochastic)

    g = golden("c1u")
    t, d = c1_models["c1u"]
    pol = HookedTree()
    out, st = SpeculativeDecoder(t, d, pol, max_context=512).generate(prompt64, 64)
    assert out == g["spec_tree:3,3,8"]["tokens"][:64]
    assert not st.fused and pol.seen == st.rounds
