"""Draft trees and the synced path (host-driven rounds over the device API; spec.py:216-374).

(a) Greedy top-k trees (StaticPolicy(3, 3, 8)) on C1 fp32: tokens equal the reference C++
    core's tree:3,3,8 run and autoregressive decoding, and the accepted total equals the
    reference's (tests/golden/c1*.json), so the tree shapes agree round by round.
(b) fused=False on a chain: the synced path gives the autoregressive tokens.
(c) Sampled trees: the same Philox stream drives the oracle's restatement of the reference
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
    assert not st.fused and st.rounds == len(st.accepted) and max(st.depths) <= 3


def test_synced_chain_equals_autoregressive(golden, c1_models, prompt64):
    from woodcock_b200 import SpeculativeDecoder, StaticPolicy

    t, d = c1_models["c1u"]
    out, st = SpeculativeDecoder(t, d, StaticPolicy(4), fused=False, max_context=512).generate(prompt64, 64)
    assert out == golden("c1u")["ar_tokens"][:64]
    assert not st.fused


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
