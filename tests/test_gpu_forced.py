"""The device round in oracle-drafter mode against the reference itself.

tests/golden/c1u_forced.json was made by the reference's C++ core (`wc_ref_driver forced`,
built from the reference's sources) on the C1u pair: drafts forced from its own greedy
continuation with a cycle of accept lengths (chains of 4 and 6) and branching draft trees.
Each round of the device path must reproduce the reference's round: accepted path, next token,
committed and drafter cache lengths, and the drafter's own head proposals with their logits
(these depend on the previous round's multi-row drafter update and on the chain steps'
drafter passes, which the forced tokens otherwise hide).
"""

from __future__ import annotations

import numpy as np
import pytest

import wc_oracle as O

pytestmark = pytest.mark.gpu

FP32_LOGIT_ATOL = 1e-4  # fp32 device path vs the reference's fp32 loops: summation order only


@pytest.fixture(scope="module")
def c1u_pair(tiny_models):
    from woodcock_b200 import Drafter, Target

    td, dd, _, _ = tiny_models["c1u"]
    return Target.load(td, feature_layers=[1, 2, 3], dtype="fp32"), Drafter.load(dd, dtype="fp32")


@pytest.mark.parametrize("name,K", [("chain4", 4), ("chain6", 6)])
def test_forced_chain_rounds_match_reference(name, K, golden, c1u_pair, prompt64):
    from woodcock_b200 import SpeculativeDecoder, StaticPolicy

    g = golden("c1u_forced")
    ref = g[name]
    t, d = c1u_pair
    V = t.cfg.vocab
    A = ref["ar"]
    templates = [O.parse_template(x) for x in ref["templates"]]
    dec = SpeculativeDecoder(t, d, StaticPolicy(K), max_context=512, max_k=8)
    emitted = [dec.prefill(prompt64)]
    assert emitted[0] == ref["first"]
    partial = 0
    for r, rr in enumerate(ref["rounds"]):
        e = len(emitted)
        drafts = [(A[e + o] + dl) % V for _, o, dl in templates[r % len(templates)]]
        assert [emitted[-1]] + drafts == rr["tokens"]
        dec.set_forced(drafts)
        acc = dec.round(K)
        assert acc[:-1] == [rr["tokens"][v] for v in rr["path"]], r
        assert acc[-1] == rr["next"], r
        props, z = dec.draft_proposals(K)
        assert props == rr["proposals"][:K], r
        np.testing.assert_allclose(z, rr["proposal_logits"][:K], rtol=0, atol=FP32_LOGIT_ATOL)
        assert dec.state() == (rr["n"], rr["drafter_len"]), r
        partial += 0 < len(rr["path"]) < K
        emitted.extend(acc[: g["max_new"] - len(emitted)])
    assert emitted == ref["tokens"]
    assert partial >= 5


def test_forced_generate_matches_reference_counts(golden, c1u_pair, prompt64):
    """The same forced chain through SpeculativeDecoder.generate (the public loop): the output and
    the accepted count per round equal the reference's."""
    from woodcock_b200 import SpeculativeDecoder, StaticPolicy

    g = golden("c1u_forced")
    ref = g["chain4"]
    t, d = c1u_pair
    A, V = ref["ar"], t.cfg.vocab
    templates = [O.parse_template(x) for x in ref["templates"]]
    dec = SpeculativeDecoder(t, d, StaticPolicy(4), max_context=512, max_k=8)
    dec.forced = lambda r, k, e: [(A[e + o] + dl) % V for _, o, dl in templates[r % len(templates)]]
    out, st = dec.generate(prompt64, g["max_new"], stop_on_eos=False)
    assert out == ref["tokens"]
    assert st.accepted == [len(x["path"]) for x in ref["rounds"]]
