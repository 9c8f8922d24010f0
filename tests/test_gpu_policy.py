"""The cost-aware chain (python/woodcock/policies.py CostAwareChain's role) driving the device
round: the chain length is chosen before every round from the acceptance estimate, so one
generate() call replays round graphs of several lengths. Forced drafts make the acceptance
swing (runs of fully accepted chains, then runs of rejected first drafts), which must move the
chosen length up and down; the output stays the greedy continuation throughout."""

from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu


def test_cost_aware_chain_changes_k_inside_generate(golden, tiny_models, prompt64):
    from woodcock_b200 import CostAwareChain, Drafter, SpeculativeDecoder, Target

    td, dd, _, _ = tiny_models["c1u"]
    t = Target.load(td, feature_layers=[1, 2, 3], dtype="fp32")
    d = Drafter.load(dd, dtype="fp32")
    ar = golden("c1u")["ar_tokens"]
    # round time grows with k: short chains win at low acceptance, long ones at high acceptance
    pol = CostAwareChain(round_ms={k: 1.0 + 0.25 * k for k in range(1, 9)}, k_max=8, alpha0=0.5, prior=2.0,
                         window=4)
    dec = SpeculativeDecoder(t, d, pol, max_context=512, max_k=8)

    def forced(r, k, emitted):
        toks = [ar[min(emitted + j, len(ar) - 1)] for j in range(k)]
        if (r // 6) % 2 == 1:  # every other run of six rounds rejects the first draft
            toks[0] = (toks[0] + 1) % t.cfg.vocab
        return toks

    dec.forced = forced
    out, st = dec.generate(prompt64, 120, stop_on_eos=False)
    assert out == ar[:120]
    assert st.drafted == pol.chosen[: st.rounds]
    assert len(set(pol.chosen)) >= 3, pol.chosen
    hi = max(pol.chosen)
    assert hi >= 6 and min(pol.chosen[6:]) <= 2, pol.chosen
    # the accepted counts follow the forced pattern: all drafts in accepting runs, none otherwise
    for r, (a, k) in enumerate(zip(st.accepted, st.drafted)):
        assert a == (0 if (r // 6) % 2 == 1 else k), (r, a, k)
