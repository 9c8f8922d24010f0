"""Host-side logic without a GPU: policies (restating tests/test_policies.py), draft trees and
masks, the host-driven sampled tree's draws, safetensors I/O, and the seeded synthetic
configs."""

from __future__ import annotations

import numpy as np
import pytest

from woodcock_b200 import synthetic as syn
from woodcock_b200.policies import CostAwareChain, StaticPolicy
from woodcock_b200.sampling import DraftTree, SamplingParams, tree_attention_mask
from woodcock_b200 import safetensors_io as st


def leviathan_factor(alpha, gamma, c):
    """arXiv:2211.17192 Thm 3.8."""
    return (1 - alpha ** (gamma + 1)) / ((1 - alpha) * (gamma * c + 1))


@pytest.mark.parametrize("alpha", [0.3, 0.6, 0.8, 0.9])
@pytest.mark.parametrize("c", [0.02, 0.1, 0.3])
def test_cost_aware_chain_reduces_to_leviathan(alpha, c):
    pol = CostAwareChain(step_ms=c, head_ms=c, verify_ms={n: 1.0 for n in range(1, 10)}, k_max=8)
    best = max(range(1, 9), key=lambda g: (leviathan_factor(alpha, g, c), -g))
    assert pol.best_depth(alpha) == best


def test_cost_aware_chain_monotonic():
    v = {n: 10.0 + 0.2 * n for n in range(1, 10)}
    pol = CostAwareChain(step_ms=1.5, head_ms=1.1, verify_ms=v)
    cheap = CostAwareChain(step_ms=0.5, head_ms=0.1, verify_ms=v)
    assert pol.best_depth(0.4) < pol.best_depth(0.8)
    assert pol.best_depth(0.7) < cheap.best_depth(0.7)


def test_cost_aware_chain_alpha_estimate_and_limits():
    """Successes and first failures with exponential forgetting over a prior."""
    pol = CostAwareChain(1.0, 0.5, {n: 10.0 for n in range(1, 10)}, alpha0=0.5, prior=2.0, window=4)
    assert pol.alpha() == pytest.approx(0.5)
    pol.observe(4, 4, 4, 0, 0)  # all accepted: 4 successes, no failure
    assert pol.alpha() == pytest.approx(4.75 / 5.5)
    pol.observe(1, 4, 4, 0, 0)  # one success, then the first rejection
    assert pol.alpha() == pytest.approx(4.5625 / (4.5625 + 1.5625))
    for _ in range(60):
        pol.observe(0, 2, 2, 0, 0)
    assert pol.alpha() == pytest.approx(0.01)  # clamped
    pol.reset()
    assert pol.alpha() == pytest.approx(0.5)
    lim = CostAwareChain(0.1, 0.05, {n: 1.0 for n in range(1, 5)}, k_max=8)
    assert lim.k_max == 3 and lim.best_depth(0.99) == 3


def test_cost_aware_chain_from_measured_round_times():
    """A cost file with this package's measured round times: T(k) = round_ms[k] directly."""
    rm = {1: 1.0, 2: 1.1, 3: 1.2, 4: 1.3, 5: 1.4, 6: 1.5}
    costs = {"ctx": 512, "drafter": {"16384": {"head_ms": 0.02, "step_ms": 0.09}},
             "verify_ms": {str(n): 1.0 for n in range(1, 10)}, "round_ms": {"16384": {str(k): v for k, v in rm.items()}}}
    pol = CostAwareChain.from_costs(costs, "16384")
    assert pol.k_max == 6
    for a in (0.2, 0.5, 0.8, 0.95):
        want = max(rm, key=lambda k: ((1 - a ** (k + 1)) / (1 - a) / rm[k], -k))
        assert pol.best_depth(a) == want
    assert pol.best_depth(0.05) == 1 and pol.best_depth(0.99) == 6
    with pytest.raises(ValueError):
        CostAwareChain()


def test_static_policy_budget_and_plan():
    assert StaticPolicy(4).budget == 4 and StaticPolicy(3, 3).budget == 12
    p = StaticPolicy(3, 2, 3).plan(10, True)
    assert [p.children_for(1.0, d) for d in range(3)] == [2, 1, 0]


def test_draft_tree_and_mask_known_answer():
    tree = DraftTree(tokens=[0, 1, 2, 4], parents=[-1, 0, 0, 2], depth=[0, 1, 1, 2])
    assert tree.children == [[1, 2], [], [3], []]
    assert tree.path_to(3) == [2, 3] and not tree.is_chain()
    m = tree_attention_mask(tree, 2)
    assert m.shape == (4, 6) and m[:, :2].all()
    assert list(m[3, 2:]) == [True, False, True, True]
    assert list(m[1, 2:]) == [True, True, False, False]
    assert SamplingParams().greedy and not SamplingParams(temperature=0.7).greedy


def test_synced_tree_draws_match_the_reference_rules(golden):
    """The host-driven sampled tree's two draws read the Philox stream exactly as the reference
    reads its Generator: a node's children by Gumbel-top-k (synced.gumbel_top_k) against the
    reference's own sample_without_replacement outputs (python/woodcock/sampling.py:196-203,
    fixture made from it), and the inverse-CDF draw (synced.inverse_cdf_draw) against the
    reference's _sample rule (sampling.py:190-193, as the oracle restates it)."""
    import wc_oracle as O
    from woodcock_b200.synced import gumbel_top_k, inverse_cdf_draw

    cases = golden("sampling")["gumbel"]
    assert cases
    for c in cases:
        tape = O.Tape(c["seed"])
        assert gumbel_top_k(np.array(c["q"]), c["k"], tape) == c["out"]
        assert tape.pos == c["uniforms_used"]
    rng = np.random.default_rng(3)
    for trial in range(64):
        p = rng.random(40) * (rng.random(40) < 0.6)
        p[trial % 40] += 0.01  # at least one positive entry
        a, b = O.Tape(trial, 5), O.Tape(trial, 5)
        assert inverse_cdf_draw(p, a) == O.sample(p, b)
        assert a.pos == b.pos == 6
    assert gumbel_top_k(np.zeros(8), 3, O.Tape(0)) == []  # nothing to draw from


def test_safetensors_roundtrip_and_bf16_rounding(tmp_path):
    rng = np.random.default_rng(0)
    a = rng.standard_normal((3, 5)).astype(np.float32)
    b = st.f32_to_bf16_bits(a)
    st.save(tmp_path / "x.safetensors", {"a": ("F32", a), "b": ("BF16", b)}, metadata={"format": "pt"})
    r = st.load(tmp_path / "x.safetensors")
    np.testing.assert_array_equal(st.to_f32(r["a"]), a)
    bf = st.to_f32(r["b"])
    assert np.all(np.abs(bf - a) <= np.abs(a) * 2.0 ** -8)
    # round-to-nearest-even on a tie
    assert st.f32_to_bf16_bits(np.array([1.0 + 2.0 ** -8], np.float32))[0] == 0x3F80


def test_synthetic_configs_are_seeded_and_shaped():
    w1 = syn.generate_weights(syn.target_tensor_specs(syn.TINY_TARGET), seed=0)
    w2 = syn.generate_weights(syn.target_tensor_specs(syn.TINY_TARGET), seed=0)
    assert all(np.array_equal(w1[k], w2[k]) for k in w1)
    assert w1["model.embed_tokens.weight"].shape == (4096, 256)
    assert "lm_head.weight" not in w1  # tied
    assert abs(float(w1["model.layers.0.mlp.up_proj.weight"].std()) - 0.02) < 1e-3
    ids = syn.trimmed_vocab_ids(151936, 16384, seed=0)
    assert len(ids) == 16384 and np.all(np.diff(ids) > 0) and {151643, 151645} <= set(ids.tolist())
    specs = dict((n, s) for n, s, _ in syn.drafter_tensor_specs(syn.Q17_DRAFTER))
    assert specs["fc.weight"] == (2048, 6144) and specs["layers.0.self_attn.aux_q.weight"] == (2048, 2048)


def test_bytes_per_round_model():
    """The algorithmic-bytes model used for the roofline (bf16 C3, k=4, ctx ~640)."""
    from woodcock_b200.roofline import round_bytes

    b = round_bytes(syn.Q17_TARGET, syn.Q17_DRAFTER, k=4, head_rows=16384, ctx=640)
    assert 4.1e9 < b["total"] < 4.4e9
    assert b["target_weights"] == pytest.approx(3.441e9, rel=0.01)
