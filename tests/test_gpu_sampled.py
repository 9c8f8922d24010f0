"""Sampled decoding on the device (temperature > 0): the chain round (spec.py:216-324 on a
chain; sampling.py:39-55, 69-82, 143-203) and the autoregressive baseline (spec.py:377-397).

(a) Tape parity: every round's draft draws, accept length and emitted token equal the
    oracle's (wc_oracle.gumbel_draw / sampled_chain_accept) on that round's own logits with
    the same Philox counters; the prefill's first token likewise.
(b) Law: the first emitted token of rounds replayed from one state follows
    p_0 = softmax(z_0 / T): Pearson chi-square of 1e5 draws in 1000 equal-mass bins, the bins
    taken over consecutive token ids and, separately, over tokens in decreasing order of p (a
    bias that follows the logit collects in the first or last rank bins), must not reject
    (p > 1e-3), while the oracle with a planted mistake (rejections drawn from p instead of the
    residual) on the same p and q must be rejected under both binnings (p < 1e-6). The draft
    vocabulary is restricted, so q is zero on most tokens and those are reached only through
    the residual.
(c) The autoregressive baseline's sampled first token follows p over many seeds, and a seed
    reproduces its stream.
(d) top-k / top-p warping of the target: tape parity of the first token and of the rounds
    with the oracle's threshold rule, and the first-token law of the warped distribution.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import wc_oracle as O

pytestmark = pytest.mark.gpu

T_TAPE = 0.8
T_LAW = 1.0  # C4: T = 1.0
N_LAW = 100_000
HEAD_IDS = np.sort(np.random.default_rng(11).choice(4096, 1024, replace=False)).tolist()


@pytest.fixture(scope="module")
def pair(tiny_models):
    from woodcock_b200 import Drafter, Target

    td, dd, _, _ = tiny_models["c1u"]
    t = Target.load(td, feature_layers=[1, 2, 3], dtype="fp32")
    d_full = Drafter.load(dd, dtype="fp32")
    d_trim = Drafter.load(dd, dtype="fp32")
    d_trim.restrict_vocab(HEAD_IDS)
    return t, d_full, d_trim


def _decoder(t, d, k):
    from woodcock_b200 import SpeculativeDecoder, StaticPolicy

    return SpeculativeDecoder(t, d, StaticPolicy(k), max_context=512, max_k=8)


@pytest.mark.parametrize("trim", [False, True])
def test_sampled_rounds_match_oracle_tape(pair, prompt64, trim):
    from woodcock_b200 import SamplingParams

    t, d_full, d_trim = pair
    d = d_trim if trim else d_full
    ids = np.asarray(HEAD_IDS) if trim else None
    k = 4
    dec = _decoder(t, d, k)
    sp = SamplingParams(temperature=T_TAPE, seed=1234)
    first = dec.prefill(prompt64, sp)
    # the first token: a draw from the last prompt row's softmax with counter base 0, stream 0
    z = t(torch.tensor(prompt64, dtype=torch.int32, device="cuda"), t.make_cache(512),
          logits_from=len(prompt64) - 1).logits.float().reshape(-1).cpu().numpy()
    assert first == O.gumbel_draw(z, T_TAPE, 1234, 0, 0)
    seen_a = set()
    for r in range(40):
        toks = dec.round(k)
        g = dec.round_logits(k)
        assert g["seed"] == 1234 and g["base"] == (r + 1) * O.RNG_ROUND_STRIDE
        for i in range(k):  # draft d_{i+1}: the Gumbel-max row of draft step i, mapped to its id
            row = O.gumbel_draw(g["zd"][i], T_TAPE, 1234, g["base"], i)
            assert g["tokens"][i + 1] == (int(ids[row]) if trim else row), (r, i)
        a, nxt = O.sampled_chain_accept(g["zt"], g["zd"], g["tokens"], T_TAPE, 1234, g["base"], vocab_ids=ids)
        assert toks == g["tokens"][1:a + 1] + [nxt], (r, toks, a, nxt)
        seen_a.add(a)
    assert 0 in seen_a and len(seen_a) > 1, seen_a  # both rejections and acceptances were exercised


def test_sampled_first_token_law_chi_square(pair, prompt64):
    from woodcock_b200 import SamplingParams

    t, _, d = pair
    k = 4
    dec = _decoder(t, d, k)
    dec.prefill(prompt64, SamplingParams(temperature=T_LAW, seed=7))
    dec.save_state()
    V = t.cfg.vocab
    counts = np.zeros(V)
    z0 = None
    for i in range(N_LAW):
        dec.restore_state()
        counts[dec.round(k)[0]] += 1
        if i in (0, N_LAW - 1):
            g = dec.round_logits(k)
            if z0 is None:
                z0, zd0 = g["zt"][0].copy(), g["zd"][0].copy()
            else:  # the replayed state gives the same target row every time
                np.testing.assert_array_equal(g["zt"][0], z0)
    x = (z0 / np.float32(T_LAW)).astype(np.float64)
    p = np.exp(x - x.max())
    p /= p.sum()
    for order in ("id", "rank"):
        stat, dof, pval = O.chi2_equal_mass(counts, p, order=order)
        assert pval > 1e-3, (order, stat, dof, pval)

    # the same test on the oracle's draws from this p and q: correct rule passes, the planted
    # mistake (no residual) fails
    xq = (zd0 / np.float32(T_LAW)).astype(np.float64)
    qd = np.exp(xq - xq.max())
    qd /= qd.sum()
    q = np.zeros(V)
    q[np.asarray(HEAD_IDS)] = qd
    rng = np.random.default_rng(3)
    drafts = rng.choice(V, N_LAW, p=q)
    accept = rng.random(N_LAW) < np.minimum(1.0, p[drafts] / q[drafts])
    r = np.maximum(p - q, 0.0)
    good = np.where(accept, drafts, rng.choice(V, N_LAW, p=r / r.sum()))
    bad = np.where(accept, drafts, rng.choice(V, N_LAW, p=p))
    for order in ("id", "rank"):
        assert O.chi2_equal_mass(np.bincount(good, minlength=V).astype(float), p, order=order)[2] > 1e-3
        assert O.chi2_equal_mass(np.bincount(bad, minlength=V).astype(float), p, order=order)[2] < 1e-6


def test_sampled_generate_runs_and_reproduces(pair, prompt64):
    from woodcock_b200 import SamplingParams

    t, _, d = pair
    sp = SamplingParams(temperature=T_LAW, seed=99)
    out1, st1 = _decoder(t, d, 4).generate(prompt64, 96, sp, stop_on_eos=False)
    out2, _ = _decoder(t, d, 4).generate(prompt64, 96, sp, stop_on_eos=False)
    assert out1 == out2 and len(out1) == 96
    assert st1.rounds > 0 and 0 < sum(st1.accepted) < 4 * st1.rounds
    out3, _ = _decoder(t, d, 4).generate(prompt64, 96, SamplingParams(temperature=T_LAW, seed=100),
                                         stop_on_eos=False)
    assert out3 != out1


def test_sampled_autoregressive_first_token_law(pair, prompt64):
    from woodcock_b200 import SamplingParams
    from woodcock_b200.spec import generate_autoregressive

    t, _, _ = pair
    prompt = prompt64[:16]
    z = t(torch.tensor(prompt, dtype=torch.int32, device="cuda"), t.make_cache(64),
          logits_from=len(prompt) - 1).logits.float().reshape(-1).cpu().numpy()
    x = (z / np.float32(T_LAW)).astype(np.float64)
    p = np.exp(x - x.max())
    p /= p.sum()
    n = 3000
    counts = np.zeros(t.cfg.vocab)
    for seed in range(n):
        out, _ = generate_autoregressive(t, prompt, 1, SamplingParams(temperature=T_LAW, seed=seed),
                                         stop_on_eos=False, max_context=64)
        if seed < 4:
            assert out[0] == O.gumbel_draw(z, T_LAW, seed, 0, 0)
        counts[out[0]] += 1
    for order in ("id", "rank"):
        assert O.chi2_equal_mass(counts, p, bins=60, order=order)[2] > 1e-3
    a, _ = generate_autoregressive(t, prompt, 24, SamplingParams(temperature=T_LAW, seed=5), stop_on_eos=False)
    b, _ = generate_autoregressive(t, prompt, 24, SamplingParams(temperature=T_LAW, seed=5), stop_on_eos=False)
    assert a == b


WARPS = [(20, 1.0), (0, 0.8), (40, 0.9)]


@pytest.mark.parametrize("top_k,top_p", WARPS)
def test_warped_rounds_match_oracle_tape(pair, prompt64, top_k, top_p):
    """top-k / top-p on the target distribution (sampling.py:39-55): the first token and every
    round's decisions and draws equal the oracle's threshold rule on the same logits."""
    from woodcock_b200 import SamplingParams

    t, _, d = pair
    ids = np.asarray(HEAD_IDS)
    k = 4
    dec = _decoder(t, d, k)
    first = dec.prefill(prompt64, SamplingParams(temperature=T_TAPE, top_k=top_k, top_p=top_p, seed=77))
    z = t(torch.tensor(prompt64, dtype=torch.int32, device="cuda"), t.make_cache(512),
          logits_from=len(prompt64) - 1).logits.float().reshape(-1).cpu().numpy()
    assert first == O.gumbel_draw_warped(z, T_TAPE, top_k, top_p, 77, 0, 0)
    for r in range(25):
        toks = dec.round(k)
        g = dec.round_logits(k)
        a, nxt = O.sampled_chain_accept(g["zt"], g["zd"], g["tokens"], T_TAPE, 77, g["base"], vocab_ids=ids,
                                        top_k=top_k, top_p=top_p)
        assert toks == g["tokens"][1:a + 1] + [nxt], (r, toks, a, nxt)


def test_warped_first_token_law_chi_square(pair, prompt64):
    from woodcock_b200 import SamplingParams

    t, _, d = pair
    k, n = 4, 20_000
    top_k, top_p = 50, 0.9
    dec = _decoder(t, d, k)
    dec.prefill(prompt64, SamplingParams(temperature=T_LAW, top_k=top_k, top_p=top_p, seed=8))
    dec.save_state()
    counts = np.zeros(t.cfg.vocab)
    for i in range(n):
        dec.restore_state()
        counts[dec.round(k)[0]] += 1
        if i == 0:
            z0 = dec.round_logits(k)["zt"][0].copy()
    p = O.warped_probs(z0, T_LAW, top_k, top_p)
    assert counts[p == 0].sum() == 0  # nothing outside the kept set is ever emitted
    for order in ("id", "rank"):
        stat, dof, pval = O.chi2_equal_mass(counts, p, bins=1000, order=order)
        assert dof >= 5 and pval > 1e-3, (order, stat, dof, pval)


def test_invalid_warping_is_refused(pair, prompt64):
    from woodcock_b200 import SamplingParams

    t, _, d = pair
    dec = _decoder(t, d, 2)
    with pytest.raises(Exception, match="top_p"):
        dec.prefill(prompt64, SamplingParams(temperature=1.0, top_p=0.0))
    with pytest.raises(Exception, match="top_k"):
        dec.prefill(prompt64, SamplingParams(temperature=1.0, top_k=-1))
