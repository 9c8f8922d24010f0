"""Edge cases of the decode path on the device (the reference's spec tests exercise the same
situations: tests/test_spec_model.py, tests/cpp/test_main.cpp):

* a one-token prompt (the drafter prefill then holds only the first generated token);
* max_new_tokens = 1 (the prefill's token, no round);
* stopping on an end-of-sequence id inside a round's accepted tokens, chain and tree paths;
* an exhausted context is an error, not a fault, and the decoder stays usable;
* bad token ids and chain lengths are refused;
* a near-zero temperature reproduces greedy decoding through the sampled round.
"""

from __future__ import annotations

import pytest
import torch

import wc_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def c1u(tiny_models):
    from woodcock_b200 import Drafter, Target

    td, dd, _, _ = tiny_models["c1u"]
    return Target.load(td, feature_layers=[1, 2, 3], dtype="fp32"), Drafter.load(dd, dtype="fp32"), td


def _ar(td, prompt, n):
    return O.generate_autoregressive(O.Qwen3.load(td, taps=[1, 2, 3]), prompt, n, stop_on_eos=False)


def test_one_token_prompt_and_single_new_token(c1u):
    from woodcock_b200 import SpeculativeDecoder, StaticPolicy

    t, d, td = c1u
    prompt = [1234]
    ar = _ar(td, prompt, 20)
    dec = SpeculativeDecoder(t, d, StaticPolicy(4), max_context=128)
    out, st = dec.generate(prompt, 20, stop_on_eos=False)
    assert out == ar
    out1, st1 = dec.generate(prompt, 1, stop_on_eos=False)
    assert out1 == ar[:1] and st1.rounds == 0


@pytest.mark.parametrize("policy", ["chain", "tree"])
def test_stop_on_eos_inside_a_round(c1u, golden, prompt64, policy):
    from woodcock_b200 import SpeculativeDecoder, StaticPolicy

    t, d, td = c1u
    ar = golden("c1u")["ar_tokens"]
    stop = ar[9]
    first = ar.index(stop)
    pol = StaticPolicy(4) if policy == "chain" else StaticPolicy(3, 3, 8)
    dec = SpeculativeDecoder(t, d, pol, max_context=512)
    saved = t.eos_token_ids
    t.eos_token_ids = {stop}
    try:
        dec.forced = None
        out, _ = dec.generate(prompt64, 64)
    finally:
        t.eos_token_ids = saved
    assert out == ar[: first + 1]  # generation ends with the end-of-sequence token


def test_context_exhaustion_is_an_error_and_the_decoder_recovers(c1u, prompt64):
    from woodcock_b200 import SpeculativeDecoder, StaticPolicy

    t, d, td = c1u
    dec = SpeculativeDecoder(t, d, StaticPolicy(4), max_context=80, max_k=4)
    with pytest.raises(RuntimeError, match="exhausted|capacity"):
        dec.generate(prompt64, 64, stop_on_eos=False)
    out, _ = dec.generate(prompt64[:16], 8, stop_on_eos=False)  # a fresh prefill still works
    assert out == _ar(td, prompt64[:16], 8)


def test_bad_inputs_are_refused(c1u, prompt64):
    from woodcock_b200 import SpeculativeDecoder, StaticPolicy

    t, d, _ = c1u
    dec = SpeculativeDecoder(t, d, StaticPolicy(4), max_context=256, max_k=4)
    with pytest.raises(ValueError):
        dec.prefill([5, 4096, 7])  # outside the 4096-token vocabulary
    with pytest.raises(ValueError):
        dec.prefill([])
    dec.prefill(prompt64)
    with pytest.raises(ValueError):
        dec.round(5)  # above max_k
    with pytest.raises(ValueError):
        dec.round(0)
    assert len(dec.round(4)) >= 1  # still usable


def test_tiny_temperature_reproduces_greedy(c1u, golden, prompt64):
    from woodcock_b200 import SamplingParams, SpeculativeDecoder, StaticPolicy

    t, d, _ = c1u
    dec = SpeculativeDecoder(t, d, StaticPolicy(4), max_context=512)
    out, _ = dec.generate(prompt64, 48, SamplingParams(temperature=1e-4, seed=3), stop_on_eos=False)
    assert out == golden("c1u")["ar_tokens"][:48]
