"""Parity of the CUDA model path with the reference (C1 fixtures made by the reference's C++
core) and with the oracle restatement: target forward, taps, drafter fuse/forward/head,
autoregressive greedy, and the fused speculative round (chain, forced drafts)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import wc_oracle as O

pytestmark = pytest.mark.gpu

FP32_LOGIT_ATOL = 1e-4  # fp32 path vs the reference: summation order only


@pytest.fixture(scope="module")
def gpu_models(tiny_models):
    from woodcock_b200 import Drafter, Target

    out = {}
    for name, (td, dd, tw, dw) in tiny_models.items():
        out[name] = (Target.load(td, feature_layers=[1, 2, 3], dtype="fp32"), Drafter.load(dd, dtype="fp32"))
    return out


@pytest.mark.parametrize("name", ["c1", "c1u"])
def test_target_forward_matches_reference(name, golden, gpu_models, prompt64):
    g = golden(name)
    t, _ = gpu_models[name]
    cache = t.make_cache(256)
    o = t(prompt64, cache, logits_from=len(prompt64) - 1)
    z = o.logits[0, -1].cpu().numpy()
    np.testing.assert_allclose(z, np.array(g["last_logits"], np.float32), rtol=0, atol=FP32_LOGIT_ATOL)
    assert int(o.argmax[-1]) == g["argmax"]
    for f in range(3):
        np.testing.assert_allclose(o.features[f][0, -1, :8].cpu().numpy(), g["taps_last_head8"][f], atol=1e-5)
    assert cache.size() == len(prompt64)


@pytest.mark.parametrize("name", ["c1", "c1u"])
def test_autoregressive_matches_reference(name, golden, gpu_models, prompt64):
    from woodcock_b200 import generate_autoregressive

    t, _ = gpu_models[name]
    out, st = generate_autoregressive(t, prompt64, 128)
    assert out == golden(name)["ar_tokens"]
    assert st.new_tokens == 128


@pytest.mark.parametrize("name", ["c1", "c1u"])
def test_speculative_chain4_matches_reference(name, golden, gpu_models, prompt64):
    from woodcock_b200 import SpeculativeDecoder, StaticPolicy

    t, d = gpu_models[name]
    g = golden(name)
    dec = SpeculativeDecoder(t, d, StaticPolicy(4), max_context=512)
    out, st = dec.generate(prompt64, 128)
    assert out == g["spec_chain:4"]["tokens"] == g["ar_tokens"]
    assert sum(st.accepted) == g["spec_chain:4"]["accepted"]
    assert st.rounds == g["spec_chain:4"]["rounds"]
    n, dl = dec.state()
    assert dl == n  # drafter holds one real entry per committed token


@pytest.mark.parametrize("K", [1, 3, 6])
def test_chain_lengths_equal_autoregressive(K, golden, gpu_models, prompt64):
    from woodcock_b200 import SpeculativeDecoder, StaticPolicy

    t, d = gpu_models["c1u"]
    out, _ = SpeculativeDecoder(t, d, StaticPolicy(K), max_context=512, max_k=8).generate(prompt64, 64)
    assert out == golden("c1u")["ar_tokens"][:64]


def forced_from_ar(ar, corrupt_every=4, vocab=4096):
    def forced(r, k, emitted):
        toks = [ar[min(emitted + j, len(ar) - 1)] for j in range(k)]
        if corrupt_every and r % corrupt_every == corrupt_every - 1 and k > 2:
            toks[2] = (toks[2] + 1) % vocab
        return toks

    return forced


@pytest.mark.parametrize("K", [4, 6])
def test_forced_drafts_partial_acceptance_matches_oracle(K, golden, tiny_models, gpu_models, prompt64):
    """Oracle-drafter mode: accepted counts per round and the output equal the oracle's, and
    the output equals autoregressive greedy; exercises the update on a+1 rows."""
    from woodcock_b200 import SpeculativeDecoder, StaticPolicy

    ar = golden("c1u")["ar_tokens"]
    t, d = gpu_models["c1u"]
    dec = SpeculativeDecoder(t, d, StaticPolicy(K), max_context=512, max_k=8)
    dec.forced = forced_from_ar(ar)
    out, st = dec.generate(prompt64, 96)
    td, dd, _, _ = tiny_models["c1u"]
    ot, od = O.Qwen3.load(td, taps=[1, 2, 3]), O.Drafter.load(dd)
    oout, ost = O.SpeculativeDecoder(ot, od, O.StaticPolicy(K)).generate(prompt64, 96, forced=forced_from_ar(ar))
    assert out == oout == ar[:96]
    assert st.accepted == ost.accepted
    assert sum(st.accepted) > 30


def test_drafter_pieces_match_oracle(tiny_models, gpu_models):
    """fuse, forward (with the aux embedding stream), logits and restrict_vocab vs the oracle."""
    td, dd, _, dw = tiny_models["c1u"]
    _, d = gpu_models["c1u"]
    od = O.Drafter.load(dd)
    rng = np.random.default_rng(3)
    L = 5
    taps = [rng.standard_normal((L, 256)).astype(np.float32) for _ in range(3)]
    g_ref = od.fuse(taps)
    g = d.fuse([torch.tensor(x, device="cuda")[None] for x in taps])[0].cpu().numpy()
    np.testing.assert_allclose(g, g_ref, rtol=1e-4, atol=1e-5)
    toks = rng.integers(0, 4096, L).tolist()
    oc = od.make_cache()
    h_ref, out_ref = od.forward(toks, g_ref, oc)
    cache = d.make_cache(64)
    h, out = d(toks, torch.tensor(g_ref, device="cuda")[None], cache)
    np.testing.assert_allclose(h[0].cpu().numpy(), h_ref, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(out[0].cpu().numpy(), out_ref, rtol=1e-4, atol=1e-4)
    z = d.logits(out)[0].cpu().numpy()
    np.testing.assert_allclose(z, od.logits(out_ref), rtol=1e-4, atol=1e-5)
    assert d.head_argmax(out).cpu().tolist() == [O.argmax(r) for r in od.logits(out_ref)]


@pytest.mark.parametrize("T", [1.0, 0.7])
def test_drafter_head_softmax_is_the_draft_distribution(tiny_models, T):
    """wc_drafter_head_softmax: softmax(z / T) of the head rows, full and restricted heads."""
    from woodcock_b200 import Drafter

    td, dd, _, _ = tiny_models["c1u"]
    d = Drafter.load(dd, dtype="fp32")
    out = torch.randn((5, 256), device="cuda")
    for restrict in (False, True):
        if restrict:
            d.restrict_vocab([1, 5, 9, 300, 2048, 4095])
        q = d.head_softmax(out, T)
        ref = torch.softmax(d.logits(out).double() / T, dim=-1)
        torch.testing.assert_close(q.double(), ref, rtol=1e-5, atol=1e-7)
        torch.testing.assert_close(q.sum(-1).double().cpu(), torch.ones(5, dtype=torch.float64), rtol=0, atol=1e-5)
    with pytest.raises(ValueError):
        d.head_softmax(out, 0.0)


def test_restricted_head_equals_gathered_full_logits(tiny_models):
    """tests/test_vocab.py:37-51 restated: restricted logits == full logits at the kept ids and
    the argmax row maps back to its token id; a second restriction is refused."""
    from woodcock_b200 import Drafter

    td, dd, _, _ = tiny_models["c1u"]
    d = Drafter.load(dd, dtype="fp32")
    out = torch.randn((4, 256), device="cuda")
    full = d.logits(out)
    ids = [3, 7, 8, 21, 49, 4000]
    d.restrict_vocab(ids)
    torch.testing.assert_close(d.logits(out), full[:, ids], rtol=0, atol=0)
    rows = torch.argmax(d.logits(out), dim=-1)
    assert d.head_argmax(out).cpu().tolist() == [ids[r] for r in rows.cpu().tolist()]
    with pytest.raises(ValueError):
        d.restrict_vocab(ids)


def test_single_token_draft_vocab_maps_rows_to_token_ids(golden, tiny_models, gpu_models, prompt64):
    """tests/test_spec_model.py:166-179 restated: with a 1-row head the drafter always proposes
    that token; it is accepted wherever the target produces it only if row 0 maps to its id."""
    from woodcock_b200 import Drafter, SpeculativeDecoder, StaticPolicy

    ar = golden("c1u")["ar_tokens"][:64]
    tok = max(set(ar), key=ar.count)
    assert tok != 0 and ar.count(tok) >= 4
    t, _ = gpu_models["c1u"]
    d = Drafter.load(tiny_models["c1u"][1], dtype="fp32")
    d.restrict_vocab([tok])
    out, st = SpeculativeDecoder(t, d, StaticPolicy(2), max_context=512).generate(prompt64, 64)
    assert out == ar
    assert sum(st.accepted) > 0


def test_bf16_target_logits_within_tolerance(tmp_path):
    """bf16 weights at Qwen3-1.7B widths (3 layers, full 151,936 vocabulary), bf16 KV cache.
    (a) vs the oracle in fp32 on the same bf16-rounded weights with bf16-rounded K/V rows:
        |dz| <= 2e-3 * max|z| + 2e-3 (only summation order and the activation split differ);
    (b) vs the oracle with an fp32 KV cache (the reference C++ core's arithmetic): the bf16
        tolerance |dz| <= 1e-2 * max|z|, and the greedy argmax agrees on every row."""
    import dataclasses

    from woodcock_b200 import Target
    from woodcock_b200 import synthetic as syn

    ts = dataclasses.replace(syn.Q17_TARGET, layers=3, tie_embeddings=True)  # three distinct taps
    w = syn.round_to_bf16(syn.generate_weights(syn.target_tensor_specs(ts), seed=0))
    t = Target.from_weights(ts.hf_config(), {k: torch.from_numpy(v).to(torch.bfloat16) for k, v in w.items()},
                            feature_layers=[0, 1, 2], dtype="bf16")
    prompt = syn.prompt_ids(24, ts.vocab, seed=1)
    z = t(prompt, t.make_cache(64), logits_from=20).logits[0].cpu().numpy()
    ot = O.Qwen3(ts.hf_config(), w, taps=[0, 1, 2])
    ot.kv_bf16 = True
    zb, _ = ot.forward(prompt, ot.make_cache(), logits_from=20)
    assert np.abs(z - zb).max() <= 2e-3 * np.abs(zb).max() + 2e-3
    ot.kv_bf16 = False
    zf, _ = ot.forward(prompt, ot.make_cache(), logits_from=20)
    assert np.abs(z - zf).max() <= 1e-2 * np.abs(zf).max()
    assert (z.argmax(-1) == zf.argmax(-1)).all()


def test_bf16_target_logits_at_4b_widths(tmp_path):
    """The same tolerances at Qwen3-4B widths (hidden 2560, 32 query heads, SwiGLU 9728): the
    projections with K = 2560 run the 80 KB activation-chunk GEMV instance without splitting
    K, the O projection (K = 4096) and down (K = 9728) split K; a 32,768-row head keeps the
    oracle's fp32 pass short."""
    import dataclasses

    from woodcock_b200 import Target
    from woodcock_b200 import synthetic as syn

    ts = dataclasses.replace(syn.Q4_TARGET, layers=3, vocab=32768, tie_embeddings=True)
    w = syn.round_to_bf16(syn.generate_weights(syn.target_tensor_specs(ts), seed=2))
    t = Target.from_weights(ts.hf_config(), {k: torch.from_numpy(v).to(torch.bfloat16) for k, v in w.items()},
                            feature_layers=[0, 1, 2], dtype="bf16")
    prompt = syn.prompt_ids(24, ts.vocab, seed=3)
    z = t(prompt, t.make_cache(64), logits_from=20).logits[0].cpu().numpy()
    ot = O.Qwen3(ts.hf_config(), w, taps=[0, 1, 2])
    ot.kv_bf16 = True
    zb, _ = ot.forward(prompt, ot.make_cache(), logits_from=20)
    assert np.abs(z - zb).max() <= 2e-3 * np.abs(zb).max() + 2e-3
    ot.kv_bf16 = False
    zf, _ = ot.forward(prompt, ot.make_cache(), logits_from=20)
    assert np.abs(z - zf).max() <= 1e-2 * np.abs(zf).max()
    assert (z.argmax(-1) == zf.argmax(-1)).all()
