"""The bf16 drafter at Qwen3-1.7B widths (the headline round's drafter) against the oracle.

Shapes of BASELINE config C2/C3: hidden 2048, 16 query / 8 KV heads of 128, SwiGLU 6144, a
6144 -> 2048 fuse over three taps, the auxiliary (token embedding) term in layer 0's Q/K/V,
and a 16,384-row trimmed head (a seeded subset of 151,936 ids) with the fused argmax. Norm
gains are drawn around 1 (not left at 1) so that every gain is exercised.

The oracle runs fp32 arithmetic on the same bf16-rounded weights with bf16-rounded K/V rows
(the device cache's storage), so the remaining difference is summation order and the
device's two-term (bf16 hi + lo) activations. Tolerance, for every compared tensor x:
|x_dev - x_oracle| <= 2e-3 * max|x_oracle| + 2e-3. The head argmax must be equal on every row
whose top-2 logit gap exceeds twice that tolerance (a near tie may legitimately flip).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import wc_oracle as O

pytestmark = pytest.mark.gpu

REL, ABS = 2e-3, 2e-3
HEAD_ROWS = 16384


def close(x_dev, x_ref, what):
    x_dev = np.asarray(x_dev, np.float64)
    x_ref = np.asarray(x_ref, np.float64)
    tol = REL * np.abs(x_ref).max() + ABS
    err = np.abs(x_dev - x_ref).max()
    assert err <= tol, f"{what}: max |diff| {err:.3e} > {tol:.3e}"


@pytest.fixture(scope="module")
def q17_drafter():
    from woodcock_b200 import Drafter
    from woodcock_b200 import synthetic as syn

    ds = syn.Q17_DRAFTER
    specs = syn.drafter_tensor_specs(ds)
    w = syn.generate_weights(specs, seed=5)
    rng = np.random.default_rng(6)
    for name, shape, is_norm in specs:
        if is_norm:
            w[name] = (1.0 + 0.2 * rng.standard_normal(shape)).astype(np.float32)
    w = syn.round_to_bf16(w)
    ids = syn.trimmed_vocab_ids(ds.vocab, HEAD_ROWS, seed=0)
    d = Drafter.from_weights(ds.config(), {k: torch.from_numpy(v).to(torch.bfloat16) for k, v in w.items()},
                             dtype="bf16")
    d.restrict_vocab(ids)
    od = O.Drafter(ds.config(), w)
    od.restrict_vocab(ids)
    od.kv_bf16 = True
    return ds, d, od, ids


def test_bf16_drafter_fuse_layer_head_at_17b_widths(q17_drafter):
    ds, d, od, ids = q17_drafter
    rng = np.random.default_rng(7)
    H, Ht = ds.hidden, ds.target_hidden

    def taps(L):  # residual-stream-like rows of growing scale, one array per tap layer
        return [(rng.standard_normal((L, Ht)) * (1.0 + 2.0 * f)).astype(np.float32) for f in range(3)]

    # the fuse (3 x 2048 -> 2048 with the per-tap norms) on a 24-row prefill and a 5-row update
    cache = d.make_cache(128)
    oc = od.make_cache()
    for L in (24, 5):
        tp = taps(L)
        g_ref = od.fuse(tp)
        g = d.fuse([torch.tensor(x, device="cuda")[None] for x in tp])[0].cpu().numpy()
        close(g, g_ref, f"fuse L={L}")
        # one drafter layer with the auxiliary embedding term, appending to a bf16 cache
        toks = rng.integers(0, ds.vocab, L).tolist()
        h_ref, out_ref = od.forward(toks, g_ref, oc)
        h, out = d(toks, torch.tensor(g_ref, device="cuda")[None], cache)
        close(h[0].cpu().numpy(), h_ref, f"drafter hidden L={L}")
        close(out[0].cpu().numpy(), out_ref, f"drafter out L={L}")
        assert cache.size() == oc.size()
    # the trimmed head over the last rows: logits and the fused argmax mapped to token ids
    o = torch.tensor(out_ref, device="cuda")[None]
    z_ref = od.logits(out_ref)
    z = d.logits(o)[0].cpu().numpy()
    assert z.shape == (5, HEAD_ROWS)
    close(z, z_ref, "head logits")
    am = d.head_argmax(o).cpu().numpy().reshape(-1)
    tol = REL * np.abs(z_ref).max() + ABS
    checked = 0
    for r in range(5):
        top2 = np.sort(z_ref[r])[-2:]
        if top2[1] - top2[0] > 2 * tol:
            assert am[r] == ids[int(np.argmax(z_ref[r]))], r
            checked += 1
    assert checked >= 3


def test_bf16_drafter_chain_rows_and_positions(q17_drafter):
    """Explicit positions and a tree mask (the drafting-phase call of spec.cpp:158-171): two
    sibling rows at the same position see the committed prefix and themselves only."""
    ds, d, od, ids = q17_drafter
    rng = np.random.default_rng(8)
    H = ds.hidden
    cache = d.make_cache(128)
    oc = od.make_cache()
    pre = 16
    g0 = (rng.standard_normal((pre, H)) * 0.5).astype(np.float32)
    toks0 = rng.integers(0, ds.vocab, pre).tolist()
    od.forward(toks0, g0, oc)
    d(toks0, torch.tensor(g0, device="cuda")[None], cache)
    g1 = (rng.standard_normal((2, H)) * 0.5).astype(np.float32)
    toks1 = rng.integers(0, ds.vocab, 2).tolist()
    mask = np.zeros((2, pre + 2), np.uint8)
    mask[:, :pre] = 1
    mask[0, pre] = mask[1, pre + 1] = 1
    h_ref, out_ref = od.forward(toks1, g1, oc, positions=[pre, pre], mask=mask)
    h, out = d(toks1, torch.tensor(g1, device="cuda")[None], cache, positions=[pre, pre], mask=mask)
    close(h[0].cpu().numpy(), h_ref, "masked hidden")
    close(out[0].cpu().numpy(), out_ref, "masked out")
