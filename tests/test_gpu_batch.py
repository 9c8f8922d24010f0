"""Batched tree verification against the single-request path.

(a) The tcgen05 GEMM against a plain PyTorch fp32 matmul of the same bf16 operands, with
    ragged M / N edges and a residual.
(b) One batched verify of three requests (different prefix lengths, random trees) against
    each request verified alone through wc_target_forward with the tree mask and positions
    (sampling.py:118-128; spec.py:313-318): logits within the bf16 tolerance below, argmax
    equal away from near ties, appended K/V rows within bf16 rounding, prefix rows untouched.
(c) Compaction: the kept rows land at lens[r] + i bit for bit (kv_cache.cpp:21-31) and a
    second round on the compacted caches still matches the single-request path.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

# bf16 activations (GEMM operands, attention inputs) against the single-request path's
# fp32-level activations: relative rounding 2^-9 per operand, summed over a few layers.
LOGIT_TOL = 2.5e-2   # |dz| <= LOGIT_TOL * max|z|
KV_TOL = 2.5e-2      # |dk| <= KV_TOL * max|k| for appended rows


@pytest.mark.parametrize("M,N,K", [(200, 300, 512), (256, 2048, 2048), (2048, 4096, 2048), (130, 6144, 1024)])
def test_gemm_bf16_matches_torch(M, N, K):
    from woodcock_b200.batch import gemm_bf16

    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    A = torch.randn((M, K), device="cuda", generator=g).to(torch.bfloat16)
    B = (torch.randn((N, K), device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    ref = A.float() @ B.float().T
    out = gemm_bf16(A, B)
    torch.cuda.synchronize()
    err = (out - ref).abs().max().item()
    assert err <= 1e-3 * ref.abs().max().item() + 1e-4, err
    R = torch.randn((M, N), device="cuda", generator=g)
    out2 = gemm_bf16(A, B, residual=R)
    torch.cuda.synchronize()
    assert (out2 - (ref + R)).abs().max().item() <= 1e-3 * ref.abs().max().item() + 1e-4


@pytest.fixture(scope="module")
def bf16_target(tmp_path_factory):
    from woodcock_b200 import Target
    from woodcock_b200 import synthetic as syn

    ts = syn.TargetSpec(hidden=512, layers=3, heads=4, kv_heads=2, head_dim=128, intermediate=1536, vocab=4096,
                        tie_embeddings=False)
    ds = syn.DrafterSpec(hidden=512, layers=1, heads=4, kv_heads=2, head_dim=128, intermediate=1536, vocab=4096,
                         target_hidden=512, feature_layers=[0, 1, 2])
    root = tmp_path_factory.mktemp("batch")
    td, _, _, _ = syn.make_pair(root, "batch", seed=5, dtype="BF16", target_spec=ts, drafter_spec=ds)
    return Target.load(td, feature_layers=[0, 1, 2], dtype="bf16")


def _tree(rng, nodes, vocab):
    parents = [-1] + [int(rng.integers(0, i)) for i in range(1, nodes)]
    tokens = [int(x) for x in rng.integers(0, vocab, nodes)]
    return tokens, parents


def _depths(parents):
    d = [0] * len(parents)
    for i in range(1, len(parents)):
        d[i] = d[parents[i]] + 1
    return d


def _mask(parents, n):
    N = len(parents)
    m = np.zeros((N, n + N), dtype=bool)
    m[:, :n] = True
    for v in range(N):
        u = v
        while u >= 0:
            m[v, n + u] = True
            u = parents[u]
    return m


def _single(t, cache, tokens, parents, n):
    pos = [n + d for d in _depths(parents)]
    out = t(torch.tensor(tokens, dtype=torch.int32, device="cuda"), cache, positions=pos, mask=_mask(parents, n))
    return out.logits[0].float().cpu().numpy()


def _check_logits(zb, zs, where):
    scale = np.abs(zs).max()
    assert np.abs(zb - zs).max() <= LOGIT_TOL * scale, (where, np.abs(zb - zs).max(), scale)
    for i in range(zs.shape[0]):
        top2 = np.sort(zs[i])[-2:]
        if top2[1] - top2[0] > 2 * LOGIT_TOL * scale:
            assert int(np.argmax(zb[i])) == int(np.argmax(zs[i])), (where, i)


def test_batch_verify_and_compaction_match_single_requests(bf16_target):
    from woodcock_b200 import synthetic as syn
    from woodcock_b200.batch import BatchVerifier

    t = bf16_target
    c = t.cfg
    rng = np.random.default_rng(1)
    lens = [37, 64, 90]
    nodes = 8
    cap = 256
    bv = BatchVerifier(t, max_requests=4, max_nodes=nodes, capacity=cap, drafter_cache=(1, 2, 128))
    singles = []
    for r, n in enumerate(lens):
        cache = t.make_cache(cap)
        t(torch.tensor(syn.prompt_ids(n, c.vocab, seed=10 + r), dtype=torch.int32, device="cuda"), cache,
          logits=False)
        bv.set_prefix(r, cache, n)
        singles.append(cache)
    before = [[bv.read_kv(r, l, n) for l in range(c.layers)] for r, n in enumerate(lens)]

    for rnd in range(2):
        trees = [_tree(rng, nodes, c.vocab) for _ in lens]
        tokens = np.array([tr[0] for tr in trees])
        parents = np.array([tr[1] for tr in trees])
        am, zb = bv.verify(tokens, parents, logits=True)
        cur = bv.lens(len(lens))
        keeps = []
        for r, (tok, par) in enumerate(trees):
            n = cur[r]
            zs = _single(t, singles[r], tok, par, n)
            _check_logits(zb[r], zs, (rnd, r))
            assert (am[r] == np.argmax(zb[r], axis=-1)).all()
            for l in range(c.layers):
                kb, vb = bv.read_kv(r, l, n + nodes)
                ks, vs = (x.cpu().numpy() for x in singles[r].read(l, n + nodes))
                for a, b_ in ((kb[n:], ks[n:]), (vb[n:], vs[n:])):
                    assert np.abs(a - b_).max() <= KV_TOL * np.abs(b_).max(), (rnd, r, l)
                if rnd == 0:  # the committed prefix is untouched by the verify
                    np.testing.assert_array_equal(kb[:n], before[r][l][0])
                    np.testing.assert_array_equal(vb[:n], before[r][l][1])
            # a root-to-node path (the greedy rule would almost never accept random drafts)
            leaf = int(rng.integers(1, nodes))
            path, u = [], leaf
            while u > 0:
                path.append(u)
                u = par[u]
            keeps.append([0] + path[::-1])
        pre = [[bv.read_kv(r, l, cur[r] + nodes) for l in range(c.layers)] for r in range(len(lens))]
        bv.commit(keeps)
        after = bv.lens(len(lens))
        for r, k in enumerate(keeps):
            n = cur[r]
            assert after[r] == n + len(k)
            for l in range(c.layers):
                ka, va = bv.read_kv(r, l, n + len(k))
                for i, src in enumerate(k):
                    np.testing.assert_array_equal(ka[n + i], pre[r][l][0][n + src])
                    np.testing.assert_array_equal(va[n + i], pre[r][l][1][n + src])
            singles[r].compact(n, k)  # the single-request cache follows the same compaction
            assert singles[r].size() == n + len(k)


@pytest.mark.parametrize("n", [37, 300, 1100])
def test_prompt_forward_matches_decode_path(bf16_target, n):
    """The prefill's target pass on the tensor cores (chunks of 1024 rows, causal attention)
    against wc_target_forward on the decode kernels: tap rows and K/V rows within the bf16
    tolerance above; the cache grows by n."""
    from woodcock_b200 import synthetic as syn
    from woodcock_b200.target import prompt_forward

    t = bf16_target
    c = t.cfg
    prompt = syn.prompt_ids(n, c.vocab, seed=n)
    ca, cb = t.make_cache(n + 8), t.make_cache(n + 8)
    ref = t(torch.tensor(prompt, dtype=torch.int32, device="cuda"), ca, capture=True, logits=False)
    taps, last = prompt_forward(t, prompt, cb)
    torch.cuda.synchronize()
    assert cb.size() == n
    for f in range(3):
        r_ = ref.features[f][0].float()
        g_ = taps[f]
        assert (g_ - r_).abs().max().item() <= KV_TOL * r_.abs().max().item(), f
    assert torch.isfinite(last).all()
    for l in range(c.layers):
        for a, b_ in zip(cb.read(l, n), ca.read(l, n)):
            assert (a - b_).abs().max().item() <= KV_TOL * b_.abs().max().item(), l

