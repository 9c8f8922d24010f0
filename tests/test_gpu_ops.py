"""The ops API (include/woodcock/ops.h counterparts) against the oracle's restatement of
src/backends/cpu_ops.cpp, on seeded inputs."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import wc_oracle as O

pytestmark = pytest.mark.gpu


def _t(x):
    return torch.tensor(x, device="cuda")


@pytest.mark.parametrize("L", [1, 5, 9, 16, 21])
@pytest.mark.parametrize("wdt", ["fp32", "bf16"])
def test_linear(L, wdt):
    from woodcock_b200 import ops, safetensors_io as st

    rng = np.random.default_rng(L)
    N, K = 384, 2304  # K spans two 2048-column chunks
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    if wdt == "bf16":
        W = st.bf16_bits_to_f32(st.f32_to_bf16_bits(W)).reshape(N, K)
    x = rng.standard_normal((L, K)).astype(np.float32)
    w = ops.Weight(torch.from_numpy(W), dtype=torch.bfloat16 if wdt == "bf16" else torch.float32)
    y = ops.linear(_t(x), w).cpu().numpy()
    ref = O.linear(x, W)
    tol = 1e-4 if wdt == "fp32" else 5e-4  # bf16 path: activations split into two bf16 terms
    np.testing.assert_allclose(y, ref, rtol=0, atol=tol * np.abs(ref).max())
    y0 = _t(np.ones((L, N), np.float32))
    ops.linear(_t(x), w, y0, accumulate=True)
    np.testing.assert_allclose(y0.cpu().numpy(), ref + 1, rtol=0, atol=tol * np.abs(ref).max() + 1e-6)


def test_rmsnorm_rope_silu_softmax_argmax():
    from woodcock_b200 import ops

    rng = np.random.default_rng(0)
    x = rng.standard_normal((7, 512)).astype(np.float32)
    w = rng.standard_normal(512).astype(np.float32)
    np.testing.assert_allclose(ops.rmsnorm(_t(x), _t(w), 1e-6).cpu().numpy(), O.rmsnorm(x, w, 1e-6), rtol=1e-5,
                               atol=1e-6)
    q = rng.standard_normal((3, 4, 128)).astype(np.float32)
    pos = [0, 17, 4095]
    np.testing.assert_allclose(ops.rope(_t(q.copy()), pos, 1e6).cpu().numpy(), O.rope(q, pos, 1e6), rtol=1e-5,
                               atol=2e-6)
    g, u = rng.standard_normal(1000).astype(np.float32), rng.standard_normal(1000).astype(np.float32)
    np.testing.assert_allclose(ops.silu_mul(_t(g.copy()), _t(u)).cpu().numpy(), O.silu_mul(g, u), rtol=1e-6,
                               atol=1e-7)
    z = rng.standard_normal((2, 151936)).astype(np.float32) * 3
    z[1, 5] = -np.inf
    np.testing.assert_allclose(ops.softmax(_t(z.copy())).cpu().numpy(), O.softmax(z), rtol=1e-5, atol=1e-12)
    z[0, 100] = z[0, 200] = z[0].max() + 1  # tie: first index wins
    assert ops.argmax(_t(z)).cpu().tolist() == [100, int(np.argmax(z[1]))]


@pytest.mark.parametrize("kvdt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("masked", [False, True])
def test_attention(kvdt, masked):
    from woodcock_b200 import ops

    rng = np.random.default_rng(1)
    L, H, Hk, D, T = 6, 16, 8, 128, 300
    q = rng.standard_normal((L, H, D)).astype(np.float32)
    K = rng.standard_normal((T, Hk, D)).astype(np.float32)
    V = rng.standard_normal((T, Hk, D)).astype(np.float32)
    mask = None
    if masked:
        mask = (rng.random((L, T)) < 0.6).astype(np.uint8)
        mask[:, -1] = 1
    Kt, Vt = _t(K).to(kvdt), _t(V).to(kvdt)
    Kr, Vr = Kt.float().cpu().numpy(), Vt.float().cpu().numpy()
    out = ops.attention(_t(q), Kt, Vt, mask=None if mask is None else _t(mask), scale=D ** -0.5).cpu().numpy()
    ref = O.attention(q, Kr, Vr, mask, D ** -0.5)
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=1e-5)


def test_kv_append_read_roundtrip():
    from woodcock_b200.cache import KVCache

    kv = KVCache.create(2, 2, 64, 32, dtype=0)
    rng = np.random.default_rng(2)
    k = rng.standard_normal((5, 2, 64)).astype(np.float32)
    v = rng.standard_normal((5, 2, 64)).astype(np.float32)
    kv.append(1, _t(k), _t(v))
    kv.commit(5)
    K, Vv = kv.read(1)
    np.testing.assert_array_equal(K.cpu().numpy(), k)
    np.testing.assert_array_equal(Vv.cpu().numpy(), v)
