"""The persistent layer-stack kernel (stack.cuh), which runs the verify pass of bf16 models
with 128-wide heads when a context is created with WC_STACK=1. Its round must append to the
target cache the same K/V rows as the per-kernel forward of the same tokens
(wc_target_forward), layer by layer, within bf16 rounding of the stored rows; and the round's
profile must show that the stack ran. The checks run in a child process that sets the switch
(contexts read it at creation)."""

from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import REPO

pytestmark = pytest.mark.gpu


def test_stack_checks_in_a_child_process():
    env = dict(os.environ, WC_STACK="1", WC_STACK_CHILD="1")
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", str(REPO / "tests" / "test_gpu_stack.py"),
                        "-k", "appends"], env=env, capture_output=True, text=True, timeout=600, cwd=str(REPO))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]

# K/V rows are stored in bf16: two paths that sum in different orders can land one bf16
# step apart (2^-8 relative); anything beyond a few steps is a real difference.
KV_RTOL = 2e-2


@pytest.fixture(scope="module")
def stack_pair(tmp_path_factory):
    from woodcock_b200 import Drafter, Target
    from woodcock_b200 import synthetic as syn

    ts = syn.TargetSpec(hidden=512, layers=4, heads=4, kv_heads=2, head_dim=128, intermediate=1536, vocab=4096,
                        tie_embeddings=False)
    ds = syn.DrafterSpec(hidden=512, layers=1, heads=4, kv_heads=2, head_dim=128, intermediate=1536, vocab=4096,
                         target_hidden=512, feature_layers=[1, 2, 3])
    root = tmp_path_factory.mktemp("stack")
    td, dd, _, _ = syn.make_pair(root, "stack", seed=3, dtype="BF16", target_spec=ts, drafter_spec=ds)
    t = Target.load(td, feature_layers=[1, 2, 3], dtype="bf16")
    d = Drafter.load(dd, dtype="bf16")
    return t, d


@pytest.mark.skipif(os.environ.get("WC_STACK_CHILD") != "1", reason="runs in the child process that sets WC_STACK=1")
@pytest.mark.parametrize("k", [1, 4])
def test_stack_verify_appends_the_forward_rows(stack_pair, k):
    from woodcock_b200 import SpeculativeDecoder, StaticPolicy
    from woodcock_b200 import synthetic as syn

    t, d = stack_pair
    prompt = syn.prompt_ids(96, 4096, seed=5)
    dec = SpeculativeDecoder(t, d, StaticPolicy(k), max_context=256, max_k=8)
    x_n = dec.prefill(prompt)
    drafts = [int(v) for v in np.random.default_rng(k).integers(0, 4096, k)]
    dec.set_forced(drafts)
    toks, prof = dec.profile_round(k)  # the instrumented graph runs the same stack plan
    assert prof["target_stack"]["launches"] == 1, "the verify pass did not use the layer stack"
    n = len(prompt)
    got = dec.target_cache()

    ref = t.make_cache(256)
    t(torch.tensor(prompt + [x_n] + drafts, dtype=torch.int32, device="cuda"), ref, logits=False)
    for layer in range(t.cfg.layers):
        gk, gv = got.read(layer, n + k + 1)
        rk, rv = ref.read(layer, n + k + 1)
        for a, b in ((gk, rk), (gv, rv)):
            a = a[n:].cpu().numpy()
            b = b[n:].cpu().numpy()
            scale = np.abs(b).max()
            assert np.abs(a - b).max() <= KV_RTOL * scale, f"layer {layer}: {np.abs(a - b).max()} vs {scale}"
    # the first emitted token is the target's greedy token after x_n (drafts are random)
    z = t(torch.tensor(prompt + [x_n], dtype=torch.int32, device="cuda"), t.make_cache(256), logits_from=n).logits
    z = z.float().reshape(-1).cpu().numpy()[-4096:]
    top2 = np.sort(z)[-2:]
    if top2[1] - top2[0] > 1e-3:  # skip the check on a near tie
        assert toks[0] == int(np.argmax(z))
