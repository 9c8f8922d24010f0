"""The prefill's drafter pass on the tensor cores (spec.py:129-141 drafter half; drafter.cpp:75-136):
fuse, the auxiliary embedding term and the layer as tcgen05 GEMMs over all prompt rows with
causal attention, against the same prefill on the decode kernels (WC_PREFILL_GEMM=0, run in a
child process because the switch is read once per process). The bf16 models have Qwen3-1.7B
widths (a 3-layer target, 32,768-token vocabulary). Compared: the drafter's K/V rows for every
prompt position within the bf16 tolerance, and the first round's draft proposals."""

from __future__ import annotations

import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

KV_TOL = 3e-2  # relative to max |row|: bf16 operands on one side, fp32-level activations on the other

SCRIPT = r"""
import dataclasses, json, sys
import numpy as np, torch
sys.path.insert(0, {repo!r})
from woodcock_b200 import Drafter, SpeculativeDecoder, StaticPolicy, Target
from woodcock_b200 import synthetic as syn
ts = dataclasses.replace(syn.Q17_TARGET, layers=3, vocab=32768, tie_embeddings=True)
ds = dataclasses.replace(syn.Q17_DRAFTER, vocab=32768, feature_layers=[0, 1, 2])
tw = syn.round_to_bf16(syn.generate_weights(syn.target_tensor_specs(ts), seed=21))
dw = syn.round_to_bf16(syn.generate_weights(syn.drafter_tensor_specs(ds), seed=22))
bf = lambda w: {{k: torch.from_numpy(v).to(torch.bfloat16) for k, v in w.items()}}
t = Target.from_weights(ts.hf_config(), bf(tw), feature_layers=[0, 1, 2], dtype="bf16")
d = Drafter.from_weights(ds.config(), bf(dw), dtype="bf16")
prompt = syn.prompt_ids({n}, ts.vocab, seed=23)
dec = SpeculativeDecoder(t, d, StaticPolicy(4), max_context={n} + 64)
first = dec.prefill(prompt)
k0, v0 = dec.drafter_cache().read(0, {n})
dec.round(4)
props, z = dec.draft_proposals(4)
np.savez({out!r}, k=k0.float().cpu().numpy(), v=v0.float().cpu().numpy(), first=first,
         props=np.array(props), z=np.array(z))
"""


def _run(n: int, out: str, gemm: bool) -> dict:
    from conftest import REPO

    env = dict(os.environ, WC_PREFILL_GEMM="1" if gemm else "0")
    r = subprocess.run([sys.executable, "-c", SCRIPT.format(repo=str(REPO), n=n, out=out)], env=env,
                       capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    return dict(np.load(out))


@pytest.mark.parametrize("n", [300])
def test_drafter_prefill_on_tensor_cores_matches_decode_kernels(tmp_path, n):
    a = _run(n, str(tmp_path / "gemm.npz"), True)
    b = _run(n, str(tmp_path / "decode.npz"), False)
    assert int(a["first"]) == int(b["first"])
    for key in ("k", "v"):
        assert a[key].shape == b[key].shape == (n, 8, 128)
        err = np.abs(a[key] - b[key]).max()
        assert err <= KV_TOL * np.abs(b[key]).max(), (key, err)
    # the first round's proposals come from the prefill's last drafter row
    assert a["props"][0] == b["props"][0]
    assert abs(float(a["z"][0]) - float(b["z"][0])) <= KV_TOL * abs(float(b["z"][0])) + 1e-3
