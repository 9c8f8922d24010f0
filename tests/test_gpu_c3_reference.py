"""The headline model at full depth against the reference itself.

tests/golden/c3_reference.json holds the reference C++ core's results on the full 28-layer
C3 target (Qwen3-1.7B architecture, the bench's seeded bf16 weights, computed in fp32 by the
reference): its greedy continuation of an 8-token prompt and, teacher-forced on that
continuation, each position's argmax, top-8 logits and the logits at 256 seeded token ids.

The device computes the same rows in bf16 (bf16 weights and K/V cache, fp32 accumulation).
Tolerance per row: |z_dev - z_ref| <= 1e-2 * max|z_ref| at every compared id. Greedy tokens
must agree wherever the reference's top-2 gap exceeds twice that tolerance; a divergence of the
device's own greedy stream is allowed only at such a near tie, and is reported with the
reference's fp32 gap there.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REL = 1e-2  # measured worst on this fixture: 6.7e-3


@pytest.fixture(scope="module")
def c3_target():
    from woodcock_b200 import Target
    from woodcock_b200 import synthetic as syn

    ts = syn.Q17_TARGET
    return Target.from_weights(ts.hf_config(), syn.device_weight_stream(syn.target_tensor_specs(ts), 0, "cuda:0"),
                               feature_layers=[2, 14, 26], dtype="bf16", device=0)


def test_c3_bf16_logits_match_reference_core(golden, c3_target):
    g = golden("c3_reference")
    t = c3_target
    P, ar = len(g["prompt"]), g["ar_tokens"]
    seq = g["prompt"] + ar[:-1]
    z = t(seq, t.make_cache(64), logits_from=P - 1).logits[0].float().cpu().numpy()
    assert z.shape[0] == len(ar) == len(g["rows"])
    sample = np.asarray(g["sample_ids"])
    worst, compared = 0.0, 0
    for i, row in enumerate(g["rows"]):
        ids = np.concatenate([np.asarray(row["top_ids"]), sample])
        ref = np.concatenate([np.asarray(row["top_logits"]), np.asarray(row["sample_logits"])])
        scale = np.abs(ref).max()
        err = np.abs(z[i, ids] - ref).max()
        worst = max(worst, err / scale)
        assert err <= REL * scale, (i, err, scale)
        gap = row["top_logits"][0] - row["top_logits"][1]
        if gap > 2 * REL * scale:
            assert int(np.argmax(z[i])) == row["argmax"], i
            compared += 1
    print(f"c3 bf16 vs reference fp32: worst |dz| / max|z| = {worst:.2e} over {len(g['rows'])} rows; "
          f"argmax compared on {compared} rows")
    assert compared >= len(g["rows"]) // 3


def test_c3_bf16_greedy_stream_against_reference(golden, c3_target):
    from woodcock_b200 import generate_autoregressive

    g = golden("c3_reference")
    ar = g["ar_tokens"]
    out, _ = generate_autoregressive(c3_target, g["prompt"], len(ar), stop_on_eos=False, max_context=64)
    div = next((i for i in range(len(ar)) if out[i] != ar[i]), None)
    if div is None:
        print(f"c3 bf16 greedy stream identical to the reference for {len(ar)} tokens")
        return
    row = g["rows"][div]
    gap = row["top_logits"][0] - row["top_logits"][1]
    scale = max(abs(x) for x in row["top_logits"] + row["sample_logits"])
    print(f"c3 bf16 greedy stream diverges from the reference at token {div}: reference fp32 top-2 gap "
          f"{gap:.3e} (tolerance {2 * REL * scale:.3e})")
    assert gap <= 2 * REL * scale, (div, gap)
