"""Trimmed draft vocabularies and the drafter export format v1 (python/woodcock/vocab.py,
python/woodcock/export.py). CPU: top_ids against the reference's own results
(tests/golden/vocab.json), the counts-file spec, manifest validation. GPU: an exported
drafter loads back and computes the same head logits; tampered weights are refused."""

from __future__ import annotations

import json

import numpy as np
import pytest


def test_top_ids_match_reference(golden):
    from woodcock_b200.vocab import coverage, top_ids

    for case in golden("vocab")["top_ids"]:
        ids = top_ids(np.array(case["counts"]), case["k"], set(case["always"]))
        assert ids.dtype == np.int32
        assert ids.tolist() == case["ids"]
        assert coverage(np.array(case["counts"]), ids) == pytest.approx(case["coverage"])


def test_top_ids_errors_and_counts_file(tmp_path):
    from woodcock_b200.vocab import load_ids, top_ids

    with pytest.raises(ValueError):
        top_ids(np.ones(5), 0)
    with pytest.raises(ValueError):
        top_ids(np.ones(5), 2, {0, 1, 2})
    counts = np.array([5, 9, 9, 1, 0, 7])
    np.savez(tmp_path / "c.npz", counts=counts, eos=np.array([4]))
    assert load_ids(f"{tmp_path / 'c.npz'}:3").tolist() == [1, 2, 4]  # 9, 9 (ids 1 < 2), then EOS 4
    with pytest.raises(ValueError):
        load_ids("no-colon")


def _plain_drafter(tmp_path):
    from woodcock_b200 import synthetic as syn

    td, dd, _, _ = syn.make_pair(tmp_path, "c1", seed=3, dtype="BF16")
    return td, dd


def test_export_manifest_and_validation(tmp_path):
    from woodcock_b200.export import FORMAT, VERSION, check_manifest, export_drafter

    _, dd = _plain_drafter(tmp_path)
    out = export_drafter(dd, tmp_path / "exp", target_name="synthetic-c1", check=False)
    m = json.loads((out / "woodcock.json").read_text())
    assert m["format"] == FORMAT and m["version"] == VERSION and m["target"]["name"] == "synthetic-c1"
    assert m["weights"]["num_params"] > 0 and len(m["weights"]["sha256"]) == 64
    assert check_manifest(out)["mode"] == "woodcock-v1"
    assert check_manifest(dd) is None  # a plain directory has no manifest

    class Cfg:
        hidden, vocab = 999, 4096
    with pytest.raises(ValueError, match="hidden size"):
        check_manifest(out, Cfg())
    w = out / "model.safetensors"
    raw = bytearray(w.read_bytes())
    raw[-1] ^= 0xFF
    w.write_bytes(bytes(raw))
    with pytest.raises(ValueError, match="sha256"):
        check_manifest(out)


@pytest.mark.gpu
def test_exported_drafter_round_trip(tmp_path):
    import torch

    from woodcock_b200 import Drafter, Target
    from woodcock_b200.export import export_drafter

    td, dd = _plain_drafter(tmp_path)
    out = export_drafter(dd, tmp_path / "exp", check=True)  # raises on any logits difference
    t = Target.load(td, feature_layers=[1, 2, 3], dtype="bf16")
    d = Drafter.load(out, target=t, vocab=[3, 7, 11, 4000])
    x = torch.randn((2, d.hidden_size), device="cuda")
    full = Drafter.load(dd, dtype="bf16").logits(x)
    torch.testing.assert_close(d.logits(x), full[:, [3, 7, 11, 4000]], rtol=0, atol=0)
