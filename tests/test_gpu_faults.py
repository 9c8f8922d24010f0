"""Failure paths, made on the host or by a bounded wait that is meant to expire (no GPU fault).

* The reference refuses bad input with exceptions (src/core/weights.cpp:22, 27, 73: files and
  headers; src/core/drafter.cpp:36, 41: drafter modes; python/woodcock/drafter.py:60-61); here
  the C ABI returns a status and the Python layer raises ValueError / RuntimeError.
* A device-side bounded wait that nobody satisfies gives up, raises the timeout bit of the
  device error word and returns; the host sees WC_ERR_DEVICE at its next synchronisation and
  the context keeps working.
"""

from __future__ import annotations

import json
import shutil
import struct

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_expires_into_a_device_error_and_the_context_survives():
    from woodcock_b200._lib import WC_ERR_DEVICE, WcError, lib
    from woodcock_b200.context import Context
    from woodcock_b200.ops import softmax

    ctx = Context.get(0)
    ctx.check(lib().wc_ctx_wait_selftest(ctx.h, 2000))
    with pytest.raises(WcError) as e:
        ctx.synchronize()
    assert e.value.status == WC_ERR_DEVICE and "32" in str(e.value)
    ctx.synchronize()  # the error word was cleared
    x = torch.randn((3, 77), device="cuda")
    want = torch.softmax(x, -1)  # ops.softmax works in place
    torch.testing.assert_close(softmax(x), want, rtol=1e-5, atol=1e-6)


@pytest.fixture()
def tiny_dirs(tiny_models, tmp_path):
    td, dd, _, _ = tiny_models["c1u"]
    t2, d2 = tmp_path / "target", tmp_path / "drafter"
    shutil.copytree(td, t2)
    shutil.copytree(dd, d2)
    return t2, d2


def _corrupt_header(path, how):
    raw = bytearray(path.read_bytes())
    if how == "length":  # header length beyond the file
        raw[:8] = struct.pack("<Q", len(raw) * 4)
    elif how == "json":  # not JSON
        n = struct.unpack("<Q", bytes(raw[:8]))[0]
        raw[8 : 8 + n] = b"{" * n
    elif how == "offsets":  # a tensor's data range outside the file
        n = struct.unpack("<Q", bytes(raw[:8]))[0]
        h = json.loads(bytes(raw[8 : 8 + n]))
        name = next(k for k in h if k != "__metadata__")
        h[name]["data_offsets"] = [0, len(raw) * 8]
        hb = json.dumps(h).encode()
        hb += b" " * (n - len(hb)) if len(hb) <= n else b""
        raw = bytearray(struct.pack("<Q", len(hb))) + hb + raw[8 + n :]
    path.write_bytes(bytes(raw))


@pytest.mark.parametrize("how", ["length", "json", "offsets"])
def test_corrupt_safetensors_is_refused(tiny_dirs, how):
    from woodcock_b200 import Target

    td, _ = tiny_dirs
    _corrupt_header(td / "model.safetensors", how)
    with pytest.raises((ValueError, RuntimeError)):
        Target.load(td, feature_layers=[1, 2, 3], dtype="fp32")


def test_missing_weight_files_are_refused(tiny_dirs):
    from woodcock_b200 import Target

    td, _ = tiny_dirs
    (td / "model.safetensors").unlink()
    with pytest.raises((ValueError, RuntimeError), match="safetensors"):
        Target.load(td, feature_layers=[1, 2, 3], dtype="fp32")


@pytest.mark.parametrize("taps", [[1, 2, 4], [-1, 1, 2], [3, 2, 1, 0]])
def test_bad_tap_layers_are_refused(tiny_dirs, taps):
    from woodcock_b200 import Target

    td, _ = tiny_dirs
    with pytest.raises(ValueError):
        Target.load(td, feature_layers=taps, dtype="fp32")


@pytest.mark.parametrize("key,value", [("residual", "hidden"), ("lowrank_rank", 8)])
def test_unsupported_drafter_modes_are_refused(tiny_dirs, key, value):
    """drafter.cpp:36, 41: a residual mode other than "feature" and a nonzero low-rank rank."""
    from woodcock_b200 import Drafter

    _, dd = tiny_dirs
    cfg = json.loads((dd / "config.json").read_text())
    cfg[key] = value
    (dd / "config.json").write_text(json.dumps(cfg))
    with pytest.raises(ValueError, match="unsupported drafter"):
        Drafter.load(dd, dtype="fp32")


def test_malformed_trees_are_refused(golden, tiny_models, prompt64):
    from woodcock_b200 import Drafter, SpeculativeDecoder, StaticPolicy, Target
    from woodcock_b200.sampling import DraftTree, verify_tree_greedy

    td, dd, _, _ = tiny_models["c1u"]
    t = Target.load(td, feature_layers=[1, 2, 3], dtype="fp32")
    d = Drafter.load(dd, dtype="fp32")
    dec = SpeculativeDecoder(t, d, StaticPolicy(3, 2, 6), max_context=256)
    dec.prefill(prompt64)
    for parents in ([-1, 0, 3, 1], [-1, 1], [0, 0, 1], [-1, 0, -1]):
        with pytest.raises(ValueError):
            dec.set_forced_tree([0] * len(parents), parents)
    with pytest.raises(ValueError):
        dec.set_forced_tree([0, 5000], [-1, 0])  # token id beyond the vocabulary
    with pytest.raises(ValueError):
        dec.tree_round(3, 17, 6)  # width above the device limit
    # a tree whose parent follows its child, given to the acceptance kernel directly
    bad = DraftTree([1, 2, 3], [-1, 2, 0], [0, 2, 1])
    with pytest.raises((ValueError, RuntimeError)):
        verify_tree_greedy(np.array([2, 3, 1]), bad)
    # the decoder is still usable after the refusals
    out = dec.tree_round(3, 2, 6)
    assert 1 <= len(out) <= 4
