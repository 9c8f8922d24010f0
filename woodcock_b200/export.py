"""Drafter export format v1 (python/woodcock/export.py:1-64), read back by `Drafter.load`.

    <dir>/
      woodcock.json       manifest: format, version, mode, target (name, hidden size,
                          vocabulary, tap layers), drafter shape, weights (file, sha256,
                          parameter count, tensor table), training metadata
      config.json         the drafter config (python/woodcock/drafter.py names)
      model.safetensors   bf16 weights under the reference's tensor names

The manifest lets a runtime check that it pairs the drafter with the right target.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np

from . import safetensors_io as st

FORMAT = "woodcock-drafter"
VERSION = 1
MODE = "woodcock-v1"


def _sha256(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 24), b""):
            h.update(block)
    return h.hexdigest()


def read_manifest(path: str | Path) -> dict | None:
    p = Path(path) / "woodcock.json"
    return json.loads(p.read_text()) if p.exists() else None


def check_manifest(path: str | Path, target_cfg=None, verify_sha: bool = True) -> dict | None:
    """Validates an exported drafter directory: format and version, the weights file's
    sha256, and (when given a target config with hidden / vocab) that the target matches.
    Returns the manifest (None for a plain directory without one); raises ValueError."""
    path = Path(path)
    m = read_manifest(path)
    if m is None:
        return None
    if m.get("format") != FORMAT:
        raise ValueError(f"not a woodcock drafter export: format {m.get('format')!r}")
    if int(m.get("version", 0)) != VERSION:
        raise ValueError(f"unsupported drafter export version {m.get('version')}")
    w = m.get("weights", {})
    wfile = path / w.get("file", "model.safetensors")
    if not wfile.exists():
        raise ValueError(f"exported weights missing: {wfile.name}")
    if verify_sha and w.get("sha256") and _sha256(wfile) != w["sha256"]:
        raise ValueError("exported weights do not match the manifest's sha256")
    tgt = m.get("target", {})
    if target_cfg is not None:
        if tgt.get("hidden_size") not in (None, target_cfg.hidden):
            raise ValueError(f"drafter was exported for target hidden size {tgt.get('hidden_size')}, "
                             f"the target has {target_cfg.hidden}")
        if tgt.get("vocab_size") not in (None, target_cfg.vocab):
            raise ValueError(f"drafter was exported for a {tgt.get('vocab_size')}-token vocabulary, "
                             f"the target has {target_cfg.vocab}")
    return m


def export_drafter(src: str | Path, out: str | Path, target_name: str | None = None, check: bool = True) -> Path:
    """Writes the v1 export of the drafter in `src` (config.json + *.safetensors) to `out`:
    bf16 weights, config and manifest. With `check`, the export is loaded back on the device
    and must compute the same head logits as the source (export.py:49-58)."""
    src_p, out_p = Path(src), Path(out)
    out_p.mkdir(parents=True, exist_ok=True)
    cfg = json.loads((src_p / "config.json").read_text())
    tensors = {}
    for f in sorted(src_p.glob("*.safetensors")):
        for name, entry in st.load(f).items():
            dt, arr = entry
            tensors[name] = ("BF16", arr if dt == "BF16" else st.f32_to_bf16_bits(st.to_f32(entry)))
    if not tensors:
        raise ValueError(f"no safetensors weights under {src_p}")
    wfile = out_p / "model.safetensors"
    st.save(wfile, tensors, metadata={"format": "woodcock-drafter-v1"})
    (out_p / "config.json").write_text(json.dumps(cfg, indent=2))
    meta_p = src_p / "meta.json"
    meta = json.loads(meta_p.read_text()) if meta_p.exists() else {}
    if target_name is None:
        target_name = meta.get("train", {}).get("target")
    manifest = {
        "format": FORMAT, "version": VERSION, "mode": MODE,
        "target": {"name": target_name, "hidden_size": cfg.get("target_hidden_size"),
                   "vocab_size": cfg.get("vocab_size"), "feature_layers": cfg.get("feature_layers")},
        "drafter": {"hidden_size": cfg.get("hidden_size"), "num_layers": cfg.get("num_layers"),
                    "post_norm": cfg.get("post_norm", True), "window": cfg.get("window")},
        "weights": {"file": wfile.name, "sha256": _sha256(wfile),
                    "num_params": int(sum(int(np.prod(a.shape)) for _, a in tensors.values())),
                    "tensors": {k: {"shape": list(a.shape), "dtype": "bfloat16"} for k, (_, a) in tensors.items()}},
        "training": meta.get("train"),
    }
    (out_p / "woodcock.json").write_text(json.dumps(manifest, indent=2))
    if check:
        import torch

        from .drafter import Drafter

        a, b = Drafter.load(src_p, dtype="bf16"), Drafter.load(out_p, dtype="bf16")
        x = torch.randn((2, a.hidden_size), device=a.ctx.device)
        if not torch.equal(a.logits(x), b.logits(x)):
            raise RuntimeError("export round trip changed the drafter's head logits")
    return out_p
