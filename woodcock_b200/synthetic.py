"""Seeded synthetic Qwen3 targets and EAGLE-3 drafters for the benchmark configs.

No checkpoints or datasets are available offline, so every workload runs on
random-init weights of the real architectures:

* C1 tiny fp32 target (4 layers, hidden 256, 4/2 heads x 64, SwiGLU 768, vocab 4096,
  tied embeddings) with a 1-layer drafter fusing taps {1, 2, 3} and a full 4096 head;
* C2/C3 Qwen3-1.7B architecture (28 layers, hidden 2048, 16/8 heads x 128, SwiGLU
  6144, vocab 151936) with a drafter reading taps {2, 14, 26} and a 16384-row head;
* C4 Qwen3-4B architecture (36 layers, hidden 2560, 32/8 heads, SwiGLU 9728).

Weights are N(0, 0.02^2) drawn in a fixed tensor order from numpy's
``default_rng(seed)``; norm gains are 1. Tensor names and config keys follow the
Hugging Face Qwen3 layout the reference loads (src/core/qwen3.cpp:22-36, 55-73) and
the drafter layout of python/woodcock/drafter.py:34-63 / src/core/drafter.cpp:18-73.
"""

from __future__ import annotations

import json
from dataclasses import asdict, dataclass, field
from pathlib import Path

import numpy as np

from . import safetensors_io as st

QWEN3_EOS = (151643, 151645)


@dataclass
class TargetSpec:
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    eps: float = 1e-6
    rope_theta: float = 1e6
    tie_embeddings: bool = True

    def hf_config(self) -> dict:
        return {
            "architectures": ["Qwen3ForCausalLM"],
            "hidden_size": self.hidden,
            "num_hidden_layers": self.layers,
            "num_attention_heads": self.heads,
            "num_key_value_heads": self.kv_heads,
            "head_dim": self.head_dim,
            "intermediate_size": self.intermediate,
            "vocab_size": self.vocab,
            "rms_norm_eps": self.eps,
            "rope_theta": self.rope_theta,
            "tie_word_embeddings": self.tie_embeddings,
        }


@dataclass
class DrafterSpec:
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    target_hidden: int
    feature_layers: list[int] = field(default_factory=list)
    num_features: int = 3
    eps: float = 1e-6
    rope_theta: float = 1e6
    post_norm: bool = True
    feature_norm: bool = True

    def config(self) -> dict:
        return {
            "hidden_size": self.hidden,
            "num_layers": self.layers,
            "num_heads": self.heads,
            "num_kv_heads": self.kv_heads,
            "head_dim": self.head_dim,
            "intermediate_size": self.intermediate,
            "vocab_size": self.vocab,
            "target_hidden_size": self.target_hidden,
            "num_features": self.num_features,
            "rms_norm_eps": self.eps,
            "rope_theta": self.rope_theta,
            "post_norm": self.post_norm,
            "feature_norm": self.feature_norm,
            "window": None,
            "feature_layers": list(self.feature_layers),
        }


TINY_TARGET = TargetSpec(hidden=256, layers=4, heads=4, kv_heads=2, head_dim=64, intermediate=768, vocab=4096)
TINY_DRAFTER = DrafterSpec(hidden=256, layers=1, heads=4, kv_heads=2, head_dim=64, intermediate=768, vocab=4096,
                           target_hidden=256, feature_layers=[1, 2, 3])
Q17_TARGET = TargetSpec(hidden=2048, layers=28, heads=16, kv_heads=8, head_dim=128, intermediate=6144, vocab=151936)
Q17_DRAFTER = DrafterSpec(hidden=2048, layers=1, heads=16, kv_heads=8, head_dim=128, intermediate=6144,
                          vocab=151936, target_hidden=2048, feature_layers=[2, 14, 26])
Q4_TARGET = TargetSpec(hidden=2560, layers=36, heads=32, kv_heads=8, head_dim=128, intermediate=9728, vocab=151936)
Q4_DRAFTER = DrafterSpec(hidden=2560, layers=1, heads=32, kv_heads=8, head_dim=128, intermediate=9728,
                         vocab=151936, target_hidden=2560, feature_layers=[2, 18, 33])

CONFIGS = {
    "c1": (TINY_TARGET, TINY_DRAFTER),
    "c3": (Q17_TARGET, Q17_DRAFTER),
    "c4": (Q4_TARGET, Q4_DRAFTER),
}


def target_tensor_specs(t: TargetSpec) -> list[tuple[str, tuple[int, ...], bool]]:
    """(name, shape, is_norm) in the fixed generation order."""
    H, D = t.hidden, t.head_dim
    out = [("model.embed_tokens.weight", (t.vocab, H), False)]
    for i in range(t.layers):
        p = f"model.layers.{i}."
        out += [
            (p + "self_attn.q_proj.weight", (t.heads * D, H), False),
            (p + "self_attn.k_proj.weight", (t.kv_heads * D, H), False),
            (p + "self_attn.v_proj.weight", (t.kv_heads * D, H), False),
            (p + "self_attn.o_proj.weight", (H, t.heads * D), False),
            (p + "self_attn.q_norm.weight", (D,), True),
            (p + "self_attn.k_norm.weight", (D,), True),
            (p + "input_layernorm.weight", (H,), True),
            (p + "post_attention_layernorm.weight", (H,), True),
            (p + "mlp.gate_proj.weight", (t.intermediate, H), False),
            (p + "mlp.up_proj.weight", (t.intermediate, H), False),
            (p + "mlp.down_proj.weight", (H, t.intermediate), False),
        ]
    out.append(("model.norm.weight", (H,), True))
    if not t.tie_embeddings:
        out.append(("lm_head.weight", (t.vocab, H), False))
    return out


def drafter_tensor_specs(d: DrafterSpec) -> list[tuple[str, tuple[int, ...], bool]]:
    H, D = d.hidden, d.head_dim
    out = [("embed_tokens.weight", (d.vocab, H), False),
           ("fc.weight", (H, d.num_features * d.target_hidden), False)]
    if d.feature_norm:
        out += [(f"feature_norms.{i}.weight", (d.target_hidden,), True) for i in range(d.num_features)]
    for i in range(d.layers):
        p = f"layers.{i}."
        out += [
            (p + "self_attn.q_proj.weight", (d.heads * D, H), False),
            (p + "self_attn.k_proj.weight", (d.kv_heads * D, H), False),
            (p + "self_attn.v_proj.weight", (d.kv_heads * D, H), False),
            (p + "self_attn.o_proj.weight", (H, d.heads * D), False),
            (p + "self_attn.q_norm.weight", (D,), True),
            (p + "self_attn.k_norm.weight", (D,), True),
            (p + "input_layernorm.weight", (H,), True),
            (p + "post_attention_layernorm.weight", (H,), True),
            (p + "mlp.gate_proj.weight", (d.intermediate, H), False),
            (p + "mlp.up_proj.weight", (d.intermediate, H), False),
            (p + "mlp.down_proj.weight", (H, d.intermediate), False),
        ]
        if i == 0:
            out += [
                (p + "self_attn.aux_q.weight", (d.heads * D, H), False),
                (p + "self_attn.aux_k.weight", (d.kv_heads * D, H), False),
                (p + "self_attn.aux_v.weight", (d.kv_heads * D, H), False),
                (p + "aux_norm.weight", (H,), True),
            ]
    out += [("norm.weight", (H,), True), ("lm_head.weight", (d.vocab, H), False)]
    return out


def generate_weights(specs, seed: int, std: float = 0.02) -> dict[str, np.ndarray]:
    """fp32 weights drawn in spec order from default_rng(seed); norms are ones."""
    rng = np.random.default_rng(seed)
    w = {}
    for name, shape, is_norm in specs:
        if is_norm:
            w[name] = np.ones(shape, np.float32)
        else:
            w[name] = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)
    return w


def write_model(dir_: str | Path, config: dict, weights: dict[str, np.ndarray], dtype: str = "F32") -> Path:
    """config.json + model.safetensors; dtype "F32" or "BF16" (norm gains stay in that dtype too)."""
    d = Path(dir_)
    d.mkdir(parents=True, exist_ok=True)
    (d / "config.json").write_text(json.dumps(config, indent=1))
    tens = {}
    for k, v in weights.items():
        tens[k] = ("BF16", st.f32_to_bf16_bits(v)) if dtype == "BF16" else ("F32", v)
    st.save(d / "model.safetensors", tens, metadata={"format": "pt"})
    return d


def round_to_bf16(weights: dict[str, np.ndarray]) -> dict[str, np.ndarray]:
    """The fp32 values a bf16 checkpoint of these weights holds."""
    return {k: st.bf16_bits_to_f32(st.f32_to_bf16_bits(v)).reshape(v.shape) for k, v in weights.items()}


def make_pair(root: str | Path, cfg: str = "c1", seed: int = 0, dtype: str = "F32",
              target_spec: TargetSpec | None = None, drafter_spec: DrafterSpec | None = None):
    """Write target/ and drafter/ under root. Returns (target_dir, drafter_dir, target_w, drafter_w)
    with the fp32 values actually stored (bf16-rounded when dtype is BF16)."""
    ts, ds = CONFIGS[cfg] if cfg in CONFIGS else (None, None)
    ts = target_spec or ts
    ds = drafter_spec or ds
    tw = generate_weights(target_tensor_specs(ts), seed)
    dw = generate_weights(drafter_tensor_specs(ds), seed + 1)
    root = Path(root)
    td = write_model(root / "target", ts.hf_config(), tw, dtype)
    dd = write_model(root / "drafter", ds.config(), dw, dtype)
    if dtype == "BF16":
        tw, dw = round_to_bf16(tw), round_to_bf16(dw)
    return td, dd, tw, dw


def trimmed_vocab_ids(vocab: int, k: int, seed: int = 0, always=QWEN3_EOS) -> np.ndarray:
    """A seeded permutation subset of [0, vocab) of size k, sorted ascending, with the
    `always` ids forced in (the shape of vocab.py:35-47's output)."""
    always = sorted(a for a in set(always) if a < vocab)
    rng = np.random.default_rng(seed)
    perm = rng.permutation(vocab)
    forced = np.zeros(vocab, bool)
    forced[always] = True
    rest = perm[~forced[perm]][: k - len(always)]
    return np.sort(np.concatenate([np.array(always, np.int64), rest])).astype(np.int32)


def prompt_ids(n: int, vocab: int, seed: int = 0) -> list[int]:
    return np.random.default_rng(seed).integers(0, vocab, n).tolist()


def spec_dict(x) -> dict:
    return asdict(x)


def device_weight_stream(specs, seed: int, device="cuda", std: float = 0.02):
    """(name, bf16 tensor on `device`) in spec order from a seeded torch generator on the device:
    the fast path for the billion-parameter configs. Norm gains are ones. The same seed yields
    the same tensors on every B200, so the reference's model files can be regenerated from it."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    for name, shape, is_norm in specs:
        if is_norm:
            yield name, torch.ones(shape, dtype=torch.bfloat16, device=device)
        else:
            yield name, (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std).to(torch.bfloat16)


def write_device_model(dir_: str | Path, config: dict, specs, seed: int, device="cuda") -> Path:
    """config.json + model.safetensors (bf16) holding the tensors of device_weight_stream(specs,
    seed, device): the same seeded weights the device-built models use, as files the
    reference's C++ core loads."""
    import torch

    d = Path(dir_)
    d.mkdir(parents=True, exist_ok=True)
    (d / "config.json").write_text(json.dumps(config))
    stream = device_weight_stream(specs, seed=seed, device=device)

    def produce(name):
        n, w = next(stream)
        assert n == name
        return w.view(torch.int16).cpu().numpy().view("uint16")

    st.save_streaming(d / "model.safetensors", [(n, "BF16", s) for n, s, _ in specs], produce)
    return d
