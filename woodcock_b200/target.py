"""Frozen Qwen3 target on the B200 (python/woodcock/target.py:42-116; include/woodcock/model.h).

``Target(tokens, cache, positions, mask)`` runs the native forward: per layer a fused
RMSNorm+QKV projection, q/k-norm + RoPE + KV append + attention in one kernel, the
o-projection with the residual add, RMSNorm+gate/up with the SwiGLU epilogue, and
the down-projection with the residual add; tap layers' block outputs are captured
in the down-projection epilogue. Logits come from the final norm fused into the
(tied) head, with the argmax fused into the same pass.
"""

from __future__ import annotations

import ctypes as C
import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from ._lib import Qwen3Config, int_array, lib, WC_BF16, WC_F32
from .cache import KVCache, compact_cache  # noqa: F401  (re-exported like the reference module)
from .context import Context, device_ints, ptr

QWEN3_EOS = frozenset({151643, 151645})


def _taps_arg(feature_layers):
    """Three tap layer indices for the C ABI (None = the reference default, target.py:26-33)."""
    if feature_layers is None:
        return None
    taps = [int(x) for x in feature_layers]
    if len(taps) != 3:
        raise ValueError(f"the drafter fuses exactly three target layers, got {len(taps)}")
    return int_array(taps)


def default_feature_layers(num_layers: int) -> tuple[int, int, int]:
    """python/woodcock/target.py:26-33."""
    return (2, num_layers // 2, num_layers - 3)


def dtype_code(dtype) -> int:
    if dtype in (None, "bf16", "bfloat16", torch.bfloat16, WC_BF16):
        return WC_BF16
    if dtype in ("fp32", "float32", "f32", torch.float32, WC_F32):
        return WC_F32
    raise ValueError(f"unsupported dtype {dtype!r}")


def _tensor_arg(v):
    """(pointer, dtype code, on_device, keepalive) for a weight given as torch or numpy."""
    if isinstance(v, torch.Tensor):
        if v.dtype == torch.bfloat16:
            code = 1
        elif v.dtype == torch.float32:
            code = 0
        else:
            v = v.float()
            code = 0
        v = v.contiguous()
        return C.c_void_p(v.data_ptr()), code, int(v.is_cuda), v
    a = np.ascontiguousarray(v)
    if a.dtype == np.uint16:
        code = 1
    else:
        a = a.astype(np.float32)
        code = 0
    return C.c_void_p(a.ctypes.data), code, 0, a


@dataclass
class TargetOutput:
    logits: torch.Tensor | None  # (1, L, V) fp32
    features: list[torch.Tensor]  # each (1, L, hidden): residual stream at the taps
    argmax: torch.Tensor | None = None  # (L,) int32


class Target:
    def __init__(self, handle: C.c_void_p, ctx: Context):
        self.h, self.ctx = handle, ctx
        cfg, taps, dt = Qwen3Config(), (C.c_int * 3)(), C.c_int()
        ctx.check(lib().wc_target_config(handle, C.byref(cfg), taps, C.byref(dt)))
        self.cfg = cfg
        self.feature_layers = tuple(int(x) for x in taps)
        self.dtype = int(dt.value)
        self.num_layers = cfg.layers
        self.hidden_size = cfg.hidden
        self.vocab_size = cfg.vocab
        self.eos_token_ids = set(QWEN3_EOS)

    @classmethod
    def load(cls, path: str | Path, feature_layers=None, dtype=None, device=0) -> "Target":
        ctx = Context.get(device)
        if dtype is None:
            dtype = _file_dtype(Path(path))
        h = C.c_void_p()
        taps = _taps_arg(feature_layers)
        ctx.check(lib().wc_target_load(ctx.h, str(path).encode(), taps, dtype_code(dtype), C.byref(h)))
        return cls(h, ctx)

    @classmethod
    def from_weights(cls, config: dict, weights: dict, feature_layers=None, dtype="bf16", device=0) -> "Target":
        """HF-style config dict + {tensor name: torch tensor / numpy array (uint16 = bf16 bits)} or an
        iterable of (name, tensor) pairs, consumed one at a time."""
        ctx = Context.get(device)
        c = Qwen3Config(hidden=config["hidden_size"], layers=config["num_hidden_layers"],
                        heads=config["num_attention_heads"], kv_heads=config["num_key_value_heads"],
                        head_dim=config.get("head_dim") or config["hidden_size"] // config["num_attention_heads"],
                        intermediate=config["intermediate_size"], vocab=config["vocab_size"],
                        eps=float(config.get("rms_norm_eps", 1e-6)), rope_theta=float(config.get("rope_theta", 1e6)),
                        tie_embeddings=int(bool(config.get("tie_word_embeddings", False))))
        h = C.c_void_p()
        taps = _taps_arg(feature_layers)
        ctx.check(lib().wc_target_create(ctx.h, C.byref(c), taps, dtype_code(dtype), C.byref(h)))
        t = cls.__new__(cls)
        try:
            for name, v in (weights.items() if isinstance(weights, dict) else weights):
                p, code, on_dev, keep = _tensor_arg(v)
                shape = (C.c_int64 * keep.ndim)(*keep.shape)
                if on_dev:
                    torch.cuda.current_stream().synchronize()
                ctx.check(lib().wc_target_set_tensor(h, name.encode(), p, code, on_dev, shape, keep.ndim))
            ctx.check(lib().wc_target_finalize(h))
        except Exception:
            lib().wc_target_destroy(h)
            raise
        t.__init__(h, ctx)
        return t

    def __del__(self):
        if getattr(self, "h", None):
            lib().wc_target_destroy(self.h)
            self.h = None

    def make_cache(self, capacity: int = 4096) -> KVCache:
        h = C.c_void_p()
        self.ctx.check(lib().wc_target_make_cache(self.h, capacity, C.byref(h)))
        return KVCache(h, self.ctx, self.cfg.layers, self.cfg.kv_heads, self.cfg.head_dim)

    def __call__(self, tokens, cache: KVCache, positions=None, mask=None, capture: bool = True,
                 logits: bool = True, logits_from: int = 0) -> TargetOutput:
        """tokens: (1, L) / (L,) ints; positions: (L,) absolute RoPE positions (None = cache offset + i);
        mask: (L, offset + L) bool, True = may attend (None = causal)."""
        dev = self.ctx.device
        tok = device_ints(tokens, dev)
        L = tok.numel()
        pos = device_ints(positions, dev) if positions is not None else None
        m = None
        if mask is not None:
            m = torch.as_tensor(np.asarray(mask.cpu() if isinstance(mask, torch.Tensor) else mask, dtype=np.uint8),
                                device=dev).contiguous()
            if tuple(m.shape) != (L, cache.size() + L):
                raise ValueError(f"mask must be ({L}, {cache.size() + L})")
        rows = L - logits_from
        with self.ctx.enter(tok, *(x for x in (pos, m) if x is not None)):
            z = torch.empty((rows, self.vocab_size), dtype=torch.float32, device=dev) if logits else None
            am = torch.empty((rows,), dtype=torch.int32, device=dev) if logits else None
            taps = torch.empty((3, L, self.hidden_size), dtype=torch.float32, device=dev) if capture else None
            self.ctx.check(lib().wc_target_forward(self.h, cache.h, ptr(tok), L, ptr(pos), ptr(m), logits_from,
                                                   ptr(z), ptr(am), ptr(taps)))
        feats = [taps[f][None] for f in range(3)] if capture else []
        return TargetOutput(logits=z[None] if logits else None, features=feats, argmax=am)


def prompt_forward(target: "Target", tokens, cache: KVCache) -> tuple[torch.Tensor, torch.Tensor]:
    """The prefill's target pass on the tensor cores (wc_target_prompt_forward): appends the
    prompt's K/V to `cache`; returns (taps [3][n][hidden], last row's residual [hidden])."""
    dev = target.ctx.device
    tok = device_ints(tokens, dev)
    n = tok.numel()
    taps = torch.empty((3, n, target.hidden_size), dtype=torch.float32, device=dev)
    last = torch.empty((target.hidden_size,), dtype=torch.float32, device=dev)
    with target.ctx.enter(tok, taps, last):
        target.ctx.check(lib().wc_target_prompt_forward(target.h, cache.h, ptr(tok), n, ptr(taps), ptr(last)))
    return taps, last


def apply_rope_positions(x: torch.Tensor, positions, base: float) -> torch.Tensor:
    """Rotate-half RoPE of x[L][heads][D] at per-row positions (target.py:119-139) on the device."""
    from .ops import rope

    return rope(x, positions, base)


def _file_dtype(path: Path) -> str:
    from . import safetensors_io as st

    files = sorted(path.glob("*.safetensors"))
    if not files:
        return "bf16"
    import struct

    with open(files[0], "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n))
    for k, v in header.items():
        if k != "__metadata__":
            return "fp32" if v["dtype"] == "F32" else "bf16"
    del st
    return "bf16"
