"""EAGLE-3 drafter on the B200 (python/woodcock/drafter.py:134-229; include/woodcock/drafter.h).

    g_t = FC([RMS_1(f_low); RMS_2(f_mid); RMS_3(f_high)])       (fuse: one GEMV, norms in its prologue)
    QKV = W_main . RMS(h) + W_aux . RMS(embed(x))             (one GEMV over [RMS(h) | RMS(e)], K = 2H)
    out = RMSNorm(h_L) feeds the head and, with post_norm, the next chain step.

The LM head can be restricted to a subset of rows (``restrict_vocab``); head rows
map back to token ids through ``vocab_ids`` on the device, inside the chain.
"""

from __future__ import annotations

import ctypes as C
import json
from pathlib import Path

import numpy as np
import torch

from ._lib import DrafterConfig, int_array, lib
from .cache import KVCache
from .context import Context, device_ints, ptr
from .target import _file_dtype, _tensor_arg, dtype_code


class Drafter:
    def __init__(self, handle: C.c_void_p, ctx: Context):
        self.h, self.ctx = handle, ctx
        self._refresh()
        self._vocab_ids: torch.Tensor | None = None

    def _refresh(self):
        cfg, dt, rows = DrafterConfig(), C.c_int(), C.c_int()
        self.ctx.check(lib().wc_drafter_config_get(self.h, C.byref(cfg), C.byref(dt), C.byref(rows)))
        self.cfg, self.dtype, self.head_rows = cfg, int(dt.value), int(rows.value)
        self.hidden_size, self.vocab_size = cfg.hidden, cfg.vocab

    @classmethod
    def load(cls, path: str | Path, dtype=None, device=0, target=None, vocab=None) -> "Drafter":
        """drafter.py:322-331. A v1 export (woodcock.json) is validated first (format, sha256,
        and the target's hidden size / vocabulary when `target` is given); `vocab` =
        '<counts.npz>:<K>' or an id list restricts the head at load (vocab.py:83-87)."""
        from .export import check_manifest

        check_manifest(path, target.cfg if target is not None else None)
        ctx = Context.get(device)
        if dtype is None:
            dtype = _file_dtype(Path(path))
        h = C.c_void_p()
        ctx.check(lib().wc_drafter_load(ctx.h, str(path).encode(), dtype_code(dtype), C.byref(h)))
        d = cls(h, ctx)
        if vocab is not None:
            from .vocab import load_ids

            d.restrict_vocab(load_ids(vocab) if isinstance(vocab, (str, Path)) else vocab)
        return d

    @classmethod
    def from_weights(cls, config: dict, weights: dict, dtype="bf16", device=0) -> "Drafter":
        ctx = Context.get(device)
        if config.get("residual", "feature") != "feature" or config.get("lowrank_rank", 0):
            raise ValueError("unsupported drafter configuration")  # drafter.py:55-63
        c = DrafterConfig(hidden=config["hidden_size"], layers=config["num_layers"], heads=config["num_heads"],
                          kv_heads=config["num_kv_heads"], head_dim=config["head_dim"],
                          intermediate=config["intermediate_size"], vocab=config["vocab_size"],
                          target_hidden=config["target_hidden_size"], num_features=config.get("num_features", 3),
                          eps=float(config.get("rms_norm_eps", 1e-6)), rope_theta=float(config.get("rope_theta", 1e6)),
                          post_norm=int(config.get("post_norm", True)), feature_norm=int(config.get("feature_norm", True)),
                          window=int(config.get("window") or 0))
        h = C.c_void_p()
        ctx.check(lib().wc_drafter_create(ctx.h, C.byref(c), dtype_code(dtype), C.byref(h)))
        try:
            for name, v in (weights.items() if isinstance(weights, dict) else weights):
                p, code, on_dev, keep = _tensor_arg(v)
                shape = (C.c_int64 * keep.ndim)(*keep.shape)
                if on_dev:
                    torch.cuda.current_stream().synchronize()
                ctx.check(lib().wc_drafter_set_tensor(h, name.encode(), p, code, on_dev, shape, keep.ndim))
            ctx.check(lib().wc_drafter_finalize(h))
        except Exception:
            lib().wc_drafter_destroy(h)
            raise
        return cls(h, ctx)

    def __del__(self):
        if getattr(self, "h", None):
            lib().wc_drafter_destroy(self.h)
            self.h = None

    # ------------------------------------------------------------ vocabulary
    @property
    def vocab_ids(self) -> torch.Tensor | None:
        return self._vocab_ids

    def restrict_vocab(self, ids) -> None:
        """drafter.py:217-229. Raises ValueError when already restricted."""
        ids = [int(x) for x in (ids.tolist() if hasattr(ids, "tolist") else ids)]
        self.ctx.check(lib().wc_drafter_restrict_vocab(self.h, int_array(ids), len(ids)))
        self._vocab_ids = torch.tensor(ids, dtype=torch.int32, device=self.ctx.device)
        self._refresh()

    def token_ids(self, rows):
        """Head rows -> token ids (drafter.py:213-215)."""
        if self._vocab_ids is None:
            return rows
        if isinstance(rows, torch.Tensor):
            return self._vocab_ids[rows.long()]
        return int(self._vocab_ids[int(rows)])

    def save(self, path):
        if self._vocab_ids is not None:
            raise ValueError("a drafter with a restricted vocabulary cannot be saved")
        raise NotImplementedError("weights live on the device in their streaming layout; export the source "
                                  "directory with woodcock_b200.export.export_drafter")

    # ------------------------------------------------------------ compute
    def make_cache(self, capacity: int = 4096) -> KVCache:
        h = C.c_void_p()
        self.ctx.check(lib().wc_drafter_make_cache(self.h, capacity, C.byref(h)))
        return KVCache(h, self.ctx, self.cfg.layers, self.cfg.kv_heads, self.cfg.head_dim)

    def fuse(self, feats: list[torch.Tensor]) -> torch.Tensor:
        """Target taps (each (1, L, D_t)) -> g (1, L, d)."""
        t = torch.stack([f.reshape(-1, self.cfg.target_hidden).float() for f in feats]).contiguous()
        L = t.shape[1]
        with self.ctx.enter(t):
            g = torch.empty((L, self.hidden_size), dtype=torch.float32, device=self.ctx.device)
            self.ctx.check(lib().wc_drafter_fuse(self.h, ptr(t), L, ptr(g)))
        return g[None]

    def __call__(self, tokens, feat: torch.Tensor, cache: KVCache, positions=None, mask=None):
        """One drafting forward: tokens (1, L), feat (1, L, d) -> (hidden, out), each (1, L, d)."""
        dev = self.ctx.device
        tok = device_ints(tokens, dev)
        L = tok.numel()
        f = feat.reshape(L, self.hidden_size).float().contiguous()
        pos = device_ints(positions, dev) if positions is not None else None
        m = None
        if mask is not None:
            m = torch.as_tensor(np.asarray(mask.cpu() if isinstance(mask, torch.Tensor) else mask, dtype=np.uint8),
                                device=dev).contiguous()
        with self.ctx.enter(tok, f, *(x for x in (pos, m) if x is not None)):
            hid = torch.empty((L, self.hidden_size), dtype=torch.float32, device=dev)
            out = torch.empty_like(hid)
            self.ctx.check(lib().wc_drafter_forward(self.h, cache.h, ptr(tok), L, ptr(f), ptr(pos), ptr(m),
                                                    ptr(hid), ptr(out)))
        return hid[None], out[None]

    def feedback(self, hidden, out):
        return out if self.cfg.post_norm else hidden

    def logits(self, out: torch.Tensor) -> torch.Tensor:
        """Logits over the head rows (full vocabulary or the restricted subset)."""
        shape = out.shape[:-1]
        x = out.reshape(-1, self.hidden_size).float().contiguous()
        with self.ctx.enter(x):
            z = torch.empty((x.shape[0], self.head_rows), dtype=torch.float32, device=self.ctx.device)
            self.ctx.check(lib().wc_drafter_logits(self.h, ptr(x), x.shape[0], ptr(z)))
        return z.reshape(*shape, self.head_rows)

    def head_softmax(self, out: torch.Tensor, temperature: float = 1.0) -> torch.Tensor:
        """The draft distribution softmax(logits / T) over the head rows (spec.py:113-125)."""
        shape = out.shape[:-1]
        x = out.reshape(-1, self.hidden_size).float().contiguous()
        with self.ctx.enter(x):
            q = torch.empty((x.shape[0], self.head_rows), dtype=torch.float32, device=self.ctx.device)
            self.ctx.check(lib().wc_drafter_head_softmax(self.h, ptr(x), x.shape[0], float(temperature), ptr(q)))
        return q.reshape(*shape, self.head_rows)

    def head_argmax(self, out: torch.Tensor) -> torch.Tensor:
        """Fused head + argmax, mapped to token ids."""
        x = out.reshape(-1, self.hidden_size).float().contiguous()
        with self.ctx.enter(x):
            tok = torch.empty((x.shape[0],), dtype=torch.int32, device=self.ctx.device)
            self.ctx.check(lib().wc_drafter_head_argmax(self.h, ptr(x), x.shape[0], ptr(tok)))
        return tok


def load_config(path: str | Path) -> dict:
    return json.loads((Path(path) / "config.json").read_text())
