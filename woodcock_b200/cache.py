"""KV cache handle (include/woodcock/cache.h:9-28; mlx-lm KVCache + compact_cache in
python/woodcock/target.py:159-175). The arena has a fixed capacity on the device,
laid out [layer][kv_head][capacity][head_dim] in the model dtype."""

from __future__ import annotations

import ctypes as C

import torch

from ._lib import int_array, lib
from .context import Context, ptr


class KVCache:
    def __init__(self, handle: C.c_void_p, ctx: Context, layers: int, kv_heads: int, head_dim: int, owned=True):
        self.h, self.ctx = handle, ctx
        self.layers, self.kv_heads, self.head_dim = layers, kv_heads, head_dim
        self._owned = owned

    @classmethod
    def create(cls, layers, kv_heads, head_dim, capacity, dtype: int, device=0) -> "KVCache":
        ctx = Context.get(device)
        h = C.c_void_p()
        ctx.check(lib().wc_kv_create(ctx.h, layers, kv_heads, head_dim, capacity, dtype, C.byref(h)))
        return cls(h, ctx, layers, kv_heads, head_dim)

    def __del__(self):
        if getattr(self, "_owned", False) and self.h:
            lib().wc_kv_destroy(self.h)
            self.h = None

    def size(self) -> int:
        return int(lib().wc_kv_size(self.h))

    @property
    def offset(self) -> int:
        return self.size()

    @offset.setter
    def offset(self, n: int) -> None:
        self.trim_to(n)

    def capacity(self) -> int:
        return int(lib().wc_kv_capacity(self.h))

    def append(self, layer: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """k, v: [L][kv_heads][head_dim] fp32 on the device, written at [size, size+L)."""
        k = k.to(torch.float32).contiguous()
        v = v.to(torch.float32).contiguous()
        with self.ctx.enter(k, v):
            self.ctx.check(lib().wc_kv_append(self.h, layer, ptr(k), ptr(v), k.shape[0]))

    def commit(self, L: int) -> None:
        self.ctx.check(lib().wc_kv_commit(self.h, L))

    def trim_to(self, n: int) -> None:
        self.ctx.check(lib().wc_kv_trim_to(self.h, n))

    def compact(self, start: int, keep: list[int]) -> None:
        """Rows start + keep[i] -> start + i (kv_cache.cpp:21-31), alias-safe on the device."""
        with self.ctx.enter():
            self.ctx.check(lib().wc_kv_compact(self.h, start, int_array(keep), len(keep)))

    def read(self, layer: int, T: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """(K, V) rows [0, T) of one layer as [T][kv_heads][head_dim] fp32."""
        T = self.size() if T is None else T
        k = torch.empty((T, self.kv_heads, self.head_dim), dtype=torch.float32, device=self.ctx.device)
        v = torch.empty_like(k)
        with self.ctx.enter(k, v):
            self.ctx.check(lib().wc_kv_read(self.h, layer, T, ptr(k), ptr(v)))
        return k, v


def compact_cache(cache: KVCache, start: int, keep: list[int]) -> None:
    """python/woodcock/target.py:159-175."""
    cache.compact(start, keep)
