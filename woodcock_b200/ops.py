"""Backend ops on the device: the woodcock::ops interface (include/woodcock/ops.h:11-22)
over torch tensors. Every call runs a native sm_100a kernel; nothing falls back to
PyTorch math."""

from __future__ import annotations

import ctypes as C

import torch

from ._lib import WC_BF16, WC_F32, lib
from .context import Context, device_ints, ptr


class Weight:
    """A projection W[out][in] in the library's streaming layout (replaces woodcock::Tensor)."""

    def __init__(self, w: torch.Tensor, dtype=torch.bfloat16, device=0):
        self.ctx = Context.get(device)
        src = w.detach().contiguous()
        if src.dtype not in (torch.float32, torch.bfloat16):
            src = src.float()
        src_code = WC_BF16 if src.dtype == torch.bfloat16 else WC_F32
        code = WC_BF16 if dtype in (torch.bfloat16, "bf16", WC_BF16) else WC_F32
        self.out_rows, self.in_cols = src.shape
        h = C.c_void_p()
        if src.is_cuda:
            torch.cuda.current_stream().synchronize()
            keep = src
            p = C.c_void_p(keep.data_ptr())
        else:
            keep = src.numpy() if src.dtype == torch.float32 else src.view(torch.int16).numpy()
            p = C.c_void_p(keep.ctypes.data)
        self.ctx.check(lib().wc_weight_create(self.ctx.h, p, src_code, int(src.is_cuda), self.out_rows,
                                              self.in_cols, code, C.byref(h)))
        self.h = h

    def __del__(self):
        if getattr(self, "h", None):
            lib().wc_weight_destroy(self.h)
            self.h = None


def linear(x: torch.Tensor, W: Weight, y: torch.Tensor | None = None, accumulate: bool = False) -> torch.Tensor:
    """y[L][out] (+)= x[L][in] . W^T (ops.h:12)."""
    ctx = W.ctx
    x2 = x.reshape(-1, W.in_cols).float().contiguous()
    L = x2.shape[0]
    if y is None:
        if accumulate:
            raise ValueError("accumulate needs y")
        y = torch.empty((L, W.out_rows), dtype=torch.float32, device=ctx.device)
    with ctx.enter(x2, y):
        ctx.check(lib().wc_linear(ctx.h, ptr(x2), L, W.in_cols, W.h, ptr(y), int(accumulate)))
    return y


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """ops.h:14; out may alias x."""
    ctx = Context.get(x.device)
    d = x.shape[-1]
    xc = x.float().contiguous()
    wc = w.float().contiguous().to(x.device)
    y = out if out is not None else torch.empty_like(xc)
    with ctx.enter(xc, wc, y):
        ctx.check(lib().wc_rmsnorm(ctx.h, ptr(xc), ptr(y), xc.numel() // d, d, ptr(wc), float(eps)))
    return y


def rope(x: torch.Tensor, positions, base: float) -> torch.Tensor:
    """ops.h:16, in place on x[L][heads][D] (fp32, contiguous)."""
    ctx = Context.get(x.device)
    if x.dtype != torch.float32 or not x.is_contiguous():
        raise ValueError("rope needs a contiguous fp32 tensor")
    L, heads, D = x.shape
    pos = device_ints(positions, x.device)
    with ctx.enter(x, pos):
        ctx.check(lib().wc_rope(ctx.h, ptr(x), L, heads, D, ptr(pos), float(base)))
    return x


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """ops.h:18, in place on gate."""
    ctx = Context.get(gate.device)
    with ctx.enter(gate, up):
        ctx.check(lib().wc_silu_mul(ctx.h, ptr(gate), ptr(up.contiguous()), gate.numel()))
    return gate


def attention(q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, mask=None, scale: float | None = None) -> torch.Tensor:
    """ops.h:20: q[L][H][D] fp32; K, V [T][Hk][D] fp32 or bf16; mask [L][T] (1 = visible)."""
    ctx = Context.get(q.device)
    L, H, D = q.shape
    T, Hk, _ = K.shape
    kvd = WC_BF16 if K.dtype == torch.bfloat16 else WC_F32
    qc = q.float().contiguous()
    Kc, Vc = K.contiguous(), V.contiguous()
    if kvd == WC_F32:
        Kc, Vc = Kc.float(), Vc.float()
    m = None if mask is None else torch.as_tensor(mask, device=q.device).to(torch.uint8).contiguous()
    out = torch.empty((L, H, D), dtype=torch.float32, device=q.device)
    s = float(scale if scale is not None else D ** -0.5)
    with ctx.enter(qc, Kc, Vc, out, *(x for x in (m,) if x is not None)):
        ctx.check(lib().wc_attention(ctx.h, ptr(qc), L, H, Hk, D, ptr(Kc), ptr(Vc), kvd, T, ptr(m), ptr(out), s))
    return out


def softmax(x: torch.Tensor) -> torch.Tensor:
    """ops.h:22, in place per row (last axis)."""
    ctx = Context.get(x.device)
    if x.dtype != torch.float32 or not x.is_contiguous():
        raise ValueError("softmax needs a contiguous fp32 tensor")
    n = x.shape[-1]
    rows = x.numel() // n
    with ctx.enter(x):
        for r in range(rows):
            ctx.check(lib().wc_softmax(ctx.h, C.c_void_p(x.data_ptr() + 4 * r * n), n))
    return x


def argmax(x: torch.Tensor) -> torch.Tensor:
    """First index of the maximum of each row (sampling.cpp:47)."""
    ctx = Context.get(x.device)
    xc = x.float().contiguous()
    n = xc.shape[-1]
    rows = xc.numel() // n
    out = torch.empty((rows,), dtype=torch.int32, device=x.device)
    with ctx.enter(xc, out):
        ctx.check(lib().wc_argmax_rows(ctx.h, ptr(xc), rows, n, ptr(out)))
    return out.reshape(xc.shape[:-1])
