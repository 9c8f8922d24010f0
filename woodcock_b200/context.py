"""Device context: one native wc_ctx per GPU, bound to a dedicated CUDA stream.

PyTorch provides the device memory of caller-owned buffers and the stream; the
native library does the compute. Calls that read torch tensors run inside
``Context.enter()``, which orders the context stream after the caller's current
stream and the caller's stream after the work it enqueued.
"""

from __future__ import annotations

import ctypes as C
from contextlib import contextmanager

import torch

from ._lib import check, lib


class Context:
    _by_device: dict[int, "Context"] = {}

    def __init__(self, device: int = 0):
        if not torch.cuda.is_available():
            raise RuntimeError("woodcock_b200 needs a CUDA device (sm_100)")
        self.device = torch.device("cuda", device)
        self.stream = torch.cuda.Stream(device=self.device)
        h = C.c_void_p()
        st = lib().wc_ctx_create(device, C.c_void_p(self.stream.cuda_stream), C.byref(h))
        if st != 0:
            msg = lib().wc_last_error(h).decode() if h else ""
            if h:
                lib().wc_ctx_destroy(h)
            raise RuntimeError(f"wc_ctx_create failed ({st}): {msg}")
        self.h = h

    @classmethod
    def get(cls, device: int | torch.device | None = None) -> "Context":
        if isinstance(device, torch.device):
            device = device.index or 0
        device = 0 if device is None else int(device)
        if device not in cls._by_device:
            cls._by_device[device] = cls(device)
        return cls._by_device[device]

    def check(self, status: int) -> None:
        check(status, self.h)

    @contextmanager
    def enter(self, *tensors: torch.Tensor):
        cur = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(cur)
        for t in tensors:
            if isinstance(t, torch.Tensor) and t.is_cuda:
                t.record_stream(self.stream)
        with torch.cuda.stream(self.stream):
            yield self
        cur.wait_stream(self.stream)

    def synchronize(self) -> None:
        self.check(lib().wc_ctx_synchronize(self.h))

    def launch_count(self) -> int:
        return int(lib().wc_ctx_launch_count(self.h))


def ptr(t: torch.Tensor | None) -> C.c_void_p:
    if t is None:
        return C.c_void_p(None)
    if not t.is_contiguous():
        raise ValueError("tensor must be contiguous")
    return C.c_void_p(t.data_ptr())


def device_ints(values, device) -> torch.Tensor:
    if isinstance(values, torch.Tensor):
        return values.to(device=device, dtype=torch.int32).contiguous().reshape(-1)
    return torch.tensor([int(v) for v in values], dtype=torch.int32, device=device)
