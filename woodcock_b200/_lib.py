"""ctypes binding of libwoodcock_b200.so (the C ABI in include/woodcock_b200.h).

There is no fallback: if the native library is missing or cannot be loaded, every
entry point raises. Build it with ``python -m woodcock_b200.build``.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libwoodcock_b200.so"

WC_OK, WC_ERR_INVALID, WC_ERR_IO, WC_ERR_CUDA, WC_ERR_OOM, WC_ERR_CAPACITY, WC_ERR_DEVICE, WC_ERR_UNSUPPORTED = range(8)
WC_F32, WC_BF16 = 0, 1
STATUS_NAMES = {0: "OK", 1: "INVALID", 2: "IO", 3: "CUDA", 4: "OOM", 5: "CAPACITY", 6: "DEVICE", 7: "UNSUPPORTED"}


class WcError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"[{STATUS_NAMES.get(status, status)}] {msg}")
        self.status = status


class WcValueError(WcError, ValueError):
    """Argument / configuration errors surface as ValueError, as in the reference's Python API."""


class Qwen3Config(C.Structure):
    _fields_ = [("hidden", C.c_int), ("layers", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int),
                ("head_dim", C.c_int), ("intermediate", C.c_int), ("vocab", C.c_int), ("eps", C.c_float),
                ("rope_theta", C.c_float), ("tie_embeddings", C.c_int)]


class DrafterConfig(C.Structure):
    _fields_ = [("hidden", C.c_int), ("layers", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int),
                ("head_dim", C.c_int), ("intermediate", C.c_int), ("vocab", C.c_int), ("target_hidden", C.c_int),
                ("num_features", C.c_int), ("eps", C.c_float), ("rope_theta", C.c_float), ("post_norm", C.c_int),
                ("feature_norm", C.c_int), ("window", C.c_int)]


class SamplingParamsC(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int), ("top_p", C.c_float), ("seed", C.c_uint64)]


class GenStatsC(C.Structure):
    _fields_ = [("prompt_tokens", C.c_int), ("new_tokens", C.c_int), ("rounds", C.c_int), ("accepted", C.c_long),
                ("verified", C.c_long), ("t_prefill", C.c_double), ("t_draft", C.c_double),
                ("t_verify", C.c_double), ("t_update", C.c_double), ("t_total", C.c_double)]


P = C.c_void_p
I32P = C.POINTER(C.c_int)
I64P = C.POINTER(C.c_int64)
S = C.c_int  # wc_status

# name -> (restype, argtypes)
SIGNATURES = {
    "wc_ctx_create": (S, [C.c_int, P, C.POINTER(P)]),
    "wc_ctx_set_stream": (S, [P, P]),
    "wc_ctx_destroy": (None, [P]),
    "wc_last_error": (C.c_char_p, [P]),
    "wc_ctx_synchronize": (S, [P]),
    "wc_ctx_launch_count": (C.c_uint64, [P]),
    "wc_weight_create": (S, [P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(P)]),
    "wc_weight_destroy": (None, [P]),
    "wc_linear": (S, [P, P, C.c_int, C.c_int, P, P, C.c_int]),
    "wc_rmsnorm": (S, [P, P, P, C.c_int, C.c_int, P, C.c_float]),
    "wc_rope": (S, [P, P, C.c_int, C.c_int, C.c_int, P, C.c_float]),
    "wc_silu_mul": (S, [P, P, P, C.c_int64]),
    "wc_attention": (S, [P, P, C.c_int, C.c_int, C.c_int, C.c_int, P, P, C.c_int, C.c_int, P, P, C.c_float]),
    "wc_softmax": (S, [P, P, C.c_int]),
    "wc_argmax_rows": (S, [P, P, C.c_int, C.c_int, P]),
    "wc_kv_create": (S, [P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(P)]),
    "wc_kv_destroy": (None, [P]),
    "wc_kv_size": (C.c_int, [P]),
    "wc_kv_capacity": (C.c_int, [P]),
    "wc_kv_append": (S, [P, C.c_int, P, P, C.c_int]),
    "wc_kv_commit": (S, [P, C.c_int]),
    "wc_kv_trim_to": (S, [P, C.c_int]),
    "wc_kv_compact": (S, [P, C.c_int, I32P, C.c_int]),
    "wc_kv_read": (S, [P, C.c_int, C.c_int, P, P]),
    "wc_target_load": (S, [P, C.c_char_p, I32P, C.c_int, C.POINTER(P)]),
    "wc_target_create": (S, [P, C.POINTER(Qwen3Config), I32P, C.c_int, C.POINTER(P)]),
    "wc_target_set_tensor": (S, [P, C.c_char_p, P, C.c_int, C.c_int, I64P, C.c_int]),
    "wc_target_finalize": (S, [P]),
    "wc_target_destroy": (None, [P]),
    "wc_target_config": (S, [P, C.POINTER(Qwen3Config), I32P, I32P]),
    "wc_target_make_cache": (S, [P, C.c_int, C.POINTER(P)]),
    "wc_target_forward": (S, [P, P, P, C.c_int, P, P, C.c_int, P, P, P]),
    "wc_drafter_load": (S, [P, C.c_char_p, C.c_int, C.POINTER(P)]),
    "wc_drafter_create": (S, [P, C.POINTER(DrafterConfig), C.c_int, C.POINTER(P)]),
    "wc_drafter_set_tensor": (S, [P, C.c_char_p, P, C.c_int, C.c_int, I64P, C.c_int]),
    "wc_drafter_finalize": (S, [P]),
    "wc_drafter_destroy": (None, [P]),
    "wc_drafter_config_get": (S, [P, C.POINTER(DrafterConfig), I32P, I32P]),
    "wc_drafter_restrict_vocab": (S, [P, I32P, C.c_int]),
    "wc_drafter_make_cache": (S, [P, C.c_int, C.POINTER(P)]),
    "wc_drafter_fuse": (S, [P, P, C.c_int, P]),
    "wc_drafter_forward": (S, [P, P, P, C.c_int, P, P, P, P, P]),
    "wc_drafter_logits": (S, [P, P, C.c_int, P]),
    "wc_drafter_head_argmax": (S, [P, P, C.c_int, P]),
    "wc_accept_greedy": (S, [P, P, P, P, C.c_int, P, P, P]),
    "wc_accept_stochastic": (S, [P, P, P, C.c_int, P, P, C.c_int, C.c_uint64, C.c_uint64, P, P, P, P]),
    "wc_accept_stochastic_noalloc": (S, [P, P, P, C.c_int, P, P, C.c_int, C.c_uint64, C.c_uint64, P, P, P, P]),
    "wc_philox_uniforms": (S, [P, C.c_uint64, C.c_uint64, C.c_int, P]),
    "wc_probs_from_logits": (S, [P, P, C.c_int, C.c_int, C.c_float, C.c_int, C.c_float, P]),
    "wc_decoder_create": (S, [P, P, C.c_int, C.c_int, C.POINTER(P)]),
    "wc_decoder_destroy": (None, [P]),
    "wc_decoder_prefill": (S, [P, I32P, C.c_int, C.POINTER(SamplingParamsC), I32P]),
    "wc_ctx_wait_selftest": (S, [P, C.c_int]),
    "wc_drafter_head_softmax": (S, [P, P, C.c_int, C.c_float, P]),
    "wc_decoder_set_forced": (S, [P, I32P, C.c_int]),
    "wc_decoder_round": (S, [P, C.c_int, I32P, I32P]),
    "wc_decoder_tree_round": (S, [P, C.c_int, C.c_int, C.c_int, I32P, I32P]),
    "wc_decoder_set_forced_tree": (S, [P, I32P, I32P, C.c_int]),
    "wc_decoder_tree_nodes": (S, [P, C.c_int, I32P, I32P, I32P, I32P, P, I32P, I32P]),
    "wc_decoder_generate": (S, [P, I32P, C.c_int, C.c_int, C.c_int, C.POINTER(SamplingParamsC), I32P, C.c_int,
                                I32P, I32P, C.POINTER(GenStatsC)]),
    "wc_generate_autoregressive": (S, [P, I32P, C.c_int, C.c_int, C.POINTER(SamplingParamsC), I32P, C.c_int,
                                       C.c_int, I32P, I32P, C.POINTER(GenStatsC)]),
    "wc_decoder_profile_round": (S, [P, C.c_int, I32P, I32P, C.POINTER(C.c_float), I32P]),
    "wc_decoder_state": (S, [P, I32P, I32P]),
    "wc_decoder_target_cache": (P, [P]),
    "wc_decoder_drafter_cache": (P, [P]),
    "wc_decoder_last_round_ms": (S, [P, C.POINTER(C.c_float)]),
    "wc_target_prompt_forward": (S, [P, P, P, C.c_int, P, P]),
    "wc_batch_create": (S, [P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(P)]),
    "wc_batch_destroy": (None, [P]),
    "wc_batch_set_prefix": (S, [P, C.c_int, P, C.c_int]),
    "wc_batch_fill_synthetic": (S, [P, C.c_int, C.c_int, C.c_uint64]),
    "wc_batch_verify": (S, [P, C.c_int, C.c_int, P, P, P, P]),
    "wc_batch_verify_profiled": (S, [P, C.c_int, C.c_int, P, P, P, P, P]),
    "wc_batch_commit": (S, [P, C.c_int, P, P, C.c_int]),
    "wc_batch_lens": (S, [P, C.c_int, P]),
    "wc_batch_read_kv": (S, [P, C.c_int, C.c_int, C.c_int, P, P]),
    "wc_gemm_bf16": (S, [P, P, P, P, C.c_int, C.c_int, C.c_int, P]),
    "wc_decoder_save_state": (S, [P]),
    "wc_decoder_restore_state": (S, [P]),
    "wc_decoder_round_logits": (S, [P, C.c_int, P, P, I32P, C.POINTER(C.c_uint64)]),
    "wc_decoder_draft_proposals": (S, [P, C.c_int, I32P, P]),
}

_lib = None


def lib() -> C.CDLL:
    """The loaded native library. Raises if it is absent: there is no CPU fallback."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m woodcock_b200.build`")
        lib_ = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(lib_, name)
            f.restype = res
            f.argtypes = args
        _lib = lib_
    return _lib


def check(status: int, ctx_handle=None) -> None:
    if status == WC_OK:
        return
    msg = lib().wc_last_error(ctx_handle).decode() if ctx_handle else ""
    if status in (WC_ERR_INVALID, WC_ERR_UNSUPPORTED):
        raise WcValueError(status, msg)
    raise WcError(status, msg)


def int_array(values) -> C.Array:
    vals = [int(v) for v in values]
    return (C.c_int * max(1, len(vals)))(*vals)
