"""The C ABI surface without a GPU: the native library loads, exports every function
include/woodcock_b200.h declares, and the ctypes binding covers exactly that set.
No compute is called here."""

from __future__ import annotations

import ctypes as C
import re
import subprocess

import pytest

from conftest import REPO

HEADER = REPO / "include" / "woodcock_b200.h"


def declared_functions() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^WC_API\s+[\w\s\*]+?\b(wc_\w+)\s*\(", text, flags=re.M))


@pytest.fixture(scope="module")
def libpath():
    from woodcock_b200 import build

    return build.build()  # no-op when up to date


def test_header_declares_the_boundary():
    fns = declared_functions()
    for required in ("wc_linear", "wc_rmsnorm", "wc_rope", "wc_silu_mul", "wc_attention", "wc_softmax",
                     "wc_kv_create", "wc_kv_append", "wc_kv_commit", "wc_kv_trim_to", "wc_kv_compact", "wc_kv_size",
                     "wc_target_load", "wc_target_forward", "wc_drafter_load", "wc_drafter_fuse",
                     "wc_drafter_forward", "wc_drafter_logits", "wc_drafter_restrict_vocab", "wc_accept_greedy",
                     "wc_accept_stochastic", "wc_decoder_create", "wc_decoder_round", "wc_decoder_generate",
                     "wc_generate_autoregressive"):
        assert required in fns, required


def test_library_exports_every_declared_symbol(libpath):
    lib = C.CDLL(str(libpath))
    missing = [f for f in sorted(declared_functions()) if not hasattr(lib, f)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", str(libpath)], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert declared_functions() <= exported
    # nothing but the C ABI is exported as code
    assert {s for s in exported if not s.startswith("wc_")} <= {"_init", "_fini"}


def test_ctypes_binding_covers_the_header(libpath):
    from woodcock_b200._lib import SIGNATURES, lib

    assert set(SIGNATURES) == declared_functions()
    lib()  # binds every signature


def test_status_codes_without_gpu(libpath):
    """Argument validation happens before any device work: null handles are rejected."""
    from woodcock_b200._lib import WC_ERR_INVALID, lib

    L = lib()
    assert L.wc_linear(None, None, 1, 1, None, None, 0) == WC_ERR_INVALID
    assert L.wc_kv_size(None) == -1
    assert L.wc_decoder_round(None, 4, None, None) == WC_ERR_INVALID
    assert L.wc_last_error(None) == b"null context"
