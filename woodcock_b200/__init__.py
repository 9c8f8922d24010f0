"""woodcock_b200: a B200-native speculative-decoding round (sm_100a CUDA behind a C ABI).

Mirrors the Python API of AtomicBot-ai/woodcock (python/woodcock/{target,drafter,
sampling,policies,spec}.py). Importing the package does not touch the GPU; the
native library (woodcock_b200/lib/libwoodcock_b200.so, built by
``python -m woodcock_b200.build``) is loaded on first use and its absence is an error.
"""

from .policies import CostAwareChain, Plan, Policy, StaticPolicy
from .sampling import DraftTree, PhiloxStream, SamplingParams, tree_attention_mask

__all__ = [
    "CostAwareChain", "DraftTree", "Drafter", "GenStats", "KVCache", "PhiloxStream", "Plan", "Policy",
    "SamplingParams", "SpeculativeDecoder", "StaticPolicy", "Target", "compact_cache", "generate_autoregressive",
    "tree_attention_mask",
]


def __getattr__(name):
    # torch-backed modules load lazily so that host-only users (policies, trees) need no GPU
    if name in ("Target",):
        from .target import Target
        return Target
    if name in ("Drafter",):
        from .drafter import Drafter
        return Drafter
    if name in ("KVCache", "compact_cache"):
        from . import cache
        return getattr(cache, name)
    if name in ("SpeculativeDecoder", "GenStats", "generate_autoregressive"):
        from . import spec
        return getattr(spec, name)
    raise AttributeError(name)
