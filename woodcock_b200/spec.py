"""Speculative decoding engine, batch size 1 (python/woodcock/spec.py:104-397;
include/woodcock/spec.h; src/core/spec.cpp:235-311).

State between rounds lives on the device (n = committed tokens before x_n = target
cache size; drafter cache of real entries 0..n-1; the root drafter output). One
chain round is one CUDA-graph replay:

  K drafter heads (fused argmax, rows mapped to token ids) and K-1 drafter layer
  passes -> target verification of [x_n, d_1..d_K] with tap capture -> acceptance
  (longest matching prefix + the target's token) -> chain compaction (rewind) ->
  drafter update on the accepted rows,

followed by the round's single host synchronisation, which returns the emitted tokens.
With temperature > 0 (SamplingParams given to the prefill / generate) the same graph
shape samples: each head draws its draft from softmax(z / T) (Gumbel-max in the
epilogue, Philox noise) and keeps its logits; verification keeps the target logits and
the acceptance kernel applies verify_tree_stochastic's chain rule (sampling.py:143-187)
with a Gumbel-max draw from the residual or the bonus row.
"""

from __future__ import annotations

import ctypes as C
import time
from dataclasses import dataclass, field

import numpy as np

from ._lib import GenStatsC, SamplingParamsC, WcValueError, WC_ERR_UNSUPPORTED, int_array, lib
from .cache import KVCache
from .drafter import Drafter
from .policies import Policy, StaticPolicy
from .sampling import SamplingParams
from .target import Target


@dataclass
class GenStats:
    prompt_tokens: int = 0
    new_tokens: int = 0
    rounds: int = 0
    accepted: list[int] = field(default_factory=list)
    drafted: list[int] = field(default_factory=list)
    depths: list[int] = field(default_factory=list)
    t_prefill: float = 0.0
    t_draft: float = 0.0
    t_verify: float = 0.0
    t_update: float = 0.0
    t_total: float = 0.0
    fused: bool = False
    round_ms_device: list[float] = field(default_factory=list)

    @property
    def mean_accepted(self) -> float:
        return float(np.mean(self.accepted)) if self.accepted else 0.0

    @property
    def tokens_per_round(self) -> float:
        return self.mean_accepted + 1.0

    @property
    def acceptance_rate(self) -> float:
        d = sum(self.drafted)
        return sum(self.accepted) / d if d else 0.0

    @property
    def decode_tps(self) -> float:
        t = self.t_total - self.t_prefill
        return (self.new_tokens - 1) / t if t > 0 else 0.0

    def as_dict(self) -> dict:
        return {
            "prompt_tokens": self.prompt_tokens, "new_tokens": self.new_tokens, "rounds": self.rounds,
            "mean_accepted": self.mean_accepted, "tokens_per_round": self.tokens_per_round,
            "acceptance_rate": self.acceptance_rate,
            "mean_verified": float(np.mean(self.drafted)) if self.drafted else 0.0,
            "mean_depth": float(np.mean(self.depths)) if self.depths else 0.0,
            "t_prefill": self.t_prefill, "t_draft": self.t_draft, "t_verify": self.t_verify,
            "t_update": self.t_update, "t_total": self.t_total, "fused": self.fused, "decode_tps": self.decode_tps,
        }


def _sp_c(sp: SamplingParams) -> SamplingParamsC:
    return SamplingParamsC(float(sp.temperature), int(sp.top_k), float(sp.top_p), int(sp.seed))


class SpeculativeDecoder:
    def __init__(self, target: Target, drafter: Drafter, policy: Policy, fused: bool = True,
                 max_context: int = 8192, max_k: int = 8):
        if target.ctx is not drafter.ctx:
            raise ValueError("target and drafter must live on the same device")
        self.t, self.d, self.policy, self.fused = target, drafter, policy, fused
        self.ctx = target.ctx
        self.max_context, self.max_k = max_context, max_k
        h = C.c_void_p()
        self.ctx.check(lib().wc_decoder_create(target.h, drafter.h, max_context, max_k, C.byref(h)))
        self.h = h
        # oracle-drafter hook: forced(round, k, emitted) -> k tokens that replace d_1..d_k after
        # the drafter computed them (the OracleDecoder pattern of tests/test_spec_model.py:59-92)
        self.forced = None
        # the same for tree rounds: forced_tree(round, emitted) -> (tokens, parents)
        self.forced_tree = None

    def __del__(self):
        if getattr(self, "h", None):
            lib().wc_decoder_destroy(self.h)
            self.h = None

    # ---------------------------------------------------------------- device state
    def state(self) -> tuple[int, int]:
        n, dl = C.c_int(), C.c_int()
        self.ctx.check(lib().wc_decoder_state(self.h, C.byref(n), C.byref(dl)))
        return n.value, dl.value

    def target_cache(self) -> KVCache:
        t = self.t.cfg
        return KVCache(lib().wc_decoder_target_cache(self.h), self.ctx, t.layers, t.kv_heads, t.head_dim, owned=False)

    def drafter_cache(self) -> KVCache:
        d = self.d.cfg
        return KVCache(lib().wc_decoder_drafter_cache(self.h), self.ctx, d.layers, d.kv_heads, d.head_dim, owned=False)

    def prefill(self, prompt: list[int], sp: SamplingParams = SamplingParams()) -> int:
        first = C.c_int()
        arr = int_array(prompt)
        self.ctx.check(lib().wc_decoder_prefill(self.h, arr, len(prompt), C.byref(_sp_c(sp)), C.byref(first)))
        return first.value

    def set_forced(self, tokens: list[int] | None) -> None:
        toks = list(tokens or [])
        self.ctx.check(lib().wc_decoder_set_forced(self.h, int_array(toks) if toks else None, len(toks)))

    def round(self, k: int) -> list[int]:
        """One fused chain round (sampled after a prefill with temperature > 0); returns d_1..d_a, next."""
        out = (C.c_int * (k + 1))()
        n = C.c_int()
        self.ctx.check(lib().wc_decoder_round(self.h, k, out, C.byref(n)))
        return list(out[: n.value])

    def tree_round(self, depth: int, width: int, budget: int) -> list[int]:
        """One greedy draft-tree round on the device (StaticPolicy(depth, width, budget) shape);
        returns d_1..d_a, next."""
        out = (C.c_int * (depth + 1))()
        n = C.c_int()
        self.ctx.check(lib().wc_decoder_tree_round(self.h, depth, width, budget, out, C.byref(n)))
        return list(out[: n.value])

    def set_forced_tree(self, tokens: list[int] | None, parents: list[int] | None = None) -> None:
        """Oracle-drafter mode for trees: the next tree rounds verify this tree (node 0 = the round's
        root, its token ignored) instead of the drafted one. None clears it."""
        if tokens is None:
            self.ctx.check(lib().wc_decoder_set_forced_tree(self.h, None, None, 0))
            return
        self.ctx.check(lib().wc_decoder_set_forced_tree(self.h, int_array(tokens), int_array(parents), len(tokens)))

    def tree_nodes(self) -> dict:
        """The last tree round's nodes (test support): tokens, parents, the drafter's own proposal
        and its logit at each node it ran on (-1 elsewhere), and the node of each verify row."""
        cap = 128
        n, nv = C.c_int(), C.c_int()
        tok, par, prop, ver = ((C.c_int * cap)() for _ in range(4))
        z = np.zeros(cap, dtype=np.float32)
        self.ctx.check(lib().wc_decoder_tree_nodes(self.h, cap, C.byref(n), tok, par, prop, z.ctypes.data, ver,
                                                   C.byref(nv)))
        k = n.value
        return {"tokens": list(tok[:k]), "parents": list(par[:k]), "proposals": list(prop[:k]),
                "proposal_logits": [float(x) for x in z[:k]], "verified": list(ver[: nv.value])}

    PROFILE_KINDS = ("target_qkv", "attention", "target_o", "target_gate_up", "target_down", "target_head",
                     "drafter_head", "drafter_layer")

    def profile_round(self, k: int) -> tuple[list[int], dict]:
        """A real round replayed from an instrumented graph: mean device ms per kernel class."""
        out = (C.c_int * (k + 1))()
        n = C.c_int()
        ms = (C.c_float * 16)()
        cnt = (C.c_int * 16)()
        self.ctx.check(lib().wc_decoder_profile_round(self.h, k, out, C.byref(n), ms, cnt))
        prof = {name: {"mean_ms": (ms[i] / cnt[i]) if cnt[i] else 0.0, "launches": cnt[i]}
                for i, name in enumerate(self.PROFILE_KINDS)}
        return list(out[: n.value]), prof

    # ---------------------------------------------------------------- test / measurement support
    def save_state(self) -> None:
        """Snapshot the device state (round state, chain root) after a prefill or round."""
        self.ctx.check(lib().wc_decoder_save_state(self.h))

    def restore_state(self) -> None:
        """Back to the snapshot; the random counter keeps running, so replays draw afresh."""
        self.ctx.check(lib().wc_decoder_restore_state(self.h))

    def round_logits(self, k: int) -> dict:
        """The last sampled round's target logits [k+1][V], draft logits [k][head rows], verify
        tokens [x_n, d_1..d_k] and (seed, counter base)."""
        V = self.t.cfg.vocab
        Vd = self.d.head_rows
        zt = np.empty((k + 1, V), dtype=np.float32)
        zd = np.empty((k, Vd), dtype=np.float32)
        toks = (C.c_int * (k + 1))()
        rng = (C.c_uint64 * 2)()
        self.ctx.check(lib().wc_decoder_round_logits(self.h, k, zt.ctypes.data, zd.ctypes.data, toks, rng))
        return {"zt": zt, "zd": zd, "tokens": list(toks), "seed": int(rng[0]), "base": int(rng[1])}

    def draft_proposals(self, k: int) -> tuple[list[int], list[float]]:
        """The drafter's own head choice (token id, logit) at each of the last greedy round's k
        chain steps, also when forced drafts replaced them (test support)."""
        toks = (C.c_int * k)()
        z = np.empty(k, dtype=np.float32)
        self.ctx.check(lib().wc_decoder_draft_proposals(self.h, k, toks, z.ctypes.data))
        return list(toks), [float(x) for x in z]

    def last_round_ms(self) -> float:
        ms = C.c_float()
        self.ctx.check(lib().wc_decoder_last_round_ms(self.h, C.byref(ms)))
        return float(ms.value)

    # ---------------------------------------------------------------- main loop
    def generate(self, prompt: list[int], max_new_tokens: int, sp: SamplingParams = SamplingParams(),
                 stop_on_eos: bool = True) -> tuple[list[int], GenStats]:
        """spec.py:151-212: returns (tokens, GenStats)."""
        chain = isinstance(self.policy, StaticPolicy) and self.policy.width == 1
        if sp.greedy and isinstance(self.policy, StaticPolicy) and (not chain or not self.fused):
            return self._generate_tree(prompt, max_new_tokens, stop_on_eos)
        if not chain or not self.fused:  # sampled trees (spec.py:168-202)
            return self._generate_host(prompt, max_new_tokens, sp, stop_on_eos)
        st = GenStats(prompt_tokens=len(prompt), fused=True)
        eos = self.t.eos_token_ids if stop_on_eos else set()
        t0 = time.perf_counter()
        x_n = self.prefill(prompt, sp)
        st.t_prefill = time.perf_counter() - t0
        out = [x_n]
        n = len(prompt)
        self.policy.reset()
        forced_active = False
        while len(out) < max_new_tokens and x_n not in eos:
            ta = time.perf_counter()
            k = self.policy.plan(context_len=n, stochastic=not sp.greedy).max_depth
            if self.forced is not None:
                self.set_forced(self.forced(st.rounds, k, len(out)))
                forced_active = True
            elif forced_active:
                self.set_forced(None)
                forced_active = False
            acc = self.round(k)
            dt = time.perf_counter() - ta
            st.t_verify += dt
            st.round_ms_device.append(self.last_round_ms())
            st.rounds += 1
            st.accepted.append(len(acc) - 1)
            st.drafted.append(k)
            st.depths.append(k)
            self.policy.observe(len(acc) - 1, k, k, 0.0, dt)
            for tok in acc:
                out.append(tok)
                if tok in eos or len(out) >= max_new_tokens:
                    break
            n += len(acc)
            x_n = out[-1]
        if forced_active:
            self.set_forced(None)
        st.t_total = time.perf_counter() - t0
        st.new_tokens = len(out)
        return out, st

    def _generate_tree(self, prompt: list[int], max_new_tokens: int, stop_on_eos: bool) -> tuple[list[int], GenStats]:
        """Greedy draft trees (and the synced path on a chain) as device tree rounds, one graph per
        (depth, width, budget) and one synchronisation per round. `forced_tree(round, emitted) ->
        (tokens, parents)` replaces the drafted tree (oracle-drafter mode)."""
        st = GenStats(prompt_tokens=len(prompt), fused=True)
        eos = self.t.eos_token_ids if stop_on_eos else set()
        t0 = time.perf_counter()
        x_n = self.prefill(prompt)
        st.t_prefill = time.perf_counter() - t0
        out = [x_n]
        n = len(prompt)
        self.policy.reset()
        forced_active = False
        while len(out) < max_new_tokens and x_n not in eos:
            ta = time.perf_counter()
            plan = self.policy.plan(context_len=n, stochastic=False)
            nodes = 1 + plan.width + (plan.max_depth - 1) * plan.width * plan.width
            verified = min(nodes - 1, plan.budget)
            if self.forced_tree is not None:
                toks, pars = self.forced_tree(st.rounds, len(out))
                self.set_forced_tree(toks, pars)
                forced_active = True
                verified = len(toks) - 1
            acc = self.tree_round(plan.max_depth, plan.width, plan.budget)
            dt = time.perf_counter() - ta
            st.t_verify += dt
            st.round_ms_device.append(self.last_round_ms())
            st.rounds += 1
            st.accepted.append(len(acc) - 1)
            st.drafted.append(verified)
            st.depths.append(plan.max_depth)
            self.policy.observe(len(acc) - 1, verified, plan.max_depth, 0.0, dt)
            for tok in acc:
                out.append(tok)
                if tok in eos or len(out) >= max_new_tokens:
                    break
            n += len(acc)
            x_n = out[-1]
        if forced_active:
            self.set_forced_tree(None)
        st.t_total = time.perf_counter() - t0
        st.new_tokens = len(out)
        return out, st

    def _generate_host(self, prompt: list[int], max_new_tokens: int, sp: SamplingParams,
                       stop_on_eos: bool) -> tuple[list[int], GenStats]:
        """Sampled trees and policies with host-side hooks: host-driven rounds over the device API
        (woodcock_b200.synced), one synchronisation per drafted level as in the reference."""
        from .sampling import PhiloxStream
        from .synced import SyncedRounds

        st = GenStats(prompt_tokens=len(prompt), fused=False)
        rng = PhiloxStream(sp.seed, device=self.ctx.device.index or 0)
        eos = self.t.eos_token_ids if stop_on_eos else set()
        t0 = time.perf_counter()
        hr = SyncedRounds(self.t, self.d, self.policy, self.max_context + 256)
        x_n = hr.prefill(prompt, sp, rng)
        st.t_prefill = time.perf_counter() - t0
        out = [x_n]
        n = len(prompt)
        self.policy.reset()
        while len(out) < max_new_tokens and x_n not in eos:
            acc = hr.round(x_n, n, sp, rng, st)
            for tok in acc:
                out.append(tok)
                if tok in eos or len(out) >= max_new_tokens:
                    break
            n += len(acc)
            x_n = out[-1]
        st.t_total = time.perf_counter() - t0
        st.new_tokens = len(out)
        return out, st

    def generate_native(self, prompt: list[int], max_new_tokens: int, k: int, sp: SamplingParams = SamplingParams(),
                        stop_on_eos: bool = True) -> tuple[list[int], GenStats]:
        """The whole generate loop inside the C ABI (wc_decoder_generate)."""
        eos = sorted(self.t.eos_token_ids) if stop_on_eos else []
        out = (C.c_int * max_new_tokens)()
        n = C.c_int()
        s = GenStatsC()
        self.ctx.check(lib().wc_decoder_generate(self.h, int_array(prompt), len(prompt), max_new_tokens, k,
                                                 C.byref(_sp_c(sp)), int_array(eos) if eos else None, len(eos),
                                                 out, C.byref(n), C.byref(s)))
        st = GenStats(prompt_tokens=s.prompt_tokens, new_tokens=s.new_tokens, rounds=s.rounds,
                      t_prefill=s.t_prefill, t_verify=s.t_verify, t_total=s.t_total, fused=True)
        st.accepted = [0] * 0
        st.drafted = [k] * s.rounds
        st.depths = [k] * s.rounds
        if s.rounds:
            base, rem = divmod(int(s.accepted), s.rounds)
            st.accepted = [base + (1 if i < rem else 0) for i in range(s.rounds)]
        return list(out[: n.value]), st


def generate_autoregressive(target: Target, prompt: list[int], max_new_tokens: int,
                            sp: SamplingParams = SamplingParams(), stop_on_eos: bool = True,
                            max_context: int = 0) -> tuple[list[int], GenStats]:
    """spec.py:377-397: plain target decoding through the same target kernels."""
    eos = sorted(target.eos_token_ids) if stop_on_eos else []
    out = (C.c_int * max_new_tokens)()
    n = C.c_int()
    s = GenStatsC()
    target.ctx.check(lib().wc_generate_autoregressive(target.h, int_array(prompt), len(prompt), max_new_tokens,
                                                      C.byref(_sp_c(sp)), int_array(eos) if eos else None, len(eos),
                                                      max_context, out, C.byref(n), C.byref(s)))
    st = GenStats(prompt_tokens=s.prompt_tokens, new_tokens=s.new_tokens, rounds=s.rounds, t_prefill=s.t_prefill,
                  t_total=s.t_total)
    return list(out[: n.value]), st
