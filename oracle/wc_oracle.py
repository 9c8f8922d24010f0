"""CPU restatement of the reference decode path in numpy.

TEST INFRASTRUCTURE ONLY. This module is the checker for the CUDA path: only
tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may import it.
The product (woodcock_b200) never imports or calls it.

Each function restates one reference function (cited path:line inside the
AtomicBot-ai/woodcock project). Arithmetic follows the reference's C++ core
(src/backends/cpu_ops.cpp): fp32 products with double-accumulated RMSNorm and
softmax sums. Matrix products go through numpy/BLAS, so their summation order
differs from the reference's sequential loops; greedy tokens are checked for
identity and logits within a tolerance, as the reference itself does between its
C++ and MLX paths (tests/cpp/test_main.cpp:101-136).

Parity pins for this restatement (tests/test_oracle.py): the reference C++ core
compiled from its own sources (oracle/_ref/wc_ref_driver, fixtures in
tests/golden/), and the reference's Python sampling functions imported here with
a uniform tape (tests/golden/make_golden.py).

Stochastic rules take a uniform tape (`Tape`) in place of numpy's Generator:
`Tape.random()` returns the Philox4x32-10 stream the CUDA acceptance kernel
reads, so accept/reject decisions can be compared bit for bit.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

F32 = np.float32

# ----------------------------------------------------------------------------- Philox tape


def _mulhilo(a: int, b: np.ndarray):
    p = np.uint64(a) * b.astype(np.uint64)
    return (p >> np.uint64(32)).astype(np.uint32), (p & np.uint64(0xFFFFFFFF)).astype(np.uint32)


def philox4x32_10(counter_lo: np.ndarray, counter_hi: np.ndarray, seed: int) -> tuple[np.ndarray, ...]:
    """Philox4x32-10 (Salmon et al., SC'11, "Parallel random numbers: as easy as 1, 2, 3")
    on counters (lo, hi, 0, 0) with key (seed lo, seed hi). Returns the four output words."""
    c0 = np.asarray(counter_lo, np.uint32).copy()
    c1 = np.asarray(counter_hi, np.uint32).copy()
    c2 = np.zeros_like(c0)
    c3 = np.zeros_like(c0)
    k0 = np.uint32(seed & 0xFFFFFFFF)
    k1 = np.uint32((seed >> 32) & 0xFFFFFFFF)
    for r in range(10):
        hi0, lo0 = _mulhilo(0xD2511F53, c0)
        hi1, lo1 = _mulhilo(0xCD9E8D57, c2)
        c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
        if r < 9:
            k0 = np.uint32((int(k0) + 0x9E3779B9) & 0xFFFFFFFF)
            k1 = np.uint32((int(k1) + 0xBB67AE85) & 0xFFFFFFFF)
    return c0, c1, c2, c3


def philox_uniforms(seed: int, start: int, n: int) -> np.ndarray:
    """Doubles in [0, 1): element i uses counter start+i and 53 bits of its first two words."""
    idx = np.arange(start, start + n, dtype=np.uint64)
    r0, r1, _, _ = philox4x32_10((idx & np.uint64(0xFFFFFFFF)).astype(np.uint32),
                                 (idx >> np.uint64(32)).astype(np.uint32), seed)
    a = (r0 >> np.uint32(5)).astype(np.float64)
    b = (r1 >> np.uint32(6)).astype(np.float64)
    return (a * 67108864.0 + b) / 9007199254740992.0


class Tape:
    """numpy-Generator-like object whose `random()` reads the Philox stream in order."""

    def __init__(self, seed: int, offset: int = 0):
        self.seed, self.pos = seed, offset

    def random(self, size=None):
        n = 1 if size is None else int(np.prod(size))
        u = philox_uniforms(self.seed, self.pos, n)
        self.pos += n
        return float(u[0]) if size is None else u.reshape(size)


# ----------------------------------------------------------------------------- sampled device rounds
# The CUDA path draws with the same rules as the reference (sampling.py:39-55, 69-82,
# 143-203) but from Philox counters instead of numpy's Generator: a draw from softmax(z / T)
# is the Gumbel-max argmax_j (z_j / T + g_j), and the residual / bonus draw is the Gumbel-max
# over log r_j. Layout per round (or autoregressive step): RNG_STREAMS streams of
# RNG_STREAM_LEN counters from the round's base; stream i < 16 = draft step i (element = head
# row), RNG_ACCEPT_STREAM = acceptance uniforms (element = draft index), RNG_RESIDUAL_STREAM =
# residual / bonus noise (element = token id). Keys are ranked as float32, as on the device.

RNG_STREAM_LEN = 1 << 21
RNG_STREAMS = 32
RNG_ROUND_STRIDE = RNG_STREAM_LEN * RNG_STREAMS
RNG_ACCEPT_STREAM = 16
RNG_RESIDUAL_STREAM = 17


def _philox_words(seed: int, start: int, n: int):
    idx = np.arange(start, start + n, dtype=np.uint64)
    return philox4x32_10((idx & np.uint64(0xFFFFFFFF)).astype(np.uint32), (idx >> np.uint64(32)).astype(np.uint32),
                         seed)


def philox_gumbel_f32(seed: int, start: int, n: int) -> np.ndarray:
    """The float64 noise of philox_gumbel_f64 rounded to float32 (the device's head-epilogue and
    first-token draws)."""
    return philox_gumbel_f64(seed, start, n).astype(F32)


def philox_gumbel_f64(seed: int, start: int, n: int) -> np.ndarray:
    """float64 Gumbel noise, u = (53 bits of words 0 and 1 + 1/2) / 2^53 on (0, 1)."""
    r0, r1, _, _ = _philox_words(seed, start, n)
    u = ((r0 >> np.uint32(5)).astype(np.float64) * 67108864.0 + (r1 >> np.uint32(6)).astype(np.float64) + 0.5) / \
        9007199254740992.0
    return -np.log(-np.log(u))


def gumbel_draw(z: np.ndarray, T: float, seed: int, base: int, stream: int) -> int:
    """Draft draw of one head row: argmax of float32 z / T + Gumbel noise (element = row)."""
    g = philox_gumbel_f32(seed, base + stream * RNG_STREAM_LEN, len(z))
    key = (np.asarray(z, F32) / F32(T)).astype(F32) + g
    return int(np.argmax(key))  # first maximum, as the device's key packing breaks ties


def warp_threshold(z: np.ndarray, T: float, top_k: int = 0, top_p: float = 1.0) -> float:
    """The device's form of probs_from_logits' warping (sampling.py:39-55): with x = z / T
    (float32), the kept tokens are x >= thr. top-k: thr = the k-th largest x; top-p: the
    largest x at which the descending inclusive softmax mass of the top-k survivors reaches
    top_p. Returns -inf when nothing is cut. Equal to the sort-based rule when no two kept
    values tie at the cut."""
    x = (np.asarray(z, F32) / F32(T)).astype(F32)
    thr = -np.inf
    if top_k and 0 < top_k < len(x):
        thr = float(np.sort(x)[-top_k])
    if top_p < 1.0:
        kept = np.sort(x[x >= thr])[::-1].astype(np.float64)
        e = np.exp(kept - kept[0])
        cs = np.cumsum(e)
        m = int(np.searchsorted(cs, top_p * cs[-1], side="left"))
        if m < len(kept):
            thr = max(thr, float(kept[m]))
    return thr


def warped_probs(z: np.ndarray, T: float, top_k: int = 0, top_p: float = 1.0) -> np.ndarray:
    x = (np.asarray(z, F32) / F32(T)).astype(F32)
    thr = warp_threshold(z, T, top_k, top_p)
    e = np.where(x >= thr, np.exp(x.astype(np.float64) - float(x.max())), 0.0)
    return e / e.sum()


def gumbel_draw_warped(z: np.ndarray, T: float, top_k: int, top_p: float, seed: int, base: int, stream: int) -> int:
    """Warped first-token / autoregressive draw: argmax over kept x of x + Gumbel (float32)."""
    x = (np.asarray(z, F32) / F32(T)).astype(F32)
    thr = warp_threshold(z, T, top_k, top_p)
    g = philox_gumbel_f32(seed, base + stream * RNG_STREAM_LEN, len(x))
    key = np.where(x >= thr, (x + g).astype(F32), -np.inf)
    return int(np.argmax(key))


def sampled_chain_accept(zt: np.ndarray, zd: np.ndarray, tokens: list[int], T: float, seed: int, base: int,
                         vocab_ids: np.ndarray | None = None, skip_residual: bool = False, top_k: int = 0,
                         top_p: float = 1.0) -> tuple[int, int]:
    """Acceptance of one sampled chain round from its logits: zt [K+1][V] target rows at
    [x_n, d_1..d_K], zd [K][Vd] draft rows (head row r is token vocab_ids[r]). p_i =
    softmax(zt_i / T), q_i = softmax(zd_i / T) scattered to token ids (spec.py:239-249);
    the chain case of verify_tree_stochastic (sampling.py:143-187). `skip_residual` plants
    the mistake a negative control must catch: a rejection draws from p instead."""
    K = len(tokens) - 1
    V = zt.shape[1]

    def probs(z):
        x = (np.asarray(z, F32) / F32(T)).astype(np.float64)
        e = np.exp(x - x.max())
        return e / e.sum()

    def target(z):  # the target rows carry the top-k / top-p warping, the draft rows only T
        return warped_probs(z, T, top_k, top_p) if (top_k or top_p < 1.0) else probs(z)

    def q_full(i):
        qd = probs(zd[i])
        q = np.zeros(V)
        if vocab_ids is None:
            q[: len(qd)] = qd
        else:
            q[np.asarray(vocab_ids)] = qd
        return q

    a = 0
    while a < K:
        x = tokens[a + 1]
        q = q_full(a)
        qx = q[x]
        if not qx > 0:
            break
        px = target(zt[a])[x]
        u = philox_uniforms(seed, base + RNG_ACCEPT_STREAM * RNG_STREAM_LEN + a, 1)[0]
        if not u < min(1.0, px / qx):
            break
        a += 1
    p = target(zt[a])
    if a < K and not skip_residual:
        r = np.maximum(p - q_full(a), 0.0)
        if not r.sum() > 1e-12:
            r = p
    else:
        r = p
    g = philox_gumbel_f64(seed, base + RNG_RESIDUAL_STREAM * RNG_STREAM_LEN, V)
    with np.errstate(divide="ignore"):
        key = np.where(r > 0, (np.log(r) + g).astype(F32), -np.inf)
    return a, int(np.argmax(key))


def chi2_equal_mass(counts: np.ndarray, p: np.ndarray, bins: int = 1000, order: str = "id") -> tuple[float, int, float]:
    """Pearson chi-square of token counts against the law p, on `bins` groups of tokens with
    (near) equal expected mass (the binning the reference's test uses where one token per cell
    would leave expected counts under 5, tests/test_sampling.py:73-76). order="id" groups
    consecutive token ids; order="rank" groups tokens in decreasing order of p, so a bias that
    grows or shrinks with the logit concentrates in the first or last bins instead of averaging
    out. Returns (statistic, degrees of freedom, p-value)."""
    from scipy.stats import chi2
    counts, p = np.asarray(counts, np.float64), np.asarray(p, np.float64)
    if order == "rank":
        perm = np.argsort(-p, kind="stable")
        counts, p = counts[perm], p[perm]
    elif order != "id":
        raise ValueError("order must be 'id' or 'rank'")
    n = counts.sum()
    c = np.cumsum(p) / p.sum()
    edges = np.searchsorted(c, np.arange(1, bins) / bins, side="left")
    b = np.concatenate([[0], edges + 1, [len(p)]])
    b = np.unique(np.clip(b, 0, len(p)))
    obs = np.add.reduceat(counts, b[:-1])
    exp = np.add.reduceat(p / p.sum(), b[:-1]) * n
    keep = exp > 0
    stat = float(((obs[keep] - exp[keep]) ** 2 / exp[keep]).sum())
    dof = int(keep.sum()) - 1
    return stat, dof, float(chi2.sf(stat, dof))


# ----------------------------------------------------------------------------- ops (cpu_ops.cpp)


def linear(x: np.ndarray, W: np.ndarray) -> np.ndarray:
    """y[L][out] = x[L][in] . W[out][in]^T (src/backends/cpu_ops.cpp:45-48)."""
    return (x.astype(F32) @ W.T).astype(F32)


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """Row RMSNorm with a double sum of squares (src/backends/cpu_ops.cpp:50-59)."""
    x = np.asarray(x, F32)
    d = x.shape[-1]
    ss = np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    inv = F32(1.0) / np.sqrt((ss / d).astype(F32) + F32(eps))
    return (x * inv.astype(F32) * np.asarray(w, F32)).astype(F32)


def rope_inv_freq(D: int, base: float) -> np.ndarray:
    """std::pow(base, -2.f * i / D) in float: the exponent is formed in float32 and the power
    rounded once from double (glibc's powf is within 1 ulp of that)."""
    i = np.arange(D // 2, dtype=F32)
    e = (F32(-2.0) * i / F32(D)).astype(F32)
    return np.power(np.float64(F32(base)), e.astype(np.float64)).astype(F32)


def rope(x: np.ndarray, positions, base: float) -> np.ndarray:
    """Rotate-half RoPE on x[L][heads][D] at per-row positions (src/backends/cpu_ops.cpp:61-77)."""
    x = np.asarray(x, F32)
    L, Hh, D = x.shape
    half = D // 2
    inv = rope_inv_freq(D, base)
    a = (np.asarray(positions, F32)[:, None] * inv[None, :]).astype(F32)  # [L][half]
    # cosf / sinf of a float angle, rounded once from double (numpy's float32 cos/sin lose
    # accuracy for angles in the thousands of radians; glibc's are correctly rounded)
    a64 = a.astype(np.float64)
    c, s = np.cos(a64).astype(F32)[:, None, :], np.sin(a64).astype(F32)[:, None, :]
    x1, x2 = x[..., :half], x[..., half:]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1).astype(F32)


def silu_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    """gate = silu(gate) * up (src/backends/cpu_ops.cpp:79-84)."""
    g = np.asarray(g, F32)
    return (g / (F32(1) + np.exp(-g)) * u).astype(F32)


def softmax(x: np.ndarray) -> np.ndarray:
    """Per row; -inf -> 0; double sum (src/backends/cpu_ops.cpp:86-96)."""
    x = np.asarray(x, F32)
    m = np.max(x, axis=-1, keepdims=True)
    e = np.where(np.isneginf(x), F32(0), np.exp(x - m)).astype(F32)
    s = np.sum(e.astype(np.float64), axis=-1, keepdims=True)
    return (e * (1.0 / s).astype(F32)).astype(F32)


def attention(q, K, V, mask, scale) -> np.ndarray:
    """q[L][H][D], K/V[T][Hk][D], mask[L][T] (1 = visible) -> out[L][H][D]
    (src/backends/cpu_ops.cpp:98-115; GQA head h reads kv head h // (H/Hk))."""
    L, H, D = q.shape
    T, Hk, _ = K.shape
    rep = H // Hk
    out = np.zeros((L, H, D), F32)
    for h in range(H):
        kh = h // rep
        S = (F32(scale) * (q[:, h, :] @ K[:, kh, :].T)).astype(F32)
        if mask is not None:
            S = np.where(np.asarray(mask, bool), S, -np.inf).astype(F32)
        P = softmax(S)
        out[:, h, :] = P @ V[:, kh, :]
    return out


def argmax(z) -> int:
    return int(np.argmax(z))  # first maximum, like std::max_element (src/sampling/sampling.cpp:47)


# ----------------------------------------------------------------------------- KV cache (kv_cache.cpp)


class KVCache:
    """Per-layer [pos][kv_head*head_dim] rows; append/commit/trim_to/compact
    (include/woodcock/cache.h:9-28, src/cache/kv_cache.cpp:8-31)."""

    def __init__(self, layers: int, kv_heads: int, head_dim: int, bf16: bool = False):
        self.bf16 = bf16  # store rows rounded to bf16, as a bf16 device cache does
        self.row = kv_heads * head_dim
        self.kv_heads, self.head_dim = kv_heads, head_dim
        self.k = [np.zeros((0, self.row), F32) for _ in range(layers)]
        self.v = [np.zeros((0, self.row), F32) for _ in range(layers)]
        self.n = 0

    def size(self) -> int:
        return self.n

    def append(self, layer: int, k: np.ndarray, v: np.ndarray) -> None:
        L = k.shape[0]
        need = self.n + L
        if self.k[layer].shape[0] < need:
            grow = max(need, 2 * self.k[layer].shape[0] + 256)
            for arr in (self.k, self.v):
                a = np.zeros((grow, self.row), F32)
                a[: arr[layer].shape[0]] = arr[layer]
                arr[layer] = a
        k, v = k.reshape(L, self.row), v.reshape(L, self.row)
        if self.bf16:
            k, v = _round_bf16(k), _round_bf16(v)
        self.k[layer][self.n : need] = k
        self.v[layer][self.n : need] = v

    def commit(self, L: int) -> None:
        self.n += L

    def trim_to(self, n: int) -> None:
        self.n = n

    def compact(self, start: int, keep: list[int]) -> None:
        """Rows start+keep[i] -> start+i in increasing i (src/cache/kv_cache.cpp:21-31)."""
        for arr in (self.k, self.v):
            for lay in arr:
                for i, kk in enumerate(keep):
                    if kk != i:
                        lay[start + i] = lay[start + kk]
        self.n = start + len(keep)

    def keys(self, layer: int, T: int) -> np.ndarray:
        return self.k[layer][:T].reshape(T, self.kv_heads, self.head_dim)

    def values(self, layer: int, T: int) -> np.ndarray:
        return self.v[layer][:T].reshape(T, self.kv_heads, self.head_dim)


def _round_bf16(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=F32).view(np.uint32)
    r = ((u + (((u >> 16) & 1) + np.uint32(0x7FFF))) >> 16) << 16
    return r.astype(np.uint32).view(F32)


def default_positions(start: int, L: int) -> list[int]:
    return list(range(start, start + L))  # src/core/qwen3.cpp:38-42


def causal_mask(prefix: int, L: int, window: int = 0) -> np.ndarray:
    """[L][prefix+L], 1 = visible (src/core/qwen3.cpp:44-53)."""
    T = prefix + L
    m = np.zeros((L, T), np.uint8)
    for l in range(L):
        q = prefix + l
        lo = max(0, q - window + 1) if window > 0 else 0
        m[l, lo : q + 1] = 1
    return m


# ----------------------------------------------------------------------------- models


def _load_dir(d: Path) -> tuple[dict, dict[str, np.ndarray]]:
    import sys

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    from woodcock_b200 import safetensors_io as st  # plain file I/O helper shared with the product

    cfg = json.loads((d / "config.json").read_text())
    w = {}
    for f in sorted(d.glob("*.safetensors")):
        for k, e in st.load(f).items():
            w[k] = st.to_f32(e)
    return cfg, w


class Qwen3:
    """Qwen3 dense decoder in fp32 (src/core/qwen3.cpp:55-114; python/woodcock/target.py:82-116)."""

    def __init__(self, cfg: dict, w: dict[str, np.ndarray], taps=None):
        self.hidden = cfg["hidden_size"]
        self.layers = cfg["num_hidden_layers"]
        self.heads = cfg["num_attention_heads"]
        self.kv_heads = cfg["num_key_value_heads"]
        self.head_dim = cfg.get("head_dim") or self.hidden // self.heads
        self.intermediate = cfg["intermediate_size"]
        self.vocab = cfg["vocab_size"]
        self.eps = float(cfg.get("rms_norm_eps", 1e-6))
        self.theta = float(cfg.get("rope_theta", 1e6))
        self.taps = list(taps) if taps is not None else [2, self.layers // 2, self.layers - 3]
        self.kv_bf16 = False  # True: model a bf16 KV cache (rows rounded on append)
        self.w = w
        tied = bool(cfg.get("tie_word_embeddings", False)) or "lm_head.weight" not in w
        self.head = w["model.embed_tokens.weight"] if tied else w["lm_head.weight"]

    @classmethod
    def load(cls, d, taps=None) -> "Qwen3":
        cfg, w = _load_dir(Path(d))
        return cls(cfg, w, taps)

    def make_cache(self) -> KVCache:
        return KVCache(self.layers, self.kv_heads, self.head_dim, bf16=self.kv_bf16)

    def forward(self, tokens, cache: KVCache, positions=None, mask=None, logits=True, logits_from=0):
        """Returns (logits [rows][V] for rows >= logits_from, taps: list of [L][hidden])."""
        w, d, H, Hk, D = self.w, self.hidden, self.heads, self.kv_heads, self.head_dim
        L = len(tokens)
        prefix = cache.size()
        T = prefix + L
        pos = positions if positions is not None else default_positions(prefix, L)
        m = mask if mask is not None else causal_mask(prefix, L)
        h = w["model.embed_tokens.weight"][np.asarray(tokens)].astype(F32)
        taps = []
        for li in range(self.layers):
            p = f"model.layers.{li}."
            x = rmsnorm(h, w[p + "input_layernorm.weight"], self.eps)
            q = linear(x, w[p + "self_attn.q_proj.weight"]).reshape(L, H, D)
            k = linear(x, w[p + "self_attn.k_proj.weight"]).reshape(L, Hk, D)
            v = linear(x, w[p + "self_attn.v_proj.weight"]).reshape(L, Hk, D)
            q = rmsnorm(q, w[p + "self_attn.q_norm.weight"], self.eps)
            k = rmsnorm(k, w[p + "self_attn.k_norm.weight"], self.eps)
            q, k = rope(q, pos, self.theta), rope(k, pos, self.theta)
            cache.append(li, k, v)
            att = attention(q, cache.keys(li, T), cache.values(li, T), m, 1.0 / np.sqrt(F32(D)))
            h = (h + linear(att.reshape(L, H * D), w[p + "self_attn.o_proj.weight"])).astype(F32)
            x = rmsnorm(h, w[p + "post_attention_layernorm.weight"], self.eps)
            g = silu_mul(linear(x, w[p + "mlp.gate_proj.weight"]), linear(x, w[p + "mlp.up_proj.weight"]))
            h = (h + linear(g, w[p + "mlp.down_proj.weight"])).astype(F32)
            for t in self.taps:
                if t == li:
                    taps.append(h.copy())
        cache.commit(L)
        z = None
        if logits:
            x = rmsnorm(h[logits_from:], w["model.norm.weight"], self.eps)
            z = linear(x, self.head)
        return z, taps


class Drafter:
    """EAGLE-3 drafter (src/core/drafter.cpp:47-141; python/woodcock/drafter.py:149-229):
    fuse = per-tap RMSNorm + FC; layer 0 adds W_aux . aux_norm(embed(token)) to Q/K/V;
    out = RMSNorm(h) feeds the head and (post_norm) the next step."""

    def __init__(self, cfg: dict, w: dict[str, np.ndarray]):
        self.cfg = cfg
        self.hidden = cfg["hidden_size"]
        self.layers = cfg["num_layers"]
        self.heads, self.kv_heads, self.head_dim = cfg["num_heads"], cfg["num_kv_heads"], cfg["head_dim"]
        self.vocab = cfg["vocab_size"]
        self.target_hidden = cfg["target_hidden_size"]
        self.num_features = cfg.get("num_features", 3)
        self.eps = float(cfg.get("rms_norm_eps", 1e-6))
        self.theta = float(cfg.get("rope_theta", 1e6))
        self.post_norm = cfg.get("post_norm", True)
        self.feature_norm = cfg.get("feature_norm", True)
        self.window = cfg.get("window") or 0
        self.kv_bf16 = False
        self.w = w
        self.head = w["lm_head.weight"]
        self.vocab_ids = None

    @classmethod
    def load(cls, d) -> "Drafter":
        cfg, w = _load_dir(Path(d))
        return cls(cfg, w)

    def restrict_vocab(self, ids) -> None:
        """Head rows of `ids`; row r maps to token ids[r] (python/woodcock/drafter.py:217-229)."""
        if self.vocab_ids is not None:
            raise ValueError("drafter vocabulary is already restricted")
        ids = np.asarray(ids, np.int64)
        self.head = self.w["lm_head.weight"][ids]
        self.vocab_ids = ids.astype(np.int32)

    def token_ids(self, rows):
        return rows if self.vocab_ids is None else int(self.vocab_ids[rows])

    def make_cache(self) -> KVCache:
        return KVCache(self.layers, self.kv_heads, self.head_dim, bf16=self.kv_bf16)

    def fuse(self, taps: list[np.ndarray]) -> np.ndarray:
        w = self.w
        parts = []
        for f, t in enumerate(taps):
            parts.append(rmsnorm(t, w[f"feature_norms.{f}.weight"], self.eps) if self.feature_norm else t)
        return linear(np.concatenate(parts, axis=-1), w["fc.weight"])

    def forward(self, tokens, feat, cache: KVCache, positions=None, mask=None):
        w, d, H, Hk, D = self.w, self.hidden, self.heads, self.kv_heads, self.head_dim
        L = len(tokens)
        prefix = cache.size()
        T = prefix + L
        pos = positions if positions is not None else default_positions(prefix, L)
        m = mask if mask is not None else causal_mask(prefix, L, self.window)
        e = w["embed_tokens.weight"][np.asarray(tokens)].astype(F32)
        h = np.asarray(feat, F32).reshape(L, d).copy()
        for li in range(self.layers):
            p = f"layers.{li}."
            x = rmsnorm(h, w[p + "input_layernorm.weight"], self.eps)
            q = linear(x, w[p + "self_attn.q_proj.weight"])
            k = linear(x, w[p + "self_attn.k_proj.weight"])
            v = linear(x, w[p + "self_attn.v_proj.weight"])
            if li == 0:
                a = rmsnorm(e, w[p + "aux_norm.weight"], self.eps)
                q = q + linear(a, w[p + "self_attn.aux_q.weight"])
                k = k + linear(a, w[p + "self_attn.aux_k.weight"])
                v = v + linear(a, w[p + "self_attn.aux_v.weight"])
            q = rmsnorm(q.reshape(L, H, D), w[p + "self_attn.q_norm.weight"], self.eps)
            k = rmsnorm(k.reshape(L, Hk, D), w[p + "self_attn.k_norm.weight"], self.eps)
            q, k = rope(q, pos, self.theta), rope(k, pos, self.theta)
            cache.append(li, k, v.reshape(L, Hk, D))
            att = attention(q, cache.keys(li, T), cache.values(li, T), m, 1.0 / np.sqrt(F32(D)))
            h = (h + linear(att.reshape(L, H * D), w[p + "self_attn.o_proj.weight"])).astype(F32)
            x = rmsnorm(h, w[p + "post_attention_layernorm.weight"], self.eps)
            g = silu_mul(linear(x, w[p + "mlp.gate_proj.weight"]), linear(x, w[p + "mlp.up_proj.weight"]))
            h = (h + linear(g, w[p + "mlp.down_proj.weight"])).astype(F32)
        cache.commit(L)
        out = rmsnorm(h, w["norm.weight"], self.eps)
        return h, out

    def feedback(self, hidden, out):
        return out if self.post_norm else hidden

    def logits(self, out_rows: np.ndarray) -> np.ndarray:
        return linear(np.atleast_2d(out_rows), self.head)


# ----------------------------------------------------------------------------- sampling (sampling.py)


@dataclass(frozen=True)
class SamplingParams:
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    seed: int = 0

    @property
    def greedy(self) -> bool:
        return self.temperature <= 0.0


def probs_from_logits(z: np.ndarray, sp: SamplingParams) -> np.ndarray:
    """Temperature / top-k / top-p warping in fp32 (python/woodcock/sampling.py:39-55)."""
    x = (np.asarray(z, F32) / F32(max(sp.temperature, 1e-6))).astype(F32)
    if sp.top_k and sp.top_k < x.shape[-1]:
        kth = np.sort(x, axis=-1)[..., -sp.top_k][..., None]
        x = np.where(x < kth, -np.inf, x).astype(F32)
    p = softmax(x)
    if sp.top_p < 1.0:
        order = np.argsort(-p, axis=-1, kind="stable")
        ps = np.take_along_axis(p, order, axis=-1)
        cs = np.cumsum(ps, axis=-1, dtype=F32)
        keep_sorted = (cs - ps) < sp.top_p
        keep = np.zeros_like(p, dtype=bool)
        np.put_along_axis(keep, order, keep_sorted, axis=-1)
        p = np.where(keep, p, F32(0)).astype(F32)
        p = (p / p.sum(axis=-1, keepdims=True)).astype(F32)
    return p


@dataclass
class DraftTree:
    """Flattened tree, node 0 = root; children in draw order (python/woodcock/sampling.py:88-115)."""

    tokens: list[int]
    parents: list[int]
    depth: list[int]
    children: list[list[int]] = field(default_factory=list)

    def __post_init__(self):
        if not self.children:
            self.children = [[] for _ in self.tokens]
            for v, p in enumerate(self.parents):
                if p >= 0:
                    self.children[p].append(v)

    def __len__(self):
        return len(self.tokens)

    def is_chain(self) -> bool:
        return all(p == i - 1 for i, p in enumerate(self.parents))


def tree_attention_mask(tree: DraftTree, prefix_len: int) -> np.ndarray:
    """(N, prefix+N): prefix + ancestors incl. self (sampling.py:118-128; sampling.cpp:85-93)."""
    N = len(tree)
    m = np.zeros((N, prefix_len + N), dtype=bool)
    m[:, :prefix_len] = True
    for v in range(N):
        u = v
        while u >= 0:
            m[v, prefix_len + u] = True
            u = tree.parents[u]
    return m


def verify_chain_greedy(target_argmax: list[int], draft_tokens: list[int]) -> tuple[int, int]:
    """(n accepted, next token) (python/woodcock/sampling.py:60-66)."""
    n = 0
    while n < len(draft_tokens) and target_argmax[n] == draft_tokens[n]:
        n += 1
    return n, int(target_argmax[n])


def verify_tree_greedy(target_argmax: list[int], tree: DraftTree) -> tuple[list[int], int]:
    """First matching child in draw order, down the tree (sampling.py:131-140; sampling.cpp:95-106)."""
    v, path = 0, []
    while True:
        want = int(target_argmax[v])
        nxt = next((c for c in tree.children[v] if tree.tokens[c] == want), None)
        if nxt is None:
            return path, want
        path.append(nxt)
        v = nxt


def residual(p: np.ndarray, q: np.ndarray) -> np.ndarray:
    """norm(max(0, p - q)); p itself when the residual mass is <= 1e-12 (sampling.py:182-187)."""
    r = np.maximum(p - q, 0.0)
    s = r.sum()
    if s <= 1e-12:
        return p / p.sum()
    return r / s


def sample(p: np.ndarray, rng) -> int:
    """Inverse-CDF draw with a sequential fp64 cumsum (sampling.py:190-193)."""
    p = np.asarray(p, dtype=np.float64)
    c = np.cumsum(p)
    return int(min(np.searchsorted(c, rng.random() * c[-1], side="right"), len(p) - 1))


def sample_without_replacement(q: np.ndarray, k: int, rng) -> list[int]:
    """Gumbel-top-k over the nonzero entries, one uniform each in id order (sampling.py:196-203)."""
    q = np.asarray(q, dtype=np.float64)
    nz = np.flatnonzero(q > 0)
    k = min(k, len(nz))
    with np.errstate(divide="ignore"):
        g = np.log(q[nz]) - np.log(-np.log(rng.random(len(nz))))
    order = np.argsort(-g, kind="stable")[:k]
    return [int(nz[i]) for i in order]


def verify_chain_stochastic(p: np.ndarray, q: np.ndarray, draft_tokens: list[int], rng) -> tuple[int, int]:
    """Leviathan et al. chain rule (sampling.py:69-82)."""
    K = len(draft_tokens)
    for i, x in enumerate(draft_tokens):
        qi = q[i, x]
        accept = False if qi <= 0 else rng.random() < min(1.0, p[i, x] / qi)
        if not accept:
            return i, sample(residual(p[i], q[i]), rng)
    return K, sample(p[K], rng)


def verify_tree_stochastic(p: dict, q: dict, tree: DraftTree, rng) -> tuple[list[int], int]:
    """Recursive rejection sampling over children drawn without replacement (sampling.py:143-177)."""
    v, path = 0, []
    while True:
        kids = tree.children[v]
        p_cur = np.asarray(p[v], np.float64)
        if not kids:
            return path, sample(p_cur, rng)
        q_cur = np.asarray(q[v], np.float64).copy()
        accepted = None
        for c in kids:
            x = tree.tokens[c]
            qx = q_cur[x]
            if qx > 0 and rng.random() < min(1.0, p_cur[x] / qx):
                accepted = c
                break
            p_cur = residual(p_cur, q_cur)
            q_cur[x] = 0.0
            s = q_cur.sum()
            if s <= 0:
                break
            q_cur /= s
        if accepted is None:
            return path, sample(p_cur, rng)
        path.append(accepted)
        v = accepted


# ----------------------------------------------------------------------------- policies (policies.py)


class StaticPolicy:
    """Fixed depth / width / budget (python/woodcock/policies.py:57-70; src/core/spec.cpp:35-45)."""

    def __init__(self, depth: int, width: int = 1, budget: int | None = None):
        self.depth, self.width = depth, width
        self.budget = budget if budget is not None else (depth if width == 1 else 4 * depth)

    def select_verify(self, nodes, stochastic):
        if stochastic or len(nodes) - 1 <= self.budget:
            return list(range(len(nodes)))
        order = sorted(range(1, len(nodes)), key=lambda v: (-nodes[v].phat, nodes[v].depth, v))[: self.budget]
        return [0] + sorted(order)


# ----------------------------------------------------------------------------- scheduler (spec.py / spec.cpp)


@dataclass
class GenStats:
    prompt_tokens: int = 0
    new_tokens: int = 0
    rounds: int = 0
    accepted: list[int] = field(default_factory=list)
    drafted: list[int] = field(default_factory=list)


@dataclass
class _Node:
    token: int
    parent: int
    depth: int
    phat: float
    out: np.ndarray | None = None
    fb: np.ndarray | None = None
    cache_idx: int = -1
    q: np.ndarray | None = None


class SpeculativeDecoder:
    """Restates SpeculativeDecoder (python/woodcock/spec.py:104-374; src/core/spec.cpp:49-280).

    `forced(round, k, emitted) -> k tokens` (oracle-drafter mode, the OracleDecoder pattern of
    tests/test_spec_model.py:59-92) gives the tokens that replace draft tokens d_1..d_k after
    the drafter computed them; `emitted` is the number of tokens generated so far. Downstream
    steps use the forced tokens, so acceptance is controlled while all draft compute runs."""

    def __init__(self, target: Qwen3, drafter: Drafter, policy: StaticPolicy, fused: bool = True):
        self.t, self.d, self.policy, self.fused = target, drafter, policy, fused

    def _prefill(self, prompt, sp, rng):
        self.tc = self.t.make_cache()
        z, feats = self.t.forward(prompt, self.tc, logits_from=len(prompt) - 1)
        first = self._sample_target(z[-1], sp, rng)
        self.dc = self.d.make_cache()
        g = self.d.fuse(feats)
        hid, out = self.d.forward(list(prompt[1:]) + [first], g, self.dc)
        self.root_out = out[-1:].copy()
        self.root_fb = self.d.feedback(hid[-1:], out[-1:]).copy()
        return first

    def _sample_target(self, z, sp, rng) -> int:
        if sp.greedy:
            return argmax(z)
        return sample(probs_from_logits(z[None], sp)[0].astype(np.float64), rng)

    def generate(self, prompt, max_new_tokens, sp=SamplingParams(), stop_on_eos=True, eos=(151643, 151645),
                 forced=None, rng=None):
        st = GenStats(prompt_tokens=len(prompt))
        rng = rng if rng is not None else Tape(sp.seed)
        eos = set(eos) if stop_on_eos else set()
        x_n = self._prefill(prompt, sp, rng)
        out = [x_n]
        n = len(prompt)
        chain = self.policy.width == 1
        r = 0
        while len(out) < max_new_tokens and x_n not in eos:
            if chain and sp.greedy:
                K = self.policy.depth
                fk = list(forced(r, K, len(out))) if forced is not None else None
                a, acc = self._chain_round(x_n, n, K, fk)
                st.accepted.append(a)
                st.drafted.append(K)
            else:
                tree, nodes = self._draft(x_n, n, sp, rng)
                if forced is not None and tree.is_chain():
                    fk = list(forced(r, len(tree) - 1, len(out)))
                    tree = DraftTree([tree.tokens[0]] + fk, tree.parents, tree.depth)
                path, nxt, feats = self._verify(tree, nodes, n, sp, rng)
                acc = [tree.tokens[v] for v in path] + [nxt]
                self._update(acc, feats)
                st.accepted.append(len(path))
                st.drafted.append(len(tree) - 1)
            st.rounds += 1
            r += 1
            for tok in acc:
                out.append(tok)
                if tok in eos or len(out) >= max_new_tokens:
                    break
            n += len(acc)
            x_n = out[-1]
            if x_n in eos:
                break
        st.new_tokens = len(out)
        return out, st

    def _chain_round(self, x_n, n, K, forced):
        """Greedy static chain (python/woodcock/spec.py:331-364)."""
        d = self.d
        base = self.dc.size()
        out, fb = self.root_out, self.root_fb
        drafts = []
        for k in range(K):
            tok = d.token_ids(argmax(d.logits(out)[0]))
            if forced is not None:
                tok = int(forced[k])
            drafts.append(tok)
            if k < K - 1:
                hid, out = d.forward([tok], fb, self.dc)
                fb = d.feedback(hid, out)
        self.dc.trim_to(base)
        seq = [x_n] + drafts
        z, feats = self.t.forward(seq, self.tc)
        am = [argmax(row) for row in z]
        a, nxt = verify_chain_greedy(am, drafts)
        acc = drafts[:a] + [nxt]
        self.tc.compact(n, list(range(a + 1)))
        self._update(acc, [f[: a + 1] for f in feats])
        return a, acc

    def _draft_dist(self, out_rows, sp):
        z = self.d.logits(out_rows)
        if sp.greedy:
            q = softmax(z)
        else:
            q = probs_from_logits(z, SamplingParams(temperature=sp.temperature))
        return self.d.vocab_ids, q

    def _draft(self, root_token, n, sp, rng):
        """Level-by-level tree drafting (python/woodcock/spec.py:216-278)."""
        pol = self.policy
        root = _Node(root_token, -1, 0, 1.0, out=self.root_out, fb=self.root_fb, cache_idx=n - 1)
        nodes = [root]
        base = self.dc.size()
        frontier = [0]
        tree_cache = 0
        remaining = pol.budget
        for depth in range(1, pol.depth + 1):
            outs = np.concatenate([nodes[v].out for v in frontier], axis=0)
            idx, q = self._draft_dist(outs, sp)
            new = []
            if sp.greedy:
                w = pol.width
                for r_, v in enumerate(frontier):
                    top = np.argsort(-q[r_], kind="stable")[:w]
                    for c in top:
                        tok = int(c) if idx is None else int(idx[c])
                        new.append(_Node(tok, v, depth, nodes[v].phat * float(q[r_, c])))
            else:
                for r_, v in enumerate(frontier):
                    qv = np.zeros(self.t.vocab)
                    if idx is None:
                        qv[: q.shape[1]] = q[r_]
                    else:
                        qv[idx] = q[r_]
                    qv /= qv.sum()
                    nodes[v].q = qv
                    m = max(min(pol.width, remaining), 0)
                    remaining -= m
                    for x in sample_without_replacement(qv, m, rng):
                        new.append(_Node(int(x), v, depth, nodes[v].phat * float(qv[x])))
            nodes.extend(new)
            level = list(range(len(nodes) - len(new), len(nodes)))
            if depth == pol.depth:
                break
            frontier = sorted(level, key=lambda v: (-nodes[v].phat, nodes[v].depth))[: pol.width]
            if not frontier:
                break
            toks = [nodes[v].token for v in frontier]
            fb = np.concatenate([nodes[nodes[v].parent].fb for v in frontier], axis=0)
            pos = [n - 1 + nodes[v].depth for v in frontier]
            mask = self._draft_mask(nodes, frontier, base, tree_cache)
            hid, out = self.d.forward(toks, fb, self.dc, positions=pos, mask=mask)
            fbk = self.d.feedback(hid, out)
            for r_, v in enumerate(frontier):
                nodes[v].out = out[r_ : r_ + 1]
                nodes[v].fb = fbk[r_ : r_ + 1]
                nodes[v].cache_idx = base + tree_cache + r_
            tree_cache += len(frontier)
        self.dc.trim_to(base)
        keep = pol.select_verify(nodes, not sp.greedy)
        remap = {v: i for i, v in enumerate(keep)}
        tree = DraftTree([nodes[v].token for v in keep], [remap.get(nodes[v].parent, -1) for v in keep],
                         [nodes[v].depth for v in keep])
        return tree, [nodes[v] for v in keep]

    def _draft_mask(self, nodes, frontier, base, tree_cache):
        """python/woodcock/spec.py:280-294."""
        m = len(frontier)
        total = base + tree_cache + m
        mask = np.zeros((m, total), dtype=np.uint8)
        w = self.d.window
        for r_, v in enumerate(frontier):
            pos = base - 1 + nodes[v].depth
            lo = 0 if not w else max(0, pos - w + 1)
            mask[r_, lo:base] = 1
            u = nodes[v].parent
            while u > 0:
                mask[r_, nodes[u].cache_idx] = 1
                u = nodes[u].parent
            mask[r_, base + tree_cache + r_] = 1
        return mask

    def _verify(self, tree: DraftTree, kept, n, sp, rng):
        """python/woodcock/spec.py:307-329."""
        if tree.is_chain():
            z, feats = self.t.forward(tree.tokens, self.tc)
        else:
            pos = [n + d for d in tree.depth]
            mask = tree_attention_mask(tree, n).astype(np.uint8)
            z, feats = self.t.forward(tree.tokens, self.tc, positions=pos, mask=mask)
        if sp.greedy:
            path, nxt = verify_tree_greedy([argmax(r) for r in z], tree)
        else:
            p_all = probs_from_logits(z, sp).astype(np.float64)
            p = {v: p_all[v] for v in range(len(tree))}
            q = {v: kept[v].q for v in range(len(tree)) if kept[v].q is not None}
            path, nxt = verify_tree_stochastic(p, q, tree, rng)
        keep = [0] + path
        self.tc.compact(n, keep)
        return path, nxt, [f[keep] for f in feats]

    def _update(self, acc, feats):
        """python/woodcock/spec.py:366-374."""
        g = self.d.fuse(feats)
        hid, out = self.d.forward(acc, g, self.dc)
        self.root_out = out[-1:].copy()
        self.root_fb = self.d.feedback(hid[-1:], out[-1:]).copy()


def generate_autoregressive(t: Qwen3, prompt, max_new_tokens, sp=SamplingParams(), stop_on_eos=True,
                            eos=(151643, 151645), rng=None):
    """python/woodcock/spec.py:377-397; src/core/spec.cpp:282-311."""
    rng = rng if rng is not None else Tape(sp.seed)
    eos = set(eos) if stop_on_eos else set()
    cache = t.make_cache()

    def pick(z):
        if sp.greedy:
            return argmax(z)
        return sample(probs_from_logits(z[None], sp)[0].astype(np.float64), rng)

    z, _ = t.forward(prompt, cache, logits_from=len(prompt) - 1)
    tok = pick(z[-1])
    out = [tok]
    while len(out) < max_new_tokens and tok not in eos:
        z, _ = t.forward([tok], cache)
        tok = pick(z[-1])
        out.append(tok)
    return out


# ----------------------------------------------------------------------------- forced draft trees


def parse_template(line: str) -> list[tuple[int, int, int]]:
    """One draft-tree template: nodes 1..N-1 as "parent:offset:delta" (see forced_tree_run)."""
    nodes = []
    for item in line.split():
        p, o, d = (int(x) for x in item.split(":"))
        if not 0 <= p <= len(nodes):
            raise ValueError(f"template node parent {p} must precede the node")
        nodes.append((p, o, d))
    return nodes


def forced_tree_run(t: Qwen3, d: Drafter, prompt, max_new: int, templates: list[str]) -> dict:
    """Oracle-drafter rounds over given draft trees, restating the `forced` mode of
    oracle/ref_driver.cpp, which runs the reference's own draft / verify / update
    (src/core/spec.cpp:86-233) with the drafts taken from templates.

    A = the greedy continuation (generate_autoregressive). Round r instantiates template
    r mod len(templates) at e = tokens emitted so far: node i gets token A[e + offset_i] plus
    delta_i (mod vocab) under its parent. The drafter runs over every internal node level by level
    (positions n-1+depth, committed entries + drafted ancestors + itself visible,
    spec.cpp:158-171); the root's and every drafted node's head argmax and its logit are
    recorded. The target verifies with positions n+depth and the tree mask (a chain: causal),
    verify_tree_greedy picks the path, the cache keeps it and the drafter is updated on the
    accepted rows."""
    tpl = [parse_template(x) for x in templates]
    max_off = max(o for tp in tpl for _, o, _ in tp)
    A = generate_autoregressive(t, prompt, max_new + max_off + 2, stop_on_eos=False)
    tc, dc = t.make_cache(), d.make_cache()
    z, feats = t.forward(prompt, tc, logits_from=len(prompt) - 1)
    first = argmax(z[-1])
    hid, out = d.forward(list(prompt[1:]) + [first], d.fuse(feats), dc)
    root_out, root_fb = out[-1:].copy(), d.feedback(hid[-1:], out[-1:]).copy()
    emitted, rounds, accepted = [first], [], 0
    r = 0
    while len(emitted) < max_new:
        n, e = tc.size(), len(emitted)
        tokens, parents, depth = [emitted[-1]], [-1], [0]
        for p, o, dl in tpl[r % len(tpl)]:
            tokens.append((A[e + o] + dl) % t.vocab)
            parents.append(p)
            depth.append(depth[p] + 1)
        N = len(tokens)
        children = [[v for v in range(N) if parents[v] == u] for u in range(N)]
        outs, fbs, cidx = {0: root_out}, {0: root_fb}, {0: n - 1}
        prop, pz = [-1] * N, [0.0] * N

        def propose(v):
            zz = d.logits(outs[v])[0]
            prop[v] = d.token_ids(argmax(zz))
            pz[v] = float(zz[argmax(zz)])

        propose(0)
        base, drafted = dc.size(), 0
        for dep in range(1, max(depth)):
            level = [v for v in range(1, N) if depth[v] == dep and children[v]]
            if not level:
                break
            m = len(level)
            mask = np.zeros((m, base + drafted + m), np.uint8)
            lo = 0 if not d.window else max(0, base - 1 + dep - d.window + 1)
            for i, v in enumerate(level):
                mask[i, lo:base] = 1
                u = parents[v]
                while u > 0:
                    mask[i, cidx[u]] = 1
                    u = parents[u]
                mask[i, base + drafted + i] = 1
            fb = np.concatenate([fbs[parents[v]] for v in level], axis=0)
            h2, o2 = d.forward([tokens[v] for v in level], fb, dc, positions=[n - 1 + dep] * m, mask=mask)
            f2 = d.feedback(h2, o2)
            for i, v in enumerate(level):
                outs[v], fbs[v], cidx[v] = o2[i : i + 1], f2[i : i + 1], base + drafted + i
                propose(v)
            drafted += m
        dc.trim_to(base)
        tree = DraftTree(tokens, parents, depth)
        if tree.is_chain():
            zt, feats = t.forward(tokens, tc)
        else:
            zt, feats = t.forward(tokens, tc, positions=[n + x for x in depth],
                                  mask=tree_attention_mask(tree, n).astype(np.uint8))
        path, nxt = verify_tree_greedy([argmax(row) for row in zt], tree)
        keep = [0] + path
        tc.compact(n, keep)
        acc = [tokens[v] for v in path] + [nxt]
        hid, out = d.forward(acc, d.fuse([f[keep] for f in feats]), dc)
        root_out, root_fb = out[-1:].copy(), d.feedback(hid[-1:], out[-1:]).copy()
        accepted += len(path)
        rounds.append({"tokens": tokens, "parents": parents, "path": path, "next": nxt, "proposals": prop,
                       "proposal_logits": pz, "n": tc.size(), "drafter_len": dc.size()})
        emitted.extend(acc[: max_new - len(emitted)])
        r += 1
    return {"first": first, "ar": A, "rounds": rounds, "tokens": emitted, "accepted": accepted}
