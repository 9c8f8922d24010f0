"""Algorithmic bytes of a speculative round, the numerator of the HBM roofline.

A round reads every weight it multiplies once per pass plus the KV rows it attends
over (BASELINE's definition: weight bytes + KV bytes read per round):

    K drafter heads + (K - 1) drafter layer passes       (the draft chain)
  + target layers + target head                          (verification of K + 1 rows)
  + fuse FC + 1 drafter layer pass                       (the drafter update)
  + target KV over the context (once)
  + drafter KV over the context (once per drafter pass: K - 1 chain steps + the update).

With the drafter's auxiliary table (bf16 drafters whose hidden size is a multiple of 512), a
drafter pass reads the layer-0 Q/K/V weights of the feature input only, plus one fp32 table row
of Q+K+V values per row it processes, instead of the auxiliary Q/K/V weights.
"""

from __future__ import annotations

import os


def _target_params(t) -> dict:
    H, D = t.hidden, t.head_dim
    per_layer = (t.heads + 2 * t.kv_heads) * D * H + H * t.heads * D + 3 * t.intermediate * H
    return {"layers": per_layer * t.layers, "head": t.vocab * H, "per_layer": per_layer}


def aux_table_on(d) -> bool:
    """Whether the library precomputes the drafter's auxiliary term per token (WC_AUX_TABLE)."""
    return os.environ.get("WC_AUX_TABLE", "1") != "0" and d.hidden % 512 == 0


def _drafter_layer_params(d) -> int:
    H, D = d.hidden, d.head_dim
    qkv = (d.heads + 2 * d.kv_heads) * D * H
    aux = 0 if aux_table_on(d) else qkv  # layer 0 carries the auxiliary Q/K/V
    return qkv + aux + H * d.heads * D + 3 * d.intermediate * H


def _aux_row_bytes(d) -> int:
    """Table bytes one row of a drafter pass reads (fp32 Q+K+V), when the table is on."""
    return (d.heads + 2 * d.kv_heads) * d.head_dim * 4 if aux_table_on(d) else 0


def round_bytes(target, drafter, k: int, head_rows: int, ctx: int, wbytes: int = 2, kvbytes: int = 2) -> dict:
    tp = _target_params(target)
    dl = _drafter_layer_params(drafter) * drafter.layers
    fc = drafter.hidden * drafter.num_features * drafter.target_hidden
    head = head_rows * drafter.hidden
    t_kv_per_tok = target.layers * 2 * target.kv_heads * target.head_dim * kvbytes
    d_kv_per_tok = drafter.layers * 2 * drafter.kv_heads * drafter.head_dim * kvbytes
    out = {
        "draft_heads": k * head * wbytes,
        "draft_layers": (k - 1) * (dl * wbytes + _aux_row_bytes(drafter)),
        "target_weights": (tp["layers"] + tp["head"]) * wbytes,
        "update": (fc + dl) * wbytes + (k + 1) * _aux_row_bytes(drafter),
        "target_kv": ctx * t_kv_per_tok,
        "drafter_kv": k * ctx * d_kv_per_tok,
    }
    out["weights"] = out["draft_heads"] + out["draft_layers"] + out["target_weights"] + out["update"]
    out["kv"] = out["target_kv"] + out["drafter_kv"]
    out["total"] = out["weights"] + out["kv"]
    return out


def draft_step_bytes(drafter, head_rows: int, ctx: int, wbytes: int = 2, kvbytes: int = 2) -> int:
    """One chain step: head + one drafter layer pass + its KV reads (scripts/time_draft_step.py `step`)."""
    dl = _drafter_layer_params(drafter) * drafter.layers
    return (head_rows * drafter.hidden + dl) * wbytes + _aux_row_bytes(drafter) + \
        ctx * drafter.layers * 2 * drafter.kv_heads * drafter.head_dim * kvbytes
