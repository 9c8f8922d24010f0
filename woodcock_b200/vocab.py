"""Frequency-truncated draft vocabularies (python/woodcock/vocab.py:35-51, 83-87): the
drafter's LM head keeps the K token ids the target generates most often, always including
the end-of-sequence ids, sorted ascending; `Drafter.restrict_vocab` gathers those head rows
on the device (drafter.py:217-229)."""

from __future__ import annotations

from pathlib import Path

import numpy as np


def top_ids(counts, k: int, always=frozenset()) -> np.ndarray:
    """The k most frequent ids (equal counts: the smaller id first) with every id of
    `always` included, as int32 in ascending order (vocab.py:35-47)."""
    counts = np.asarray(counts)
    if not 0 < k <= len(counts):
        raise ValueError(f"vocabulary size {k} not in 1..{len(counts)}")
    forced = sorted({int(a) for a in always})
    if len(forced) > k:
        raise ValueError("more forced ids than k")
    # descending counts, ties by ascending id: sort the keys (-count, id)
    order = np.lexsort((np.arange(len(counts)), -counts.astype(np.int64)))
    taken = np.zeros(len(counts), dtype=bool)
    taken[forced] = True
    rest = order[~taken[order]][: k - len(forced)]
    return np.sort(np.concatenate([np.asarray(forced, dtype=np.int64), rest])).astype(np.int32)


def coverage(counts, ids) -> float:
    """Share of the counted tokens that the kept ids cover (vocab.py:50-52)."""
    counts = np.asarray(counts)
    total = counts.sum()
    return float(counts[np.asarray(ids)].sum() / total) if total else 0.0


def load_ids(spec: str) -> np.ndarray:
    """'<counts.npz>:<K>' (arrays `counts` and `eos`) -> draft vocabulary ids (vocab.py:83-87)."""
    path, sep, k = str(spec).rpartition(":")
    if not sep or not path:
        raise ValueError("vocabulary spec must be '<counts.npz>:<K>'")
    with np.load(Path(path)) as z:
        return top_ids(z["counts"], int(k), {int(e) for e in z["eos"]})
