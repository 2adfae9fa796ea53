"""Host-side routing policy and row buckets, the behaviour of gx/gx_ingest.py:55-108
and gx/gx_expert_worker.py:563-594 in the reference.

Id -1 is the unrouted/padded sentinel: served as a zero contribution. Any other
id outside [0, E) names no expert: the post is refused (RoutingError) before any
compute, because a partial output cannot be taken back once published.
"""

from __future__ import annotations

import numpy as np

E = 384
TOPK = 6
GRAPH_MAX = 16
EXACT_ROWS = frozenset({6})


class RoutingError(RuntimeError):
    """A post's routing names an expert that does not exist: the round is refused."""


def bucket_of(n: int) -> int:
    """Smallest power of two >= n (n >= 1) (gx_ingest.py:61-63)."""
    return 1 << max(0, (n - 1).bit_length())


def graph_rows(n: int) -> int:
    """Rows a captured step for n valid rows computes: exact for the decode's six,
    else the power-of-two bucket (gx_ingest.py:66-74)."""
    return n if n in EXACT_ROWS else bucket_of(n)


def classify_ids(ids: np.ndarray, n_experts: int = E) -> tuple[int, int]:
    """(padding slots, corrupt slots) in one post (gx_ingest.py:77-85)."""
    ids = np.asarray(ids)
    return int((ids == -1).sum()), int(((ids < -1) | (ids >= n_experts)).sum())


def routing_gate(ids: np.ndarray, n_experts: int = E, what: str = "post") -> int:
    """Padding count of a post; raise RoutingError if any id names no expert
    (gx_expert_worker.py:577-594)."""
    pad, bad = classify_ids(ids, n_experts)
    if bad:
        n = int(np.asarray(ids).size)
        raise RoutingError(f"{what}: {bad} of {n} routing slots name no expert "
                           f"(ids must be -1 or in [0, {n_experts})); refusing to serve a partial result")
    return pad
