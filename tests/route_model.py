"""CPU model of the decode kernel's routing tables (route_sort in
qmesh-afd-tp3_b200/csrc/qx_decode_tc.cu), step for step at lane level: a warp of
32 lanes holds K keys each (pair lane + 32 j: expert << 9 | pair, no pair = all
ones); a bitonic network sorts them (element i = K lane + j); each pair's run
start and end come from a max scan and a suffix min scan over the sorted order,
its rank and group from the run; a group's first pair writes the group record.

Test infrastructure only: it restates the kernel's algorithm so that the tests
can check it against the direct grouping the reference uses (unique experts
ascending, an expert's pairs in (row, slot) order, split evenly into groups of
at most min(6, rows); gx/gx_decode_swz.py:148-179)."""

from __future__ import annotations

import numpy as np

NONE = 0xFFFFFFFF
XT_STAGE = 4096
SK = 8


def route_sort(ids: np.ndarray, rows: int, n_tiles: int, n_experts: int) -> tuple[list, list, int]:
    """ids [rows * topk] (any int; outside [0, E) = no pair) -> (groups, pair order, valid pairs);
    groups as (expert, gsz, pair_off, ab_off)."""
    P = ids.size
    K = 2 if P <= 64 else 4 if P <= 128 else 8 if P <= 256 else 16
    gmax = min(6, rows)
    N = 32 * K
    lane = np.arange(32)[:, None]
    j = np.arange(K)[None, :]
    q = lane + 32 * j
    e_in = np.full((32, K), -1, dtype=np.int64)
    e_in[q < P] = ids[q[q < P]]
    e_in[(e_in < 0) | (e_in >= n_experts)] = -1
    v = np.where(e_in >= 0, (e_in << 9) | q, NONE).astype(np.uint64)
    i = K * lane + j                                        # element index after the sort
    k = 2
    while k <= N:
        s = k >> 1
        while s > 0:
            if s >= K:                                      # partner in lane ^ (s / K)
                o = v[np.arange(32) ^ (s // K)]
                keep_min = ((i & k) == 0) == ((i & s) == 0)
                v = np.where(keep_min, np.minimum(v, o), np.maximum(v, o))
            else:                                           # partner in slot j ^ s
                o = v[:, np.arange(K) ^ s]
                asc = (i & k) == 0
                lower = (np.arange(K) & s) == 0
                v = np.where(asc == lower[None, :], np.minimum(v, o), np.maximum(v, o))
            s >>= 1
        k <<= 1
    flat = v.reshape(-1)                                    # flat[K lane + j]
    valid = flat != NONE
    e = np.where(valid, (flat >> 9).astype(np.int64), -1)
    Pv = int(valid.sum())
    idx = np.arange(N)
    f = valid & np.concatenate([[True], e[1:] != e[:-1]])   # first pair of an expert's run
    st = np.maximum.accumulate(np.where(f, idx, -1))
    nxt = np.where(f, idx, np.iinfo(np.int64).max)
    en = np.minimum.accumulate(nxt[::-1])[::-1]             # first start at or after i
    en = np.concatenate([en[1:], [np.iinfo(np.int64).max]])  # ... strictly after i
    end = np.minimum(en, Pv)
    c = np.where(valid, end - st, 1)
    r = idx - st
    ng = (c + gmax - 1) // gmax
    gk = ((r + 1) * ng - 1) // c
    gcount = np.cumsum(np.where(f, ng, 0))                  # inclusive group count
    abs_ = ((n_tiles + SK - 1) // SK) * XT_STAGE
    groups = {}
    for pos in np.flatnonzero(valid):
        lo = gk[pos] * c[pos] // ng[pos]
        if r[pos] == lo:
            gsz = (gk[pos] + 1) * c[pos] // ng[pos] - lo
            g = int(gcount[pos] - ng[pos] + gk[pos])
            assert g not in groups
            groups[g] = (int(e[pos]), int(gsz), int(pos), int(pos) * abs_)
    G = int(gcount[-1])
    assert sorted(groups) == list(range(G))
    order = [int(x & 511) for x in flat[valid]]
    return [groups[g] for g in range(G)], order, Pv


def direct_grouping(ids: np.ndarray, rows: int, n_tiles: int, n_experts: int) -> tuple[list, list, int]:
    gmax = min(6, rows)
    abs_ = ((n_tiles + SK - 1) // SK) * XT_STAGE
    groups, order, off = [], [], 0
    ok = [(q, int(x)) for q, x in enumerate(ids) if 0 <= x < n_experts]
    for ex in sorted({x for _, x in ok}):
        qs = [q for q, x in ok if x == ex]
        c = len(qs)
        ng = (c + gmax - 1) // gmax
        for kk in range(ng):
            lo, hi = kk * c // ng, (kk + 1) * c // ng
            groups.append((ex, hi - lo, off + lo, (off + lo) * abs_))
        order += qs
        off += c
    return groups, order, off
