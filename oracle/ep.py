"""Expert-parallel exchange — CPU restatement, TEST INFRASTRUCTURE ONLY.

The reference runs every routed expert on one device (Gemma4MoeBlock::forward,
src/model/moe.rs:361-466); its answer for a token is the oracle's
moe_experts().  This file restates, in numpy, the split that libfmoe's
expert-parallel path performs (experts contiguous over R ranks, a token sent
once to each rank that owns one of its experts, per-rank fp32 partial sums
added back in ascending rank order and rounded to bf16 once), so that tests
can check the
exchange layout rank by rank and the whole split against the single-device
answer.  Only tests/ use it.

Layout (the same as the library's):
    slots[r, t]  position of token t in rank r's block, -1 if none of its
                 experts is on r; positions count earlier tokens routed to r
    counts[r]    tokens routed to rank r
    send blocks  [R, cap, .]: rows 0..counts[r]-1 in slot order; the id rows of
                 the padding (counts[r]..cap-1) are -1
"""
from __future__ import annotations

import numpy as np

from . import f32_to_bf16, moe_experts


def plan(ids: np.ndarray, R: int, per_rank: int, cap: int):
    """-> slots int32 [R, cap] (-1 past T), counts int32 [R]."""
    T = ids.shape[0]
    owner = ids // per_rank  # [T, k]; ids < 0 give owner < 0
    slots = np.full((R, cap), -1, np.int32)
    counts = np.zeros(R, np.int32)
    for r in range(R):
        hit = np.any((owner == r) & (ids >= 0), axis=1)
        pos = np.cumsum(hit) - 1
        slots[r, :T] = np.where(hit, pos, -1)
        counts[r] = int(hit.sum())
    return slots, counts


def pack(x: np.ndarray, ids: np.ndarray, wts: np.ndarray, slots: np.ndarray, counts: np.ndarray, cap: int):
    """-> send_x uint16 [R, cap, H], send_ids int32 [R, cap, k], send_wts f32 [R, cap, k]."""
    R = slots.shape[0]
    T, H = x.shape
    k = ids.shape[1] if ids.ndim == 2 else 0
    sx = np.zeros((R, cap, H), np.uint16)
    sids = np.full((R, cap, k), -1, np.int32)
    swts = np.zeros((R, cap, k), np.float32)
    for r in range(R):
        for t in range(T):
            s = slots[r, t]
            if s >= 0:
                sx[r, s] = x[t]
                sids[r, s] = ids[t]
                swts[r, s] = wts[t]
    return sx, sids, swts


def local_partial(rx: np.ndarray, rids: np.ndarray, rwts: np.ndarray, buf: np.ndarray, stride: int, offsets,
                  hidden: int, inter: int, first: int, n: int) -> np.ndarray:
    """fp32 [rows, H]: sum over the row's experts in [first, first + n) of
    w * expert(x) (ascending expert id); rows with no local expert give 0.
    buf is the WHOLE table (global ids index it)."""
    rows = rx.shape[0]
    out = np.zeros((rows, hidden), np.float32)
    if rows == 0:
        return out
    local = (rids >= first) & (rids < first + n)
    ids = np.where(local, rids, first).astype(np.int32)   # non-local slots: weight 0 on a local expert
    w = np.where(local, rwts, 0.0).astype(np.float32)
    keep = local.any(axis=1)
    if keep.any():
        y32, _ = moe_experts(rx[keep], ids[keep], w[keep], buf, stride, offsets, hidden, inter)
        out[keep] = y32
    return out


def combine(ret: np.ndarray, slots: np.ndarray, T: int) -> np.ndarray:
    """y bf16 [T, H] = bf16(sum over r ascending of ret[r, slots[r, t]]) (fp32 partials and sums)."""
    R, _, H = ret.shape
    acc = np.zeros((T, H), np.float32)
    for r in range(R):
        for t in range(T):
            s = slots[r, t]
            if s >= 0:
                acc[t] += ret[r, s]
    return f32_to_bf16(acc)


def simulate(xs, idss, wtss, R: int, buf, stride, offsets, hidden: int, inter: int, num_experts: int, cap: int):
    """The whole exchange for R ranks in one process: xs / idss / wtss are the
    per-rank token rows and routing.  Returns the per-rank outputs (bf16)."""
    per = num_experts // R
    plans = [plan(ids, R, per, cap) for ids in idss]
    sends = [pack(x, ids, w, s, c, cap) for x, ids, w, (s, c) in zip(xs, idss, wtss, plans)]
    # dispatch: rank p receives block p of every sender q (only counts[p] rows matter)
    parts = []
    for p in range(R):
        rx = np.concatenate([sends[q][0][p] for q in range(R)])
        rids = np.concatenate([sends[q][1][p] for q in range(R)])
        rwts = np.concatenate([sends[q][2][p] for q in range(R)])
        parts.append(local_partial(rx, rids, rwts, buf, stride, offsets, hidden, inter, p * per, per)
                     .reshape(R, cap, hidden))
    # combine: sender q gets, from every p, the partials of its own block p
    outs = []
    for q in range(R):
        ret = np.stack([parts[p][q] for p in range(R)])
        outs.append(combine(ret, plans[q][0], xs[q].shape[0]))
    return outs


def simulate_p2p(xs, idss, wtss, R: int, buf, stride, offsets, hidden: int, inter: int, num_experts: int, cap: int,
                 stale_seed: int = 0):
    """The peer-memory exchange (FMOE_EP_P2P) restated on per-rank windows that
    still hold an earlier exchange's rows (stale data): sender `me` stores each
    routed row into block `me` of the owner's window at its slot, writes ids -1
    over the rest of that block and its count into rx_cnt[me] (the dispatch
    kernel); every rank runs its experts on its whole window; rank `me` stores
    the first rx_cnt[r] partial rows of block r into block `me` of rank r's
    returned rows (the return kernel); each rank combines from its own window.
    Must give simulate()'s outputs exactly.  (The ids -1 over a block's tail
    only keep stale rows from selecting experts — work, not results: their
    partial rows are never returned.)"""
    per = num_experts // R
    k = idss[0].shape[1]
    g = np.random.default_rng(stale_seed)
    wins = [{"rx": g.integers(0, 0x3F80, (R * cap, hidden), dtype=np.uint16),  # finite stale bf16 rows
             "rids": g.integers(0, num_experts, (R * cap, k)).astype(np.int32),
             "rwts": g.random((R * cap, k), dtype=np.float32),
             "ret": g.standard_normal((R * cap, hidden)).astype(np.float32),
             "rx_cnt": np.full(R, -7, np.int32)} for _ in range(R)]
    plans = [plan(ids, R, per, cap) for ids in idss]
    for me in range(R):  # dispatch
        slots, counts = plans[me]
        for r in range(R):
            w = wins[r]
            w["rx_cnt"][me] = counts[r]
            for t in range(xs[me].shape[0]):
                s = slots[r, t]
                if s >= 0:
                    row = me * cap + s
                    w["rx"][row], w["rids"][row], w["rwts"][row] = xs[me][t], idss[me][t], wtss[me][t]
            w["rids"][me * cap + counts[r]:(me + 1) * cap] = -1
            w["rwts"][me * cap + counts[r]:(me + 1) * cap] = 0.0
    ypart = [local_partial(w["rx"], w["rids"], w["rwts"], buf, stride, offsets, hidden, inter, p * per, per)
             for p, w in enumerate(wins)]
    for me in range(R):  # return
        for r in range(R):
            n = int(wins[me]["rx_cnt"][r])
            wins[r]["ret"][me * cap:me * cap + n] = ypart[me][r * cap:r * cap + n]
    return [combine(wins[q]["ret"].reshape(R, cap, hidden), plans[q][0], xs[q].shape[0]) for q in range(R)]
