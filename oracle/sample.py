"""Next-token sampling — CPU restatement, TEST INFRASTRUCTURE ONLY.

Restates the engine's sample() (src/engine.rs:302-355) in numpy fp32 for
libfmoe's fmoe_sample, with the random draw made reproducible: the reference
draws through MLX's categorical (engine.rs:352-354); here the draw is the
Gumbel-max argmax of log(p + 1e-10) + G, G = -log(E), E = -log(u), with u from
a splitmix64 hash keyed by (seed, call number, row, token) — the same draw the
library makes, so tests can compare tokens, and a draw has the distribution
P(token) proportional to p + 1e-10 that the reference samples from.  Parity
with the reference itself is unpinned (MLX is not available here).  Only
tests/ use it.
"""
from __future__ import annotations

import numpy as np

M64 = (1 << 64) - 1


def mix64(z: np.ndarray) -> np.ndarray:
    """splitmix64's output function (Steele, Lea & Flood 2014), uint64 arrays."""
    z = np.asarray(z, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def row_key(seed: int, step: int, row: int) -> np.uint64:
    a = np.uint64(seed & M64) ^ np.uint64((step * 0x9E3779B97F4A7C15) & M64)
    b = mix64(a) ^ np.uint64((row * 0xD1B54A32D192ED03) & M64)
    return mix64(b)


def uniforms(seed: int, step: int, row: int, vocab: int) -> np.ndarray:
    """u[token] = (k + 0.5) / 2^23, k = the top 23 bits of the token's hash."""
    key = row_key(seed, step, row)
    idx = np.arange(vocab, dtype=np.uint64)
    with np.errstate(over="ignore"):
        b = mix64(key + idx * np.uint64(0xA0761D6478BD642F))
    k = (b >> np.uint64(41)).astype(np.float32)
    return (k + np.float32(0.5)) * np.float32(1.0 / 8388608.0)


def penalize(logits: np.ndarray, recent, penalty: float) -> np.ndarray:
    """engine.rs:305-327: each distinct recent token inside the vocabulary once;
    logit >= 0 divided by the penalty, negative multiplied (fp32)."""
    z = np.array(logits, dtype=np.float32, copy=True)
    if penalty > 1.0 and recent is not None and len(recent):
        p = np.float32(penalty)
        seen = set()
        for t in recent:
            t = int(t)
            if t < 0 or t >= z.shape[0] or t in seen:
                continue
            seen.add(t)
            z[t] = z[t] / p if z[t] >= 0 else z[t] * p
    return z


def kept_prefix(z: np.ndarray, top_p: float):
    """engine.rs:335-350 -> (descending order (stable), number kept, max).
    A token is dropped when cumulative - p > top_p (cumulative = running fp32 sum
    of p in that order); the kept tokens form a prefix of the order."""
    order = np.argsort(-z, kind="stable")
    m = np.float32(z.max())
    e = np.exp((z[order] - m).astype(np.float32)).astype(np.float32)
    p = (e / np.float32(e.sum(dtype=np.float32))).astype(np.float32)
    cum = np.cumsum(p, dtype=np.float32)
    drop = (cum - p) > np.float32(top_p)
    kept = int(np.argmax(drop)) if drop.any() else z.shape[0]
    assert not drop[:kept].any() and drop[kept:].all(), "cut is not a prefix"
    return order, kept, m


def scores(logits_row: np.ndarray, recent, temperature: float, top_p: float, penalty: float, seed: int,
           step: int, row: int, kept_override: int | None = None) -> np.ndarray:
    """Per-token Gumbel-max score (p' + 1e-10) / E of one row (temperature > 0).
    kept_override replaces the top-p cut's token count (near-tie analysis)."""
    z = penalize(logits_row, recent, penalty) / np.float32(temperature)
    z = z.astype(np.float32)
    V = z.shape[0]
    m = np.float32(z.max())
    e = np.exp((z - m).astype(np.float32)).astype(np.float32)
    if top_p < 1.0:
        order, kept, _ = kept_prefix(z, top_p)
        if kept_override is not None:
            kept = min(max(kept_override, 1), V)
        mask = np.zeros(V, bool)
        mask[order[:kept]] = True
        s = np.float32(e[mask].sum(dtype=np.float32))
        p = np.where(mask, e / s, np.float32(0)).astype(np.float32)
    else:
        p = (e / np.float32(e.sum(dtype=np.float32))).astype(np.float32)
    E = -np.log(uniforms(seed, step, row, V)).astype(np.float32)
    return ((p + np.float32(1e-10)) / E).astype(np.float32)


def sample(logits: np.ndarray, recent, temperature: float, top_p: float, penalty: float, seed: int = 0,
           step: int = 0) -> np.ndarray:
    """logits [rows, V] fp32, recent [rows, n] int (or None) -> tokens int32 [rows]."""
    rows = logits.shape[0]
    out = np.empty(rows, np.int32)
    for r in range(rows):
        rc = None if recent is None else recent[r]
        if temperature == 0.0:
            out[r] = int(np.argmax(penalize(logits[r], rc, penalty)))
        else:
            out[r] = int(np.argmax(scores(logits[r], rc, temperature, top_p, penalty, seed, step, r)))
    return out


def margin(logits_row, recent, temperature, top_p, penalty, seed, step, row, cut_tol: float = 2e-5) -> float:
    """How far a draw is from a near tie: the relative gap between the best and
    second-best score; 0 when, with top_p < 1, the winner changes as the cut
    moves over the tokens whose running sum before them lies within cut_tol of
    top_p (fp32 sums in another order can place the cut anywhere there).
    Moving the cut only adds or drops the tokens in between, so the two
    extreme cuts cover every cut in the range (up to the renormalisation, a
    relative change far below the score gap checked)."""
    if temperature == 0.0:
        z = np.sort(penalize(logits_row, recent, penalty))[::-1]
        return float((z[0] - z[1]) / max(abs(z[0]), 1e-30)) if z.shape[0] > 1 else 1.0
    sc = scores(logits_row, recent, temperature, top_p, penalty, seed, step, row)
    s = np.sort(sc)[::-1]
    g = float((s[0] - s[1]) / s[0]) if s.shape[0] > 1 else 1.0
    if top_p < 1.0:
        z = (penalize(logits_row, recent, penalty) / np.float32(temperature)).astype(np.float32)
        order, kept, m = kept_prefix(z, top_p)
        e = np.exp((z[order] - m).astype(np.float64))
        excl = np.cumsum(e / e.sum()) - e / e.sum()
        near = np.flatnonzero(np.abs(excl - top_p) <= cut_tol)
        lo = min(kept, int(near.min())) if near.size else kept
        hi = max(kept, int(near.max()) + 1) if near.size else kept
        win = int(np.argmax(sc))
        for k in {lo, hi, kept - 1, kept + 1}:
            if int(np.argmax(scores(logits_row, recent, temperature, top_p, penalty, seed, step, row,
                                    kept_override=k))) != win:
                return 0.0
    return g
