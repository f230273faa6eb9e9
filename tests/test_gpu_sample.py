"""GPU parity of fmoe_sample (the engine's sample(), src/engine.rs:302-355)
against oracle/sample.py on the same logits and the same keyed draw.

Tokens must equal the oracle's wherever the oracle's draw is not a near tie
(best / second-best score, or the top-p cut, within 1e-5 relative): the
library's fp32 sums run in another order than numpy's.  Temperature 0 is an
exact argmax.  The draw's distribution is checked on the GPU over many rows.
"""
import numpy as np
import pytest
import torch

from oracle import sample as osmp

pytestmark = pytest.mark.gpu
NEAR = 1e-5


def _logits(rows, V, seed, scale=3.0):
    g = np.random.default_rng(seed)
    return (g.standard_normal((rows, V)) * scale).astype(np.float32)


def _recent(rows, n, V, seed):
    g = np.random.default_rng(seed)
    r = g.integers(-1, V + 3, size=(rows, n)).astype(np.int32)  # empty slots and out-of-range entries
    if n > 2:
        r[:, 1] = r[:, 0]  # a duplicate
    return r


CASES = [  # rows, vocab, temperature, top_p, penalty, n_recent
    (1, 64, 0.0, 1.0, 1.0, 0),
    (3, 1000, 0.0, 0.9, 1.3, 16),
    (2, 1000, 0.7, 1.0, 1.0, 0),
    (2, 1000, 1.3, 0.9, 1.2, 64),
    (4, 5000, 1.0, 0.5, 1.1, 64),
    (1, 4096, 0.8, 0.95, 1.0, 0),
    (1, 4097, 0.8, 0.95, 1.0, 0),
    (2, 262144, 0.8, 0.9, 1.1, 64),
    (2, 262144, 1.0, 1.0, 1.0, 0),
    (1, 262144, 0.0, 1.0, 1.5, 64),
]


@pytest.mark.parametrize("rows,V,T,top_p,pen,n", CASES)
def test_sample_matches_oracle(fm, dev, rows, V, T, top_p, pen, n):
    lg = _logits(rows, V, 100 + V + rows)
    rc = _recent(rows, n, V, 7 + n) if n else None
    ws = fm._Workspace()
    checked = 0
    for step in range(3):
        st = torch.tensor([step], dtype=torch.int64, device=dev)
        got = fm.sample_tokens(torch.from_numpy(lg).to(dev), T, top_p, pen,
                               None if rc is None else torch.from_numpy(rc).to(dev), seed=1234, step=st,
                               workspace=ws).cpu().numpy()
        assert int(st.item()) == step + 1  # the call counter advanced
        want = osmp.sample(lg, rc, T, top_p, pen, seed=1234, step=step)
        for r in range(rows):
            if T == 0.0 or osmp.margin(lg[r], None if rc is None else rc[r], T, top_p, pen, 1234, step, r) > NEAR:
                assert got[r] == want[r], (step, r, got[r], want[r])
                checked += 1
    assert checked >= 2 * rows  # most draws are far from a tie


def test_sample_distribution(fm, dev):
    """4096 rows with the same logits: each row's draw has its own key, so the
    token frequencies estimate P(token) proportional to p' + 1e-10."""
    p = np.array([0.02, 0.3, 0.05, 0.25, 0.18, 0.1, 0.06, 0.04], np.float64)
    rows = 4096
    lg = np.tile(np.log(p).astype(np.float32), (rows, 1))
    for top_p, drop in [(1.0, []), (0.8, [0, 2, 6, 7])]:  # running sums before: .3 .55 .73 .83 ...
        toks = []
        st = torch.zeros(1, dtype=torch.int64, device=dev)
        for _ in range(4):
            toks.append(fm.sample_tokens(torch.from_numpy(lg).to(dev), 1.0, top_p, 1.0, seed=5, step=st).cpu())
        toks = torch.cat(toks).numpy()
        want = p.copy()
        want[drop] = 0
        want = want / want.sum() + 1e-10
        want /= want.sum()
        n = toks.size
        freq = np.bincount(toks, minlength=8) / n
        assert np.all(np.abs(freq - want) <= 4.5 * np.sqrt(want * (1 - want) / n) + 1e-4), (top_p, freq, want)


def test_sampler_ring_and_graph_replay(fm, dev):
    """Sampler pushes each drawn token into its ring (slot = call number % window)
    and advances the call counter on the device; a CUDA graph replay draws the
    next keyed sample each time, as the oracle does with the ring's contents."""
    rows, V, win = 2, 3000, 4
    lg = _logits(rows, V, 99, scale=1.0)
    lt = torch.from_numpy(lg).to(dev)
    smp = fm.Sampler(rows, V, temperature=0.9, top_p=0.95, rep_penalty=1.3, seed=42, window=win, device=dev)
    out = torch.empty(rows, dtype=torch.int32, device=dev)
    smp(lt, out=out)  # eager call 0 (library set-up outside the capture)
    torch.cuda.synchronize()
    ring = np.full((rows, win), -1, np.int32)
    first = osmp.sample(lg, ring, 0.9, 0.95, 1.3, seed=42, step=0)
    assert out.cpu().numpy().tolist() == first.tolist()
    ring[:, 0] = first
    assert np.array_equal(smp.recent.cpu().numpy(), ring)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    got = []
    try:
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                smp(lt, out=out)
        torch.cuda.current_stream().wait_stream(s)
        for _ in range(6):
            graph.replay()
            torch.cuda.synchronize()
            got.append((out.cpu().numpy().copy(), smp.recent.cpu().numpy().copy()))
    finally:
        torch.cuda.synchronize()
        del graph
    assert int(smp.step.item()) == 7
    for i, (toks, r_after) in enumerate(got):
        step = i + 1
        want = osmp.sample(lg, ring, 0.9, 0.95, 1.3, seed=42, step=step)
        for r in range(rows):
            if osmp.margin(lg[r], ring[r], 0.9, 0.95, 1.3, 42, step, r) > NEAR:
                assert toks[r] == want[r], (step, r)
        ring[:, step % win] = toks  # the library's own draw goes into the ring
        assert np.array_equal(r_after, ring), step


def test_decode_step_with_sampler(fm, dev):
    """A two-layer model: set_sampler(temperature 0) gives the greedy ids; with
    temperature / top-p the step's ids equal the oracle's draw from the step's
    logits (the first call sees an empty ring)."""
    cfg = dict(fm.GEMMA4_26B, vocab=4096, full_every=2)
    m = fm.Gemma4Model.random(cfg, batch=2, max_positions=256, seed=31, device=dev, n_layers=2)
    m.ids.copy_(torch.tensor([3, 9], dtype=torch.int32))
    m.set_position(0)
    greedy = m.decode_step().clone()
    lg = m.logits.cpu().numpy()
    assert greedy.cpu().numpy().tolist() == osmp.sample(lg, None, 0.0, 1.0, 1.0).tolist()
    m2 = fm.Gemma4Model(cfg, m.embed, m.layers, m.final_norm, 2, 256, device=dev).set_sampler(0.8, 0.9, 1.2, seed=3)
    m2.ids.copy_(torch.tensor([3, 9], dtype=torch.int32))
    m2.set_position(0)
    got = m2.decode_step().cpu().numpy()
    lg2 = m2.logits.cpu().numpy()
    want = osmp.sample(lg2, np.full((2, 64), -1, np.int32), 0.8, 0.9, 1.2, seed=3, step=0)
    for r in range(2):
        if osmp.margin(lg2[r], None, 0.8, 0.9, 1.2, 3, 0, r) > NEAR:
            assert got[r] == want[r], r


def test_sample_rejects_bad_arguments(fm, dev):
    lg = torch.zeros(2, 10, device=dev)
    with pytest.raises(fm.FmoeError):
        fm.sample_tokens(lg, -1.0)
    with pytest.raises(fm.FmoeError):
        fm.sample_tokens(lg, 1.0, rep_penalty=0.0)
    ring = torch.full((2, 4), -1, dtype=torch.int32, device=dev)
    with pytest.raises(fm.FmoeError):  # a ring push needs the call counter
        fm.sample_tokens(lg, 1.0, recent=ring, push=True)
