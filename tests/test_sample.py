"""CPU checks of the sampling oracle (oracle/sample.py): the generator against
splitmix64's published outputs, the repetition penalty, temperature 0, the
top-p cut, and the draw's distribution (P(token) proportional to p' + 1e-10,
engine.rs:352-354)."""
import numpy as np
import pytest

from oracle import sample as smp


def test_mix64_matches_splitmix64_published_sequence():
    # splitmix64 seeded with 0: state += 0x9E3779B97F4A7C15, output = mix(state)
    state, out = 0, []
    for _ in range(3):
        state = (state + 0x9E3779B97F4A7C15) % (1 << 64)
        out.append(int(smp.mix64(np.uint64(state))))
    assert out == [0xE220A8397B1DCDAF, 0x6E789E6AA1B965F4, 0x06C45D188009454F]


def test_uniforms_open_interval_and_keyed():
    u = smp.uniforms(7, 3, 1, 100000)
    assert u.dtype == np.float32 and u.min() > 0 and u.max() < 1
    assert np.all(u == smp.uniforms(7, 3, 1, 100000))
    assert not np.all(u == smp.uniforms(7, 4, 1, 100000))  # another call number
    assert not np.all(u == smp.uniforms(7, 3, 2, 100000))  # another row
    assert abs(float(u.mean()) - 0.5) < 0.01


def test_penalty_each_distinct_token_once():
    z = np.array([2.0, -2.0, 1.0, 0.0, 4.0], np.float32)
    out = smp.penalize(z, [0, 1, 0, 0, 7, -1, 3], 2.0)  # duplicates, out of range, empty slot
    assert out.tolist() == [1.0, -4.0, 1.0, 0.0, 4.0]
    assert smp.penalize(z, [0, 1], 1.0).tolist() == z.tolist()  # penalty <= 1: untouched


def test_temperature_zero_is_first_argmax():
    lg = np.array([[1.0, 3.0, 3.0, 2.0], [5.0, 1.0, 1.0, 5.0]], np.float32)
    assert smp.sample(lg, None, 0.0, 1.0, 1.0).tolist() == [1, 0]
    # the penalty can move the argmax
    assert smp.sample(lg, np.array([[1, 1], [0, 0]]), 0.0, 1.0, 2.0).tolist() == [2, 3]


def test_top_p_cut():
    z = np.log(np.array([0.15, 0.5, 0.05, 0.3], np.float32)).astype(np.float32)
    order, kept, _ = smp.kept_prefix(z, 0.7)  # running sums before each: 0, .5, .8, .95
    assert order.tolist() == [1, 3, 0, 2] and kept == 2
    assert smp.kept_prefix(z, 0.0)[1] == 1  # the most likely token always stays
    assert smp.kept_prefix(z, 0.99)[1] == 4


@pytest.mark.parametrize("top_p", [1.0, 0.7])
def test_draw_distribution(top_p):
    p = np.array([0.15, 0.5, 0.05, 0.3], np.float64)
    lg = np.log(p).astype(np.float32)[None]
    n = 20000
    draws = np.array([smp.sample(lg, None, 1.0, top_p, 1.0, seed=11, step=s)[0] for s in range(n)])
    want = p.copy()
    if top_p < 1.0:
        want[[0, 2]] = 0
    want = (want / want.sum() + 1e-10)
    want /= want.sum()
    freq = np.bincount(draws, minlength=4) / n
    assert np.all(np.abs(freq - want) <= 4 * np.sqrt(want * (1 - want) / n) + 1e-4), (freq, want)


def test_sample_abi_rejects_bad_arguments_before_any_launch(fm):
    """Argument checks run on the host before any CUDA call (no GPU needed)."""
    L = fm.lib()
    assert L.fmoe_sample_workspace_bytes(0, 10) == 0 and L.fmoe_sample_workspace_bytes(70000, 10) == 0
    bad = [  # logits, rows, vocab, recent, n_recent, temperature, top_p, penalty, step, push, out
        (None, 2, 10, None, 0, 1.0, 1.0, 1.0, None, 0, 0x1000),      # null logits
        (0x1000, 0, 10, None, 0, 1.0, 1.0, 1.0, None, 0, 0x1000),    # no rows
        (0x1000, 2, 10, None, 0, -1.0, 1.0, 1.0, None, 0, 0x1000),   # negative temperature
        (0x1000, 2, 10, None, 0, 1.0, 1.0, 0.0, None, 0, 0x1000),    # penalty 0
        (0x1000, 2, 10, None, 4, 1.0, 1.0, 1.2, None, 0, 0x1000),    # recent count without a list
        (0x1000, 2, 10, 0x1000, 4, 1.0, 1.0, 1.2, None, 1, 0x1000),  # ring push without the counter
    ]
    for lg, rows, V, rc, n, T, tp, pen, step, push, out in bad:
        assert L.fmoe_sample(lg, rows, V, rc, n, T, tp, pen, 0, step, push, out, None, 0, None) == -1


def test_oracle_against_committed_fixture():
    """Regression of the sampling oracle against tests/golden/sample_small.npz
    (made by tests/golden/make_golden.py)."""
    import os

    d = np.load(os.path.join(os.path.dirname(__file__), "golden", "sample_small.npz"))
    assert np.array_equal(smp.uniforms(99, 0, 0, 8), d["uniforms"])
    for c, (T, top_p, pen) in enumerate(d["cases"]):
        for s in range(3):
            got = smp.sample(d["logits"], d["recent"], float(T), float(top_p), float(pen), seed=99, step=s)
            assert np.array_equal(got, d["tokens"][c, s]), (c, s)
