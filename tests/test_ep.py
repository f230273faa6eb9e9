"""Expert parallelism on the CPU: the exchange layout and the whole split,
restated in oracle/ep.py, against the single-device oracle MoE
(src/model/moe.rs:424-466); the two-rank exchange protocol over gloo; the
host-side liveness check; and the library's argument checks (no GPU calls).
The CUDA kernels are held to the same restatement by tests/test_gpu_ep.py.

Tolerance: max |split - single| / max |single| <= 1e-2 (the split only
reassociates the fp32 sum over experts)."""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import oracle
from oracle import ep as oep

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TOL = 1e-2


def _table():
    d = np.load(os.path.join(GOLD, "moe_small.npz"))
    H, I, E, k, _ = (int(v) for v in d["dims"])
    return d, H, I, E, k


def _tokens(n, H, seed):
    rng = np.random.default_rng(seed)
    return oracle.f32_to_bf16(rng.standard_normal((n, H)).astype(np.float32))


def _route(d, x, k, bias=None):
    if x.shape[0] == 0:
        return np.zeros((0, k), np.int32), np.zeros((0, k), np.float32)
    ids, w, _ = oracle.router(x, d["wr"], k, logit_bias=bias)
    return ids, w


def _single(d, x, ids, w, H, I):
    if x.shape[0] == 0:
        return np.zeros((0, H), np.float32)
    y32, _ = oracle.moe_experts(x, ids, w, d["buf"], int(d["stride"]), d["offsets"], H, I)
    return y32


def _rel(a, b):
    if a.size == 0:
        return 0.0
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def test_plan_and_pack_layout():
    # 4 experts per rank, 2 ranks; token 2 has both experts on rank 1, token 3 none valid
    ids = np.array([[0, 5], [1, 2], [6, 7], [-1, -1], [4, 3]], np.int32)
    wts = np.arange(10, dtype=np.float32).reshape(5, 2)
    slots, counts = oep.plan(ids, R=2, per_rank=4, cap=6)
    assert counts.tolist() == [3, 3]
    assert slots[0].tolist() == [0, 1, -1, -1, 2, -1]
    assert slots[1].tolist() == [0, -1, 1, -1, 2, -1]
    x = np.arange(5 * 8, dtype=np.uint16).reshape(5, 8)
    sx, sids, swts = oep.pack(x, ids, wts, slots, counts, cap=6)
    assert (sx[1, 1] == x[2]).all() and (sids[1, 1] == ids[2]).all() and (swts[1, 1] == wts[2]).all()
    assert (sids[0, 3:] == -1).all() and (sids[1, 3:] == -1).all()  # padding selects no expert


@pytest.mark.parametrize("R", [1, 2, 4, 8])
def test_simulated_split_matches_single_device(R):
    d, H, I, E, k = _table()
    sizes = [5, 0, 3, 7, 1, 4, 2, 6][:R]  # ragged, one rank without tokens when R > 1
    xs = [_tokens(n, H, 10 + r) for r, n in enumerate(sizes)]
    routed = [_route(d, x, k) for x in xs]
    outs = oep.simulate(xs, [r[0] for r in routed], [r[1] for r in routed], R, d["buf"], int(d["stride"]),
                        d["offsets"], H, I, E, cap=max(sizes))
    for x, (ids, w), y in zip(xs, routed, outs):
        assert y.shape == (x.shape[0], H)
        assert _rel(oracle.bf16_to_f32(y), _single(d, x, ids, w, H, I)) <= TOL


@pytest.mark.parametrize("R", [2, 4])
def test_peer_memory_windows_match_the_exchange(R):
    """The P2P mode's window protocol (stores at block `me` of the owner's
    window, ids -1 over the rest of the block, partial sums returned for the
    first rx_cnt rows only) over windows holding stale rows gives the same
    outputs as the send/recv exchange, bit for bit."""
    d, H, I, E, k = _table()
    sizes = [5, 0, 3, 7][:R]
    xs = [_tokens(n, H, 50 + r) for r, n in enumerate(sizes)]
    routed = [_route(d, x, k) for x in xs]
    args = ([r[0] for r in routed], [r[1] for r in routed], R, d["buf"], int(d["stride"]), d["offsets"], H, I, E)
    want = oep.simulate(xs, *args, cap=max(sizes))
    got = oep.simulate_p2p(xs, *args, cap=max(sizes), stale_seed=R)
    for a, b in zip(got, want):
        assert np.array_equal(a, b)


def test_simulated_split_all_tokens_to_one_rank():
    """Every token routed to experts of the last rank: the other ranks receive
    nothing but still take part."""
    d, H, I, E, k = _table()
    R = 4
    bias = np.zeros(E, np.float32)
    bias[E - 2:] = 1e4
    xs = [_tokens(3, H, 30 + r) for r in range(R)]
    routed = [_route(d, x, k, bias) for x in xs]
    assert all(set(np.unique(r[0]).tolist()) == {E - 2, E - 1} for r in routed)
    outs = oep.simulate(xs, [r[0] for r in routed], [r[1] for r in routed], R, d["buf"], int(d["stride"]),
                        d["offsets"], H, I, E, cap=3)
    for x, (ids, w), y in zip(xs, routed, outs):
        assert _rel(oracle.bf16_to_f32(y), _single(d, x, ids, w, H, I)) <= TOL


# ---------------------------------------------------------------------------
# two ranks over gloo: the exchange protocol with real collectives


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _exchange_worker(rank, world, port, exact, q):
    import torch
    import torch.distributed as dist

    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        d, H, I, E, k = _table()
        sizes = [4, 6]
        cap = max(sizes)
        x = _tokens(sizes[rank], H, 50 + rank)
        ids, w = _route(d, x, k)
        per = E // world
        slots, counts = oep.plan(ids, world, per, cap)
        sx, sids, swts = oep.pack(x, ids, w, slots, counts, cap)
        if exact:  # counts first, then only the routed rows
            rc = torch.zeros(world, dtype=torch.int32)
            dist.all_to_all_single(rc, torch.from_numpy(counts))
            send_n, recv_n = counts.tolist(), rc.tolist()
        else:      # every block is cap rows
            send_n, recv_n = [cap] * world, [cap] * world

        def a2a(blocks, width, dtype, sn, rn):
            src = torch.from_numpy(np.concatenate([blocks[p][:sn[p]] for p in range(world)]).reshape(-1, width))
            dst = torch.empty(sum(rn), width, dtype=dtype)
            dist.all_to_all_single(dst, src, output_split_sizes=rn, input_split_sizes=sn)
            return dst.numpy()

        rx = a2a(sx.view(np.uint8), 2 * H, torch.uint8, send_n, recv_n).view(np.uint16)
        rids = a2a(sids, k, torch.int32, send_n, recv_n)
        rwts = a2a(swts, k, torch.float32, send_n, recv_n)
        part = oep.local_partial(rx, rids, rwts, d["buf"], int(d["stride"]), d["offsets"], H, I, rank * per, per)
        # back: my partials of sender p's rows go to p, into its block for me
        offs = np.concatenate([[0], np.cumsum(recv_n)])
        back = a2a([part[offs[p]:offs[p + 1]] for p in range(world)], H, torch.float32, recv_n, send_n)
        ret = np.zeros((world, cap, H), np.float32)
        o = 0
        for p in range(world):
            ret[p, :send_n[p]] = back[o:o + send_n[p]]
            o += send_n[p]
        y = oep.combine(ret, slots, x.shape[0])
        err = _rel(oracle.bf16_to_f32(y), _single(d, x, ids, w, H, I))
        dist.destroy_process_group()
        q.put((rank, err, None))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, None, repr(e)))


@pytest.mark.parametrize("exact", [False, True])
def test_gloo_two_rank_exchange(exact):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, exact, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            rank, err, exc = q.get(timeout=120)
            res[rank] = (err, exc)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for rank, (err, exc) in res.items():
        assert exc is None, f"rank {rank}: {exc}"
        assert err <= TOL, (rank, err)


# ---------------------------------------------------------------------------
# failure detection on the host: a rank that leaves between steps


def _watch_worker(rank, world, port, q):
    import torch.distributed as dist

    import __graft_entry__

    fm = __graft_entry__.load_package()
    store = dist.TCPStore("127.0.0.1", port, world, is_master=rank == 0, timeout=__import__("datetime").timedelta(
        seconds=30))
    watch = fm.PeerWatch(store, rank, world, prefix="t")
    try:
        watch.arrive(timeout_s=20)       # step 0: everyone
        if rank == 1:
            q.put((rank, "left"))
            return                        # rank 1 leaves between steps
        watch.arrive(timeout_s=1.5)      # step 1: rank 1 never checks in
        q.put((rank, "no error"))
    except fm.PeerLost as e:
        q.put((rank, f"PeerLost: {e}"))
    except Exception as e:
        q.put((rank, repr(e)))


def test_peer_watch_reports_a_lost_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_watch_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            rank, msg = q.get(timeout=120)
            res[rank] = msg
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert res[1] == "left"
    assert res[0].startswith("PeerLost") and "[1]" in res[0], res[0]


# ---------------------------------------------------------------------------
# library argument checks (return before any device work)


def test_ep_abi_argument_checks(fm):
    L = fm.lib()
    H, I, E = 256, 128, 16
    offs, _, stride = fm.ecb_layout(H, I)
    full = fm.ExpertsC(0x1000, stride, (ctypes.c_int64 * 9)(*offs), E, 0, H, I, 4, 64)
    part = fm.ExpertsC(0x1000, stride, (ctypes.c_int64 * 9)(*offs), E // 2, E // 2, H, I, 4, 64)
    r = fm.RouterC(fm.QWeightC(0x1000, None, None, E, H, 16, 64), None, None, None, H ** -0.5, 1e-6, 0, 4)
    small = L.fmoe_ep_moe_workspace_bytes(2, 8, ctypes.byref(r), ctypes.byref(part))
    big = L.fmoe_ep_moe_workspace_bytes(2, 512, ctypes.byref(r), ctypes.byref(part))
    assert 0 < small < big
    assert L.fmoe_ep_moe_workspace_bytes(0, 8, ctypes.byref(r), ctypes.byref(part)) == 0
    assert L.fmoe_ep_moe_workspace_bytes(2, 0, ctypes.byref(r), ctypes.byref(part)) == 0
    # null communicator -> FMOE_ERR_INVALID
    rc = L.fmoe_ep_moe_forward(None, 0x1000, 4, 8, ctypes.byref(r), ctypes.byref(full), None, 0x1000, None, None, 0,
                               None, 0, None)
    assert rc == -1 and "communicator" in fm.last_error()
    assert L.fmoe_ep_comm_init(None, 2, 0, None, 0) in (-1, -7)
    # the peer-memory windows need a communicator (FMOE_ERR_NCCL where libnccl is absent)
    assert L.fmoe_ep_p2p_init(None, 4, 2816, 8) in (-1, -7)
    with pytest.raises(ValueError):
        fm.shard_range(128, 3, 0)
    assert fm.shard_range(128, 8, 7) == (112, 16)
