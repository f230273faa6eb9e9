"""GPU parity of the expert-parallel MoE block and decoder (fmoe_ep_* /
fmoe_decoder_layer_forward_ep) against the CPU oracle and the single-device
path.

One GPU: a one-rank NCCL communicator runs the whole exchange (plan, pack,
grouped send/recv to itself, local experts, return, combine); mode 2 (the
peer-memory exchange) stores into the rank's own window.  Two GPUs (when
present): one process per GPU, 64 experts each; every rank checks its own
tokens against the single-device block holding all 128 experts.

Routing ids must equal the single-device ones; outputs within max |a - b| /
max |b| <= 1e-2 of the oracle (evaluated on the GPU's routing).  With one rank
the partial sum is the single-device sum, so decode outputs are bit-identical.
"""
import os
import queue
import socket
import time

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from gpu_util import max_rel_err, to_np_bf16

pytestmark = pytest.mark.gpu
TOL = 1e-2
H, I, E, K = 2816, 704, 128, 8


@pytest.fixture(scope="module")
def comm1(fm, dev):
    c = fm.EPComm(rank=0, world=1)
    yield c
    torch.cuda.synchronize()
    c.close()


@pytest.fixture(scope="module")
def layer(fm, dev):
    table = fm.ExpertTable.random(E, H, I, seed=2002, device=dev)
    g = torch.Generator(device=dev).manual_seed(2002)
    wr = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    bias = torch.randn(E, generator=g, device=dev)
    return table, wr, bias, table.buf.cpu().numpy()


def _oracle(orc, table, host, x, ids, w):
    y32, _ = orc.moe_experts(to_np_bf16(x), ids.cpu().numpy(), w.cpu().numpy(), host, table.stride, table.offsets,
                             table.hidden, table.inter)
    return y32


@pytest.mark.parametrize("T,cap,mode", [(5, 8, 0), (64, 64, 1), (300, 300, 0), (200, 256, 1), (0, 4, 0), (5, 8, 2),
                                        (300, 300, 2), (0, 4, 2)])
def test_ep_one_rank_matches_oracle(fm, orc, dev, comm1, layer, T, cap, mode):
    table, wr, bias, host = layer
    g = torch.Generator(device=dev).manual_seed(700 + T)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    router = fm.QuantizedLinear(wr, bits=16)
    ep = fm.ExpertParallelMoeBlock(comm1, router, table.shard(0, 1), cap=cap, top_k=K, mode=mode, logit_bias=bias)
    y, ids, w = ep.forward(x, return_routing=True)
    torch.cuda.synchronize()
    comm1.status()
    assert y.shape == (T, H)
    if T == 0:
        return
    ref = fm.Gemma4MoeBlock(router, table, top_k=K, logit_bias=bias)
    r_ids, r_w, _ = ref.route(x)
    assert torch.equal(ids, r_ids) and torch.equal(w, r_w)
    err = max_rel_err(y.float().cpu().numpy(), _oracle(orc, table, host, x, ids, w))
    assert err <= TOL, err
    assert torch.equal(y, ep.forward(x))  # deterministic


def _decoder_pair(fm, dev, comm, mode=0):
    cfg = dict(fm.GEMMA4_26B, vocab=4096, full_every=2)
    ctx = 300
    m1 = fm.Gemma4Model.random(cfg, batch=1, max_positions=1024, seed=21, device=dev, n_layers=2)
    m2 = fm.Gemma4Model(cfg, m1.embed, m1.layers, m1.final_norm, 1, 1024, device=dev, ep=comm, ep_mode=mode)
    g = torch.Generator(device=dev).manual_seed(22)
    for L, c1, c2 in zip(m1.layers, m1.caches, m2.caches):
        kv = torch.randn(2, 1, L.num_kv_heads, ctx, L.head_dim, generator=g, device=dev).to(torch.bfloat16)
        c1.update(kv[0], kv[1])
        c2.update(kv[0], kv[1])
    for m in (m1, m2):
        m.ids.fill_(5)
        m.set_position(ctx)
    want = [(m1.decode_step().clone(), m1.logits.clone()) for _ in range(3)]
    torch.cuda.synchronize()
    return m2, want


@pytest.mark.parametrize("mode", [0, 2])
def test_ep_decoder_one_rank_is_the_local_decoder(fm, dev, comm1, mode):
    """Two decoder layers: the expert-parallel layer call with one rank gives
    bit-identical tokens and logits to the local call (NCCL or peer-memory
    exchange)."""
    m2, want = _decoder_pair(fm, dev, comm1, mode)
    got = []
    for _ in range(3):
        got.append((m2.decode_step().clone(), m2.logits.clone()))
    torch.cuda.synchronize()
    comm1.status()
    for step, ((gi, gl), (wi, wl)) in enumerate(zip(got, want)):
        assert torch.equal(gl, wl), (step, float((gl - wl).abs().max()))
        assert torch.equal(gi, wi), step


@pytest.mark.parametrize("mode", [0, 2])
def test_ep_decoder_graph_replay(fm, dev, comm1, mode):
    """The same from a CUDA graph that captured the exchanges (position on the
    device; the peer-memory exchange's sequence counter lives on the device
    too).  The graph is released before any check, so a failure cannot leave
    the communicator with captured work outstanding."""
    m2, want = _decoder_pair(fm, dev, comm1, mode)
    got = []
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    try:
        with torch.cuda.stream(s):
            ids0, pos0 = m2.ids.clone(), m2.pos_dev.clone()
            m2.decode_step(device_pos=True)  # outside capture: library attribute setup
            torch.cuda.synchronize()
            m2.ids.copy_(ids0)
            m2.pos_dev.copy_(pos0)
            torch.cuda.synchronize()
            with torch.cuda.graph(graph, stream=s, capture_error_mode="thread_local"):
                m2.decode_step(device_pos=True)
        torch.cuda.current_stream().wait_stream(s)
        for _ in range(3):
            graph.replay()
            torch.cuda.synchronize()
            got.append((m2.ids.clone(), m2.logits.clone()))
    finally:
        torch.cuda.synchronize()
        del graph
        torch.cuda.synchronize()
    comm1.status()
    for step, ((gi, gl), (wi, wl)) in enumerate(zip(got, want)):
        assert torch.equal(gl, wl), (step, float((gl - wl).abs().max()))
        assert torch.equal(gi, wi), step


# ---------------------------------------------------------------------------
# two GPUs, one process each


def _prefill_pair(fm, dev, comm, rank=0, world=1, T=200):
    """A 2-layer model (window 64 < prompt) prefilled locally and, on the same
    weights with this rank's expert slice, through the expert-parallel layer
    prefill; returns (local logits, ids, expert-parallel model)."""
    cfg = dict(fm.GEMMA4_26B, vocab=4096, full_every=2, window=64)
    m1 = fm.Gemma4Model.random(cfg, batch=1, max_positions=512, seed=31, device=dev, n_layers=2)
    layers = []
    for L in m1.layers:  # the same weights, expert slice only
        layers.append(fm.Gemma4DecoderLayer(L.q_proj, L.k_proj, L.v_proj, L.o_proj, L.q_norm, L.k_norm, L.norms,
                                            L.mlp, L.router, L.experts.shard(rank, world) if world > 1 else L.experts,
                                            L.num_heads, L.num_kv_heads, L.head_dim, L.rope_dims, L.rope_theta,
                                            L.k_eq_v, L.eps, L.layer_scalar, L.attn_scale, L.top_k))
    m2 = fm.Gemma4Model(cfg, m1.embed, layers, m1.final_norm, 1, 512, device=dev, ep=comm, ep_mode=0)
    prompt = torch.randint(0, cfg["vocab"], (T,), generator=torch.Generator().manual_seed(7 + rank)).to(torch.int32)
    m1.prefill(prompt.to(dev))
    want_lg, want_id = m1.logits.clone(), m1.ids.clone()
    m2.prefill(prompt.to(dev))
    torch.cuda.synchronize()
    return want_lg, want_id, m2


def test_ep_prefill_one_rank_matches_local(fm, dev, comm1):
    """The whole-decoder prefill with the routed experts through the
    expert-parallel MoE (exact exchange; one rank) matches the local prefill:
    last-position logits and the next token."""
    want_lg, want_id, m2 = _prefill_pair(fm, dev, comm1)
    comm1.status()
    err = max_rel_err(m2.logits.cpu().numpy(), want_lg.cpu().numpy())
    assert err <= TOL, err
    top = torch.topk(want_lg[0], 2).values
    if top[0] - top[1] > 1e-3 * top[0].abs():
        assert torch.equal(m2.ids, want_id)


def _two_rank_prefill_worker(rank, world, port, q):
    """Two decoder layers prefilled over a 200-token prompt per rank with the
    experts split over two GPUs, against the same model with all experts local."""
    import torch.distributed as dist

    import __graft_entry__

    comm = None
    try:
        fm = __graft_entry__.load_package()
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        comm = fm.EPComm()
        want_lg, want_id, m2 = _prefill_pair(fm, dev, comm, rank, world)
        top = torch.topk(want_lg[0], 2).values
        sure = bool(top[0] - top[1] > 1e-3 * top[0].abs())
        res = (bool(torch.equal(m2.ids, want_id)) or not sure,
               max_rel_err(m2.logits.cpu().numpy(), want_lg.cpu().numpy()))
        comm.status()
        torch.cuda.synchronize()
        comm.close()
        dist.destroy_process_group()
        q.put((rank, res, None))
    except Exception as e:
        import traceback

        q.put((rank, None, repr(e) + "\n" + traceback.format_exc()))
        if comm is not None:
            comm.abort()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _two_rank_worker(rank, world, port, q):
    import torch.distributed as dist

    import __graft_entry__

    comm = None
    try:
        fm = __graft_entry__.load_package()
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        comm = fm.EPComm()
        table = fm.ExpertTable.random(E, H, I, seed=2002, device=dev)  # the same on every rank
        g = torch.Generator(device=dev).manual_seed(2002)
        wr = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        bias = torch.randn(E, generator=g, device=dev)
        router = fm.QuantizedLinear(wr, bits=16)
        ref = fm.Gemma4MoeBlock(router, table, top_k=K, logit_bias=bias)
        errs = []
        for T, cap, mode in [(4, 4, 0), (3, 4, 1), (200, 256, 0), (150, 256, 1), (4, 4, 2), (200, 256, 2),
                             (1, 4, 2)]:
            Tr = T if rank == 0 else max(T - 1, 0)  # ragged token counts
            gx = torch.Generator(device=dev).manual_seed(900 + 10 * T + rank)
            x = torch.randn(Tr, H, generator=gx, device=dev).to(torch.bfloat16)
            ep = fm.ExpertParallelMoeBlock(comm, router, table.shard(rank, world), cap=cap, top_k=K, mode=mode,
                                           logit_bias=bias)
            y, ids, w = ep.forward(x, return_routing=True)
            if Tr == 0:  # this rank only serves the other's tokens: nothing of its own to compare
                assert y.shape == (0, H)
                continue
            want, r_ids, _ = ref.forward(x, return_routing=True) if Tr <= 128 else ref.forward_prefill(
                x, return_routing=True)
            torch.cuda.synchronize()
            same = bool(torch.equal(ids, r_ids))
            errs.append((T, mode, same, max_rel_err(y.float().cpu().numpy(), want.float().cpu().numpy())))
        comm.status()
        torch.cuda.synchronize()
        comm.close()
        dist.destroy_process_group()
        q.put((rank, errs, None))
    except Exception as e:
        import traceback

        q.put((rank, None, repr(e) + "\n" + traceback.format_exc()))
        if comm is not None:  # frees this rank's NCCL state; the peer is then reported as silent
            comm.abort()


def _two_rank_decoder_worker(rank, world, port, q, mode=0):
    """Two decoder layers (sliding + full attention) with the experts split over
    two GPUs, one sequence per GPU; checked against the same model with all
    experts local on this GPU."""
    import torch.distributed as dist

    import __graft_entry__

    comm = None
    try:
        fm = __graft_entry__.load_package()
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        comm = fm.EPComm()
        cfg = dict(fm.GEMMA4_26B, vocab=4096, full_every=2)
        ctx = 300
        m1 = fm.Gemma4Model.random(cfg, batch=1, max_positions=1024, seed=21, device=dev, n_layers=2)
        layers = []
        for L in m1.layers:  # the same weights, expert slice only
            L2 = fm.Gemma4DecoderLayer(L.q_proj, L.k_proj, L.v_proj, L.o_proj, L.q_norm, L.k_norm, L.norms, L.mlp,
                                       L.router, L.experts.shard(rank, world), L.num_heads, L.num_kv_heads,
                                       L.head_dim, L.rope_dims, L.rope_theta, L.k_eq_v, L.eps, L.layer_scalar,
                                       L.attn_scale, L.top_k)
            layers.append(L2)
        m2 = fm.Gemma4Model(cfg, m1.embed, layers, m1.final_norm, 1, 1024, device=dev, ep=comm, ep_mode=mode)
        g = torch.Generator(device=dev).manual_seed(22 + rank)
        for L, c1, c2 in zip(m1.layers, m1.caches, m2.caches):
            kv = torch.randn(2, 1, L.num_kv_heads, ctx, L.head_dim, generator=g, device=dev).to(torch.bfloat16)
            c1.update(kv[0], kv[1])
            c2.update(kv[0], kv[1])
        for m in (m1, m2):
            m.ids.fill_(5 + rank)
            m.set_position(ctx)
        res = []
        for _ in range(3):
            a = m1.decode_step().clone()
            la = m1.logits.clone()
            b = m2.decode_step().clone()
            torch.cuda.synchronize()
            top = torch.topk(la[0], 2).values
            sure = bool(top[0] - top[1] > 1e-3 * top[0].abs())  # ids compared where the argmax is clear
            res.append((bool(torch.equal(a, b)) or not sure,
                        max_rel_err(m2.logits.cpu().numpy(), la.cpu().numpy())))
            m2.ids.copy_(a)  # continue both from the same token
        assert m2.status() == 0, fm.last_error()  # no bounded exchange wait gave up
        comm.status()
        torch.cuda.synchronize()
        comm.close()
        dist.destroy_process_group()
        q.put((rank, res, None))
    except Exception as e:
        import traceback

        q.put((rank, None, repr(e) + "\n" + traceback.format_exc()))
        if comm is not None:  # frees this rank's NCCL state; the peer is then reported as silent
            comm.abort()


def _spawn_two(target, *extra):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    env_nvls = os.environ.get("NCCL_NVLS_ENABLE")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    procs = [ctx.Process(target=target, args=(r, 2, port, q) + extra) for r in range(2)]
    res = {}
    deadline = time.monotonic() + 200  # well inside the per-test timeout, so a stuck rank is reported
    try:
        for p in procs:
            p.start()
        for _ in range(2):
            try:
                rank, out, exc = q.get(timeout=max(1.0, deadline - time.monotonic()))
            except queue.Empty:
                break
            res[rank] = (out, exc)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
                p.join(timeout=30)
        if env_nvls is None:
            os.environ.pop("NCCL_NVLS_ENABLE", None)
        else:
            os.environ["NCCL_NVLS_ENABLE"] = env_nvls
    for r in range(2):
        res.setdefault(r, (None, "no answer within 200 s (waiting in a collective for a rank that failed?)"))
    return res


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", [0, 2])
def test_ep_two_rank_decoder_matches_local(mode):
    out = _spawn_two(_two_rank_decoder_worker, mode)
    assert all(exc is None for _, exc in out.values()), "\n".join(f"rank {r}: {e}" for r, (_, e) in out.items())
    for rank, (res, exc) in out.items():
        for step, (same_ids, err) in enumerate(res):
            assert err <= TOL, (rank, step, err)
            assert same_ids, (rank, step)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_two_ranks_match_single_device():
    out = _spawn_two(_two_rank_worker)
    assert all(exc is None for _, exc in out.values()), "\n".join(f"rank {r}: {e}" for r, (_, e) in out.items())
    for rank, (errs, exc) in out.items():
        for T, mode, same, err in errs:
            assert same, (rank, T, mode)
            assert err <= TOL, (rank, T, mode, err)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_two_rank_prefill_matches_local():
    out = _spawn_two(_two_rank_prefill_worker)
    assert all(exc is None for _, exc in out.values()), "\n".join(f"rank {r}: {e}" for r, (_, e) in out.items())
    for rank, ((same_ids, err), exc) in out.items():
        assert err <= TOL, (rank, err)
        assert same_ids, rank
