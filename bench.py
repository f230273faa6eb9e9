#!/usr/bin/env python
"""Benchmark of the B200 quantised-MoE hot path (one JSON line on rank 0).

Workloads (synthetic data, random-init weights of the Gemma-4 26B-A4B shapes):
  decode30_b1       (default) one greedy decode step of the whole 30-layer
                    decoder for one sequence after a 2048-position context:
                    6-bit embedding row, per layer 8-bit q/k/v/o projections
                    with q/k/v norms, RoPE and a KV-cache append (default:
                    TurboQuant 3-bit round trip, the reference's), decode
                    attention (sliding window 1024 / full), the 4-bit dense
                    MLP, the bf16 router and 8 of 128 4-bit experts, then the
                    final norm, the tied 6-bit lm_head with softcap and argmax.
                    The context comes from a random 2048-token prompt run
                    through the whole decoder (Gemma4Model.prefill), whose
                    time is reported as the decoder_prefill key.
  moe30_decode_b1   the routed-expert path of the same decoder alone: per
                    layer the bf16 router [128, 2816] (softmax, top-8,
                    renormalise) and 8 of 128 MLX-affine 4-bit experts
                    (gate/up 2816->704, GELU-tanh gating, down 704->2816,
                    weighted combine), 30 layers.
  moe30_decode_b32  the same with 32 tokens per step.
Weights resident in HBM (about 15 GB) are far above L2, so no flush is needed.
A step is captured once in a CUDA graph and replayed.  `value` is tokens/s
with inputs resident in HBM; `e2e` adds the pinned-host -> device copy of the
step's input and the device -> host copy of its result inside the timed region.

--impl reference times the CPU port of the reference's path (oracle/, C++
OpenMP on all host cores) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, I, E, K, LAYERS = 2816, 704, 128, 8, 30
ROUTER_BYTES = E * H * 2                                   # bf16 router weight per layer
GATE_UP_BYTES = 2 * (I * H // 2 + 2 * I * (H // 64) * 2)   # per selected expert: 2,230,272
DOWN_BYTES = H * I // 2 + 2 * H * (I // 64) * 2            # per selected expert: 1,115,136
WORKLOADS = {"decode30_b1": 1, "decode30_b32": 32, "moe30_decode_b1": 1, "moe30_decode_b32": 32}
# total tokens per step (split evenly over the GPUs), default exchange mode
EP_WORKLOADS = {"ep_moe30_decode_b256": (256, "p2p"), "ep_moe30_prefill_8192": (8192, "exact")}
# config 5 measured inside a multi-GPU decode30 run (workload, exchange mode)
EP_EXTRA = [("ep_moe30_decode_b256", "fixed"), ("ep_moe30_decode_b256", "p2p"), ("ep_moe30_prefill_8192", "exact")]
CTX = 2048                                                 # decode context (positions in every KV cache)
# decode30's KV cache: "turbo3" (bf16 rows through the TurboQuant 3-bit round trip on
# append, the reference's default cache), "bf16" or "affine" (WHT + K4 / V8); --kv-cache
KV_KINDS = ("turbo3", "bf16", "affine")
DECODE_KV = "turbo3"
KV_DESC = {"turbo3": "bf16 rows through the TurboQuant 3-bit round trip on append (the reference's default cache)",
           "bf16": "bf16 rows", "affine": "WHT-rotated MLX-affine K 4-bit / V 8-bit"}
EXPERT_BYTES = GATE_UP_BYTES + DOWN_BYTES                  # 3,345,408


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode30_b1", choices=sorted(WORKLOADS) + sorted(EP_WORKLOADS))
    ap.add_argument("--ep-mode", default=None, choices=["fixed", "exact", "p2p"],
                    help="expert-parallel exchange (default: p2p for decode, exact for prefill; p2p = fixed's "
                         "layout stored into the peers' memory by the library's kernels; decode30 at N > 1 takes "
                         "fixed or p2p)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kv-cache", default="turbo3", choices=list(KV_KINDS),
                    help="decode30's KV cache (default turbo3, the reference's default); the other two are "
                         "measured as the kv_cache_variants key at N = 1")
    ap.add_argument("--sample", action="store_true",
                    help="decode30: draw each token on the device with the reference generate command's defaults "
                         "(temperature 0.7, top_p 0.9, repetition penalty 1.15 over the last 64 tokens) instead of "
                         "the greedy argmax")
    ap.add_argument("--profile-step", action="store_true",
                    help="after warm-up, run one eager step between cudaProfilerStart / Stop and exit (for "
                         "ncu --profile-from-start off launch lists of the decode30 / ep_* workloads)")
    ap.add_argument("--profile-prefill", action="store_true",
                    help="decode30: after one warm-up prefill of the 2048-token context, run one more prefill "
                         "between cudaProfilerStart / Stop and exit (ncu launch lists of the prefill)")
    ap.add_argument("--no-ep-extra", action="store_true",
                    help="decode30 at N > 1: skip the expert-parallel config-5 sub-measurements")
    ap.add_argument("--no-attn", action="store_true", help="skip the quantised-KV decode-attention sub-measurement")
    ap.add_argument("--qlinear-case", default=None, metavar="OUT:IN:BITS:T",
                    help="run only fmoe_qlinear on one shape: four launches, L2 flushed before each, the last one "
                         "timed (a small case for profilers)")
    ap.add_argument("--attn-case", default=None, metavar="MODE:B:T",
                    help="run only one decode-attention case (mode affine|bf16, batch, context): four launches, "
                         "L2 flushed before each, the last one timed (a small case for profilers)")
    ap.add_argument("--prefill-case", type=int, default=None, metavar="T",
                    help="run only the prefill MoE block (BASELINE config 2: T tokens, Zipf-skewed routing) on the "
                         "tcgen05 path: four calls, L2 flushed before each, the last one timed (a small case for "
                         "profilers)")
    ap.add_argument("--pf-attn-case", default=None, metavar="D:HKV:HQ:WINDOW:T",
                    help="run only the prefill attention (fmoe_attn_prefill) of a T-token prompt from position 0 "
                         "(WINDOW 0: full causal): four launches, the last one timed (a small case for profilers)")
    ap.add_argument("--layers", type=int, default=30,
                    help="decoder layers in the step (30 = the model; fewer only for small profiling cases)")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def load_peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        self.first = ""
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            # the timed region starts once sampling runs (the first line is printed)
            import select
            if select.select([self.proc.stdout], [], [], 5.0)[0]:
                self.first = self.proc.stdout.readline()
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
        if not self.out.strip():
            self.out = self.first  # a region shorter than one period: the sample taken as it began

    def summary(self):
        sms, maxs, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (getattr(self, "out", "") or "").splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sms.append(float(f[1]))
                maxs.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxs), "reasons": sorted(reasons),
                "samples": len(sms)}


# ---------------------------------------------------------------------------
# our arm


def build_layers(fm, torch, dev, seed, n_layers):
    layers = []
    g = torch.Generator(device=dev)
    for l in range(n_layers):
        g.manual_seed(seed + l)
        wr = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        table = fm.ExpertTable.random(E, H, I, seed=seed + 1000 + l, device=dev)
        layers.append(fm.Gemma4MoeBlock(fm.QuantizedLinear(wr, bits=16), table, top_k=K))
    return layers


class MoeStack:
    """Prepared C-ABI calls for the 30 layers (structs and workspaces built once)."""

    def __init__(self, fm, torch, layers, T, dev):
        import ctypes
        self.fm, self.torch, self.ctypes = fm, torch, ctypes
        self.T = T
        self.x = torch.zeros(T, H, dtype=torch.bfloat16, device=dev)
        self.ys = [torch.empty(T, H, dtype=torch.bfloat16, device=dev) for _ in layers]
        self.ids = [torch.empty(T, K, dtype=torch.int32, device=dev) for _ in layers]
        self.wts = [torch.empty(T, K, dtype=torch.float32, device=dev) for _ in layers]
        self.rc = [l.router_cstruct() for l in layers]
        self.ec = [l.experts.cstruct() for l in layers]
        nbytes = max(fm.lib().fmoe_moe_block_workspace_bytes(T, ctypes.byref(r), ctypes.byref(e))
                     for r, e in zip(self.rc, self.ec))
        self.ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)  # router counters start at zero
        self.layers = layers

    def run(self, stream):
        lib, ct = self.fm.lib(), self.ctypes
        s = stream.cuda_stream
        for i in range(len(self.layers)):
            rc = lib.fmoe_moe_block_forward(self.x.data_ptr(), self.T, ct.byref(self.rc[i]), ct.byref(self.ec[i]),
                                            self.ys[i].data_ptr(), self.ids[i].data_ptr(), self.wts[i].data_ptr(),
                                            self.ws.data_ptr(), self.ws.numel(), s)
            if rc:
                self.fm.check(rc)


def ncu_traffic(workload, kernel):
    """DRAM bytes per launch of `kernel` from the committed ncu captures (profiles/), or None."""
    try:
        return json.load(open(os.path.join(ROOT, "profiles", "ncu_traffic.json"))).get(workload, {}).get(kernel)
    except Exception:
        return None


def profiled_step(torch, fn):
    """One eager step between cudaProfilerStart / Stop (ncu --profile-from-start off)."""
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStart()
    fn()
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    print(json.dumps({"profile_step": "done"}), flush=True)


def qlin_bytes(q):
    return q.weight.numel() * q.weight.element_size() + (q.scales.numel() + q.biases.numel()) * 2


def decoder_step_bytes(m, T, ctx):
    """Algorithmic bytes of one decode step: every weight byte the step needs
    once (the experts the step routes to: 8 distinct per token at T = 1), the
    KV positions attended plus the appended one, and the embedding row."""
    per = {"attention": 0, "dense": 0, "router": 0, "experts": 0, "kv": 0, "lm_head": 0}
    for L, c in zip(m.layers, m.caches):
        per["attention"] += sum(qlin_bytes(q) for q in (L.q_proj, L.k_proj, L.o_proj))
        if not L.k_eq_v:
            per["attention"] += qlin_bytes(L.v_proj)
        per["dense"] += sum(qlin_bytes(q) for q in L.mlp)
        w = L.router["proj"].weight
        per["router"] += w.numel() * w.element_size()
        # distinct experts a step reads: 8 at T = 1; for T > 1 the expectation
        # under uniform routing, E (1 - (1 - K/E)^T) (112.6 of 128 at T = 32)
        per["experts"] += (K if T == 1 else E * (1.0 - (1.0 - K / E) ** T)) * EXPERT_BYTES
        n = min(ctx + 1, c.capacity)
        per["kv"] += T * L.num_kv_heads * L.head_dim * 2 * 2 * (n + 1)
    per["lm_head"] = qlin_bytes(m.embed) + T * qlin_bytes(m.embed) // m.embed.out_features
    return sum(per.values()), per


DECODER_METRIC = "decode tok/s, batch 1 (30-layer Gemma-4 26B-A4B-shaped decoder, full step incl. lm_head)"


def decoder_metric(args):
    T = WORKLOADS[args.workload]
    return DECODER_METRIC if T == 1 else DECODER_METRIC.replace("batch 1", f"batch {T}")
MOE_METRIC = "decode tok/s (routed-expert path of the 30-layer Gemma-4 26B-A4B-shaped decoder)"


def decoder_config(args, world):
    """The decode30 workload's `config` (both arms print this dict)."""
    T = WORKLOADS[args.workload]
    par = "single GPU" if world == 1 else (
        f"expert-parallel x{world}: {E // world} experts per GPU, routed tokens dispatched / combined "
        + ("by NCCL send/recv" if args.ep_mode == "fixed"
           else "by stores into the peers' exchange windows (CUDA IPC, flag-synchronised)")
        + " over NVLink (fixed capacity, in the CUDA graph); attention, dense MLP, router, embedding "
        f"replicated; one sequence per GPU")
    return {"workload": args.workload, "layers": args.layers, "hidden": H, "experts": E, "top_k": K,
            "batch": T, "context": CTX, "kv_cache": f"{args.kv_cache}: {KV_DESC[args.kv_cache]}",
            "attention_bits": 8, "expert_bits": 4,
            "dense_bits": 4, "embed_bits": 6, "router": "bf16",
            "parallelism": par,
            "l2": "weights (about 15 GB) far larger than L2; no flush",
            "graph": "one CUDA graph per step, position on the device",
            "next_token": ("sampled (fmoe_sample on the device; the oracle's sampler on the CPU): temperature "
                           "0.7, top_p 0.9, repetition penalty 1.15 over the last 64 tokens" if args.sample
                           else "greedy argmax (fused in the lm_head)")}


def moe_config(args, world):
    """The moe30_decode_* workloads' `config`."""
    return {"workload": args.workload, "layers": args.layers, "hidden": H, "experts": E, "top_k": K,
            "expert_intermediate": I, "tokens_per_step": WORKLOADS[args.workload], "router": "bf16",
            "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
            "l2": "inputs larger than L2 (30 x 428 MB of experts resident)",
            "graph": "one CUDA graph per step"}


def ep_mode_name(args):
    return args.ep_mode or EP_WORKLOADS[args.workload][1]


def ep_metric(args):
    total = EP_WORKLOADS[args.workload][0]
    return (("prefill tok/s" if "prefill" in args.workload else "decode tok/s") +
            f" (MoE half of the 30-layer Gemma-4 26B-A4B-shaped model, {total} tokens per step, experts "
            f"split over the GPUs)")


def ep_config(args, world):
    """The ep_moe30_* workloads' `config` (config 5: experts split over the GPUs)."""
    total = EP_WORKLOADS[args.workload][0]
    mode_name = ep_mode_name(args)
    T = total // world
    row_b = H * 2 + K * 8
    return {"workload": args.workload, "layers": args.layers, "hidden": H, "experts": E, "top_k": K,
            "expert_intermediate": I, "tokens_per_step": total, "tokens_per_gpu": T,
            "parallelism": f"expert-parallel x{world}: {E // world} experts per GPU, "
                           + ("peer-memory stores (CUDA IPC windows)" if mode_name == "p2p"
                              else "NCCL grouped send/recv")
                           + f" dispatch + combine ({mode_name} exchange); router replicated, tokens split",
            "exchange_bytes_per_layer_per_gpu": (world * T * row_b * 2) if mode_name in ("fixed", "p2p") else None,
            "graph": "one CUDA graph per step" if mode_name in ("fixed", "p2p")
                     else "eager (exact mode syncs per layer)",
            "l2": "inputs larger than L2 (expert slices resident)"}


def run_decoder(args, rank, world, local):
    import torch
    import __graft_entry__

    fm = __graft_entry__.load_package()
    fm.lib()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    ep = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        ep = fm.EPComm()  # experts split E / world per GPU, exchanged over NVLink
    T = WORKLOADS[args.workload]
    cfg = dict(fm.GEMMA4_26B)
    # the same weights on every rank (each keeps its expert slice); per-rank sequences
    # default exchange at N > 1: peer-memory stores (measured faster than NCCL
    # send / recv at N = 2 and 4); --ep-mode fixed selects NCCL
    ep_mode = fm.FMOE_EP_FIXED if args.ep_mode == "fixed" else fm.FMOE_EP_P2P
    if args.ep_mode == "exact":
        raise SystemExit("decode30: the exact exchange syncs the host per layer and cannot be captured")
    # one layout per weight: the decoder's GEMVs read the plain MLX-affine rows
    m = fm.Gemma4Model.random(cfg, batch=T, max_positions=CTX + 64, seed=4000, device=dev, n_layers=args.layers,
                              ep=ep, ep_mode=ep_mode, **kv_kwargs(fm, args.kv_cache))
    if args.sample:
        m.set_sampler(0.7, 0.9, 1.15, seed=4200 + rank)
    g = torch.Generator(device=dev).manual_seed(4100 + rank)
    peaks, peaks_kind = load_peaks()
    pf_result = None
    prompt = torch.randint(0, cfg["vocab"], (T, CTX), generator=g, device=dev, dtype=torch.int32)
    if ep is None:
        # BASELINE config 4's context: a CTX-token prompt per sequence prefilled
        # through the whole decoder, which fills every KV cache
        quiet = args.profile_step or args.profile_prefill
        pf_result = decoder_prefill(torch, m, prompt, peaks, timed_reps=0 if quiet else 3)
        if args.profile_prefill:
            m.set_position(0)
            profiled_step(torch, lambda: m.prefill(prompt))
            return
    else:
        # expert-parallel models have no whole-decoder prefill
        random_context(torch, m, T, g, dev)
    ids0 = torch.randint(0, cfg["vocab"], (T,), generator=g, device=dev, dtype=torch.int32)
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream())

    if args.profile_step:
        with torch.cuda.stream(stream):
            m.ids.copy_(ids0)
            m.set_position(CTX)
            for _ in range(3):
                m.decode_step()
            torch.cuda.synchronize()
            profiled_step(torch, m.decode_step)
        if ep is not None:
            ep.close()
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    # per-kernel device times of eager steps (profiling on)
    with torch.cuda.stream(stream):
        m.ids.copy_(ids0)
        m.set_position(CTX)
        m.decode_step()
        torch.cuda.synchronize()
        fm.profile_read(reset=True)
        fm.profile_enable(True)
        nprof = 3
        for _ in range(nprof):
            m.decode_step()
        torch.cuda.synchronize()
        fm.profile_enable(False)
    prof = fm.profile_read(reset=True)
    launches_per_step = sum(v[0] for v in prof.values()) // nprof

    # one step in a CUDA graph; the position lives on the device and advances per replay
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        m.ids.copy_(ids0)
        m.set_position(CTX)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream, capture_error_mode="thread_local"):
            m.decode_step(device_pos=True)

    def timed(n, e2e, host_in=None, host_out=None):
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            m.ids.copy_(ids0)
            m.set_position(CTX)
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            start.record(stream)
            for i in range(n):
                if e2e:
                    m.ids.copy_(host_in[i % host_in.shape[0]], non_blocking=True)
                graph.replay()
                if e2e:
                    host_out[i % host_out.shape[0]].copy_(m.ids, non_blocking=True)
            stop.record(stream)
        torch.cuda.synchronize()
        ms = start.elapsed_time(stop)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    timed(args.warmup, False)
    clocks = ClockSampler(local)
    with clocks:
        ms = timed(args.steps, False)
    host_in = torch.randint(0, cfg["vocab"], (64, T), dtype=torch.int32).pin_memory()
    host_out = torch.empty(64, T, dtype=torch.int32).pin_memory()
    timed(min(args.warmup, 3), True, host_in, host_out)
    ms_e2e = timed(args.steps, True, host_in, host_out)
    if m.status() != 0:  # a bounded device wait (exchange flag, copy) gave up: the step did not run as timed
        raise SystemExit(f"rank {rank}: device status: {fm.last_error()}")
    assert int(m.pos_dev[0]) == CTX + args.steps

    ms_step = ms / args.steps
    value = world * T / (ms_step / 1e3)
    e2e_value = world * T / (ms_e2e / args.steps / 1e3)
    step_bytes, parts = decoder_step_bytes(m, T, CTX)
    step_gbs = step_bytes / (ms_step / 1e3) / 1e9

    # roofline of the dominant kernel (most device time per step)
    name, (n_l, tot_ms) = max(prof.items(), key=lambda kv: kv[1][1])
    by_kernel = {"rgemv_kernel<8>": parts["attention"], "rgemv_kernel<4>": parts["dense"],
                 "qgemv_kernel<8>": parts["attention"], "qgemv_kernel<4>": parts["dense"],
                 "dl_lm_kernel": parts["lm_head"], "qgemv_kernel<6>": parts["lm_head"], "attn_bf16_kernel": parts["kv"],
                 "moe_gate_up_kernel": parts["experts"] * 2 / 3, "moe_down_kernel": parts["experts"] / 3}
    alg = by_kernel[name] / (n_l / nprof) if name in by_kernel else None
    achieved = alg / (tot_ms / n_l / 1e3) / 1e9 if alg else None
    result = {
        "metric": decoder_metric(args),
        "value": round(value, 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "u8/u4/u6-affine weights x bf16 activations, fp32 accumulate",
        "data": "synthetic (random-init weights MLX-affine quantised; random token ids; the 2048-position "
                "context prefilled from a random prompt%s)" % ("" if ep is None else
                                                              " — here random bf16 K/V rows (expert-parallel)"),
        "config": decoder_config(args, world),
        "e2e": {"value": round(e2e_value, 2), "unit": "tok/s", "h2d_bytes_per_step": T * 4,
                "d2h_bytes_per_step": T * 4,
                "api": "Gemma4Model.decode_step (embedding, fmoe_decoder_layer_forward%s x30, fmoe_lm_head) "
                       "captured in a CUDA graph + pinned host copies of the token ids" % ("_ep" if ep else "")},
        "gpu_launches": launches_per_step * args.steps,
        "step_alg_bytes": int(step_bytes),
        "step_alg_bytes_parts": {k: int(v) for k, v in parts.items()},
        "step_hbm_gbs": round(step_gbs, 1),
        "step_roofline_frac": round(step_gbs / peaks["hbm_gbs"], 4),
        "roofline": {"bound": "hbm", "kernel": name,
                     "achieved": round(achieved, 1) if achieved else None,
                     "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4) if achieved else None,
                     "peak_source": f"{peaks_kind} (MEASURED_PEAKS.json hbm_gbs)" if peaks_kind == "measured"
                     else "fallback 6.65 TB/s",
                     "alg_bytes_per_launch": int(alg) if alg else None,
                     "avg_launch_us": round(tot_ms / n_l * 1e3, 3), "traffic": ncu_traffic(args.workload, name)},
        "kernels": {k: {"launches_per_step": v[0] // nprof, "avg_us": round(v[1] / v[0] * 1e3, 3),
                        "us_per_step": round(v[1] / nprof * 1e3, 1)}
                    for k, v in sorted(prof.items(), key=lambda kv: -kv[1][1])},
        "clocks": clocks.summary(),
    }
    del graph  # graphs holding NCCL work go before the communicators
    torch.cuda.synchronize()
    if ep is not None:
        ep.close()
    if pf_result is not None and rank == 0:
        result["decoder_prefill"] = pf_result
    if rank == 0 and world == 1 and not args.profile_step:
        # the other KV caches on the same weights: decode tok/s of each
        result["kv_cache_variants"] = {k: kv_variant(fm, torch, m, cfg, T, k, prompt, ids0, stream, dev, g)
                                       for k in KV_KINDS if k != args.kv_cache}
    if rank == 0 and world == 1 and not args.profile_step and T == 1:
        # BASELINE config 4's batch 32 on the same weights and cache kind (its own
        # prompts, prefilled), as an extra key of the headline line
        B = WORKLOADS["decode30_b32"]
        p32 = torch.randint(0, cfg["vocab"], (B, CTX), generator=g, device=dev, dtype=torch.int32)
        i32 = torch.randint(0, cfg["vocab"], (B,), generator=g, device=dev, dtype=torch.int32)
        r32 = kv_variant(fm, torch, m, cfg, B, args.kv_cache, p32, i32, stream, dev, g, steps=20, warmup=3)
        r32["workload"] = "decode30_b32"
        r32["context"] = f"{B} random {CTX}-token prompts, prefilled"
        r32["api"] = ("Gemma4Model.decode_step at batch 32: one fmoe_decoder_layer_forward per layer (attention "
                      "half per group of 8, router / experts / dense MLP over all 32), fmoe_lm_head per group of 8")
        result["decode30_b32"] = r32
    if rank == 0 and world == 1 and not args.no_attn:
        # BASELINE configs 3 and 2 on the same box, as extra keys of the headline line
        result["kv_attention"] = attn_submeasure(fm, torch, dev, peaks["hbm_gbs"])
        result["moe_prefill"] = prefill_submeasure(fm, torch, dev, peaks)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_decoder_baseline(T, sampled=args.sample)
    if world > 1 and not args.no_ep_extra:
        # BASELINE config 5 (experts split over the GPUs) on the same ranks, as extra keys
        torch.cuda.empty_cache()
        result["ep_config5"] = {}
        for wl, mode in EP_EXTRA:
            sub = argparse.Namespace(**{**vars(args), "workload": wl, "ep_mode": mode, "steps": 10, "warmup": 3,
                                        "no_cpu_baseline": True, "profile_step": False})
            r = ep_measure(sub, rank, world, local, own_pg=False)
            if rank == 0:
                result["ep_config5"][f"{wl}:{mode}"] = {k: r[k] for k in ("metric", "value", "unit", "ms_per_step",
                                                                           "steps", "warmup", "scaling", "e2e",
                                                                           "roofline", "config")}
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def run_ours(args, rank, world, local):
    import torch
    import __graft_entry__

    fm = __graft_entry__.load_package()
    fm.lib()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    T = WORKLOADS[args.workload]
    layers = build_layers(fm, torch, dev, seed=4000, n_layers=args.layers)
    stack = MoeStack(fm, torch, layers, T, dev)
    g = torch.Generator(device=dev).manual_seed(5000 + rank)
    nin = max(args.steps + args.warmup, 16)
    xs = torch.randn(nin, T, H, generator=g, device=dev).to(torch.bfloat16)
    stream = torch.cuda.Stream(device=dev)

    # per-kernel device times (eager, profiling on) for the roofline
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for i in range(3):
            stack.x.copy_(xs[i])
            stack.run(stream)
        torch.cuda.synchronize()
        fm.profile_read(reset=True)
        fm.profile_enable(True)
        nprof = 5
        uniq = []
        for i in range(nprof):
            stack.x.copy_(xs[i])
            stack.run(stream)
            torch.cuda.synchronize()
            uniq.append([int(torch.unique(ids).numel()) for ids in stack.ids])
        fm.profile_enable(False)
    prof = fm.profile_read(reset=True)

    # capture one step
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        stack.x.copy_(xs[0])
        stack.run(stream)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            stack.run(stream)
    launches_per_step = sum(v[0] for v in prof.values()) // nprof

    def timed(n, e2e, host_in=None, host_out=None):
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            start.record(stream)
            for i in range(n):
                if e2e:
                    stack.x.copy_(host_in[i % host_in.shape[0]], non_blocking=True)
                else:
                    stack.x.copy_(xs[args.warmup + (i % args.steps)])
                graph.replay()
                if e2e:
                    host_out.copy_(stack.ys[-1], non_blocking=True)
            stop.record(stream)
        torch.cuda.synchronize()
        ms = start.elapsed_time(stop)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            stack.x.copy_(xs[i])
            graph.replay()
    clocks = ClockSampler(local)
    with clocks:
        ms = timed(args.steps, False)
    host_in = xs[: min(nin, 64)].cpu().pin_memory()
    host_out = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
    timed(min(args.warmup, 3), True, host_in, host_out)
    ms_e2e = timed(args.steps, True, host_in, host_out)

    ms_step = ms / args.steps
    value = world * T / (ms_step / 1e3)
    e2e_value = world * T / (ms_e2e / args.steps / 1e3)

    # roofline of the dominant kernel
    peaks, peaks_kind = load_peaks()
    name, (n_l, tot_ms) = max(prof.items(), key=lambda kv: kv[1][1])
    nl = args.layers
    avg_u = sum(sum(u) for u in uniq) / nprof  # unique experts per step summed over layers
    if name == "moe_gate_up_kernel":
        alg = avg_u * GATE_UP_BYTES / nl + T * H * 2 + avg_u / nl * T * I * 2
    elif name == "moe_down_kernel":
        alg = avg_u * DOWN_BYTES / nl + T * H * 2
    else:
        alg = ROUTER_BYTES
    achieved = alg / (tot_ms / n_l / 1e3) / 1e9
    traffic = None
    try:
        tr = json.load(open(os.path.join(ROOT, "profiles", "ncu_traffic.json")))
        traffic = tr.get(args.workload, {}).get(name)
    except Exception:
        pass
    step_bytes = avg_u * (GATE_UP_BYTES + DOWN_BYTES) + nl * ROUTER_BYTES
    result = {
        "metric": MOE_METRIC,
        "value": round(value, 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "u4-affine weights x bf16 activations, fp32 accumulate",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights MLX-affine 4-bit quantised; random init)",
        "config": moe_config(args, world),
        "e2e": {"value": round(e2e_value, 2), "unit": "tok/s", "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2,
                "api": "fmoe_moe_block_forward x30 (captured in a CUDA graph) + pinned host copies"},
        "gpu_launches": launches_per_step * args.steps,
        "step_weight_bytes": int(step_bytes),
        "step_hbm_gbs": round(step_bytes / (ms_step / 1e3) / 1e9, 1),
        "roofline": {"bound": "hbm", "kernel": name, "achieved": round(achieved, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "peak_source": f"{peaks_kind} (MEASURED_PEAKS.json hbm_gbs)" if peaks_kind == "measured"
                     else "fallback 6.65 TB/s",
                     "alg_bytes_per_launch": int(alg), "avg_launch_us": round(tot_ms / n_l * 1e3, 3),
                     "traffic": traffic},
        "kernels": {k: {"launches_per_step": v[0] // nprof, "avg_us": round(v[1] / v[0] * 1e3, 3)}
                    for k, v in sorted(prof.items(), key=lambda kv: -kv[1][1])},
        "clocks": clocks.summary(),
    }
    if rank == 0 and world == 1 and not args.no_attn:
        del graph, stack, layers
        torch.cuda.empty_cache()
        result["kv_attention"] = attn_submeasure(fm, torch, dev, peaks["hbm_gbs"])
        graph = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(None, T)
    if rank == 0:
        print(json.dumps(result), flush=True)
    del graph
    if world > 1:
        torch.distributed.destroy_process_group()


# ---------------------------------------------------------------------------
# expert parallelism: the MoE half of the 30-layer model
# with its 128 experts split over the GPUs, total tokens fixed (strong scaling)


def run_ep_moe(args, rank, world, local):
    result = ep_measure(args, rank, world, local, own_pg=True)
    if rank == 0 and result is not None:
        print(json.dumps(result), flush=True)


def ep_measure(args, rank, world, local, own_pg):
    """One expert-parallel workload on every rank; rank 0 gets the result dict.
    own_pg: create / destroy the process group here (False: the caller's)."""
    import datetime

    import torch
    import torch.distributed as dist
    import __graft_entry__

    fm = __graft_entry__.load_package()
    fm.lib()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    total, mode_name = EP_WORKLOADS[args.workload]
    mode_name = args.ep_mode or mode_name
    mode = {"fixed": fm.FMOE_EP_FIXED, "exact": fm.FMOE_EP_EXACT, "p2p": fm.FMOE_EP_P2P}[mode_name]
    if total % world or E % world:
        raise SystemExit(f"{total} tokens / {E} experts do not split over {world} GPUs")
    T = total // world
    if world > 1 and own_pg:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    comm = fm.EPComm()
    nl = args.layers
    g = torch.Generator(device=dev)
    shared = fm._Workspace()  # one exchange workspace for every layer (calls are sequential)
    blocks = []
    for l in range(nl):
        g.manual_seed(6000 + l)
        wr = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        bias = torch.randn(E, generator=g, device=dev)  # config 2's Zipf-like per-expert skew
        table = fm.ExpertTable.random(E, H, I, seed=7000 + l, device=dev).shard(rank, world, copy=True)
        b = fm.ExpertParallelMoeBlock(comm, fm.QuantizedLinear(wr, bits=16), table, cap=T, top_k=K, mode=mode,
                                      logit_bias=bias)
        b._ws = shared
        blocks.append(b)
        torch.cuda.empty_cache()
    gx = torch.Generator(device=dev).manual_seed(5000 + rank)
    x = torch.randn(T, H, generator=gx, device=dev).to(torch.bfloat16)
    ys = [torch.empty(T, H, dtype=torch.bfloat16, device=dev) for _ in range(nl)]
    ids = [None] * nl
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream())

    def step(keep_ids=False):
        for l, b in enumerate(blocks):
            if keep_ids:
                _, ids[l], _ = b.forward(x, return_routing=True, out=ys[l])
            else:
                b.forward(x, out=ys[l])

    if args.profile_step:
        with torch.cuda.stream(stream):
            for _ in range(2):
                step()
            torch.cuda.synchronize()
            profiled_step(torch, step)
        comm.close()
        if world > 1 and own_pg:
            dist.destroy_process_group()
        return None
    with torch.cuda.stream(stream):
        step(keep_ids=True)
        torch.cuda.synchronize()
        fm.profile_read(reset=True)
        fm.profile_enable(True)
        nprof = 2
        for _ in range(nprof):
            step()
        torch.cuda.synchronize()
        fm.profile_enable(False)
    prof = fm.profile_read(reset=True)
    launches_per_step = sum(v[0] for v in prof.values()) // nprof
    # pairs each rank computes: every rank's routing, counted on the expert owners
    all_ids = torch.stack(ids)  # [layers, T, K]
    if world > 1:
        gathered = [torch.empty_like(all_ids) for _ in range(world)]
        dist.all_gather(gathered, all_ids)
        all_ids = torch.cat(gathered, dim=1)
    per = E // world
    local = (all_ids >= rank * per) & (all_ids < (rank + 1) * per)
    pairs_local = int(local.sum()) / nl
    uniq_local = sum(int(torch.unique(all_ids[l][local[l]]).numel()) for l in range(nl)) / nl

    graph = None
    if mode in (fm.FMOE_EP_FIXED, fm.FMOE_EP_P2P):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            torch.cuda.synchronize()
            with torch.cuda.graph(graph, stream=stream, capture_error_mode="thread_local"):
                step()

    def timed(n, e2e, host_in=None, host_out=None):
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            start.record(stream)
            for i in range(n):
                if e2e:
                    x.copy_(host_in, non_blocking=True)
                if graph is not None:
                    graph.replay()
                else:
                    step()
                if e2e:
                    host_out.copy_(ys[-1], non_blocking=True)
            stop.record(stream)
        torch.cuda.synchronize()
        ms = start.elapsed_time(stop)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    timed(args.warmup, False)
    clocks = ClockSampler(local)
    with clocks:
        ms = timed(args.steps, False)
    host_in = x.cpu().pin_memory()
    host_out = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
    timed(min(args.warmup, 3), True, host_in, host_out)
    ms_e2e = timed(args.steps, True, host_in, host_out)
    if fm.lib().fmoe_workspace_status(shared.buf.data_ptr(), 0, fm._stream()) != 0:
        raise SystemExit(f"rank {rank}: device status: {fm.last_error()}")
    ms_step = ms / args.steps
    value = total / (ms_step / 1e3)
    e2e_value = total / (ms_e2e / args.steps / 1e3)

    peaks, peaks_kind = load_peaks()
    name, (n_l, tot_ms) = max(prof.items(), key=lambda kv: kv[1][1])
    avg_s = tot_ms / n_l / 1e3
    prefill = total > 1024
    if name.startswith("tc_gemm_kernel") and prefill:  # tensor-bound: fp32-accumulated bf16 MMA FLOPs
        fl = 2 * pairs_local * H * 2 * I if "gate_up" in name else 2 * pairs_local * I * H
        roof = {"bound": "tensor", "achieved": round(fl / avg_s / 1e12, 2), "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": round(fl / avg_s / 1e12 / peaks["bf16_tflops"], 4),
                "alg_flops_per_launch": int(fl)}
    else:  # HBM-bound: the local experts' weights once
        wb = GATE_UP_BYTES if "gate_up" in name else DOWN_BYTES
        alg = uniq_local * wb if ("gate_up" in name or "down" in name) else None
        roof = {"bound": "hbm", "achieved": round(alg / avg_s / 1e9, 1) if alg else None, "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": round(alg / avg_s / 1e9 / peaks["hbm_gbs"], 4) if alg else None,
                "alg_bytes_per_launch": int(alg) if alg else None}
    roof.update({"kernel": name, "avg_launch_us": round(avg_s * 1e6, 3), "traffic": None,
                 "peak_source": f"{peaks_kind} (MEASURED_PEAKS.json)" if peaks_kind == "measured" else "fallback"})
    result = {
        "metric": ep_metric(args),
        "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "u4-affine weights x bf16 activations, fp32 accumulate",
        "data": "synthetic (seeded N(0,1) activations; N(0,0.02) weights MLX-affine 4-bit; router logit bias N(0,1) "
                "per expert)",
        "config": ep_config(args, world),
        "e2e": {"value": round(e2e_value, 2), "unit": "tok/s", "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2,
                "api": "ExpertParallelMoeBlock.forward x30 (fmoe_ep_moe_forward) + pinned host copies"},
        "gpu_launches": launches_per_step * args.steps,
        "local_pairs_per_layer": round(pairs_local, 1), "local_unique_experts_per_layer": round(uniq_local, 2),
        "roofline": roof,
        "kernels": {k: {"launches_per_step": v[0] // nprof, "avg_us": round(v[1] / v[0] * 1e3, 3)}
                    for k, v in sorted(prof.items(), key=lambda kv: -kv[1][1])},
        "clocks": clocks.summary(),
    }
    del graph  # graphs holding NCCL work go before the communicator
    torch.cuda.synchronize()
    comm.close()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(None, EP_WORKLOADS[args.workload][0])
    del blocks, ys, shared
    torch.cuda.empty_cache()
    if world > 1 and own_pg:
        dist.destroy_process_group()
    return result if rank == 0 else None


# ---------------------------------------------------------------------------
# quantised-KV decode attention: 16 query heads, 8 KV heads,
# head_dim 256; K/V N(0,1) with 1% outlier channels x20; WHT-rotated affine
# 4-bit K / 8-bit V (the benchmark's cache) and the reference's bf16 cache.

ATTN_CASES = [  # (mode, batch, positions appended, sliding window or None)
    ("affine", 1, 32768, None), ("affine", 1, 32768, 1024), ("affine", 32, 8192, None),
    ("affine", 32, 32768, None), ("affine", 32, 32768, 1024), ("bf16", 32, 32768, None),
]


def attn_submeasure(fm, torch, dev, peak_gbs, iters=20, cases=ATTN_CASES):
    D, HKV, HQ = 256, 8, 16
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)  # > L2 (126 MB)
    out = []
    for mode, B, T, win in cases:
        cap = win or T
        if mode == "affine":
            cache = fm.KVCache.new_affine(B, HKV, D, cap, window=win, device=dev)
            per_pos = D // 2 + D + 4 * (D // 64) * 2
        else:
            cache = fm.KVCache(B, HKV, D, cap, window=win, device=dev)
            per_pos = 4 * D
        g = torch.Generator(device=dev).manual_seed(77)
        ch = torch.randperm(D, generator=torch.Generator().manual_seed(78))[:3].to(dev)
        step = max(1, (1 << 27) // (B * HKV * D * 2))
        done = 0
        while done < T:
            t = min(step, T - done)
            kv = torch.randn(2, B, HKV, t, D, generator=g, device=dev)
            kv[..., ch] *= 20.0
            kv = kv.to(torch.bfloat16)
            cache.update(kv[0], kv[1])
            done += t
        q = torch.randn(B, HQ, D, generator=g, device=dev).to(torch.bfloat16)
        times = []
        for i in range(iters + 3):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            st = torch.cuda.current_stream()
            a.record(st)
            cache.attend(q, 1.0)
            b.record(st)
            torch.cuda.synchronize()
            if i >= 3:
                times.append(a.elapsed_time(b) * 1e3)
        us = statistics.median(times)
        n = cache.stored_len()
        alg = B * HKV * n * per_pos + 2 * B * HQ * D * 2
        out.append({"cache": mode, "batch": B, "context": T, "window": win, "attended": n, "us": round(us, 1),
                    "alg_bytes": alg, "gbs": round(alg / us / 1e3, 1), "frac": round(alg / us / 1e3 / peak_gbs, 3)})
        del cache
        torch.cuda.empty_cache()
    return {"kernel": "attn_affine_kernel / attn_bf16_kernel (one launch per call, split-KV with in-kernel merge)",
            "shape": "Hq 16, Hkv 8, head_dim 256, scale 1.0; L2 flushed before each timed launch; median of 20",
            "cases": out}


# ---------------------------------------------------------------------------
# CPU baseline / reference arm (oracle port of the reference's path)


def cpu_sample_setup(T, seed=4000):
    import numpy as np
    import oracle
    rng = np.random.default_rng(seed)
    x = oracle.f32_to_bf16(rng.standard_normal((T, H)).astype(np.float32))
    wr = oracle.f32_to_bf16((rng.standard_normal((E, H)) * 0.02).astype(np.float32))
    # one layer's 128 experts: the CPU time does not depend on the code values,
    # so random codes with N(0.01, 0.001)-sized bf16 scales/biases stand in
    offs, sizes, stride = ecb(H, I)
    buf = rng.integers(0, 256, size=E * stride, dtype=np.uint8)
    view = buf.reshape(E, stride)
    for j in (1, 2, 4, 5, 7, 8):
        n = sizes[j] // 2
        sb = oracle.f32_to_bf16((0.01 + 0.001 * rng.standard_normal((E, n))).astype(np.float32))
        view[:, offs[j]:offs[j] + sizes[j]] = sb.view(np.uint8).reshape(E, -1)
    return x, wr, buf, offs, stride


def ecb(hidden, inter):
    sizes = [inter * hidden // 2, inter * hidden // 32, inter * hidden // 32] * 2 + \
            [hidden * inter // 2, hidden * inter // 32, hidden * inter // 32]
    offs = [0]
    for s in sizes[:-1]:
        offs.append(offs[-1] + s)
    return offs, sizes, sum(sizes)


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def oracle_all_cores():
    """The oracle on every host core this process may use, whatever
    OMP_NUM_THREADS says (torchrun sets it to 1)."""
    import oracle
    oracle.set_num_threads(host_cores())
    return oracle.num_threads()


def cpu_layer(x, wr, buf, offs, stride):
    import oracle
    ids, w, _ = oracle.router(x, wr, K)
    oracle.moe_experts(x, ids, w, buf, stride, offs, H, I)


def cpu_moe_step(sample, n_layers=LAYERS):
    """One whole step of the routed-expert workloads on the oracle: n_layers MoE
    blocks (router + 8 experts + combine) over the sample's tokens.  The CPU
    cost does not depend on which layer's weights are read (every layer's table
    is far above the host caches), so one table stands in for all of them."""
    for _ in range(n_layers):
        cpu_layer(*sample)


def cpu_moe_tokens(T, budget_s, n_steps):
    """Tokens per CPU step so that n_steps whole 30-layer steps fit budget_s
    (the oracle's cost is linear in routed pairs, i.e. in tokens)."""
    probe = cpu_sample_setup(1)
    cpu_layer(*probe)
    t0 = time.perf_counter()
    cpu_layer(*probe)
    per_tok = (time.perf_counter() - t0) * LAYERS
    return max(1, min(T, int(budget_s / max(n_steps * per_tok, 1e-9))))


def cpu_baseline(_layers, T, budget_s=15.0):
    """Routed-expert workloads: whole 30-layer steps on the oracle within budget_s."""
    cores = oracle_all_cores()
    Ts = cpu_moe_tokens(T, budget_s, 3)
    sample = cpu_sample_setup(Ts)
    cpu_moe_step(sample)
    n, t0 = 0, time.perf_counter()
    while n < 1 or time.perf_counter() - t0 < budget_s:
        cpu_moe_step(sample)
        n += 1
    step_s = (time.perf_counter() - t0) / n
    return {"value": round(Ts / step_s, 3), "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"{n} whole steps ({LAYERS} MoE layers: router + 8 experts + combine) of {Ts} of the "
                      f"workload's {T} tokens on the oracle (C++ OpenMP, fp64 accumulation), {step_s * 1e3:.1f} ms "
                      f"per step"}


def cpu_decoder_sample(seed=4000, T=1, kv=None):
    """Numpy weights for the oracle's decoder layer (one sliding, one full) and
    the 6-bit lm_head at the model's shapes, with caches of the run's KV kind
    (DECODE_KV unless given).  The CPU time does not depend on the code values,
    so uniform random codes with small bf16 scales stand in."""
    kv = DECODE_KV if kv is None else kv
    import numpy as np
    import oracle
    rng = np.random.default_rng(seed)

    def ql(out_f, in_f, bits):
        wq = rng.integers(0, 2 ** 32, size=(out_f, in_f * bits // 32), dtype=np.uint32)
        sc = oracle.f32_to_bf16((0.001 + 0.0001 * rng.standard_normal((out_f, in_f // 64))).astype(np.float32))
        bi = oracle.f32_to_bf16(np.full((out_f, in_f // 64), -0.01, np.float32))
        return (wq, sc, bi, in_f, bits)

    def nrm(n):
        return oracle.f32_to_bf16((1 + 0.1 * rng.standard_normal(n)).astype(np.float32))

    offs, sizes, stride = ecb(H, I)
    experts = (rng.integers(0, 256, size=E * stride, dtype=np.uint8), stride, offs)
    layers = []
    for full in (False, True):
        Hq, Hkv, D = 16, (2 if full else 8), (512 if full else 256)
        L = {"q": ql(Hq * D, H, 8), "k": ql(Hkv * D, H, 8), "v": None if full else ql(Hkv * D, H, 8),
             "o": ql(H, Hq * D, 8), "q_norm": nrm(D), "k_norm": nrm(D),
             "gate": ql(2112, H, 4), "up": ql(2112, H, 4), "down": ql(H, 2112, 4),
             "router": (oracle.f32_to_bf16(rng.standard_normal((E, H)).astype(np.float32)), 16, nrm(H), nrm(E),
                        H ** -0.5),
             "experts": experts}
        for k in ("input_norm", "post_attn_norm", "pre_ff_norm", "post_ff_norm_1", "pre_ff_norm_2",
                  "post_ff_norm_2", "post_ff_norm"):
            L[k] = nrm(H)
        cap = CTX + 16 if full else 1024
        ck = oracle.f32_to_bf16(rng.standard_normal((T, Hkv, cap, D)).astype(np.float32))
        cfg = {"heads": Hq, "kv_heads": Hkv, "head_dim": D, "rope_dims": 128 if full else 256,
               "rope_theta": 1e6 if full else 1e4, "eps": 1e-6, "k_eq_v": full, "scalar": 1.0, "attn_scale": 1.0,
               "top_k": K, "hidden": H, "inter_expert": I, "turbo_bits": 3 if kv == "turbo3" else 0}
        if kv == "affine":
            cfg["kv_mode"] = "affine"
            kq = tuple(a.reshape(T, Hkv, cap, -1) for a in oracle.kv_quant_affine(ck, 4))
            vq = tuple(a.reshape(T, Hkv, cap, -1) for a in oracle.kv_quant_affine(ck, 8))
            layers.append((L, kq, vq, cfg))
        else:
            layers.append((L, ck, ck.copy(), cfg))
    embed = ql(262144, H, 6)
    x = oracle.f32_to_bf16(rng.standard_normal((T, H)).astype(np.float32))
    return layers, embed, nrm(H), x


def cpu_sampler_setup(vocab=262144, seed=1, T=1):
    import numpy as np
    rng = np.random.default_rng(seed)
    return rng.integers(0, vocab, (T, 64)).astype(np.int32)


def cpu_decoder_step(sample, step, recent=None):
    """One whole decode step (one token per sequence of the sample) on the oracle: the 30 layers in the
    model's order (every fifth one full attention, the rest sliding), the
    final norm + tied lm_head with softcap and argmax, and — with `recent` —
    the sampler at the generate defaults (temperature 0.7, top_p 0.9,
    repetition penalty 1.15 over the last 64 tokens).  Each layer appends its
    K / V row at position CTX of its cache, as the GPU step does."""
    import oracle
    layers, embed, fnorm, x = sample
    h = x
    for i in range(LAYERS):
        L, ck, cv, cfg = layers[1 if (i + 1) % 5 == 0 else 0]
        h, _ = oracle.decoder_layer(h, L, ck, cv, CTX, cfg)
    lg, ids = oracle.lm_head(h, embed, fnorm, 1e-6, 30.0)
    if recent is not None:
        from oracle import sample as osmp
        osmp.sample(lg, recent, 0.7, 0.9, 1.15, seed=1, step=step)
    return ids


def cpu_decoder_baseline(T, budget_s=15.0, sampled=False):
    """decode30: whole decode steps on the oracle for about budget_s (at least one)."""
    cores = oracle_all_cores()
    Ts = cpu_decoder_tokens(T, budget_s, 2)
    sample = cpu_decoder_sample(T=Ts)
    recent = cpu_sampler_setup(T=Ts) if sampled else None
    cpu_decoder_step(sample, 0, recent)
    n, t0 = 0, time.perf_counter()
    while n < 1 or time.perf_counter() - t0 < budget_s:
        cpu_decoder_step(sample, n, recent)
        n += 1
    step_s = (time.perf_counter() - t0) / n
    return {"value": round(Ts / step_s, 3), "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"{n} whole decode steps of {Ts} of the workload's {T} sequences at context {CTX} on the "
                      f"oracle (C++ OpenMP / numpy), {DECODE_KV} KV cache: 24 sliding + 6 full layers + lm_head"
                      + (" + the sampler" if sampled else "") + f", {step_s * 1e3:.1f} ms per step"}


def cpu_decoder_tokens(T, budget_s, n_steps):
    """Sequences per CPU decode step so that n_steps whole steps fit budget_s
    (the oracle's step cost grows about linearly with the sequences)."""
    if T == 1:
        return 1
    s1 = cpu_decoder_sample(T=1)
    cpu_decoder_step(s1, 0)
    t0 = time.perf_counter()
    cpu_decoder_step(s1, 0)
    t1 = time.perf_counter() - t0
    return max(1, min(T, int(budget_s / max(n_steps * t1, 1e-9))))


REF_BUDGET_S = 150.0  # the reference arm's whole run (warm-up + timed steps) stays within a few minutes


def run_reference(args, rank, world):
    """The reference arm: the oracle (the repository's C++ / numpy port of the
    reference's path) on all host cores, rank 0 alone, same metric / unit /
    config as the GPU arm.  decode30: every step is one whole decode step.
    Routed-expert workloads: every step is one whole 30-layer step over a
    bounded number of the workload's tokens (the CPU cost is linear in tokens),
    sized so that warm-up + timed steps fit REF_BUDGET_S."""
    if rank != 0:
        return
    cores = oracle_all_cores()
    n_runs = args.steps + args.warmup
    if args.workload.startswith("decode30"):
        T = WORKLOADS[args.workload]
        tokens = cpu_decoder_tokens(T, REF_BUDGET_S, n_runs)
        sample = cpu_decoder_sample(T=tokens)
        recent = cpu_sampler_setup(T=tokens) if args.sample else None
        step = lambda i: cpu_decoder_step(sample, i, recent)  # noqa: E731
        metric, config = decoder_metric(args), decoder_config(args, world)
        dtype = "u8/u4/u6-affine weights x bf16 activations, fp32/fp64 accumulate (CPU)"
        desc = (f"each step = one whole decode step of {tokens} of the workload's {T} sequences at context {CTX} on "
                f"the oracle: 24 sliding + 6 full layers + lm_head"
                + (" + the sampler (temperature 0.7, top_p 0.9, penalty 1.15)" if args.sample else ""))
    else:
        if args.workload in EP_WORKLOADS:
            T = EP_WORKLOADS[args.workload][0]
            metric, config = ep_metric(args), ep_config(args, world)
        else:
            T = WORKLOADS[args.workload]
            metric, config = MOE_METRIC, moe_config(args, world)
        tokens = cpu_moe_tokens(T, REF_BUDGET_S, n_runs)
        sample = cpu_sample_setup(tokens)
        step = lambda i: cpu_moe_step(sample)  # noqa: E731
        dtype = "u4-affine weights x bf16 activations, fp64 accumulate (CPU)"
        desc = (f"each step = one whole {LAYERS}-layer step (router + 8 experts + combine per layer) over {tokens} "
                f"of the workload's {T} tokens on the oracle")
    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(args.warmup + i)
    step_s = (time.perf_counter() - t0) / max(args.steps, 1)
    value = tokens / step_s
    out = {
        "impl": "reference", "metric": metric, "value": round(value, 3), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_s * 1e3, 3),
        "higher_is_better": True, "scaling": "strong" if args.workload in EP_WORKLOADS else "weak",
        "vs_baseline": None, "dtype": dtype, "data": "synthetic (seeded)", "config": config,
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": cores, "kind": "port", "sample": desc},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference (Rust + MLX/Metal) cannot run here; this is the repository's C++ / numpy port of "
                "its path (oracle/), timed on the host cores",
    }
    print(json.dumps(out), flush=True)


def run_attn_case(args):
    import torch
    import __graft_entry__

    fm = __graft_entry__.load_package()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    mode, B, T = args.attn_case.split(":")
    peaks, _ = load_peaks()
    res = attn_submeasure(fm, torch, dev, peaks["hbm_gbs"], iters=1, cases=[(mode, int(B), int(T), None)])
    print(json.dumps({"attn_case": args.attn_case, **res}), flush=True)


def run_pf_attn_case(args):
    import torch
    import __graft_entry__

    fm = __graft_entry__.load_package()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    D, Hkv, Hq, win, T = (int(v) for v in args.pf_attn_case.split(":"))
    g = torch.Generator(device=dev).manual_seed(12)
    cache = fm.KVCache(1, Hkv, D, max(T, win or T), window=win or None, device=dev)
    q = (torch.randn(T, Hq, D, generator=g, device=dev) * 0.08).to(torch.bfloat16)
    kn = torch.randn(Hkv, T, D, generator=g, device=dev).to(torch.bfloat16)
    vn = torch.randn(Hkv, T, D, generator=g, device=dev).to(torch.bfloat16)
    for _ in range(4):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        cache.attend_prefill(q, kn, vn, 0, window=win)
        b.record()
        torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3
    keys = sum(min(t + 1, win) if win else t + 1 for t in range(T))
    flops = 4.0 * Hq * D * keys
    print(json.dumps({"pf_attn_case": args.pf_attn_case, "us": round(us, 1), "alg_flops": int(flops),
                      "tflops": round(flops / us / 1e6, 1)}), flush=True)


def run_qlinear_case(args):
    import torch
    import __graft_entry__

    fm = __graft_entry__.load_package()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    out_f, in_f, bits, T = (int(v) for v in args.qlinear_case.split(":"))
    g = torch.Generator(device=dev).manual_seed(11)
    w = torch.randn(out_f, in_f, generator=g, device=dev) * 0.02
    ql = fm.QuantizedLinear.from_float(w, bits)
    del w
    x = torch.randn(T, in_f, generator=g, device=dev).to(torch.bfloat16)
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    for _ in range(4):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        ql.forward(x)
        b.record()
        torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3
    nbytes = out_f * in_f * bits // 8 + 2 * out_f * (in_f // 64) * 2
    print(json.dumps({"qlinear_case": args.qlinear_case, "us": round(us, 1), "weight_bytes": nbytes,
                      "gbs": round(nbytes / us / 1e3, 1), "tflops": round(2.0 * T * out_f * in_f / us / 1e6, 1)}),
          flush=True)


def kv_kwargs(fm, kind):
    """Gemma4Model arguments of a decode30 KV-cache kind."""
    if kind == "affine":
        return {"kv_mode": fm.KV_AFFINE}
    return {"turbo_bits": 3 if kind == "turbo3" else 0}


def random_context(torch, m, T, g, dev):
    """CTX random bf16 K/V positions appended to every cache (through the cache's own
    append: TurboQuant round trip or affine quantisation as the cache has it)."""
    for L, c in zip(m.layers, m.caches):
        chunk = 256
        for p0 in range(0, CTX, chunk):
            kv = torch.randn(2, T, L.num_kv_heads, chunk, L.head_dim, generator=g, device=dev).to(torch.bfloat16)
            c.update(kv[0], kv[1])


def kv_variant(fm, torch, m, cfg, T, kind, prompt, ids0, stream, dev, g, steps=50, warmup=5):
    """decode30 with another KV-cache kind on the same weights (new caches only):
    context from the same prompt (prefill); one CUDA graph per step, `steps`
    replays timed with CUDA events after `warmup`."""
    v = fm.Gemma4Model(cfg, m.embed, m.layers, m.final_norm, T, CTX + 64, device=dev, **kv_kwargs(fm, kind))
    with torch.cuda.stream(stream):
        v.set_position(0)
        v.prefill(prompt)
        v.ids.copy_(ids0)
        v.set_position(CTX)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream, capture_error_mode="thread_local"):
            v.decode_step(device_pos=True)
        v.set_position(CTX)
        for _ in range(warmup):
            graph.replay()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(steps):
            graph.replay()
        b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    if v.status() != 0:
        raise SystemExit(f"kv variant {kind}: device status: {fm.last_error()}")
    del graph
    return {"kv_cache": KV_DESC[kind], "value": round(T / (ms / 1e3), 2), "unit": "tok/s", "ms_per_step": round(ms, 5),
            "context": "prefilled from the same prompt",
            "timing": f"{steps} CUDA-graph replays after {warmup}"}


def prefill_flops(m, T):
    """Algorithmic FLOPs of one T-token prompt through the decoder: projections,
    dense MLP, router, 8 routed experts per token, causal / sliding attention
    (QK and PV over the admitted keys), and the lm_head of the last position."""
    cfg = m.cfg
    fl = 0.0
    for L in m.layers:
        D, Hq = L.head_dim, L.num_heads
        qkv = L.q_proj.out_features + L.k_proj.out_features + (0 if L.k_eq_v else L.v_proj.out_features)
        per_tok = 2 * H * qkv + 2 * Hq * D * H + 2 * 3 * H * L.mlp[0].out_features + 2 * H * E + 2 * K * 3 * H * I
        full = getattr(L, "full_attention", L.k_eq_v)
        keys = sum(t + 1 if full else min(t + 1, cfg["window"]) for t in range(T))
        fl += T * per_tok + 4.0 * Hq * D * keys
    return fl + 2.0 * H * cfg["vocab"]


def decoder_prefill(torch, m, prompt, peaks, timed_reps=3):
    """Gemma4Model.prefill of every sequence's prompt (fills the caches; the first
    call builds the prefill buffers), then `timed_reps` CUDA-event timed prefills
    of the same prompts from position 0 (they rewrite the same rows).  Returns
    the sub-measurement for the JSON line, or None when untimed."""
    B, T = prompt.shape
    m.set_position(0)
    m.prefill(prompt)
    torch.cuda.synchronize()
    if timed_reps <= 0:
        return None
    times = []
    for _ in range(timed_reps):
        m.set_position(0)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        m.prefill(prompt)
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    ms = statistics.median(times)
    flops = B * prefill_flops(m, T)
    tf = flops / (ms / 1e3) / 1e12
    return {"metric": "prefill tok/s (whole decoder, %d-token prompt%s)" % (T, "" if B == 1 else " x %d" % B),
            "value": round(B * T / (ms / 1e3), 1), "unit": "tok/s", "ms": round(ms, 3), "tokens": B * T,
            "roofline": {"bound": "tensor", "alg_flops": int(flops), "achieved_tflops": round(tf, 1),
                         "peak_tflops": peaks["bf16_tflops_sustained"],
                         "frac": round(tf / peaks["bf16_tflops_sustained"], 4)},
            "api": "Gemma4Model.prefill (fmoe_embed_rows, fmoe_decoder_layer_prefill x layers, fmoe_lm_head)",
            "timing": f"median of {timed_reps} CUDA-event timed prefills after one warm-up prefill"}


def prefill_setup(fm, torch, dev, seed=2002):
    """BASELINE config 2's layer: 128 MLX-affine 4-bit experts, bf16 router
    N(0, 0.02), per-expert logit bias N(0, 1) (Zipf-like load skew)."""
    table = fm.ExpertTable.random(E, H, I, seed=seed, device=dev)
    g = torch.Generator(device=dev).manual_seed(seed)
    wr = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    bias = torch.randn(E, generator=g, device=dev)
    return fm.Gemma4MoeBlock(fm.QuantizedLinear(wr, bits=16), table, top_k=K, logit_bias=bias), g


def prefill_time(fm, torch, dev, block, g, T, iters):
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    y, ids, w = block.forward_prefill(x, return_routing=True)
    uniq = int(torch.unique(ids).numel())
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    times = []
    for i in range(iters):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        block.forward_prefill(x)
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b) * 1e3)
    return times, uniq


def prefill_submeasure(fm, torch, dev, peaks, T=512, iters=10):
    """the prefill MoE block (router + Zipf-skewed top-8 +
    grouped 4-bit expert GEMMs + combine) over T tokens, L2 flushed between
    runs; median of `iters` device-timed calls of Gemma4MoeBlock.forward_prefill."""
    block, g = prefill_setup(fm, torch, dev)
    times, uniq = prefill_time(fm, torch, dev, block, g, T, iters + 2)
    us = statistics.median(times[2:])
    flops = 2.0 * T * K * 3 * H * I                      # gate, up, down of every routed pair
    nbytes = uniq * EXPERT_BYTES + ROUTER_BYTES + 2 * T * H * 2
    t_fl = flops / (peaks["bf16_tflops"] * 1e12) * 1e6
    t_by = nbytes / (peaks["hbm_gbs"] * 1e9) * 1e6
    del block
    torch.cuda.empty_cache()
    return {"metric": "prefill tok/s (MoE block, one layer)", "tokens": T, "value": round(T / us * 1e6, 1),
            "unit": "tok/s", "us": round(us, 1), "unique_experts": uniq,
            "roofline": {"bound": "tensor" if t_fl > t_by else "hbm", "alg_flops": int(flops),
                         "alg_bytes": int(nbytes), "floor_us": round(max(t_fl, t_by), 1),
                         "frac": round(max(t_fl, t_by) / us, 4)},
            "timing": f"median of {iters} CUDA-event timed calls, 512 MB L2 flush before each"}


def run_prefill_case(args):
    import torch
    import __graft_entry__

    fm = __graft_entry__.load_package()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    block, g = prefill_setup(fm, torch, dev)
    times, uniq = prefill_time(fm, torch, dev, block, g, args.prefill_case, 4)
    print(json.dumps({"prefill_case": args.prefill_case, "us": round(times[-1], 1), "unique_experts": uniq}),
          flush=True)


def main():
    global DECODE_KV
    args = parse()
    DECODE_KV = args.kv_cache
    rank, world, local = dist_env()
    if args.prefill_case:
        run_prefill_case(args)
    elif args.attn_case:
        run_attn_case(args)
    elif args.qlinear_case:
        run_qlinear_case(args)
    elif args.pf_attn_case:
        run_pf_attn_case(args)
    elif args.impl == "reference":
        run_reference(args, rank, world)
    elif args.workload.startswith("decode30"):
        run_decoder(args, rank, world, local)
    elif args.workload in EP_WORKLOADS:
        run_ep_moe(args, rank, world, local)
    else:
        run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
