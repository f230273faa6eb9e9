"""Expert parallelism over libfmoe: the experts of every MoE layer split
contiguously over the GPUs of one box (one process per GPU), tokens exchanged
by NCCL inside the library (fmoe_ep_* in include/fmoe.h).

The reference has no multi-device path (Gemma4MoeBlock::forward,
src/model/moe.rs:315-470, runs every routed expert on its one device); this
module adds the split that BASELINE config 5 asks for:

    EPComm                    the NCCL communicator (unique id over torch.distributed)
    ExpertTable.shard(r, n)   experts [r*E/n, (r+1)*E/n) of a layer (package __init__)
    ExpertParallelMoeBlock    Gemma4MoeBlock's interface with the experts on their owners
    PeerWatch                 host-side liveness check between steps (a lost rank is
                              reported before the next exchange is launched)

torch.distributed is plumbing only (rendezvous, the id broadcast, barriers);
the dispatch and combine exchanges are the library's grouped ncclSend/ncclRecv,
or (FMOE_EP_P2P) the library's own kernels storing rows straight into the
peers' exchange windows over NVLink.
"""
from __future__ import annotations

import ctypes
import time

import torch

from . import (ExpertTable, FmoeError, QuantizedLinear, _need_cuda, _ptr, _stream, _Workspace, check, lib)

FMOE_EP_FIXED = 0  # every rank exchanges cap rows with every rank (graph-capturable)
FMOE_EP_EXACT = 1  # counts cross first (one host sync), then only the routed rows
FMOE_EP_P2P = 2    # FIXED's exchange as stores into the peers' memory (CUDA IPC windows); EPComm.p2p_init
UNIQUE_ID_BYTES = 128


def shard_range(num_experts: int, world: int, rank: int) -> tuple[int, int]:
    """(first expert, count) held by `rank`: contiguous, num_experts / world each."""
    if world < 1 or num_experts % world:
        raise ValueError(f"{num_experts} experts do not split evenly over {world} ranks")
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside [0, {world})")
    n = num_experts // world
    return rank * n, n


class EPComm:
    """The expert-parallel group's NCCL communicator on the current CUDA device.

    rank / world default to torch.distributed's; with world > 1 rank 0's NCCL
    unique id is broadcast over torch.distributed (any backend).  Every rank must
    make the same sequence of expert-parallel calls.  close() (or abort() from a
    watchdog) frees it; release CUDA graphs that captured its exchanges first."""

    def __init__(self, rank: int | None = None, world: int | None = None, group=None):
        import torch.distributed as dist

        if world is None:
            world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        if rank is None:
            rank = dist.get_rank(group) if world > 1 else 0
        self.rank, self.world = rank, world
        uid = ctypes.create_string_buffer(UNIQUE_ID_BYTES)
        if rank == 0:
            check(lib().fmoe_ep_unique_id(uid, UNIQUE_ID_BYTES))
        if world > 1:
            obj = [uid.raw if rank == 0 else None]
            dist.broadcast_object_list(obj, src=0, group=group)
            uid = ctypes.create_string_buffer(obj[0], UNIQUE_ID_BYTES)
        self._h = ctypes.c_void_p()
        self.p2p_shape = None
        check(lib().fmoe_ep_comm_init(ctypes.byref(self._h), world, rank, uid, UNIQUE_ID_BYTES))

    @property
    def handle(self) -> ctypes.c_void_p:
        if not self._h:
            raise RuntimeError("EPComm: communicator closed")
        return self._h

    def p2p_init(self, cap: int, hidden: int, top_k: int) -> None:
        """Collective: (re)creates the peer-memory exchange windows for
        FMOE_EP_P2P calls with this cap / hidden / top_k.  Re-creating frees
        the previous windows: release CUDA graphs that captured P2P exchanges
        on them first."""
        self.p2p_shape = None
        check(lib().fmoe_ep_p2p_init(self.handle, cap, hidden, top_k))
        self.p2p_shape = (cap, hidden, top_k)

    def ensure_p2p(self, cap: int, hidden: int, top_k: int) -> None:
        if self.p2p_shape != (cap, hidden, top_k):
            self.p2p_init(cap, hidden, top_k)

    def status(self) -> None:
        """Raises FmoeError if NCCL recorded an asynchronous error."""
        check(lib().fmoe_ep_comm_status(self.handle))

    def close(self) -> None:
        """Collective once p2p_init ran (every rank calls it); after a lost rank use abort()."""
        if self._h:
            h, self._h = self._h, ctypes.c_void_p()
            check(lib().fmoe_ep_comm_destroy(h))

    def abort(self) -> None:
        """Ends outstanding exchanges with an error and frees the communicator."""
        if self._h:
            h, self._h = self._h, ctypes.c_void_p()
            check(lib().fmoe_ep_comm_abort(h))

    def shard(self, num_experts: int) -> tuple[int, int]:
        return shard_range(num_experts, self.world, self.rank)


class PeerLost(RuntimeError):
    """A rank of the expert-parallel group did not reach a step in time."""


class PeerWatch:
    """Liveness check between steps over the torch.distributed store: every
    rank checks in under a per-step key and waits, with a deadline, for all
    others.  A rank that died or left is reported as PeerLost (naming it) on
    the host, before any exchange of that step is launched, so no collective is
    left waiting on the GPU."""

    def __init__(self, store, rank: int, world: int, prefix: str = "fmoe_ep"):
        self.store, self.rank, self.world, self.prefix = store, rank, world, prefix
        self.step = 0

    def arrive(self, timeout_s: float = 30.0) -> int:
        """Check in for the next step; returns its index or raises PeerLost."""
        s = self.step
        self.store.set(f"{self.prefix}/{s}/{self.rank}", "1")
        deadline = time.monotonic() + timeout_s
        missing = [r for r in range(self.world) if r != self.rank]
        while missing:
            missing = [r for r in missing if not self.store.check([f"{self.prefix}/{s}/{r}"])]
            if not missing:
                break
            if time.monotonic() > deadline:
                raise PeerLost(f"step {s}: rank(s) {missing} did not check in within {timeout_s:.1f} s")
            time.sleep(0.002)
        self.step += 1
        return s


class ExpertParallelMoeBlock:
    """Gemma4MoeBlock (src/model/moe.rs:298-470) with the layer's experts split
    over the group: `experts` is this rank's slice (ExpertTable.shard), the
    router is the full replicated one, and forward(x) serves this rank's tokens.

    cap: the most tokens any rank passes per call (FIXED exchanges cap rows per
    peer); mode FMOE_EP_FIXED (no host sync, capturable), FMOE_EP_EXACT (only
    routed rows cross; one host sync per call) or FMOE_EP_P2P (FIXED's layout,
    stored straight into the peers' windows; capturable; sets up the comm's
    windows for this cap, collectively, when they differ)."""

    def __init__(self, comm: EPComm, router_proj: QuantizedLinear, experts: ExpertTable, cap: int, top_k=8,
                 mode=FMOE_EP_FIXED, router_scale=None, per_expert_scale=None, root_size=None, rms_norm_eps=1e-6,
                 use_norm=False, logit_bias=None):
        from . import Gemma4MoeBlock

        first, n = comm.shard(router_proj.out_features)
        if experts.first_expert != first or experts.num_experts != n:
            raise ValueError(f"rank {comm.rank}: expected experts [{first}, {first + n}), got "
                             f"[{experts.first_expert}, {experts.first_expert + experts.num_experts})")
        self.comm, self.cap, self.mode = comm, cap, mode
        if mode == FMOE_EP_P2P:
            comm.ensure_p2p(cap, router_proj.in_features, top_k)
        # the router half of the single-device block (same fields and argument meaning)
        self._block = Gemma4MoeBlock(router_proj, experts, top_k, router_scale, per_expert_scale, root_size,
                                     rms_norm_eps, use_norm, logit_bias)
        self.experts, self.top_k = experts, top_k
        self._ws = _Workspace()
        self._prep = None

    def _prepared(self, device):
        if self.comm.world * self.cap <= 128:
            return None  # the decode expert kernels serve every call
        if self._prep is None:
            self._prep = self._block._prepared(device)
        return self._prep

    def workspace_bytes(self) -> int:
        r = self._block.router_cstruct()
        e = self.experts.cstruct()
        return lib().fmoe_ep_moe_workspace_bytes(self.comm.world, self.cap, ctypes.byref(r), ctypes.byref(e))

    def forward(self, x: torch.Tensor, return_routing=False, out=None):
        _need_cuda(x)
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        T = x2.shape[0]
        if T > self.cap:
            raise ValueError(f"{T} tokens above the exchange capacity {self.cap}")
        y = torch.empty_like(x2) if out is None else out.view(-1, shape[-1])
        if T == 0:  # no tokens here: this rank still takes part in both exchanges
            x2 = torch.zeros(1, shape[-1], dtype=x.dtype, device=x.device)
            y = torch.empty_like(x2)
        ids = torch.empty(max(T, 1), self.top_k, dtype=torch.int32, device=x.device)
        w = torch.empty(max(T, 1), self.top_k, dtype=torch.float32, device=x.device)
        r = self._block.router_cstruct()
        e = self.experts.cstruct()
        prep = self._prepared(x.device)
        nbytes = self.workspace_bytes()
        if nbytes == 0:
            raise FmoeError(-1, "ExpertParallelMoeBlock: unsupported router / expert configuration")
        buf = self._ws.get(nbytes, x.device)
        check(lib().fmoe_ep_moe_forward(self.comm.handle, _ptr(x2), T, self.cap, ctypes.byref(r), ctypes.byref(e),
                                        _ptr(prep), _ptr(y), _ptr(ids), _ptr(w), self.mode, _ptr(buf), buf.numel(),
                                        _stream()))
        y = y[:T].reshape(shape)
        return (y, ids[:T], w[:T]) if return_routing else y

    __call__ = forward
