"""Next-token sampling on the device (fmoe_sample): the engine's sample()
(src/engine.rs:302-355) — repetition penalty over the recent tokens,
temperature, top-p, categorical draw — without the reference's host round trip
per token.

    sample_tokens(logits, ...)  one call: logits [rows, vocab] fp32 -> tokens int32 [rows]
    Sampler                     the decode loop's state: a device ring of the last
                                `window` tokens per row (the engine's REP_WINDOW = 64,
                                engine.rs:153-155), the call counter that keys the
                                random draw, and the workspace; capturable in a CUDA
                                graph (the counter and the ring live on the device)
"""
from __future__ import annotations

import torch

from . import _need_cuda, _ptr, _stream, _Workspace, check, lib


def sample_tokens(logits: torch.Tensor, temperature: float = 0.0, top_p: float = 1.0, rep_penalty: float = 1.0,
                  recent: torch.Tensor | None = None, seed: int = 0, step: torch.Tensor | None = None,
                  push: bool = False, out: torch.Tensor | None = None,
                  workspace: _Workspace | None = None) -> torch.Tensor:
    """logits [rows, vocab] fp32 -> next tokens int32 [rows].  recent: int32
    [rows, n] device tokens (-1 = empty slot); step: device uint64 [1] call
    counter (advanced by one; the draw is keyed by (seed, step, row, token));
    push: store each drawn token into recent[row, step % n]."""
    _need_cuda(logits)
    if logits.dim() != 2 or logits.dtype != torch.float32 or not logits.is_contiguous():
        raise ValueError("sample: contiguous fp32 logits [rows, vocab] expected")
    rows, vocab = logits.shape
    n_recent = 0
    if recent is not None:
        if recent.dtype != torch.int32 or recent.dim() != 2 or recent.shape[0] != rows or not recent.is_contiguous():
            raise ValueError("sample: recent must be contiguous int32 [rows, n]")
        n_recent = recent.shape[1]
    if step is not None and (step.dtype not in (torch.int64, torch.uint64) or step.numel() != 1):
        raise ValueError("sample: step must be a one-element 64-bit device tensor")
    out = torch.empty(rows, dtype=torch.int32, device=logits.device) if out is None else out
    nbytes = lib().fmoe_sample_workspace_bytes(rows, vocab)
    if nbytes == 0:
        raise ValueError(f"sample: unsupported shape [{rows}, {vocab}]")
    ws = (workspace or _Workspace()).get(nbytes, logits.device)
    check(lib().fmoe_sample(_ptr(logits), rows, vocab, _ptr(recent), n_recent, float(temperature), float(top_p),
                            float(rep_penalty), seed & ((1 << 64) - 1), _ptr(step), int(push), _ptr(out), _ptr(ws),
                            ws.numel(), _stream()))
    return out


class Sampler:
    """Decode-loop sampling state for `rows` sequences over a `vocab`-token
    head: ring of the last `window` drawn tokens per row (starts empty, as the
    reference's first draw after the prompt passes no recent tokens,
    engine.rs:95), the device call counter, a fixed workspace."""

    def __init__(self, rows: int, vocab: int, temperature: float = 0.0, top_p: float = 1.0,
                 rep_penalty: float = 1.0, seed: int = 0, window: int = 64, device="cuda"):
        self.temperature, self.top_p, self.rep_penalty, self.seed = temperature, top_p, rep_penalty, seed
        self.rows, self.vocab = rows, vocab
        device = torch.device(device)
        if device.type == "cuda" and device.index is None:  # the workspace is keyed by the indexed device
            device = torch.device("cuda", torch.cuda.current_device())
        self.recent = torch.full((rows, window), -1, dtype=torch.int32, device=device)
        self.step = torch.zeros(1, dtype=torch.int64, device=device)
        self._ws = _Workspace()
        self._ws.get(lib().fmoe_sample_workspace_bytes(rows, vocab), device)  # allocated once, outside any capture

    def reset(self) -> None:
        self.recent.fill_(-1)
        self.step.zero_()

    def __call__(self, logits: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        return sample_tokens(logits, self.temperature, self.top_p, self.rep_penalty, self.recent, self.seed,
                             self.step, push=True, out=out, workspace=self._ws)
