"""Helpers shared by the GPU parity tests."""
import numpy as np
import torch


def to_np_bf16(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def to_np_u32(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().numpy().view(np.uint32)


def max_rel_err(got, want) -> float:
    """max |got - want| / max |want|  (the tolerance metric of the benchmark spec)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))


def topk_gap(logits: np.ndarray, k: int) -> np.ndarray:
    """Per-token gap between the k-th and (k+1)-th largest logit."""
    s = -np.sort(-logits, axis=1)
    return s[:, k - 1] - s[:, k]


def bf16_round(x) -> np.ndarray:
    """fp32 -> nearest bf16 (ties to even), returned as fp32."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def topk_sure(logits: np.ndarray, k: int, gap: float = 1e-3, margin: float = 2e-5) -> np.ndarray:
    """Tokens whose top-k routing is decided robustly under the router rule
    (bf16-rounded logits, descending, ties to the lower id): the k-th and
    (k+1)-th bf16 logits differ by more than `gap` (the benchmark's 1e-3), and
    none of the top k+1 fp32 logits lies within `margin` (relative) of a bf16
    rounding midpoint, so fp32 accumulation-order noise cannot change which
    bf16 values the experts get (hence neither the ids nor the weights)."""
    lg = np.asarray(logits, np.float32)
    b = bf16_round(lg)
    order = np.argsort(-b, axis=1, kind="stable")
    top = np.take_along_axis(lg, order[:, :k + 1], axis=1)
    tb = np.take_along_axis(b, order[:, :k + 1], axis=1)
    mid = (np.ascontiguousarray(top).view(np.uint32) & np.uint32(0xFFFF0000)) | np.uint32(0x8000)
    dist = np.abs(top - mid.view(np.float32)) / np.maximum(np.abs(top), 1e-30)
    return (tb[:, k - 1] - tb[:, k] > gap) & (dist > margin).all(axis=1)
