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
