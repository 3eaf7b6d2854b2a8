"""Shared helpers of the parity tests."""
import numpy as np
import torch

ATOL = 2e-3  # max-abs vs the fp32-or-better reference, fp16 I/O


def np16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy()


def max_abs(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b))) if a.size else 0.0


def ulp_distance_fp16(got: np.ndarray, ref64: np.ndarray) -> np.ndarray:
    """Distance in fp16 ulps between got (fp16) and ref (float64) rounded to fp16."""
    r = ref64.astype(np.float16).view(np.int16).astype(np.int64)
    g = np.asarray(got, dtype=np.float16).view(np.int16).astype(np.int64)
    # map sign-magnitude to a monotone integer line
    r = np.where(r < 0, -(r & 0x7FFF), r)
    g = np.where(g < 0, -(g & 0x7FFF), g)
    return np.abs(r - g)


def to_dev(case_tensors, device="cuda"):
    return [t.to(device) for t in case_tensors]
