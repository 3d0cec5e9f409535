"""Helpers for the GPU parity tests: device buffers through torch (plumbing)."""
import numpy as np
import torch


def dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t: torch.Tensor) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy()


def empty_f32(n: int) -> torch.Tensor:
    # NaN-filled, so an element a kernel forgot to write cannot pass as correct
    return torch.full((n,), float("nan"), dtype=torch.float32, device="cuda")


def same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    """Bit equality, with every NaN equal to every NaN (payloads are not
    observable through Mapal's print, which renders all NaNs as "NaN")."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    if a.shape != b.shape:
        return False
    na, nb = np.isnan(a), np.isnan(b)
    if not np.array_equal(na, nb):
        return False
    return np.array_equal(a[~na].view(np.uint32), b[~nb].view(np.uint32))


def first_diff(a, b) -> str:
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    bad = np.nonzero(a.view(np.uint32) != b.view(np.uint32))[0]
    if bad.size == 0:
        return "no difference"
    i = bad[0]
    return f"{bad.size} differ; first at {i}: {a[i]!r} vs {b[i]!r}"
