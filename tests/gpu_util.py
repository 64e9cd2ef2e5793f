"""Helpers shared by the GPU parity tests (device buffers through torch, calls
through the C-ABI)."""
import numpy as np
import torch

from channel_b200 import _lib as L


def dev(a: np.ndarray) -> torch.Tensor:
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    elif a.dtype == np.uint16:
        a = a.view(np.int16)
    elif a.dtype == np.uint64:
        a = a.view(np.int64)
    return torch.from_numpy(a).cuda()


def empty(n, dtype=torch.float32) -> torch.Tensor:
    return torch.empty(int(n), dtype=dtype, device="cuda")


def host(t: torch.Tensor, dtype=None) -> np.ndarray:
    a = t.cpu().numpy()
    return a.view(dtype) if dtype is not None else a


def call(fn, *args):
    torch.cuda.synchronize()
    L.check(fn(*args))


def rel_err(y, ref) -> float:
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.linalg.norm(y - ref) / max(np.linalg.norm(ref), 1e-30))


# parity bar from the spec: 1e-3 relative (norm-wise), fp32 accumulate
REL_TOL = 1e-3


def assert_close(y, ref, tol=REL_TOL, what=""):
    e = rel_err(y, ref)
    assert e < tol, f"{what}: relative error {e:.3e} >= {tol}"
    amax = float(np.max(np.abs(np.asarray(y, np.float64) - np.asarray(ref, np.float64))))
    assert amax <= tol * float(np.max(np.abs(ref))) + 1e-30, f"{what}: max abs err {amax:.3e}"
    return e
