"""Shared helpers for the GPU tests (torch is used only to hold device memory)."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")


def require_gpu():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.max(np.abs(b))
    return float(np.max(np.abs(a - b)) / (den if den > 0 else 1.0))
