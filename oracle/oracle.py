"""ctypes loader for the CPU oracle (oracle/oracle.cpp).

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()`` and
by bench.py's cpu_baseline / reference arm, always as the checker or the timed
CPU baseline, never as the thing measured or shipped.
Each wrapper names the pkt function it restates (file:line in Marco-Christiani/pkt).
"""
import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


def build():
    subprocess.check_call(["make", "-s", "-C", _HERE, "all"])


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        L.orc_pkt_make_linear_data.argtypes = [ctypes.c_int] * 3 + [_f32p] * 3
        L.orc_pkt_host_mse.argtypes = [_f32p, _f32p, ctypes.c_longlong]
        L.orc_pkt_host_mse.restype = ctypes.c_float
        L.orc_pkt_cpu_train_linear.argtypes = [_f32p, _f32p, _f32p] + [ctypes.c_int] * 4 + [ctypes.c_float, _f32p]
        L.orc_axpy.argtypes = [_f32p, _f32p, ctypes.c_float, ctypes.c_longlong]
        L.orc_sgd.argtypes = [_f32p, _f32p, ctypes.c_float, ctypes.c_longlong]
        L.orc_bf16_round.argtypes = [ctypes.c_float]
        L.orc_bf16_round.restype = ctypes.c_float
        L.orc_num_threads.restype = ctypes.c_int
        L.orc_set_num_threads.argtypes = [ctypes.c_int]
        vp = ctypes.c_void_p
        L.orc_mlp_train.argtypes = [ctypes.c_int, _i32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                    _f32p, _f32p, _f32p, vp, ctypes.c_float, ctypes.c_int,
                                    _f32p, vp, vp, vp]
        L.orc_mlp_train.restype = ctypes.c_int
        L.orc_make_linear_task.argtypes = [ctypes.c_int] * 3 + [ctypes.c_uint, ctypes.c_float] + [_f32p] * 4
        _LIB = L
    return _LIB


def pkt_make_linear_data(m, n, batch):
    """examples/train_linear.cu:41-76 (mt19937(42) data generator)."""
    W = np.empty(m * n, np.float32)
    x = np.empty(batch * n, np.float32)
    t = np.empty(batch * m, np.float32)
    lib().orc_pkt_make_linear_data(m, n, batch, W, x, t)
    return W.reshape(m, n), x.reshape(batch, n), t.reshape(batch, m)


def pkt_host_mse(y, t):
    """examples/train_linear.cu:78-86."""
    y = np.ascontiguousarray(y, np.float32).ravel()
    t = np.ascontiguousarray(t, np.float32).ravel()
    return float(lib().orc_pkt_host_mse(y, t, y.size))


def pkt_cpu_train_linear(W, x, t, steps, lr):
    """examples/train_linear.cu:101-151, bit-identical loop order. Returns (W, losses)."""
    W = np.array(W, np.float32, copy=True, order="C")
    m, n = W.shape
    batch = x.shape[0]
    losses = np.zeros(steps, np.float32)
    lib().orc_pkt_cpu_train_linear(W, np.ascontiguousarray(x, np.float32),
                                   np.ascontiguousarray(t, np.float32), batch, m, n, steps,
                                   lr, losses)
    return W, losses


def axpy(x, y, a):
    """include/ops/axpy.cuh:33-46 (single-rounding fma)."""
    y = np.array(y, np.float32, copy=True)
    lib().orc_axpy(np.ascontiguousarray(x, np.float32), y, a, y.size)
    return y


def sgd(W, dW, lr):
    """include/ops/sgd.cuh:33-44."""
    W = np.array(W, np.float32, copy=True)
    lib().orc_sgd(W, np.ascontiguousarray(dW, np.float32), lr, W.size)
    return W


MODE = {"fp32": 0, "tf32": 1, "bf16": 2}


def mlp_train(dims, x, t, Ws, bs, lr, steps, mode="fp32", want_grads=False, want_acts=False,
              relu_last=False):
    """Multi-layer extension of examples/train_linear.cu:101-151 (bias, ReLU, dgrad).

    Ws: list of [d_{l+1}, d_l] arrays, bs: list of [d_{l+1}] arrays or None.
    Returns dict(W=list, b=list|None, losses, dW=list, db=list, acts=list).
    """
    L = len(dims) - 1
    dims_a = np.asarray(dims, np.int32)
    batch = x.shape[0]
    Wc = np.concatenate([np.asarray(w, np.float32).ravel() for w in Ws])
    bc = None if bs is None else np.concatenate([np.asarray(b, np.float32).ravel() for b in bs])
    losses = np.zeros(max(steps, 1), np.float32)
    gW = np.zeros_like(Wc) if want_grads else None
    gb = np.zeros_like(bc) if (want_grads and bc is not None) else None
    acts = np.zeros(sum(batch * d for d in dims[1:]), np.float32) if want_acts else None
    ptr = lambda a: None if a is None else a.ctypes.data_as(ctypes.c_void_p)
    rc = lib().orc_mlp_train(L, dims_a, batch, MODE[mode], int(relu_last),
                             np.ascontiguousarray(x, np.float32).ravel(),
                             np.ascontiguousarray(t, np.float32).ravel(), Wc, ptr(bc), lr, steps,
                             losses, ptr(gW), ptr(gb), ptr(acts))
    assert rc == 0
    out = {"losses": losses[:steps]}

    def split(flat, shapes):
        res, o = [], 0
        for s in shapes:
            k = int(np.prod(s))
            res.append(flat[o:o + k].reshape(s))
            o += k
        return res

    wshapes = [(dims[l + 1], dims[l]) for l in range(L)]
    out["W"] = split(Wc, wshapes)
    out["b"] = None if bc is None else split(bc, [(dims[l + 1],) for l in range(L)])
    if want_grads:
        out["dW"] = split(gW, wshapes)
        out["db"] = None if gb is None else split(gb, [(dims[l + 1],) for l in range(L)])
    if want_acts:
        out["acts"] = split(acts, [(batch, d) for d in dims[1:]])
    return out


def make_linear_task(inp, out, batch, seed=0, noise=0.01):
    """Seeded single-Linear problem: mt19937(seed); x~N(0,1), W~U(+-1/sqrt(in)), b=0,
    target = x W*^T + b* + N(0, noise^2) with W*, b* ~ N(0,1)."""
    x = np.empty(batch * inp, np.float32)
    W = np.empty(out * inp, np.float32)
    b = np.empty(out, np.float32)
    t = np.empty(batch * out, np.float32)
    lib().orc_make_linear_task(inp, out, batch, seed, noise, x, W, b, t)
    return x.reshape(batch, inp), W.reshape(out, inp), b, t.reshape(batch, out)
