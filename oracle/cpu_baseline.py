"""Timed CPU baseline: ctypes wrapper of oracle/cpu_mlp.cpp (fp32 OpenMP restatement
of pkt's host training loop, examples/train_linear.cu:101-151, extended to the MLP)
and of pkt's own single-threaded loop (oracle.cpp ``orc_pkt_cpu_train_linear``).

BENCHMARK / TEST INFRASTRUCTURE ONLY: used by bench.py's cpu_baseline leg and its
reference arm, and by tests/. Both libraries are compiled with -O3 -march=native
on the machine that runs them (``make -C oracle native``), so the timing uses that
machine's vector units; nothing here is shipped or called by the product path.
"""
import ctypes
import os
import platform
import subprocess
import time

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_NATIVE = os.path.join(_HERE, "_native")
_LIBS = {}
FLAGS = "g++ -O3 -march=native -fopenmp"


def ensure_built():
    subprocess.check_call(["make", "-s", "-C", _HERE, "native"], stdout=subprocess.DEVNULL)


def _lib(name):
    if name not in _LIBS:
        ensure_built()
        L = ctypes.CDLL(os.path.join(_NATIVE, name))
        if name == "libcpu_mlp.so":
            L.cpu_mlp_create.restype = ctypes.c_void_p
            L.cpu_mlp_create.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int]
            L.cpu_mlp_destroy.argtypes = [ctypes.c_void_p]
            L.cpu_mlp_step.restype = ctypes.c_float
            L.cpu_mlp_step.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_float]
            L.cpu_mlp_num_threads.restype = ctypes.c_int
            L.cpu_mlp_set_num_threads.argtypes = [ctypes.c_int]
        else:
            f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
            L.orc_pkt_cpu_train_linear.argtypes = [f32p, f32p, f32p] + [ctypes.c_int] * 4 + [ctypes.c_float, f32p]
            L.orc_set_num_threads.argtypes = [ctypes.c_int]
        _LIBS[name] = L
    return _LIBS[name]


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


class MLPStep:
    """fp32 MLP training step on the host cores (weights updated in place)."""

    def __init__(self, dims, batch, Ws, bs, threads=0):
        self.L = _lib("libcpu_mlp.so")
        if threads:
            self.L.cpu_mlp_set_num_threads(int(threads))
        self.threads = self.L.cpu_mlp_num_threads()
        self.dims = np.asarray(dims, np.int32)
        self.batch = batch
        self.W = np.concatenate([np.ascontiguousarray(w, np.float32).ravel() for w in Ws])
        self.b = None if bs is None else np.concatenate([np.ascontiguousarray(v, np.float32).ravel() for v in bs])
        self.h = self.L.cpu_mlp_create(len(dims) - 1, self.dims.ctypes.data, batch)
        if not self.h:
            raise ValueError("bad MLP configuration")

    def step(self, x, t, lr):
        return float(self.L.cpu_mlp_step(self.h, x.ctypes.data, t.ctypes.data, self.W.ctypes.data,
                                         None if self.b is None else self.b.ctypes.data, float(lr)))

    def close(self):
        if self.h:
            self.L.cpu_mlp_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()


def time_mlp(dims, x, t, Ws, bs, lr, max_steps, budget_s, warmup=1, threads=0):
    """Full-batch steps on the host cores: `warmup` untimed, then timed steps until
    `max_steps` or until `budget_s` seconds have been spent. Returns a dict with
    samples/s, the steps and seconds actually timed, the threads and the losses."""
    x = np.ascontiguousarray(x, np.float32)
    t = np.ascontiguousarray(t, np.float32)
    m = MLPStep(dims, x.shape[0], Ws, bs, threads)
    for _ in range(warmup):
        m.step(x, t, lr)
    losses, n = [], 0
    t0 = time.perf_counter()
    while n < max(1, max_steps):
        losses.append(m.step(x, t, lr))
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    secs = time.perf_counter() - t0
    m.close()
    return {"samples_per_s": x.shape[0] * n / secs, "steps": n, "seconds": secs,
            "threads": m.threads, "losses": losses}


def time_pkt_loop(W, x, t, steps, lr):
    """pkt's own host loop (single-threaded; no bias), native build. Returns
    (samples/s, seconds, final loss)."""
    L = _lib("liboracle.so")
    L.orc_set_num_threads(1)
    W = np.array(W, np.float32, copy=True, order="C")
    m, n = W.shape
    batch = x.shape[0]
    losses = np.zeros(steps, np.float32)
    t0 = time.perf_counter()
    L.orc_pkt_cpu_train_linear(W, np.ascontiguousarray(x, np.float32), np.ascontiguousarray(t, np.float32),
                               batch, m, n, steps, lr, losses)
    secs = time.perf_counter() - t0
    return batch * steps / secs, secs, float(losses[-1])
