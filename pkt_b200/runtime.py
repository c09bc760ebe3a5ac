"""Python mirror of pkt's host API over the C-ABI.

Same names, argument meaning and behaviour as pkt's C++ headers:
  * OpCode / TaskHeader / Task / encode_args / decode_args  (include/task.cuh:11-66)
  * ZeroMemoryArgs, AxpyArgs, LinearForwardArgs, LinearBackwardArgs, MSELossArgs,
    SGDUpdateArgs  (include/ops/*.cuh)
  * Runtime.initialize / submit_tasks / set_segments / set_segment_window_size /
    launch / synchronize / fetch_task_counter / set_task_accounting_enabled /
    set_perf_enabled / last_launch_blocks / fetch_perf_blocks / get_num_sms
    (include/runtime.hpp:27-329)
Differences: errors raise PktError instead of passing silently, and
Runtime.status() exposes the device status word (timeouts, bad opcodes).
"""
import ctypes
import enum

from . import _lib
from ._lib import GemmDesc, PktError, Task, TaskHeader, check

c_float, c_int, c_void_p = ctypes.c_float, ctypes.c_int, ctypes.c_void_p


class OpCode(enum.IntEnum):
    Invalid = 0
    ZeroMemory = 1
    Axpy = 2
    Gemm = 3
    LinearForward = 10
    MSELoss = 11
    LinearBackward = 12
    SGDUpdate = 13
    BiasSGD = 20
    LossReduce = 21
    SGDMixed = 22


class ZeroMemoryArgs(ctypes.Structure):
    _fields_ = [("ptr", c_void_p), ("size", c_int)]


class AxpyArgs(ctypes.Structure):
    _fields_ = [("x", c_void_p), ("y", c_void_p), ("a", c_float), ("n", c_int)]


class LinearForwardArgs(ctypes.Structure):
    _fields_ = [("W", c_void_p), ("x", c_void_p), ("y", c_void_p)] + [
        (n, c_int) for n in ("batch", "m", "n", "tile_m_start", "tile_m_count", "tile_n_start",
                             "tile_n_count")]


class LinearBackwardArgs(ctypes.Structure):
    _fields_ = [("dy", c_void_p), ("x", c_void_p), ("dW", c_void_p)] + [
        (n, c_int) for n in ("batch", "m", "n", "tile_m_start", "tile_m_count", "tile_n_start",
                             "tile_n_count")]


class MSELossArgs(ctypes.Structure):
    _fields_ = [("y", c_void_p), ("target", c_void_p), ("dy", c_void_p), ("loss", c_void_p),
                ("batch", c_int), ("m", c_int)]


class SGDUpdateArgs(ctypes.Structure):
    _fields_ = [("W", c_void_p), ("dW", c_void_p), ("lr", c_float), ("size", c_int)]


class GemmTileArgs(ctypes.Structure):
    _fields_ = [("gemm", ctypes.c_uint32), ("tile_m", ctypes.c_uint32),
                ("tile_n", ctypes.c_uint32), ("pad", ctypes.c_uint32)]


class BiasSGDArgs(ctypes.Structure):
    _fields_ = [("partials", c_void_p), ("bias", c_void_p), ("grad_out", c_void_p),
                ("num_partials", c_int), ("ld", c_int), ("col_begin", c_int), ("col_end", c_int),
                ("lr", c_float), ("pad", c_int)]


class LossReduceArgs(ctypes.Structure):
    _fields_ = [("partials", c_void_p), ("loss", c_void_p), ("count", c_int), ("scale", c_float),
                ("step", c_void_p)]


class SGDMixedArgs(ctypes.Structure):
    _fields_ = [("w", c_void_p), ("g", c_void_p), ("w_out", c_void_p), ("w_bf16", c_void_p),
                ("n", ctypes.c_longlong), ("lr", c_float), ("pad", c_int)]


_ARG_SIZES = {ZeroMemoryArgs: 16, AxpyArgs: 24, LinearForwardArgs: 56, LinearBackwardArgs: 56,
              MSELossArgs: 40, SGDUpdateArgs: 24}
for _k, _v in _ARG_SIZES.items():
    assert ctypes.sizeof(_k) == _v, (_k, ctypes.sizeof(_k))


def encode_args(task, opcode, args):
    """include/task.cuh:50-66: set opcode/arg_bytes, clear dependency fields, copy args."""
    n = ctypes.sizeof(args)
    if n > 64:
        raise ValueError("Args size exceeds task payload capacity")
    task.header.opcode = int(opcode)
    task.header.arg_bytes = n
    task.header.buffer_read_id = 0
    task.header.buffer_write_id = 0
    task.header.wait_count = 0
    task.header.read_epoch = 0
    task.header.write_epoch = 0
    task.header.ext_ids = 0
    task.header.ext_wait_count = 0
    ctypes.memset(task.args, 0, 64)
    ctypes.memmove(task.args, ctypes.addressof(args), n)
    return task


def decode_args(task, args_type):
    """include/task.cuh:43-47."""
    return args_type.from_buffer_copy(bytes(task.args)[:ctypes.sizeof(args_type)])


def make_tasks(n):
    return (Task * n)()


class Runtime:
    """pk::Runtime (include/runtime.hpp:22-450) over libpkt_b200."""

    def __init__(self, device=None):
        L = _lib.load()
        if device is None:
            device = _current_device()
        self.device = device
        h = c_void_p()
        check(L.pkt_runtime_create(device, ctypes.byref(h)))
        self._h = h
        self._L = L
        self._accounting = False
        self._perf = False

    def close(self):
        if self._h:
            self._L.pkt_runtime_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def initialize(self, max_tasks):
        check(self._L.pkt_runtime_initialize(self._h, int(max_tasks)))

    def submit_tasks(self, tasks):
        n = len(tasks)
        if n == 0:
            check(self._L.pkt_runtime_submit(self._h, None, 0))
            return
        if not isinstance(tasks, ctypes.Array):
            arr = (Task * n)(*tasks)
        else:
            arr = tasks
        check(self._L.pkt_runtime_submit(self._h, ctypes.cast(arr, c_void_p), n))

    def set_segments(self, segments):
        flat = (c_int * (2 * len(segments)))(*[v for s in segments for v in s])
        check(self._L.pkt_runtime_set_segments(self._h, ctypes.cast(flat, c_void_p), len(segments)))

    def set_segment_window_size(self, window):
        check(self._L.pkt_runtime_set_segment_window_size(self._h, int(window)))

    def launch(self, num_blocks, stream=None):
        check(self._L.pkt_runtime_launch(self._h, int(num_blocks), stream))

    def synchronize(self):
        check(self._L.pkt_runtime_synchronize(self._h))

    def status(self):
        code, task, detail = c_int(), c_int(), c_int()
        check(self._L.pkt_runtime_status(self._h, ctypes.byref(code), ctypes.byref(task),
                                         ctypes.byref(detail)))
        return code.value, task.value, detail.value

    def set_timeout_ns(self, ns):
        check(self._L.pkt_runtime_set_timeout_ns(self._h, int(ns)))

    def set_cta_pair(self, pair):
        """1: each CTA runs its own 128-row GEMM tiles; 2: CTA pairs share 256-row tiles."""
        check(self._L.pkt_runtime_set_cta_pair(self._h, int(pair)))

    def set_task_accounting_enabled(self, enabled):
        self._accounting = bool(enabled)
        check(self._L.pkt_runtime_set_task_accounting(self._h, int(bool(enabled))))

    def fetch_task_counter(self):
        if not self._accounting:
            return None
        v = ctypes.c_ulonglong()
        check(self._L.pkt_runtime_fetch_task_counter(self._h, ctypes.byref(v)))
        return v.value

    def set_perf_enabled(self, enabled):
        self._perf = bool(enabled)
        check(self._L.pkt_runtime_set_perf(self._h, int(bool(enabled))))

    def last_launch_blocks(self):
        return self._L.pkt_runtime_last_launch_blocks(self._h)

    def fetch_perf_blocks(self):
        if not self._perf:
            return None
        nb = self.last_launch_blocks()
        buf = (ctypes.c_ulonglong * (_lib.PERF_WORDS * max(nb, 1)))()
        got = c_int()
        check(self._L.pkt_runtime_fetch_perf(self._h, ctypes.cast(buf, c_void_p), nb,
                                             ctypes.byref(got)))
        w = _lib.PERF_WORDS
        return [list(buf[i * w:(i + 1) * w]) for i in range(got.value)]

    def register_gemms(self, descs):
        n = len(descs)
        arr = (GemmDesc * n)(*descs)
        first = c_int()
        check(self._L.pkt_runtime_register_gemms(self._h, ctypes.cast(arr, c_void_p), n,
                                                 ctypes.byref(first)))
        return list(range(first.value, first.value + n))

    def clear_gemms(self):
        check(self._L.pkt_runtime_clear_gemms(self._h))

    @staticmethod
    def get_num_sms(device=None):
        rc = _lib.load().pkt_num_sms(_current_device() if device is None else device)
        if rc < 0:
            check(rc)
        return rc


def gemm_tiles(desc):
    tm, tn = c_int(), c_int()
    check(_lib.load().pkt_gemm_tiles(ctypes.byref(desc), ctypes.byref(tm), ctypes.byref(tn)))
    return tm.value, tn.value


def axpy(x_ptr, y_ptr, a, n, stream=None):
    """y = a*x + y over n floats of device memory (examples/axpy_example.cu workload)."""
    check(_lib.load().pkt_axpy(x_ptr, y_ptr, float(a), int(n), stream))


def _current_device():
    try:
        import torch
        if torch.cuda.is_available():
            return torch.cuda.current_device()
    except Exception:
        pass
    return 0


def axpy_noalloc(x_ptr, y_ptr, a, n, stream=None):
    """pkt_axpy for callers that must not allocate: scratch in a fixed array of the
    library (n <= 67,108,864); calls that overlap on the GPU race on that array."""
    check(_lib.load().pkt_axpy_noalloc(x_ptr, y_ptr, float(a), int(n), stream))


def axpy_noalloc_status():
    """(code, task, detail) of the last pkt_axpy_noalloc launch on the current device
    (all 0 after a clean run); synchronises the device first."""
    code, task, detail = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    check(_lib.load().pkt_axpy_noalloc_status(ctypes.byref(code), ctypes.byref(task), ctypes.byref(detail)))
    return code.value, task.value, detail.value
