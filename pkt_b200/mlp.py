"""MLP training engine (the hot path) over the C-ABI.

One training step = one persistent megakernel launch over a tile-granular task
DAG: tcgen05 forward tiles with fused bias+ReLU, MSE + dY fused into the last
layer's epilogue, ReLU-masked dgrad tiles, weight-gradient tiles with the SGD
update fused into their epilogue, bias SGD from column partials.
This is the multi-layer generalisation of pkt's train_linear
(examples/train_linear.cu:482-607).
"""
import ctypes

import numpy as np

from . import _lib
from ._lib import PKT_DTYPE_BF16, PKT_DTYPE_TF32, MlpConfig, check

c_int, c_void_p = ctypes.c_int, ctypes.c_void_p

DTYPES = {"bf16": PKT_DTYPE_BF16, "tf32": PKT_DTYPE_TF32}


def to_bf16_bits(a):
    """fp32 -> bf16 bits (round to nearest even) as uint16."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def from_bf16_bits(h):
    return (np.asarray(h, np.uint16).astype(np.uint32) << 16).view(np.float32)


class MLP:
    def __init__(self, dims, batch, dtype="bf16", lr=1e-3, bias=True, relu_last=False,
                 grad_mode=0, max_bn=0, cta_pair=0, device=None):
        L = _lib.load()
        self._L = L
        self.dims = list(dims)
        self.batch = batch
        self.dtype = dtype
        self.storage = np.uint16 if dtype == "bf16" else np.float32
        self._dims_c = (c_int * len(dims))(*dims)
        cfg = MlpConfig(len(dims) - 1, self._dims_c, batch, DTYPES[dtype], int(bias),
                        int(relu_last), float(lr), int(grad_mode), int(max_bn), int(cta_pair))
        if device is None:
            from .runtime import _current_device
            device = _current_device()
        h = c_void_p()
        check(L.pkt_mlp_create(device, ctypes.byref(cfg), ctypes.byref(h)))
        self._h = h
        self.has_bias = bias
        self.grad_mode = grad_mode

    def close(self):
        if self._h:
            self._L.pkt_mlp_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def num_layers(self):
        return len(self.dims) - 1

    def _wsize(self):
        return sum(self.dims[i] * self.dims[i + 1] for i in range(self.num_layers))

    def _bsize(self):
        return sum(self.dims[1:])

    def set_params(self, Ws, bs=None):
        W = np.concatenate([np.ascontiguousarray(w, np.float32).ravel() for w in Ws])
        b = None if bs is None else np.concatenate([np.ascontiguousarray(x, np.float32).ravel() for x in bs])
        check(self._L.pkt_mlp_set_params(self._h, W.ctypes.data_as(c_void_p),
                                         None if b is None else b.ctypes.data_as(c_void_p)))

    def get_params(self):
        W = np.zeros(self._wsize(), np.float32)
        b = np.zeros(self._bsize(), np.float32)
        check(self._L.pkt_mlp_get_params(self._h, W.ctypes.data_as(c_void_p), b.ctypes.data_as(c_void_p)))
        return self._split_w(W), self._split_b(b)

    def get_grads(self):
        W = np.zeros(self._wsize(), np.float32)
        b = np.zeros(self._bsize(), np.float32)
        check(self._L.pkt_mlp_get_grads(self._h, W.ctypes.data_as(c_void_p), b.ctypes.data_as(c_void_p)))
        return self._split_w(W), self._split_b(b)

    def _split_w(self, W):
        out, o = [], 0
        for i in range(self.num_layers):
            k = self.dims[i] * self.dims[i + 1]
            out.append(W[o:o + k].reshape(self.dims[i + 1], self.dims[i]))
            o += k
        return out

    def _split_b(self, b):
        out, o = [], 0
        for d in self.dims[1:]:
            out.append(b[o:o + d])
            o += d
        return out

    def storage_array(self, a):
        """fp32 array -> the engine's storage representation (bf16 bits or fp32)."""
        return to_bf16_bits(a) if self.dtype == "bf16" else np.ascontiguousarray(a, np.float32)

    def load_batch(self, x, t, stream=None):
        """x, t: host arrays in storage representation (see storage_array), or raw
        device pointers (ints) with on_device semantics."""
        if isinstance(x, int):
            check(self._L.pkt_mlp_load_batch(self._h, x, t, 1, stream))
            return
        x = np.ascontiguousarray(x)
        t = np.ascontiguousarray(t)
        assert x.dtype == self.storage and t.dtype == self.storage
        assert x.shape == (self.batch, self.dims[0]) and t.shape == (self.batch, self.dims[-1])
        self._hold = (x, t)  # keep host buffers alive until the copy ran
        check(self._L.pkt_mlp_load_batch(self._h, x.ctypes.data_as(c_void_p),
                                         t.ctypes.data_as(c_void_p), 0, stream))

    def load_batch_ptr(self, x_ptr, t_ptr, on_device, stream=None):
        check(self._L.pkt_mlp_load_batch(self._h, x_ptr, t_ptr, int(on_device), stream))

    def train(self, steps=1, stream=None):
        check(self._L.pkt_mlp_train(self._h, int(steps), stream))

    def forward_backward(self, stream=None):
        check(self._L.pkt_mlp_forward_backward(self._h, stream))

    def apply_update(self, stream=None):
        check(self._L.pkt_mlp_apply_update(self._h, stream))

    def backward_segments(self):
        """Number of launches the segmented step takes (grad_mode 1): L."""
        n = ctypes.c_int()
        check(self._L.pkt_mlp_backward_segments(self._h, ctypes.byref(n)))
        return n.value

    def forward_backward_segment(self, segment, stream=None):
        """Segment s of the step (grad_mode 1); after it, layer L-1-s's gradient
        bucket (grad_bucket) is final and can be all-reduced on another stream."""
        check(self._L.pkt_mlp_forward_backward_segment(self._h, int(segment), stream))

    def grad_bucket(self, layer):
        """(offset, count) in floats of layer `layer`'s dW and db in grad_buffer()."""
        o, n = ctypes.c_longlong(), ctypes.c_longlong()
        check(self._L.pkt_mlp_grad_bucket(self._h, int(layer), ctypes.byref(o), ctypes.byref(n)))
        return o.value, n.value

    def set_reserved_sms(self, sms):
        """Leave `sms` SMs out of the persistent grid (room for a collective kernel)."""
        check(self._L.pkt_mlp_set_reserved_sms(self._h, int(sms)))

    def grad_buffer(self):
        p, n = c_void_p(), ctypes.c_longlong()
        check(self._L.pkt_mlp_grad_buffer(self._h, ctypes.byref(p), ctypes.byref(n)))
        return p.value, n.value

    # ---- fused data parallel (grad_mode 2)
    DP_HANDLE_BYTES = 64

    def dp_handle(self):
        """This rank's exchange-region handle (CUDA IPC, 64 bytes) for its peers."""
        buf = ctypes.create_string_buffer(self.DP_HANDLE_BYTES)
        check(self._L.pkt_mlp_dp_handle(self._h, ctypes.cast(buf, c_void_p)))
        return buf.raw

    def dp_connect(self, rank, world, handles=None):
        """Maps every peer's exchange region; handles: the ranks' dp_handle()
        bytes in rank order (None for world 1)."""
        if world > 1:
            assert len(handles) == world and all(len(h) == self.DP_HANDLE_BYTES for h in handles)
            buf = ctypes.create_string_buffer(b"".join(handles), self.DP_HANDLE_BYTES * world)
            check(self._L.pkt_mlp_dp_connect(self._h, int(rank), int(world), ctypes.cast(buf, c_void_p)))
        else:
            check(self._L.pkt_mlp_dp_connect(self._h, int(rank), int(world), None))

    def set_grad_scale(self, s):
        check(self._L.pkt_mlp_set_grad_scale(self._h, float(s)))

    def set_output_capture(self, on=True):
        check(self._L.pkt_mlp_set_output_capture(self._h, int(bool(on))))

    def get_output(self):
        y = np.zeros((self.batch, self.dims[-1]), np.float32)
        check(self._L.pkt_mlp_get_output(self._h, y.ctypes.data_as(c_void_p)))
        return y

    def losses(self, max_n=1 << 16):
        buf = np.zeros(max_n, np.float32)
        n = c_int()
        check(self._L.pkt_mlp_losses(self._h, buf.ctypes.data_as(c_void_p), max_n, ctypes.byref(n)))
        return buf[:n.value].copy()

    def reset_losses(self):
        check(self._L.pkt_mlp_reset_losses(self._h))

    def loss_ptr(self, i):
        p = c_void_p()
        check(self._L.pkt_mlp_loss_ptr(self._h, int(i), ctypes.byref(p)))
        return p.value

    def status(self):
        code, task, detail = c_int(), c_int(), c_int()
        check(self._L.pkt_mlp_status(self._h, ctypes.byref(code), ctypes.byref(task), ctypes.byref(detail)))
        return code.value, task.value, detail.value

    def clock_stats(self, reset=False):
        """(SM cycles, nanoseconds, launches) summed over the engine's launches since
        the last reset; cycles * 1000 / ns is the mean SM clock in MHz."""
        buf = (ctypes.c_ulonglong * 3)()
        check(self._L.pkt_mlp_clock_stats(self._h, ctypes.cast(buf, c_void_p), int(reset)))
        return int(buf[0]), int(buf[1]), int(buf[2])

    TRACE_NAMES = ["cta", "dequeue", "ready", "load", "mma0", "mma1", "exec", "done"]

    def set_trace(self, enabled=True):
        """Record per-task stage timestamps of every launch (pkt_mlp_set_trace)."""
        check(self._L.pkt_mlp_set_trace(self._h, int(enabled)))

    def fetch_trace(self):
        """Records of the last launch: uint64 array [tasks, 8] (see TRACE_NAMES)."""
        n_max = self.step_info()["tasks"]
        buf = np.zeros((max(n_max, 1), _lib.TRACE_WORDS), np.uint64)
        got = c_int()
        check(self._L.pkt_mlp_fetch_trace(self._h, buf.ctypes.data_as(c_void_p), n_max, ctypes.byref(got)))
        return buf[:got.value]

    PERF_NAMES = ["tasks", "gemm_tiles", "ctrl_dep_wait", "ctrl_slot_wait", "load_stage_wait",
                  "mma_full_wait", "mma_tmem_wait", "epi_tmem_wait", "epi_gemm", "epi_simt", "total", "mma_slot_wait", "mma_issue",
                  "kblocks"]

    def set_perf(self, on=True):
        check(self._L.pkt_mlp_set_perf(self._h, int(bool(on))))

    def fetch_perf(self, max_blocks=1024):
        """Per-CTA counters of the last launch: list of dicts (cycles unless a count)."""
        buf = (ctypes.c_ulonglong * (_lib.PERF_WORDS * max_blocks))()
        got = c_int()
        check(self._L.pkt_mlp_fetch_perf(self._h, ctypes.cast(buf, c_void_p), max_blocks, ctypes.byref(got)))
        w = _lib.PERF_WORDS
        return [dict(zip(self.PERF_NAMES, buf[i * w:i * w + len(self.PERF_NAMES)])) for i in range(got.value)]

    def step_info(self):
        t, g, f = c_int(), c_int(), ctypes.c_double()
        check(self._L.pkt_mlp_step_info(self._h, ctypes.byref(t), ctypes.byref(g), ctypes.byref(f)))
        return {"tasks": t.value, "gemm_tiles": g.value, "flops": f.value}
