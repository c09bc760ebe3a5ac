"""ctypes binding of the C-ABI in include/pkt_b200.h (libpkt_b200.so, built in-tree).

There is no fallback: if the shared library is missing, importing the package
raises. The CUDA work always runs in the sm_100a kernels of that library.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpkt_b200.so")

c_int, c_float, c_void_p, c_longlong = ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_longlong
c_u16, c_u32, c_u64 = ctypes.c_uint16, ctypes.c_uint32, ctypes.c_uint64

PKT_OK, PKT_ERR_ARGS, PKT_ERR_CUDA, PKT_ERR_TIMEOUT, PKT_ERR_OPCODE = 0, -1, -2, -3, -4
PKT_DTYPE_BF16, PKT_DTYPE_TF32, PKT_DTYPE_F32 = 1, 2, 3
PKT_MAJOR_K, PKT_MAJOR_MN = 0, 1
EPI_STORE, EPI_BIAS_ACT, EPI_MSE, EPI_DGRAD_RELU, EPI_WGRAD_SGD, EPI_WGRAD_STORE = range(6)
DEV_OK, DEV_TIMEOUT_DEPS, DEV_TIMEOUT_PIPE, DEV_BAD_OPCODE, DEV_BAD_ARGS = range(5)
PERF_WORDS = 16
TRACE_WORDS = 8


class PktError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"pkt_b200 error {code}: {msg}")
        self.code = code


class TaskHeader(ctypes.Structure):
    _fields_ = [("opcode", c_u16), ("arg_bytes", c_u16), ("user_tag", c_u32),
                ("buffer_read_id", c_u16), ("buffer_write_id", c_u16), ("wait_count", c_u32),
                ("read_epoch", c_u32), ("write_epoch", c_u32), ("ext_ids", c_u32),
                ("ext_wait_count", c_u32)]


class Task(ctypes.Structure):
    _fields_ = [("header", TaskHeader), ("args", ctypes.c_uint8 * 64)]


assert ctypes.sizeof(TaskHeader) == 32 and ctypes.sizeof(Task) == 96


class GemmDesc(ctypes.Structure):
    _fields_ = [("M", c_int), ("N", c_int), ("K", c_int), ("bn", c_int), ("in_dtype", c_int),
                ("a", c_void_p), ("lda", c_int), ("a_major", c_int),
                ("b", c_void_p), ("ldb", c_int), ("b_major", c_int),
                ("epilogue", c_int), ("out", c_void_p), ("ldo", c_int), ("out_dtype", c_int),
                ("relu", c_int), ("bias", c_void_p), ("aux", c_void_p), ("ldaux", c_int),
                ("scale", c_float), ("loss_partials", c_void_p), ("colsum", c_void_p),
                ("ldcol", c_int), ("w_in", c_void_p), ("w_out", c_void_p), ("w_shadow", c_void_p),
                ("ldw", c_int), ("lr", c_float), ("y_out", c_void_p), ("ldy", c_int),
                ("cta_pair", c_int)]


class MlpConfig(ctypes.Structure):
    _fields_ = [("num_layers", c_int), ("dims", ctypes.POINTER(c_int)), ("batch", c_int),
                ("dtype", c_int), ("has_bias", c_int), ("relu_last", c_int), ("lr", c_float),
                ("grad_mode", c_int), ("max_bn", c_int), ("cta_pair", c_int)]


_P = c_void_p
_SIGS = {
    "pkt_last_error": ([], ctypes.c_char_p),
    "pkt_num_sms": ([c_int], c_int),
    "pkt_runtime_create": ([c_int, ctypes.POINTER(_P)], c_int),
    "pkt_runtime_destroy": ([_P], c_int),
    "pkt_runtime_initialize": ([_P, c_int], c_int),
    "pkt_runtime_submit": ([_P, _P, c_int], c_int),
    "pkt_runtime_submit_async": ([_P, _P, c_int, _P], c_int),
    "pkt_runtime_set_segments": ([_P, _P, c_int], c_int),
    "pkt_runtime_set_segment_window_size": ([_P, c_int], c_int),
    "pkt_runtime_launch": ([_P, c_int, _P], c_int),
    "pkt_runtime_synchronize": ([_P], c_int),
    "pkt_runtime_status": ([_P, _P, _P, _P], c_int),
    "pkt_runtime_register_gemms": ([_P, _P, c_int, ctypes.POINTER(c_int)], c_int),
    "pkt_runtime_clear_gemms": ([_P], c_int),
    "pkt_gemm_tiles": ([_P, ctypes.POINTER(c_int), ctypes.POINTER(c_int)], c_int),
    "pkt_runtime_set_timeout_ns": ([_P, ctypes.c_ulonglong], c_int),
    "pkt_runtime_set_task_accounting": ([_P, c_int], c_int),
    "pkt_runtime_set_cta_pair": ([_P, c_int], c_int),
    "pkt_runtime_fetch_task_counter": ([_P, ctypes.POINTER(ctypes.c_ulonglong)], c_int),
    "pkt_runtime_set_perf": ([_P, c_int], c_int),
    "pkt_runtime_fetch_perf": ([_P, _P, c_int, ctypes.POINTER(c_int)], c_int),
    "pkt_runtime_last_launch_blocks": ([_P], c_int),
    "pkt_runtime_clock_stats": ([_P, _P, c_int], c_int),
    "pkt_runtime_prepare_launch": ([_P, c_int, _P, _P, c_int, ctypes.POINTER(c_int), ctypes.POINTER(c_int)], c_int),
    "pkt_runtime_set_trace": ([_P, c_int], c_int),
    "pkt_runtime_fetch_trace": ([_P, _P, c_int, ctypes.POINTER(c_int)], c_int),
    "pkt_axpy": ([_P, _P, c_float, c_longlong, _P], c_int),
    "pkt_axpy_noalloc": ([_P, _P, c_float, c_longlong, _P], c_int),
    "pkt_axpy_noalloc_status": ([_P, _P, _P], c_int),
    "pkt_mlp_create": ([c_int, _P, ctypes.POINTER(_P)], c_int),
    "pkt_mlp_destroy": ([_P], c_int),
    "pkt_mlp_set_params": ([_P, _P, _P], c_int),
    "pkt_mlp_get_params": ([_P, _P, _P], c_int),
    "pkt_mlp_get_grads": ([_P, _P, _P], c_int),
    "pkt_mlp_load_batch": ([_P, _P, _P, c_int, _P], c_int),
    "pkt_mlp_train": ([_P, c_int, _P], c_int),
    "pkt_mlp_losses": ([_P, _P, c_int, ctypes.POINTER(c_int)], c_int),
    "pkt_mlp_reset_losses": ([_P], c_int),
    "pkt_mlp_loss_ptr": ([_P, c_int, ctypes.POINTER(_P)], c_int),
    "pkt_mlp_get_output": ([_P, _P], c_int),
    "pkt_mlp_status": ([_P, _P, _P, _P], c_int),
    "pkt_mlp_step_info": ([_P, _P, _P, _P], c_int),
    "pkt_mlp_set_output_capture": ([_P, c_int], c_int),
    "pkt_mlp_grad_buffer": ([_P, ctypes.POINTER(_P), ctypes.POINTER(c_longlong)], c_int),
    "pkt_mlp_set_grad_scale": ([_P, c_float], c_int),
    "pkt_mlp_dp_handle": ([_P, _P], c_int),
    "pkt_mlp_dp_connect": ([_P, c_int, c_int, _P], c_int),
    "pkt_mlp_forward_backward": ([_P, _P], c_int),
    "pkt_mlp_apply_update": ([_P, _P], c_int),
    "pkt_mlp_backward_segments": ([_P, ctypes.POINTER(c_int)], c_int),
    "pkt_mlp_forward_backward_segment": ([_P, c_int, _P], c_int),
    "pkt_mlp_grad_bucket": ([_P, c_int, ctypes.POINTER(c_longlong), ctypes.POINTER(c_longlong)], c_int),
    "pkt_mlp_set_reserved_sms": ([_P, c_int], c_int),
    "pkt_mlp_set_perf": ([_P, c_int], c_int),
    "pkt_mlp_fetch_perf": ([_P, _P, c_int, ctypes.POINTER(c_int)], c_int),
    "pkt_mlp_clock_stats": ([_P, _P, c_int], c_int),
    "pkt_mlp_set_trace": ([_P, c_int], c_int),
    "pkt_mlp_fetch_trace": ([_P, _P, c_int, ctypes.POINTER(c_int)], c_int),
}

EXPORTS = sorted(_SIGS)
_lib = None


def load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run __graft_entry__.build() or "
                              "python pkt_b200/build.py (no CPU fallback exists)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def check(rc):
    if rc != PKT_OK:
        msg = load().pkt_last_error()
        raise PktError(rc, msg.decode() if msg else "")
    return rc
