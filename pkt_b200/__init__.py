"""pkt_b200: B200-native (sm_100a) persistent training megakernel with pkt's host API.

Everything here calls libpkt_b200.so through its C-ABI (include/pkt_b200.h).
"""
from ._lib import PktError, load as _load  # noqa: F401
from .runtime import (AxpyArgs, GemmDesc, LinearBackwardArgs, LinearForwardArgs, MSELossArgs,  # noqa: F401
                      OpCode, Runtime, SGDUpdateArgs, Task, ZeroMemoryArgs, axpy, decode_args,
                      encode_args, make_tasks)
from .mlp import MLP, from_bf16_bits, to_bf16_bits  # noqa: F401

_load()
