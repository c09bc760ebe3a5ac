"""The C-ABI boundary without a GPU: libpkt_b200.so loads, exports every
function include/pkt_b200.h declares, and the Python binding table (_lib._SIGS)
covers exactly that set. No compute call is made."""
import ctypes
import os
import re

import pkt_b200._lib as L

HERE = os.path.dirname(os.path.abspath(__file__))
HEADER = os.path.join(HERE, "..", "include", "pkt_b200.h")


def declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int|const\s+char\s*\*)\s+(pkt_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_entry_points():
    names = declared()
    for must in ("pkt_runtime_create", "pkt_runtime_launch", "pkt_axpy", "pkt_axpy_noalloc",
                 "pkt_mlp_create", "pkt_mlp_train", "pkt_mlp_dp_handle", "pkt_mlp_dp_connect"):
        assert must in names


def test_library_exports_every_declared_function():
    lib = ctypes.CDLL(L.LIB_PATH)
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_bindings_mirror_the_header():
    assert set(L.EXPORTS) == set(declared())
