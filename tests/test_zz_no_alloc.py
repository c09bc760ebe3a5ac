"""pkt_axpy_noalloc: the axpy entry point for callers that cannot allocate device
memory (for example code running under a caching allocator that owns the memory
budget, or code that must not synchronise the device the way cudaMalloc/cudaFree
can). It keeps its scratch in a fixed array inside the library. Here its output
must equal pkt_axpy's bit for bit (both compute one fused multiply-add per
element), on two calls in a row, so leftovers of a previous call cannot leak in.
This file is collected last on purpose."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from tests._gpu import dev, host, require_gpu  # noqa: E402


@pytest.fixture(scope="module")
def pk():
    require_gpu()
    import pkt_b200
    return pkt_b200


@pytest.mark.parametrize("n", [1000, (1 << 22) + 5])
def test_noalloc_matches_allocating_entry_point_twice(pk, n):
    from pkt_b200.runtime import axpy, axpy_noalloc, axpy_noalloc_status
    rng = np.random.default_rng(n)
    hx = rng.uniform(-1, 1, n).astype(np.float32)
    hy = rng.uniform(-1, 1, n).astype(np.float32)
    x = dev(hx)
    y_ref, y_new = dev(hy), dev(hy)
    for a in (2.5, -0.75):  # two calls in a row on the same buffers
        axpy(x.data_ptr(), y_ref.data_ptr(), a, n)
        axpy_noalloc(x.data_ptr(), y_new.data_ptr(), a, n)
        assert axpy_noalloc_status() == (0, 0, 0)  # the launch's device status words
        assert np.array_equal(host(y_new), host(y_ref))


def test_noalloc_rejects_sizes_beyond_its_scratch(pk):
    from pkt_b200.runtime import axpy_noalloc
    with pytest.raises(pk.PktError, match="fixed scratch limit"):
        axpy_noalloc(16, 16, 1.0, 2048 * 32768 + 1)
