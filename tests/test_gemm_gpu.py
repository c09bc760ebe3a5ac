"""tcgen05 GEMM tiles (pkt's reserved OpCode::Gemm) against an fp64 host product
of the same rounded operands. Covers bf16 and TF32, K-major and MN-major
operands, every tile width, ragged shapes (TMA zero fill + epilogue predication)
and each epilogue. fp32 accumulation: tolerance 2e-3 of the tensor's max."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

from tests._gpu import dev, host, ptr, rel_err, require_gpu, torch  # noqa: E402

TOL = 2e-3


@pytest.fixture(scope="module")
def pk():
    require_gpu()
    import pkt_b200
    return pkt_b200


def bf16r(a):
    from pkt_b200.mlp import from_bf16_bits, to_bf16_bits
    return from_bf16_bits(to_bf16_bits(a)).reshape(np.shape(a))


def tf32r(a):
    """fp32 -> TF32 by round-to-nearest-even (what the TMA loads feed the MMA)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0xFFF + ((u >> 13) & 1)) & 0xFFFFE000
    return u.astype(np.uint32).view(np.float32).reshape(np.shape(a))


def stored(a, dtype, ld):
    """logical [rows, cols] fp32 -> padded device tensor in storage type."""
    rows, cols = a.shape
    if dtype == "bf16":
        from pkt_b200.mlp import to_bf16_bits
        buf = np.zeros((rows, ld), np.uint16)
        buf[:, :cols] = to_bf16_bits(a).reshape(rows, cols)
        return dev(buf.view(np.int16))
    buf = np.zeros((rows, ld), np.float32)
    buf[:, :cols] = a
    return dev(buf)


def pad(n, m=64):
    return (n + m - 1) // m * m


def run_gemm(pk, desc, rt=None):
    rt = rt or pk.Runtime()
    rt.set_cta_pair(2 if desc.cta_pair == 2 else 1)
    gid = rt.register_gemms([desc])[0]
    from pkt_b200.runtime import gemm_tiles, GemmTileArgs
    tm, tn = gemm_tiles(desc)
    tasks = pk.make_tasks(tm * tn)
    k = 0
    for i in range(tm):
        for j in range(tn):
            pk.encode_args(tasks[k], pk.OpCode.Gemm, GemmTileArgs(gid, i, j, 0))
            k += 1
    rt.initialize(tm * tn)
    rt.submit_tasks(tasks)
    rt.launch(0)
    rt.synchronize()
    return rt


CASES = [
    # dtype, M, N, K, a_major, b_major, bn
    ("bf16", 256, 256, 128, 0, 0, 256),
    ("bf16", 128, 128, 64, 0, 0, 128),
    ("bf16", 384, 512, 320, 0, 1, 128),
    ("bf16", 256, 192, 256, 1, 1, 64),
    ("bf16", 200, 80, 100, 0, 0, 16),
    ("bf16", 300, 130, 77, 0, 0, 32),
    ("bf16", 1000, 777, 4099, 1, 1, 256),
    ("bf16", 4099, 1000, 3000, 0, 1, 128),
    ("tf32", 256, 256, 128, 0, 0, 256),
    ("tf32", 256, 128, 96, 0, 1, 64),
    ("tf32", 160, 96, 200, 1, 1, 32),
    ("tf32", 4099, 10, 777, 0, 0, 16),
    ("tf32", 777, 1000, 4099, 1, 1, 128),
]


PAIR_CASES = [
    ("bf16", 512, 512, 256, 0, 0, 256),
    ("bf16", 256, 256, 128, 0, 1, 128),
    ("bf16", 384, 256, 320, 1, 1, 256),
    ("bf16", 300, 130, 77, 0, 0, 32),
    ("bf16", 4099, 1000, 3000, 0, 1, 128),
    ("bf16", 1000, 777, 4099, 1, 1, 256),
    ("tf32", 256, 256, 128, 0, 0, 256),
    ("tf32", 256, 128, 96, 0, 1, 64),
    ("tf32", 160, 128, 200, 1, 1, 128),
    ("tf32", 4099, 10, 777, 0, 0, 32),
]


@pytest.mark.parametrize("case", PAIR_CASES, ids=lambda c: "pair_%s_%dx%dx%d_a%d_b%d_bn%d" % c)
def test_gemm_store_cta_pair(pk, case):
    _gemm_store(pk, case, 2)


@pytest.mark.parametrize("case", CASES, ids=lambda c: "%s_%dx%dx%d_a%d_b%d_bn%d" % c)
def test_gemm_store(pk, case):
    _gemm_store(pk, case, 1)


def _gemm_store(pk, case, pair):
    dt, M, N, K, am, bm, bn = case
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    A = rng.standard_normal((M, K)).astype(np.float32)
    Bm = rng.standard_normal((N, K)).astype(np.float32)
    rnd = bf16r if dt == "bf16" else tf32r
    ref = rnd(A).astype(np.float64) @ rnd(Bm).astype(np.float64).T
    # stored layouts: K-major = [rows][K]; MN-major = [K][rows]
    a_t = stored(A if am == 0 else A.T.copy(), dt, pad(K if am == 0 else M))
    b_t = stored(Bm if bm == 0 else Bm.T.copy(), dt, pad(K if bm == 0 else N))
    out = dev(np.zeros((M, pad(N)), np.float32))
    d = pk.GemmDesc()
    d.M, d.N, d.K, d.bn = M, N, K, bn
    d.in_dtype = 1 if dt == "bf16" else 2
    d.a, d.lda, d.a_major = a_t.data_ptr(), a_t.shape[1], am
    d.b, d.ldb, d.b_major = b_t.data_ptr(), b_t.shape[1], bm
    d.epilogue = 0
    d.out, d.ldo, d.out_dtype = out.data_ptr(), out.shape[1], 3
    d.cta_pair = pair
    run_gemm(pk, d)
    got = host(out)[:, :N]
    assert rel_err(got, ref) < TOL
    assert np.all(host(out)[:, N:] == 0)  # predication: nothing written past N


def test_gemm_bias_relu_bf16_out(pk):
    M, N, K = 256, 320, 192
    rng = np.random.default_rng(1)
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = rng.standard_normal((N, K)).astype(np.float32) * 0.1
    b = rng.standard_normal(N).astype(np.float32)
    a_t, w_t = stored(A, "bf16", pad(K)), stored(W, "bf16", pad(K))
    out = dev(np.zeros((M, pad(N)), np.int16))
    bias = dev(b)
    d = pk.GemmDesc()
    d.M, d.N, d.K, d.bn, d.in_dtype = M, N, K, 64, 1
    d.a, d.lda, d.a_major, d.b, d.ldb, d.b_major = a_t.data_ptr(), a_t.shape[1], 0, w_t.data_ptr(), w_t.shape[1], 0
    d.epilogue, d.relu, d.bias = 1, 1, bias.data_ptr()
    d.out, d.ldo, d.out_dtype = out.data_ptr(), out.shape[1], 1
    run_gemm(pk, d)
    from pkt_b200.mlp import from_bf16_bits
    got = from_bf16_bits(host(out).view(np.uint16))[:, :N] if False else \
        from_bf16_bits(host(out).view(np.uint16).ravel()).reshape(M, -1)[:, :N]
    ref = np.maximum(bf16r(A).astype(np.float64) @ bf16r(W).astype(np.float64).T + b, 0)
    assert rel_err(got, ref) < 1e-2  # bf16 output rounding


def test_gemm_wgrad_sgd_epilogue(pk):
    # dW = dY^T H (both MN-major), W_out = W_in - lr dW, bf16 shadow of W_out
    B, n_out, n_in, lr = 512, 192, 256, 0.05
    rng = np.random.default_rng(2)
    dY = rng.standard_normal((B, n_out)).astype(np.float32)
    H = rng.standard_normal((B, n_in)).astype(np.float32)
    W0 = rng.standard_normal((n_out, n_in)).astype(np.float32)
    dy_t, h_t = stored(dY, "bf16", pad(n_out)), stored(H, "bf16", pad(n_in))
    w_in = dev(np.pad(W0, ((0, 0), (0, pad(n_in) - n_in))))
    w_out = dev(np.zeros((n_out, pad(n_in)), np.float32))
    shadow = dev(np.zeros((n_out, pad(n_in)), np.int16))
    d = pk.GemmDesc()
    d.M, d.N, d.K, d.bn, d.in_dtype = n_out, n_in, B, 128, 1
    d.a, d.lda, d.a_major = dy_t.data_ptr(), dy_t.shape[1], 1
    d.b, d.ldb, d.b_major = h_t.data_ptr(), h_t.shape[1], 1
    d.epilogue = 4
    d.w_in, d.w_out, d.w_shadow, d.ldw, d.lr = w_in.data_ptr(), w_out.data_ptr(), shadow.data_ptr(), pad(n_in), lr
    run_gemm(pk, d)
    dW = bf16r(dY).astype(np.float64).T @ bf16r(H).astype(np.float64)
    ref = W0 - lr * dW
    got = host(w_out)[:, :n_in]
    assert rel_err(got - W0, ref - W0) < TOL
    from pkt_b200.mlp import from_bf16_bits, to_bf16_bits
    sh = from_bf16_bits(host(shadow).view(np.uint16).ravel()).reshape(n_out, -1)[:, :n_in]
    assert np.array_equal(sh, from_bf16_bits(to_bf16_bits(got)).reshape(sh.shape))
