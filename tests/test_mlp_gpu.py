"""MLP engine (forward / MSE / dgrad / wgrad / SGD megakernel step) against the
CPU oracle on identical seeded inputs.

Tolerances (per tensor, max|a-b| / max|b|): bf16 paths 2e-2, TF32 paths 1e-3 on
gradients after one step; loss curves within 1% relative.
"""
import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

from tests._gpu import rel_err, require_gpu  # noqa: E402

TOL = {"bf16": 2e-2, "tf32": 1e-3}


@pytest.fixture(scope="module")
def pk():
    require_gpu()
    import pkt_b200
    return pkt_b200


def problem(dims, batch, seed, onehot=False):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((batch, dims[0])).astype(np.float32)
    if onehot:
        t = np.zeros((batch, dims[-1]), np.float32)
        t[np.arange(batch), rng.integers(0, dims[-1], batch)] = 1.0
    else:
        t = rng.standard_normal((batch, dims[-1])).astype(np.float32)
    Ws = [rng.uniform(-1, 1, (dims[i + 1], dims[i])).astype(np.float32) * np.sqrt(6.0 / dims[i])
          for i in range(len(dims) - 1)]
    bs = [rng.uniform(-0.1, 0.1, dims[i + 1]).astype(np.float32) for i in range(len(dims) - 1)]
    return x, t, Ws, bs


def make(pk, dims, batch, dtype, lr, grad_mode, x, t, Ws, bs, bias=True, cta_pair=2):
    m = pk.MLP(dims, batch, dtype=dtype, lr=lr, bias=bias, grad_mode=grad_mode, cta_pair=cta_pair)
    m.set_params(Ws, bs if bias else None)
    m.load_batch(m.storage_array(x), m.storage_array(t))
    return m


CONFIGS = [
    ("bf16", [256, 512, 384, 128], 256),
    ("bf16", [512, 512, 512], 1024),
    ("bf16", [128, 64], 256),
    ("tf32", [100, 300, 77, 10], 409),
    ("tf32", [128, 64], 256),
]


@pytest.mark.parametrize("cfg", CONFIGS, ids=lambda c: c[0] + "_" + "x".join(map(str, c[1])) + "_b%d" % c[2])
def test_one_step_gradients(pk, cfg):
    dtype, dims, batch = cfg
    x, t, Ws, bs = problem(dims, batch, 11)
    ref = orc.mlp_train(dims, x, t, Ws, bs, 0.0, 1, mode=dtype, want_grads=True)
    m = make(pk, dims, batch, dtype, 0.0, 1, x, t, Ws, bs)
    m.train(1)
    loss = m.losses()
    dW, db = m.get_grads()
    assert abs(loss[0] - ref["losses"][0]) / ref["losses"][0] < 1e-3
    for l in range(len(dims) - 1):
        assert rel_err(dW[l], ref["dW"][l]) < TOL[dtype], ("dW", l)
        assert rel_err(db[l], ref["db"][l]) < TOL[dtype], ("db", l)


@pytest.mark.parametrize("cfg", CONFIGS, ids=lambda c: c[0] + "_" + "x".join(map(str, c[1])) + "_b%d" % c[2])
def test_fused_sgd_step_matches_oracle(pk, cfg):
    dtype, dims, batch = cfg
    lr = 0.05
    x, t, Ws, bs = problem(dims, batch, 12)
    ref = orc.mlp_train(dims, x, t, Ws, bs, lr, 1, mode=dtype)
    m = make(pk, dims, batch, dtype, lr, 0, x, t, Ws, bs)
    m.train(1)
    W1, b1 = m.get_params()
    for l in range(len(dims) - 1):
        # compare the update itself (W1 - W0), the part the step computed
        assert rel_err(W1[l] - Ws[l], ref["W"][l] - Ws[l]) < TOL[dtype], ("W", l)
        assert rel_err(b1[l] - bs[l], ref["b"][l] - bs[l]) < TOL[dtype], ("b", l)


@pytest.mark.parametrize("dtype,grad_mode,pair", [("bf16", 0, 2), ("tf32", 0, 2), ("bf16", 1, 2),
                                                   ("bf16", 0, 1), ("tf32", 1, 1)])
def test_loss_curve_within_one_percent(pk, dtype, grad_mode, pair):
    dims, batch, steps, lr = [64, 256, 256, 32], 512, 30, 0.05
    x, t, Ws, bs = problem(dims, batch, 5)
    ref = orc.mlp_train(dims, x, t, Ws, bs, lr, steps, mode=dtype)
    m = make(pk, dims, batch, dtype, lr, grad_mode, x, t, Ws, bs, cta_pair=pair)
    m.train(steps)
    got = m.losses()
    assert len(got) == steps
    assert np.max(np.abs(got - ref["losses"]) / ref["losses"]) < 0.01
    assert got[-1] < got[0]


def test_no_bias_single_linear_matches_pkt_loop(pk):
    """pkt's own train_linear problem (no bias, m=64, n=128, batch 64) through the
    TF32 engine: loss curve within 1% of the bit-exact restatement of pkt's CPU loop."""
    m_, n_, batch, steps, lr = 64, 128, 64, 50, 0.01
    W, x, t = orc.pkt_make_linear_data(m_, n_, batch)
    _, lref = orc.pkt_cpu_train_linear(W, x, t, steps, lr)
    m = pk.MLP([n_, m_], batch, dtype="tf32", lr=lr, bias=False)
    m.set_params([W])
    m.load_batch(m.storage_array(x), m.storage_array(t))
    m.train(steps)
    got = m.losses()
    assert np.max(np.abs(got - lref) / lref) < 0.01


def test_output_capture_matches_forward(pk):
    dims, batch = [96, 160, 48], 300
    x, t, Ws, bs = problem(dims, batch, 3)
    ref = orc.mlp_train(dims, x, t, Ws, bs, 0.0, 1, mode="tf32", want_acts=True)
    m = make(pk, dims, batch, "tf32", 0.0, 0, x, t, Ws, bs)
    m.set_output_capture(True)
    m.train(1)
    assert rel_err(m.get_output(), ref["acts"][-1]) < 1e-3
