"""The timed CPU baseline (oracle/cpu_mlp.cpp, fp32 OpenMP) computes the same
training step as the oracle, and the product's seeded train_linear data generator
(pkt_b200/data.py) reproduces the oracle's <random>-based one bit for bit."""
import numpy as np

from oracle import cpu_baseline as cb
from oracle import mlp_np
from oracle import oracle as orc


def test_cpu_mlp_step_matches_oracle_fp32():
    rng = np.random.default_rng(7)
    dims, batch, lr = [100, 300, 77, 10], 409, 0.01
    x = rng.standard_normal((batch, dims[0])).astype(np.float32)
    t = rng.standard_normal((batch, dims[-1])).astype(np.float32)
    Ws = [rng.uniform(-0.2, 0.2, (dims[i + 1], dims[i])).astype(np.float32) for i in range(3)]
    bs = [rng.uniform(-0.1, 0.1, dims[i + 1]).astype(np.float32) for i in range(3)]
    m = cb.MLPStep(dims, batch, Ws, bs)
    got = [m.step(x, t, lr) for _ in range(3)]
    ref = mlp_np.mlp_train(dims, x, t, Ws, bs, lr, 3, mode="fp32")
    np.testing.assert_allclose(got, ref["losses"], rtol=1e-5)
    W = np.concatenate([w.ravel() for w in ref["W"]])
    assert np.max(np.abs(m.W - W)) < 1e-6
    b = np.concatenate(ref["b"])
    assert np.max(np.abs(m.b - b)) < 1e-6


def test_cpu_baseline_times_full_batches():
    rng = np.random.default_rng(8)
    dims = [64, 128, 32]
    x = rng.standard_normal((512, 64)).astype(np.float32)
    t = rng.standard_normal((512, 32)).astype(np.float32)
    Ws = [rng.uniform(-0.2, 0.2, (dims[i + 1], dims[i])).astype(np.float32) for i in range(2)]
    r = cb.time_mlp(dims, x, t, Ws, None, 0.01, max_steps=3, budget_s=10.0)
    assert r["steps"] == 3 and r["samples_per_s"] > 0 and r["threads"] >= 1
    assert r["losses"][-1] < r["losses"][0]


def test_linear_task_generator_matches_oracle():
    from pkt_b200.data import make_linear_task
    got = make_linear_task(128, 64, 256, seed=0, noise=0.01)
    want = orc.make_linear_task(128, 64, 256, seed=0, noise=0.01)
    for g, w in zip(got, want):
        assert np.array_equal(g, w)
