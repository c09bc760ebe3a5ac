"""Pins the CPU oracle against Marco-Christiani/pkt's own outputs.

tests/golden/pkt_train_linear_cpu.txt holds what pkt's train_linear binary
(examples/train_linear.cu, built from the reference sources by oracle/Makefile)
printed for several configurations: its data generator's first values, the
initial host loss and its CPU training loop's first/final loss. The oracle's
restatement must reproduce every printed digit.
"""
import os
import re

import numpy as np
import pytest

from oracle import oracle as orc

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "pkt_train_linear_cpu.txt")


def _cases():
    cases, cur = [], None
    for line in open(GOLDEN):
        line = line.rstrip("\n")
        if line.startswith("### args:"):
            toks = line.split()[2:]
            args = {toks[i].lstrip("-"): toks[i + 1] for i in range(0, len(toks), 2)}
            cur = {"args": args}
            cases.append(cur)
        elif ":" in line or "=" in line:
            if line.startswith("x[0:5]"):
                cur["x"] = [float(v) for v in line.split("=")[1].split()]
            elif line.startswith("target[0:5]"):
                cur["t"] = [float(v) for v in line.split("=")[1].split()]
            elif line.startswith("Host expected y[0]"):
                cur["y0"] = float(line.split("=")[1])
            else:
                k, v = line.split(":")
                cur[k.strip()] = float(v)
    return cases


def _fmt6(v):
    # std::cout default formatting: 6 significant digits (%g)
    return float("%g" % v)


@pytest.mark.parametrize("case", _cases(), ids=lambda c: "m{m}_n{n}_b{batch}".format(**c["args"]))
def test_oracle_matches_pkt_cpu_loop(case):
    a = case["args"]
    m, n, batch = int(a["m"]), int(a["n"]), int(a["batch"])
    steps, lr = int(a["steps"]), float(a["lr"])
    W, x, t = orc.pkt_make_linear_data(m, n, batch)
    assert [_fmt6(v) for v in x.ravel()[:5]] == case["x"]
    assert [_fmt6(v) for v in t.ravel()[:5]] == case["t"]
    # "Host expected y[0]" is printf("%f") of a float dot product in index order
    acc = np.float32(0)
    for j in range(n):
        acc = np.float32(acc + np.float32(W[0, j] * x[0, j]))
    assert float("%f" % acc) == case["y0"]
    # initial host loss: host forward (float accumulation) + host_mse
    y0 = np.zeros((batch, m), np.float32)
    Wt, losses = orc.pkt_cpu_train_linear(W, x, t, steps, lr)
    assert _fmt6(losses[0]) == case["CPU first step loss"]
    assert _fmt6(losses[-1]) == case["CPU final loss"]


def test_oracle_mlp_fp32_single_layer_matches_pkt_loop():
    # The MLP oracle with one layer, no bias and fp32 mode is cpu_train_linear
    # with fp64 accumulation: agree to fp32 rounding.
    W, x, t = orc.pkt_make_linear_data(64, 128, 64)
    Wp, lp = orc.pkt_cpu_train_linear(W, x, t, 5, 0.01)
    r = orc.mlp_train([128, 64], x, t, [W], None, 0.01, 5, mode="fp32")
    np.testing.assert_allclose(r["losses"], lp, rtol=1e-4)
    np.testing.assert_allclose(r["W"][0], Wp, rtol=1e-5, atol=1e-6)


def test_oracle_mlp_gradients_match_finite_differences():
    rng = np.random.default_rng(3)
    dims = [6, 5, 4]
    x = rng.standard_normal((7, 6)).astype(np.float32)
    t = rng.standard_normal((7, 4)).astype(np.float32)
    Ws = [rng.uniform(-0.5, 0.5, (dims[i + 1], dims[i])).astype(np.float32) for i in range(2)]
    bs = [rng.uniform(-0.1, 0.1, dims[i + 1]).astype(np.float32) for i in range(2)]
    r = orc.mlp_train(dims, x, t, Ws, bs, 0.0, 1, want_grads=True)

    def loss(Ws_, bs_):
        h = x.astype(np.float64)
        for l in range(2):
            h = h @ Ws_[l].T.astype(np.float64) + bs_[l]
            if l == 0:
                h = np.maximum(h, 0)
        return np.mean((h - t) ** 2)

    eps = 1e-4
    for l in range(2):
        for (i, j) in [(0, 0), (1, 2), (dims[l + 1] - 1, dims[l] - 1)]:
            Wp = [w.astype(np.float64).copy() for w in Ws]
            Wm = [w.astype(np.float64).copy() for w in Ws]
            Wp[l][i, j] += eps
            Wm[l][i, j] -= eps
            fd = (loss(Wp, bs) - loss(Wm, bs)) / (2 * eps)
            assert abs(fd - r["dW"][l][i, j]) < 1e-4 * max(1, abs(fd))
        bp = [b.astype(np.float64).copy() for b in bs]
        bm = [b.astype(np.float64).copy() for b in bs]
        bp[l][1] += eps
        bm[l][1] -= eps
        fd = (loss(Ws, bp) - loss(Ws, bm)) / (2 * eps)
        assert abs(fd - r["db"][l][1]) < 1e-4 * max(1, abs(fd))


def test_oracle_axpy_is_fma():
    rng = np.random.default_rng(42)
    x = rng.uniform(-1, 1, 1000).astype(np.float32)
    y = rng.uniform(-1, 1, 1000).astype(np.float32)
    out = orc.axpy(x, y, 2.5)
    ref = (np.float64(2.5) * x.astype(np.float64) + y.astype(np.float64)).astype(np.float32)
    assert np.array_equal(out, ref)  # fma == exact product+sum rounded once


def test_bf16_round_is_rne():
    assert orc.lib().orc_bf16_round(1.0 + 2.0 ** -8) == 1.0  # tie -> even
    assert orc.lib().orc_bf16_round(1.0 + 3 * 2.0 ** -8) == 1.0 + 2.0 ** -6


@pytest.mark.parametrize("mode", ["fp32", "tf32", "bf16"])
def test_numpy_restatement_matches_c_oracle(mode):
    """oracle/mlp_np.py (fp64 numpy GEMMs, used for the full-size configs) against
    oracle.cpp's loops: gradients, losses and updated weights of two steps agree
    to fp32 rounding of differently ordered fp64 sums (and the rare bf16 rounding
    flip such a difference can cause)."""
    from oracle import mlp_np
    rng = np.random.default_rng(3)
    dims, batch, lr = [48, 96, 40, 8], 70, 0.05
    x = rng.standard_normal((batch, dims[0])).astype(np.float32)
    t = rng.standard_normal((batch, dims[-1])).astype(np.float32)
    Ws = [rng.uniform(-0.4, 0.4, (dims[i + 1], dims[i])).astype(np.float32) for i in range(3)]
    bs = [rng.uniform(-0.1, 0.1, dims[i + 1]).astype(np.float32) for i in range(3)]
    a = orc.mlp_train(dims, x, t, Ws, bs, lr, 2, mode=mode, want_grads=True)
    b = mlp_np.mlp_train(dims, x, t, Ws, bs, lr, 2, mode=mode, want_grads=True)
    tol = 1e-5 if mode != "bf16" else 2e-3
    np.testing.assert_allclose(b["losses"], a["losses"], rtol=1e-5)
    for l in range(3):
        den = np.max(np.abs(a["dW"][l]))
        assert np.max(np.abs(b["dW"][l] - a["dW"][l])) / den < tol, ("dW", l)
        assert np.max(np.abs(b["db"][l] - a["db"][l])) / np.max(np.abs(a["db"][l])) < tol, ("db", l)
        assert np.max(np.abs(b["W"][l] - a["W"][l])) < 1e-6, ("W", l)


def test_numpy_rounding_helpers_match_c():
    from oracle import mlp_np
    rng = np.random.default_rng(4)
    v = (rng.standard_normal(4096) * 10.0 ** rng.integers(-8, 8, 4096)).astype(np.float32)
    got = mlp_np.bf16_round(v)
    want = np.array([orc.lib().orc_bf16_round(float(f)) for f in v], np.float32)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
