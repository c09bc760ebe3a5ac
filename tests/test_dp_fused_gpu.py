"""Fused data parallel (MLP grad_mode 2): weight-gradient tiles cross to their
owner rank over peer memory inside the step launch; the owner reduces, applies
SGD and writes the new bf16 weights into every rank.

* world 1 on one GPU: the same arithmetic as the SGD fused into the gradient
  epilogue (grad_mode 0), so weights, biases and losses are bit-identical.
* world 2 on two GPUs (skipped with one): bit-identical to grad_mode 1, where
  NCCL sums the fp32 gradient buffers (a sum of two partials has one result
  whatever the order), and identical on both ranks; so is grad_mode 1 run in
  backward segments with one NCCL all-reduce per layer on a side stream.
* backward segments on one GPU: the step in L launches gives the same gradient
  buffer, weights and losses as the step in one launch.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

from _gpu import require_gpu, torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _train(pk, grad_mode, dims, batch, steps, lr=0.05, seed=3):
    rng = np.random.default_rng(seed)
    Ws = [(rng.uniform(-1, 1, (dims[i + 1], dims[i])) * np.sqrt(6.0 / dims[i])).astype(np.float32)
          for i in range(len(dims) - 1)]
    bs = [rng.standard_normal(dims[i + 1]).astype(np.float32) * 0.1 for i in range(len(dims) - 1)]
    x = rng.standard_normal((batch, dims[0])).astype(np.float32)
    t = rng.standard_normal((batch, dims[-1])).astype(np.float32)
    e = pk.MLP(dims, batch, lr=lr, grad_mode=grad_mode)
    e.set_params(Ws, bs)
    e.load_batch(e.storage_array(x), e.storage_array(t))
    if grad_mode == 2:
        e.dp_connect(0, 1)
    e.train(steps)
    torch.cuda.synchronize()
    assert e.status()[0] == 0
    W, b = e.get_params()
    out = (np.concatenate([w.ravel() for w in W]), np.concatenate([v.ravel() for v in b]), e.losses())
    e.close()
    return out


@pytest.mark.parametrize("dims,batch", [([384, 512, 320, 128], 1024), ([256, 1024, 256], 700)])
def test_fused_dp_world1_matches_fused_sgd(dims, batch):
    require_gpu()
    import pkt_b200 as pk
    W0, b0, l0 = _train(pk, 0, dims, batch, 4)
    W2, b2, l2 = _train(pk, 2, dims, batch, 4)
    assert np.array_equal(l0, l2)
    assert np.array_equal(b0, b2)
    assert np.array_equal(W0, W2)


@pytest.mark.parametrize("dims,batch,dtype", [([384, 512, 320, 128], 1024, "bf16"),
                                              ([1000, 3000, 777, 10], 600, "tf32"),
                                              ([512] * 7, 2048, "bf16")])
def test_backward_segments_match_one_launch(dims, batch, dtype):
    require_gpu()
    import pkt_b200 as pk
    rng = np.random.default_rng(11)
    Ws = [(rng.uniform(-1, 1, (dims[i + 1], dims[i])) * np.sqrt(6.0 / dims[i])).astype(np.float32)
          for i in range(len(dims) - 1)]
    bs = [rng.standard_normal(dims[i + 1]).astype(np.float32) * 0.1 for i in range(len(dims) - 1)]
    x = rng.standard_normal((batch, dims[0])).astype(np.float32)
    t = rng.standard_normal((batch, dims[-1])).astype(np.float32)
    out = []
    for segmented in (False, True):
        e = pk.MLP(dims, batch, lr=0.01, grad_mode=1, dtype=dtype)
        e.set_params(Ws, bs)
        e.load_batch(e.storage_array(x), e.storage_array(t))
        if segmented:
            e.set_reserved_sms(16)
        L = len(dims) - 1
        grads = []
        for _ in range(2):
            if segmented:
                assert e.backward_segments() == L
                for s in range(L):
                    e.forward_backward_segment(s)
            else:
                e.forward_backward()
            torch.cuda.synchronize()
            dW, db = e.get_grads()
            grads.append(np.concatenate([g.ravel() for g in dW] + [g.ravel() for g in db]))
            e.apply_update()
        torch.cuda.synchronize()
        assert e.status()[0] == 0
        W, b = e.get_params()
        out.append((grads, np.concatenate([w.ravel() for w in W]), np.concatenate([v.ravel() for v in b]),
                    e.losses()))
        e.close()
    (g0, W0, b0, l0), (g1, W1, b1, l1) = out
    for a, c in zip(g0, g1):
        assert np.array_equal(a, c)
    assert np.array_equal(W0, W1)
    assert np.array_equal(b0, b1)
    assert np.array_equal(l0, l1)


def test_grad_buckets_tile_the_buffer():
    require_gpu()
    import pkt_b200 as pk
    dims = [384, 512, 320, 128]
    e = pk.MLP(dims, 512, grad_mode=1)
    _, total = e.grad_buffer()
    o = 0
    for l in range(3):
        off, n = e.grad_bucket(l)
        assert off == o and n >= dims[l] * dims[l + 1] + dims[l + 1]
        o += n
    assert o == total
    with pytest.raises(RuntimeError):
        e.forward_backward_segment(3)
    e.close()


def test_fused_dp_needs_connect():
    require_gpu()
    import pkt_b200 as pk
    e = pk.MLP([256, 256, 128], 512, grad_mode=2)
    with pytest.raises(RuntimeError):
        e.train(1)
    e.close()


def test_fused_dp_two_gpus_matches_nccl(tmp_path):
    require_gpu()
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT="29531", WORLD_SIZE="2",
               NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "dp_fused_worker.py"), str(tmp_path)],
                              env=dict(env, RANK=str(r), LOCAL_RANK=str(r))) for r in range(2)]
    rcs = [p.wait(timeout=300) for p in procs]
    assert rcs == [0, 0]
    r = [np.load(tmp_path / f"rank{k}.npz") for k in range(2)]
    for k in range(2):
        assert r[k]["status2"][0] == 0
        assert np.array_equal(r[k]["W2"], r[k]["W1"])
        assert np.array_equal(r[k]["b2"], r[k]["b1"])
        assert np.array_equal(r[k]["loss2"], r[k]["loss1"])
        assert r[k]["status3"][0] == 0
        assert np.array_equal(r[k]["W3"], r[k]["W1"])
        assert np.array_equal(r[k]["b3"], r[k]["b1"])
        assert np.array_equal(r[k]["loss3"], r[k]["loss1"])
    assert np.array_equal(r[0]["W2"], r[1]["W2"])
    assert np.array_equal(r[0]["b2"], r[1]["b2"])
