"""Data-parallel step logic on CPU ranks (gloo, world_size 2, 127.0.0.1).

The GPU data-parallel path (bench.py --gpus N) runs, per rank, the engine's
forward/backward on its batch shard with per-rank mean-squared-error scaling
2/(B_rank * n), all-reduces the fp32 gradients with a SUM, and applies SGD
with lr * 1/world_size (pkt_mlp_set_grad_scale). Here the same arithmetic runs
with the CPU oracle's gradients on two gloo ranks and must equal one
full-batch step of the oracle."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as orc

DIMS, B, LR = [16, 32, 8], 64, 0.05


def _problem():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((B, DIMS[0])).astype(np.float32)
    t = rng.standard_normal((B, DIMS[-1])).astype(np.float32)
    Ws = [rng.uniform(-0.5, 0.5, (DIMS[i + 1], DIMS[i])).astype(np.float32) for i in range(2)]
    bs = [rng.uniform(-0.1, 0.1, DIMS[i + 1]).astype(np.float32) for i in range(2)]
    return x, t, Ws, bs


def _rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    x, t, Ws, bs = _problem()
    shard = slice(rank * B // world, (rank + 1) * B // world)
    g = orc.mlp_train(DIMS, x[shard], t[shard], Ws, bs, 0.0, 1, want_grads=True)
    flat = torch.from_numpy(np.concatenate([a.ravel() for a in g["dW"] + g["db"]]))
    dist.all_reduce(flat)  # SUM, as the NCCL all-reduce of the engine's gradient buffer
    loss = torch.tensor([float(g["losses"][0])])
    dist.all_reduce(loss)
    scale = 1.0 / world
    new, o = [], 0
    for p in Ws + bs:
        k = p.size
        new.append(p - LR * scale * flat[o:o + k].numpy().reshape(p.shape))
        o += k
    if rank == 0:
        out.put(([a.tolist() for a in new], float(loss.item()) / world))
    dist.destroy_process_group()


def test_two_rank_step_equals_full_batch_step():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 300
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    new, loss = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x, t, Ws, bs = _problem()
    ref = orc.mlp_train(DIMS, x, t, Ws, bs, LR, 1)
    for got, want in zip(new, ref["W"] + ref["b"]):
        np.testing.assert_allclose(np.array(got, np.float32), want, rtol=1e-5, atol=1e-6)
    assert abs(loss - ref["losses"][0]) < 1e-6 * max(1.0, abs(ref["losses"][0]))
