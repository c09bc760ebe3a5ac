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


# ---- fused data parallel (MLP grad_mode 2): the exchange protocol on CPU ranks
#
# On the GPU every weight-gradient tile t (tiles numbered across layers) has an
# owner rank t % world. A non-owner sends its fp32 partial tile to the owner;
# the owner sums the ranks' partials in rank order, updates its shard of the
# fp32 masters with lr * 1/world and sends the new weights to every rank. Bias
# gradients go from every rank to every rank and each rank sums them in rank
# order. Here point-to-point gloo messages stand in for the peer-memory stores.
TILE = (8, 8)


def _tiles(shapes):
    out, t = [], 0
    for l, (m, n) in enumerate(shapes):
        for i in range(0, m, TILE[0]):
            for j in range(0, n, TILE[1]):
                out.append((t, l, i, j))
                t += 1
    return out


def _fused_rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    x, t, Ws, bs = _problem()
    shard = slice(rank * B // world, (rank + 1) * B // world)
    g = orc.mlp_train(DIMS, x[shard], t[shard], Ws, bs, 0.0, 1, want_grads=True)
    lr = np.float32(LR / world)
    masters = [w.copy() for w in Ws]
    new_w = [np.full_like(w, np.nan) for w in Ws]  # every entry must arrive
    for (tid, l, i, j) in _tiles([w.shape for w in Ws]):
        owner = tid % world
        part = np.ascontiguousarray(g["dW"][l][i:i + TILE[0], j:j + TILE[1]], np.float32)
        if rank != owner:
            dist.send(torch.from_numpy(part), dst=owner)
            upd = torch.empty(part.shape, dtype=torch.float32)
            dist.recv(upd, src=owner)
            new_w[l][i:i + TILE[0], j:j + TILE[1]] = upd.numpy()
        else:
            parts = {rank: part}
            for src in range(world):
                if src != rank:
                    buf = torch.empty(part.shape, dtype=torch.float32)
                    dist.recv(buf, src=src)
                    parts[src] = buf.numpy()
            acc = np.zeros_like(part)
            for src in range(world):  # rank order
                acc = acc + parts[src]
            m = masters[l][i:i + TILE[0], j:j + TILE[1]]
            m[...] = m - lr * acc
            new_w[l][i:i + TILE[0], j:j + TILE[1]] = m
            for dst in range(world):
                if dst != rank:
                    dist.send(torch.from_numpy(np.ascontiguousarray(m)), dst=dst)
    new_b = []
    for l, b in enumerate(bs):
        mine = torch.from_numpy(np.ascontiguousarray(g["db"][l], np.float32))
        allv = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allv, mine)
        acc = np.zeros_like(b)
        for src in range(world):
            acc = acc + allv[src].numpy()
        new_b.append(b - lr * acc)
    out.put((rank, [a.tolist() for a in new_w + new_b]))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_fused_exchange_equals_full_batch_step(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29900 + os.getpid() % 90 + world
    procs = [ctx.Process(target=_fused_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(1, world):  # replicated weights stay identical on every rank
        for a, b in zip(res[0], res[r]):
            assert np.array_equal(np.array(a, np.float32), np.array(b, np.float32))
    x, t, Ws, bs = _problem()
    ref = orc.mlp_train(DIMS, x, t, Ws, bs, LR, 1)
    for got, want in zip(res[0], ref["W"] + ref["b"]):
        np.testing.assert_allclose(np.array(got, np.float32), want, rtol=1e-5, atol=1e-6)
