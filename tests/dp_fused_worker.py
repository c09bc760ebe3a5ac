"""One rank of the fused data-parallel parity check (run by test_dp_fused_gpu.py).

Each rank trains the same small MLP on its own shard twice: through grad_mode 1
(fp32 gradients, NCCL all-reduce, separate update launch) and through grad_mode
2 (partial weight tiles sent to their owner rank over peer memory, reduced and
applied inside the step launch), and a third time through grad_mode 1 in
backward segments, one NCCL all-reduce per layer on a side stream overlapped
with the following segments. With two ranks a sum of two partials does not
depend on order, so all paths must give the same bits. Results go to
<out>/rank<r>.npz.
"""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import pkt_b200  # noqa: E402

DIMS = [384, 512, 320, 128]
BATCH = 1024
STEPS = 3
LR = 0.05


def wrap_f32(ptr, count, device):
    class _CAI:
        def __init__(self):
            self.__cuda_array_interface__ = {"shape": (count,), "typestr": "<f4",
                                             "data": (ptr, False), "version": 3, "strides": None}
    return torch.as_tensor(_CAI(), device=torch.device("cuda", device))


def params(seed=7):
    rng = np.random.default_rng(seed)
    Ws = [(rng.uniform(-1, 1, (DIMS[i + 1], DIMS[i])) * np.sqrt(6.0 / DIMS[i])).astype(np.float32)
          for i in range(len(DIMS) - 1)]
    bs = [rng.standard_normal(DIMS[i + 1]).astype(np.float32) * 0.1 for i in range(len(DIMS) - 1)]
    return Ws, bs


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    out = sys.argv[1]
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    rng = np.random.default_rng(100 + rank)
    x = rng.standard_normal((BATCH, DIMS[0])).astype(np.float32)
    t = rng.standard_normal((BATCH, DIMS[-1])).astype(np.float32)
    Ws, bs = params()
    res = {}

    # ---- grad_mode 1: NCCL all-reduce of the fp32 gradient buffer
    e1 = pkt_b200.MLP(DIMS, BATCH, lr=LR, grad_mode=1, device=rank)
    e1.set_grad_scale(1.0 / world)
    e1.set_params(Ws, bs)
    e1.load_batch(e1.storage_array(x), e1.storage_array(t))
    gptr, gcount = e1.grad_buffer()
    g = wrap_f32(gptr, gcount, rank)
    for _ in range(STEPS):
        e1.forward_backward()
        dist.all_reduce(g)  # default stream, as the engine's
        e1.apply_update()
    torch.cuda.synchronize()
    res["W1"], res["b1"] = [np.concatenate([a.ravel() for a in v]) for v in e1.get_params()]
    res["loss1"] = e1.losses()
    e1.close()

    # ---- grad_mode 1 in backward segments: one all-reduce per layer, overlapped
    e3 = pkt_b200.MLP(DIMS, BATCH, lr=LR, grad_mode=1, device=rank)
    e3.set_grad_scale(1.0 / world)
    e3.set_params(Ws, bs)
    e3.load_batch(e3.storage_array(x), e3.storage_array(t))
    e3.set_reserved_sms(16)
    gptr, gcount = e3.grad_buffer()
    g3 = wrap_f32(gptr, gcount, rank)
    L = e3.backward_segments()
    main_s = torch.cuda.current_stream()
    side = torch.cuda.Stream()
    for _ in range(STEPS):
        for s in range(L):
            e3.forward_backward_segment(s)
            ev = torch.cuda.Event()
            ev.record(main_s)
            side.wait_event(ev)
            o, n = e3.grad_bucket(L - 1 - s)
            with torch.cuda.stream(side):
                dist.all_reduce(g3[o:o + n])
        main_s.wait_stream(side)
        e3.apply_update()
    torch.cuda.synchronize()
    res["status3"] = np.array(e3.status())
    res["W3"], res["b3"] = [np.concatenate([a.ravel() for a in v]) for v in e3.get_params()]
    res["loss3"] = e3.losses()
    e3.close()

    # ---- grad_mode 2: fused over peer memory
    e2 = pkt_b200.MLP(DIMS, BATCH, lr=LR, grad_mode=2, device=rank)
    e2.set_grad_scale(1.0 / world)
    e2.set_params(Ws, bs)
    e2.load_batch(e2.storage_array(x), e2.storage_array(t))
    handles = [None] * world
    dist.all_gather_object(handles, e2.dp_handle())
    e2.dp_connect(rank, world, handles)
    torch.cuda.synchronize()
    dist.barrier()
    e2.train(STEPS)
    torch.cuda.synchronize()
    res["status2"] = np.array(e2.status())
    dist.barrier()
    res["W2"], res["b2"] = [np.concatenate([a.ravel() for a in v]) for v in e2.get_params()]
    res["loss2"] = e2.losses()
    torch.cuda.synchronize()
    dist.barrier()  # no rank frees its region while another still reads it
    e2.close()
    np.savez(os.path.join(out, f"rank{rank}.npz"), **res)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
