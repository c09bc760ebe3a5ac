"""Per-role cycle counters of one MLP training step (pkt's profiling ranges).

    python -m pkt_b200.perf_report --dims 1024,4096,4096,4096,1024 --batch 8192
    python -m torch.distributed.run --nproc-per-node 8 -m pkt_b200.perf_report --grad-mode 2
    python -m pkt_b200.perf_report --axpy 268435456
    python -m pkt_b200.perf_report --sgd 268435456

Times `--steps` steps with CUDA events, then runs one more step with the
per-CTA counters on and prints, for the leader CTA of every CTA pair, the mean
and maximum over CTAs of each counter (cycles unless a count): the controller's
dependency and slot waits, the loader's stage waits, the MMA issuer's waits for
full stages / free accumulators / tasks and its issue time, and the epilogue
warps' accumulator waits and work. Under torch.distributed.run (WORLD_SIZE > 1)
the engine runs data parallel: grad_mode 2 (default there) reduces the weight
gradients inside the step over peer memory, grad_mode 1 with an NCCL all-reduce
between the backward and the update launch; every rank prints its step time and
rank 0 its counters.

--axpy N instead times pkt_axpy (y = a*x + y over N floats already on the device,
12 bytes per element: read x, read y, write y) and prints its HBM bandwidth;
--sgd N the SGDMixed update pass over N parameters (14 bytes per parameter).
"""
import argparse
import os
import sys

import numpy as np


def _wrap_f32(ptr, count, device):
    import torch

    class _CAI:
        def __init__(self):
            self.__cuda_array_interface__ = {"shape": (count,), "typestr": "<f4",
                                             "data": (ptr, False), "version": 3, "strides": None}
    return torch.as_tensor(_CAI(), device=torch.device("cuda", device))


def axpy_report(args):
    import torch
    import pkt_b200

    n = args.axpy
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    x = torch.rand(n, device="cuda")
    y = torch.rand(n, device="cuda")
    for _ in range(args.warmup):
        pkt_b200.axpy(x.data_ptr(), y.data_ptr(), 0.5, n)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    ev[0].record()
    for i in range(args.steps):
        pkt_b200.axpy(x.data_ptr(), y.data_ptr(), 0.5, n)
        ev[i + 1].record()
    torch.cuda.synchronize()
    per = sorted(ev[i].elapsed_time(ev[i + 1]) for i in range(args.steps))
    ms = per[len(per) // 2]
    print(f"axpy n={n}: {ms:.3f} ms per call (median of {args.steps}), "
          f"{12.0 * n / ms / 1e6:.0f} GB/s (12 B per element)")


def sgd_report(args):
    """SGDMixed tasks (fp32 master w -= lr * g in place, bf16 copy of the new w
    written alongside: 14 bytes per parameter -- read w, read g, write w, write
    the copy) over N parameters already on the device, in chunks of 2^16 per task
    (as the MLP engine's grad_mode 1 update list; many tasks per SM, so the last
    wave is short), one persistent launch per pass."""
    import torch
    import pkt_b200
    from pkt_b200 import runtime as R

    n = args.sgd
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    w = torch.rand(n, device="cuda")
    g = torch.rand(n, device="cuda") * 1e-3
    wb = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    chunk = 1 << 16
    ntask = (n + chunk - 1) // chunk
    tasks = R.make_tasks(ntask)
    for i in range(ntask):
        k = min(chunk, n - i * chunk)
        a = R.SGDMixedArgs(w.data_ptr() + 4 * i * chunk, g.data_ptr() + 4 * i * chunk, w.data_ptr() + 4 * i * chunk,
                           wb.data_ptr() + 2 * i * chunk, k, 1e-3, 0)
        R.encode_args(tasks[i], R.OpCode.SGDMixed, a)
    rt = pkt_b200.Runtime()
    rt.initialize(ntask)
    per = []
    for it in range(args.warmup + args.steps):
        rt.submit_tasks(tasks)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        rt.launch(0)
        e1.record()
        rt.synchronize()
        if it >= args.warmup:
            per.append(e0.elapsed_time(e1))
    per.sort()
    ms = per[len(per) // 2]
    print(f"sgd_mixed n={n}: {ms:.3f} ms per pass (median of {args.steps}), "
          f"{14.0 * n / ms / 1e6:.0f} GB/s (14 B per parameter)")


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--dims", default="1024,4096,4096,4096,1024")
    ap.add_argument("--batch", type=int, default=8192)
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "tf32"])
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--grad-mode", type=int, default=None, choices=[0, 1, 2],
                    help="0: SGD fused into the gradient epilogue (one GPU); 1: NCCL all-reduce; "
                         "2: fused peer-memory reduce (default with WORLD_SIZE > 1)")
    ap.add_argument("--axpy", type=int, default=0, metavar="N",
                    help="time pkt_axpy over N floats instead of an MLP step")
    ap.add_argument("--sgd", type=int, default=0, metavar="N",
                    help="time the SGDMixed update pass over N parameters instead of an MLP step")
    args = ap.parse_args(argv)
    if args.axpy:
        return axpy_report(args)
    if args.sgd:
        return sgd_report(args)

    import torch
    import pkt_b200

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    gm = args.grad_mode if args.grad_mode is not None else (2 if world > 1 else 0)
    if world > 1 and gm == 0:
        sys.exit("grad_mode 0 has no gradient exchange: use 1 or 2 with several ranks")
    dims = [int(v) for v in args.dims.split(",")]
    B = args.batch
    eng = pkt_b200.MLP(dims, B, dtype=args.dtype, lr=1e-3, bias=True, grad_mode=gm, device=local)
    if world > 1:
        eng.set_grad_scale(1.0 / world)
    rng = np.random.default_rng(0)
    Ws = [(rng.uniform(-1, 1, (dims[i + 1], dims[i])) * np.sqrt(6.0 / dims[i])).astype(np.float32)
          for i in range(len(dims) - 1)]
    eng.set_params(Ws)
    rng = np.random.default_rng(1 + rank)
    x = rng.standard_normal((B, dims[0])).astype(np.float32)
    t = rng.standard_normal((B, dims[-1])).astype(np.float32)
    eng.load_batch(eng.storage_array(x), eng.storage_array(t))
    grad = None
    if gm == 2:
        handles = [eng.dp_handle()]
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, eng.dp_handle())
        eng.dp_connect(rank, world, handles if world > 1 else None)
    elif gm == 1:
        p, n = eng.grad_buffer()
        grad = _wrap_f32(p, n, local)

    def step():
        if gm == 1:
            eng.forward_backward()
            if dist is not None:
                dist.all_reduce(grad)
            eng.apply_update()
        else:
            eng.train(1)

    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / max(1, args.steps)
    flops = eng.step_info()["flops"]
    print(f"rank {rank}: {ms:.3f} ms/step, {flops / ms / 1e9:.0f} TFLOP/s", flush=True)
    if dist is not None:
        dist.barrier()
    eng.set_perf(True)
    step()
    torch.cuda.synchronize()
    blocks = eng.fetch_perf()
    if rank == 0:
        lead = blocks[0::2] if len(blocks) > 1 else blocks
        print(f"per-CTA counters of one step ({len(lead)} leader CTAs; cycles unless a count):")
        for k in eng.PERF_NAMES:
            vals = [b[k] for b in lead]
            print(f"  {k:18s} mean {np.mean(vals):12.0f}   max {np.max(vals):12.0f}")
    if dist is not None:
        dist.barrier()  # no rank frees its exchange region while another still reads it
    eng.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
