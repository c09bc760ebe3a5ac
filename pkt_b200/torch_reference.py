"""PyTorch comparison of the MLP training step (the multi-layer form of pkt's
scripts/benchmark_linear.py:37-92, which times the same Linear step in PyTorch
beside the megakernel and compares their losses).

The same step as the engine, written with torch on the GPU: cuBLAS GEMMs with
the engine's rounding points (bf16 storage of x, targets, activations, output
gradients and the weight copy, fp32 accumulation through ``torch.mm(...,
out_dtype=torch.float32)``; TF32 mode: operands rounded to TF32 (nearest even),
then fp32 GEMMs on the tensor cores), fp32 bias add / ReLU / MSE / SGD on fp32
master weights. It is an independent third-party implementation of the same
arithmetic: tests use its distance from the fp64 oracle as the accuracy an
fp32-accumulating tensor-core GEMM reaches on a given problem, and

    python -m pkt_b200.torch_reference [--dims ...] [--batch ...] [--steps N]

times it against the engine on the benchmark configuration and prints both
step times and their numeric agreement.
"""
import argparse
import time

import numpy as np


def _bf16(t):
    import torch
    return t.to(torch.bfloat16).to(torch.float32)


def _tf32(t):
    """fp32 -> TF32 (10 explicit mantissa bits), round to nearest even."""
    import torch
    u = t.contiguous().view(torch.int32)
    special = (u & 0x7F800000) == 0x7F800000
    r = (u + 0xFFF + ((u >> 13) & 1)) & ~0x1FFF
    return torch.where(special, u, r).view(torch.float32)


def _mm(a, b, mode):
    """fp32 result of the GEMM a @ b on operands already carrying their rounding."""
    import torch
    if mode == "bf16":
        return torch.mm(a.to(torch.bfloat16), b.to(torch.bfloat16), out_dtype=torch.float32)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = mode == "tf32"
    try:
        return torch.mm(a, b)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def mlp_train(dims, x, t, Ws, bs, lr, steps, mode="bf16", want_grads=False, device="cuda"):
    """Same contract as the oracle's mlp_train; returns numpy arrays."""
    import torch
    dev = torch.device(device)
    store = _bf16 if mode == "bf16" else (lambda v: v)
    operand = _bf16 if mode == "bf16" else (_tf32 if mode == "tf32" else (lambda v: v))
    L = len(dims) - 1
    B = x.shape[0]
    W = [torch.tensor(np.asarray(w, np.float32), device=dev) for w in Ws]
    b = None if bs is None else [torch.tensor(np.asarray(v, np.float32), device=dev) for v in bs]
    H0 = store(torch.tensor(np.asarray(x, np.float32), device=dev))
    tq = store(torch.tensor(np.asarray(t, np.float32), device=dev))
    scale = torch.tensor(2.0 / (float(B) * float(dims[L])), dtype=torch.float32, device=dev)
    losses, dW, db = [], None, None
    for _ in range(steps):
        Wop = [operand(w) for w in W]
        H = [H0]
        for l in range(L):
            p = _mm(operand(H[l]), Wop[l].t().contiguous(), mode)
            if b is not None:
                p = p + b[l][None, :]
            if l < L - 1:
                p = torch.clamp_min(p, 0.0)
            H.append(p if l == L - 1 else store(p))
        diff = H[L] - tq
        losses.append(float((diff.double() ** 2).sum() / (B * dims[L])))
        dY = store(scale * diff)
        dW, db = [None] * L, [None] * L
        for l in range(L - 1, -1, -1):
            dYop = operand(dY)
            dW[l] = _mm(dYop.t().contiguous(), operand(H[l]), mode)
            if b is not None:
                db[l] = dY.double().sum(0).float()
            if l > 0:
                v = _mm(dYop, Wop[l], mode)
                dY = store(torch.where(H[l] > 0, v, torch.zeros_like(v)))
        for l in range(L):
            W[l] = W[l] - lr * dW[l]
            if b is not None:
                b[l] = b[l] - lr * db[l]
    out = {"losses": np.asarray(losses, np.float32), "W": [w.cpu().numpy() for w in W],
           "b": None if b is None else [v.cpu().numpy() for v in b]}
    if want_grads:
        out["dW"] = [g.cpu().numpy() for g in dW]
        out["db"] = None if b is None else [g.cpu().numpy() for g in db]
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--dims", default="1024,4096,4096,4096,1024")
    ap.add_argument("--batch", type=int, default=8192)
    ap.add_argument("--dtype", default="bf16")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--lr", type=float, default=1e-3)
    args = ap.parse_args()
    import torch
    import pkt_b200
    dims = [int(v) for v in args.dims.split(",")]
    B = args.batch
    rng = np.random.default_rng(0)
    x = rng.standard_normal((B, dims[0]), dtype=np.float32)
    t = rng.standard_normal((B, dims[-1]), dtype=np.float32)
    Ws = [(rng.uniform(-1, 1, (dims[l + 1], dims[l])) * np.sqrt(6.0 / dims[l])).astype(np.float32)
          for l in range(len(dims) - 1)]
    bs = [np.zeros(dims[l + 1], np.float32) for l in range(len(dims) - 1)]
    flops = sum(2.0 * B * dims[l] * dims[l + 1] * (3 if l else 2) for l in range(len(dims) - 1))

    def timed(fn):
        fn(2)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        out = fn(args.steps)
        torch.cuda.synchronize()
        return out, (time.perf_counter() - t0) / args.steps

    ref, t_torch = timed(lambda n: mlp_train(dims, x, t, Ws, bs, args.lr, n, mode=args.dtype))
    m = pkt_b200.MLP(dims, B, dtype=args.dtype, lr=args.lr)
    m.set_params(Ws, bs)
    m.load_batch(m.storage_array(x), m.storage_array(t))

    def ours(n):
        m.reset_losses()
        m.train(n)
        return m.losses()

    _, t_ours = timed(ours)
    m.set_params(Ws, bs)  # the numeric comparison starts from the same weights as torch's run
    got = ours(args.steps)
    rel = float(np.max(np.abs(got - ref["losses"]) / ref["losses"]))
    print(f"dims {dims} batch {B} {args.dtype}, {args.steps} steps")
    print(f"torch (cuBLAS, same rounding): {t_torch * 1e3:.3f} ms/step  {flops / t_torch / 1e12:.0f} TFLOP/s "
          f"(host-timed, includes its element-wise kernels)")
    print(f"pkt_b200 megakernel:           {t_ours * 1e3:.3f} ms/step  {flops / t_ours / 1e12:.0f} TFLOP/s")
    print(f"loss curves: max relative difference {rel:.2e}; last loss torch {ref['losses'][-1]:.6f} "
          f"pkt_b200 {got[-1]:.6f}")


if __name__ == "__main__":
    main()
