"""Per-task trace of one MLP training step: where the tensor pipe waits.

    python -m pkt_b200.trace_report --dims 1024,4096,4096,4096,1024 --batch 8192
    python -m pkt_b200.trace_report --dims 512x17 --batch 2048 --json trace.json
    python -m torch.distributed.run --nproc-per-node 2 -m pkt_b200.trace_report --grad-mode 2

Runs `--warmup` steps, then one step with the per-task trace on
(pkt_mlp_set_trace) and prints, from the %globaltimer stamps of every task:

  * per GEMM (forward / dgrad / weight gradient of each layer): tiles, mean MMA
    issue window (first MMA to last commit), mean first-load-to-first-MMA latency,
    mean epilogue time (accumulator complete to task done);
  * for the MMA issuer of every CTA (pair leader): the gaps between one tile's
    last commit and the next tile's first MMA, split by what the next tile was
    waiting for -- its dependencies (controller), its first stage (loads), or a
    free accumulator (the epilogue of the tile before) -- and the idle time at the
    start and end of the launch;
  * the layer-to-layer hops of the forward and dgrad chains: for each row block,
    from the last producer tile's end (and the spread of the producers' ends) to
    the consumer tiles' dependencies satisfied, first load, first MMA, last MMA,
    epilogue start and end;
  * the SIMT tasks by opcode (count, mean and maximum run time); the fused
    data-parallel reduce task also stamps the end of its wait for the ranks'
    partials, so its wait and its work are shown apart.

Under torch.distributed.run (WORLD_SIZE > 1) every rank runs the data-parallel
step (--grad-mode 2, the fused peer-memory reduce, by default; 1: NCCL) and
prints its own report (the ranks' %globaltimer clocks are not comparable).
"""
import argparse
import json
import os
import sys

import numpy as np

W_CTA, W_DEQ, W_READY, W_LOAD, W_MMA0, W_MMA1, W_EXEC, W_DONE = range(8)
OP_GEMM = 3
OP_NAMES = {1: "zero", 2: "axpy", 10: "linear_fwd", 11: "mse", 12: "linear_bwd", 13: "sgd",
            20: "bias_sgd", 21: "loss_reduce", 22: "sgd_mixed", 30: "dp_wait", 31: "dp_bias_send",
            32: "dp_bias_apply", 33: "dp_reduce"}
OP_DP_REDUCE = 33


def gemm_names(dims):
    """Names of the GEMMs one build registers, in the engine's registration order
    (pkt_b200/csrc/mlp.cu Mlp::build): forward 0..L-1, then per layer from the
    last: dgrad (layers >= 1), weight gradient."""
    L = len(dims) - 1
    names = [f"fwd{l}" for l in range(L)]
    for l in range(L - 1, -1, -1):
        if l >= 1:
            names.append(f"dgrad{l}")
        names.append(f"wgrad{l}")
    return names


def analyse(tr, dims):
    tr = np.asarray(tr, np.uint64)
    w0 = tr[:, W_CTA]
    cta = (w0 & 0xFFFF).astype(np.int64)
    op = ((w0 >> 16) & 0xFFFF).astype(np.int64)
    gid = ((w0 >> 32) & 0xFFFF).astype(np.int64)
    ts = tr[:, 1:].astype(np.int64)
    t0 = int(ts[ts > 0].min())
    t_end = int(ts.max())
    rel = np.where(ts > 0, ts - t0, -1)
    names = gemm_names(dims)
    per_build = len(names)
    is_gemm = op == OP_GEMM
    out = {"launch_us": (t_end - t0) / 1e3, "tasks": int(len(tr)), "gemm_tiles": int(is_gemm.sum())}
    # ---- per GEMM
    rows = {}
    for i in np.nonzero(is_gemm)[0]:
        name = names[gid[i] % per_build]
        r = rel[i]
        d = rows.setdefault(name, {"tiles": 0, "mma_us": 0.0, "load_to_mma_us": 0.0, "epi_us": 0.0,
                                   "ready_to_done_us": 0.0})
        d["tiles"] += 1
        d["mma_us"] += (r[W_MMA1 - 1] - r[W_MMA0 - 1]) / 1e3
        d["load_to_mma_us"] += (r[W_MMA0 - 1] - r[W_LOAD - 1]) / 1e3
        d["epi_us"] += (r[W_DONE - 1] - r[W_EXEC - 1]) / 1e3
        d["ready_to_done_us"] += (r[W_DONE - 1] - r[W_READY - 1]) / 1e3
    for d in rows.values():
        for k in ("mma_us", "load_to_mma_us", "epi_us", "ready_to_done_us"):
            d[k] /= d["tiles"]
    out["gemms"] = {n: rows[n] for n in names if n in rows}
    # ---- MMA issuer gaps per CTA
    cats = {"dependency": 0.0, "first_stage": 0.0, "accumulator": 0.0, "start": 0.0, "end": 0.0,
            "busy": 0.0}
    ctas = sorted(set(cta[is_gemm].tolist()))
    for c in ctas:
        idx = np.nonzero(is_gemm & (cta == c))[0]
        idx = idx[np.argsort(rel[idx, W_MMA0 - 1])]
        if len(idx) == 0:
            continue
        m0 = rel[idx, W_MMA0 - 1]
        m1 = rel[idx, W_MMA1 - 1]
        cats["start"] += m0[0]
        cats["end"] += (t_end - t0) - m1[-1]
        cats["busy"] += float(np.sum(m1 - m0))
        for k in range(1, len(idx)):
            gap = m0[k] - m1[k - 1]
            if gap <= 0:
                continue
            nxt = rel[idx[k]]
            prev2_done = rel[idx[k - 2], W_DONE - 1] if k >= 2 else -1
            if nxt[W_READY - 1] > m1[k - 1]:
                cats["dependency"] += gap
            elif prev2_done > m1[k - 1]:
                cats["accumulator"] += gap
            else:
                cats["first_stage"] += gap
    n = max(1, len(ctas))
    out["mma_issuer_per_cta_us"] = {k: v / n / 1e3 for k, v in cats.items()}
    out["ctas"] = n
    out["hops"] = hop_breakdown(rel, op, gid, ((w0 >> 48) & 0xFF).astype(np.int64), names, dims)
    # ---- SIMT tasks
    simt = {}
    for code in sorted(set(op[~is_gemm].tolist())):
        m = (op == code) & ~is_gemm
        run = (rel[m, W_DONE - 1] - rel[m, W_EXEC - 1]) / 1e3
        d = {"tasks": int(m.sum()), "run_us_mean": float(run.mean()), "run_us_max": float(run.max())}
        if code == OP_DP_REDUCE:
            wait = (rel[m, W_LOAD - 1] - rel[m, W_EXEC - 1]) / 1e3
            d["wait_us_mean"] = float(wait.mean())
            d["work_us_mean"] = float((run - wait).mean())
        simt[OP_NAMES.get(code, str(code))] = d
    out["simt"] = simt
    return out


def hop_breakdown(rel, op, gid, tile_m, names, dims):
    """Mean latencies (us) of the forward and dgrad chain hops: per row block, the
    last producer tile's end to the consumer tiles' stages."""
    per_build = len(names)
    L = len(dims) - 1
    gname = np.array([names[g % per_build] if o == OP_GEMM else "" for g, o in zip(gid, op)])
    out = {}
    for kind, layers, prev in (("fwd", range(1, L), lambda l: f"fwd{l - 1}"),
                               ("dgrad", range(L - 2, 0, -1), lambda l: f"dgrad{l + 1}")):
        rows = []
        for l in layers:
            for i in sorted(set(tile_m[gname == f"{kind}{l}"].tolist())):
                pm = (gname == prev(l)) & (tile_m == i)
                cm = (gname == f"{kind}{l}") & (tile_m == i)
                if not pm.any() or not cm.any():
                    continue
                pd = rel[pm, W_DONE - 1]
                done = pd.max()
                c = rel[cm]
                rows.append([pd.max() - pd.min(), (c[:, W_READY - 1] - done).mean(),
                             (c[:, W_LOAD - 1] - c[:, W_READY - 1]).mean(),
                             (c[:, W_MMA0 - 1] - c[:, W_LOAD - 1]).mean(),
                             (c[:, W_MMA1 - 1] - c[:, W_MMA0 - 1]).mean(),
                             (c[:, W_EXEC - 1] - c[:, W_MMA1 - 1]).mean(),
                             (c[:, W_DONE - 1] - c[:, W_EXEC - 1]).mean(),
                             c[:, W_DONE - 1].max() - done])
        if rows:
            r = np.array(rows).mean(0) / 1e3
            out[kind] = dict(zip(["producer_spread", "to_ready", "ready_to_load", "load_to_mma",
                                  "mma", "mma_to_epilogue", "epilogue", "hop"], map(float, r)))
    return out


def print_report(rep):
    mhz = rep.get("sm_mhz")
    print(f"launch {rep['launch_us']:.1f} us, {rep['tasks']} tasks, {rep['gemm_tiles']} GEMM tiles, "
          f"{rep['ctas']} MMA issuers" + (f", SM clock {mhz:.0f} MHz" if mhz else ""))
    print(f"{'gemm':>8} {'tiles':>6} {'mma us':>8} {'load->mma':>10} {'epilogue':>9} {'ready->done':>12}")
    for name, d in rep["gemms"].items():
        print(f"{name:>8} {d['tiles']:6d} {d['mma_us']:8.2f} {d['load_to_mma_us']:10.2f} "
              f"{d['epi_us']:9.2f} {d['ready_to_done_us']:12.2f}")
    m = rep["mma_issuer_per_cta_us"]
    tot = rep["launch_us"]
    print("MMA issuer, mean per CTA (us, share of the launch):")
    for k in ("busy", "dependency", "first_stage", "accumulator", "start", "end"):
        print(f"  {k:>12}: {m[k]:9.1f}  {100 * m[k] / tot:5.1f} %")
    if rep.get("hops"):
        print("layer hops, mean per row block (us): producers' spread | last producer end -> "
              "dependencies satisfied | -> first load | -> first MMA | MMA | -> epilogue | epilogue | hop")
        for kind, h in rep["hops"].items():
            print(f"  {kind:>6}: {h['producer_spread']:5.2f} | {h['to_ready']:5.2f} | {h['ready_to_load']:5.2f} | "
                  f"{h['load_to_mma']:5.2f} | {h['mma']:5.2f} | {h['mma_to_epilogue']:5.2f} | "
                  f"{h['epilogue']:5.2f} | {h['hop']:5.2f}")
    if rep.get("simt"):
        print("SIMT tasks (us):")
        for name, d in rep["simt"].items():
            extra = (f", wait {d['wait_us_mean']:.2f} + work {d['work_us_mean']:.2f}"
                     if "wait_us_mean" in d else "")
            print(f"  {name:>14}: {d['tasks']:5d} tasks, run mean {d['run_us_mean']:7.2f} max "
                  f"{d['run_us_max']:7.2f}{extra}")


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--dims", default="1024,4096,4096,4096,1024",
                    help="comma-separated widths, or WxN for N equal widths")
    ap.add_argument("--batch", type=int, default=8192)
    ap.add_argument("--dtype", default="bf16")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--cta-pair", type=int, default=0)
    ap.add_argument("--grad-mode", type=int, default=None, choices=[0, 1, 2],
                    help="0: SGD fused into the gradient epilogue (one GPU, default there); 1: NCCL "
                         "all-reduce between two launches (the first is traced); 2: fused peer-memory "
                         "reduce (default with WORLD_SIZE > 1)")
    ap.add_argument("--json", default=None, help="write report and raw trace (rank suffix under torchrun)")
    args = ap.parse_args(argv)
    if "x" in args.dims:
        w, n = args.dims.split("x")
        dims = [int(w)] * int(n)
    else:
        dims = [int(v) for v in args.dims.split(",")]
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
    rng = np.random.default_rng(0)
    m = pkt_b200.MLP(dims, args.batch, dtype=args.dtype, lr=1e-3, cta_pair=args.cta_pair, grad_mode=gm,
                     device=local)
    if world > 1:
        m.set_grad_scale(1.0 / world)
    Ws = [(rng.uniform(-1, 1, (dims[l + 1], dims[l])) * np.sqrt(6.0 / dims[l])).astype(np.float32)
          for l in range(len(dims) - 1)]
    m.set_params(Ws)
    rng = np.random.default_rng(1 + rank)  # per-rank data shard (rank 0: the single-GPU data)
    x = rng.standard_normal((args.batch, dims[0])).astype(np.float32)
    t = rng.standard_normal((args.batch, dims[-1])).astype(np.float32)
    m.load_batch(m.storage_array(x), m.storage_array(t))
    grad = None
    if gm == 2:
        handles = None
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, m.dp_handle())
        m.dp_connect(rank, world, handles)
    elif gm == 1:
        p, n = m.grad_buffer()

        class _CAI:
            __cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (p, False), "version": 3,
                                        "strides": None}
        grad = torch.as_tensor(_CAI(), device=torch.device("cuda", local))

    def step(traced=False):
        if gm != 1:
            m.train(1)
            return
        m.forward_backward()  # the traced launch (the trace keeps the last launch)
        if traced:
            torch.cuda.synchronize()
            return
        if dist is not None:
            dist.all_reduce(grad)
        m.apply_update()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    m.set_trace(True)
    m.clock_stats(reset=True)
    step(traced=True)
    torch.cuda.synchronize()
    tr = m.fetch_trace()
    cyc, ns, _ = m.clock_stats()
    m.set_trace(False)
    rep = analyse(tr, dims)
    rep["sm_mhz"] = cyc * 1000.0 / ns if ns else None
    for r in range(world):  # one rank's report at a time
        if r == rank:
            head = f"rank {rank} of {world}, grad_mode {gm}: " if world > 1 else ""
            print(f"{head}dims {dims} batch {args.batch} {args.dtype}", flush=True)
            print_report(rep)
            sys.stdout.flush()
        if dist is not None:
            dist.barrier()
    if args.json:
        path = args.json if world == 1 else f"{os.path.splitext(args.json)[0]}_rank{rank}.json"
        with open(path, "w") as f:
            json.dump({"dims": dims, "batch": args.batch, "grad_mode": gm, "rank": rank, "world": world,
                       "report": rep, "trace": tr.tolist()}, f)
    if dist is not None:
        dist.barrier()  # no rank frees its exchange region while another still reads it
    m.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
