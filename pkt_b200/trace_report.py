"""Per-task trace of one MLP training step: where the tensor pipe waits.

    python -m pkt_b200.trace_report --dims 1024,4096,4096,4096,1024 --batch 8192
    python -m pkt_b200.trace_report --dims 512x17 --batch 2048 --json gpurun_out/trace.json

Runs `--warmup` steps, then one step with the per-task trace on
(pkt_mlp_set_trace) and prints, from the %globaltimer stamps of every task:

  * per GEMM (forward / dgrad / weight gradient of each layer): tiles, mean MMA
    issue window (first MMA to last commit), mean first-load-to-first-MMA latency,
    mean epilogue time (accumulator complete to task done);
  * for the MMA issuer of every CTA (pair leader): the gaps between one tile's
    last commit and the next tile's first MMA, split by what the next tile was
    waiting for -- its dependencies (controller), its first stage (loads), or a
    free accumulator (the epilogue of the tile before) -- and the idle time at the
    start and end of the launch.
"""
import argparse
import json

import numpy as np

W_CTA, W_DEQ, W_READY, W_LOAD, W_MMA0, W_MMA1, W_EXEC, W_DONE = range(8)
OP_GEMM = 3


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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--dims", default="1024,4096,4096,4096,1024",
                    help="comma-separated widths, or WxN for N equal widths")
    ap.add_argument("--batch", type=int, default=8192)
    ap.add_argument("--dtype", default="bf16")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--cta-pair", type=int, default=0)
    ap.add_argument("--json", default=None)
    args = ap.parse_args()
    if "x" in args.dims:
        w, n = args.dims.split("x")
        dims = [int(w)] * int(n)
    else:
        dims = [int(v) for v in args.dims.split(",")]
    import torch
    import pkt_b200
    torch.cuda.set_device(0)
    rng = np.random.default_rng(0)
    m = pkt_b200.MLP(dims, args.batch, dtype=args.dtype, lr=1e-3, cta_pair=args.cta_pair)
    Ws = [(rng.uniform(-1, 1, (dims[l + 1], dims[l])) * np.sqrt(6.0 / dims[l])).astype(np.float32)
          for l in range(len(dims) - 1)]
    m.set_params(Ws)
    x = rng.standard_normal((args.batch, dims[0])).astype(np.float32)
    t = rng.standard_normal((args.batch, dims[-1])).astype(np.float32)
    m.load_batch(m.storage_array(x), m.storage_array(t))
    m.train(args.warmup)
    m.set_trace(True)
    m.clock_stats(reset=True)
    m.train(1)
    tr = m.fetch_trace()
    cyc, ns, _ = m.clock_stats()
    m.set_trace(False)
    rep = analyse(tr, dims)
    rep["sm_mhz"] = cyc * 1000.0 / ns if ns else None
    print(f"dims {dims} batch {args.batch} {args.dtype}")
    print_report(rep)
    if args.json:
        with open(args.json, "w") as f:
            json.dump({"dims": dims, "batch": args.batch, "report": rep, "trace": tr.tolist()}, f)


if __name__ == "__main__":
    main()
