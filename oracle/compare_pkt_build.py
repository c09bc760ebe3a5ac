"""pkt's own build (oracle/_ref, compiled from the reference sources for sm_100a)
timed beside this build on the same GPU in the same process run.

COMPARISON INFRASTRUCTURE (like the rest of oracle/): pkt's binaries and its
kernel library are the thing compared against, never part of the product path.

    python oracle/compare_pkt_build.py [--json out.json]

  * axpy: pkt's persistent kernel (pktref_axpy_time: Axpy tasks over device
    buffers, one launch per repetition, CUDA events around the launch) against
    pkt_axpy at the same sizes -- pkt's example size (1000 x 1024 floats) and a
    bandwidth-sized one (4096 tasks x 65536 floats = 1 GiB of x and y); GB/s at
    12 bytes per element (read x, read y, write y);
  * train_linear in pkt's domain (no bias, batch <= 64, n <= 1024): pkt's own
    train_linear binary (its "Time per step" line, all steps in one launch) and
    this build's examples/train_linear with --engine tasks (pkt's DAG on the
    B200 runtime) and --engine mlp (tcgen05 engine), at pkt's defaults
    (1024 x 1024, batch 64, 20 steps) and at the single-Linear benchmark shape
    128 -> 64 with batch 64.
"""
import argparse
import ctypes
import json
import os
import re
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
REF = os.path.join(HERE, "_ref")


def _time_per_step(out):
    m = re.search(r"Time per step: ([0-9.eE+-]+) ms", out)
    return float(m.group(1)) if m else None


def run(cmd, timeout=600):
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout)
    return r.returncode, r.stdout + r.stderr


def axpy_rows():
    import torch
    sys.path.insert(0, ROOT)
    import pkt_b200
    lib = ctypes.CDLL(os.path.join(REF, "libpkt_ref.so"))
    lib.pktref_axpy_time.argtypes = [ctypes.c_int] * 4 + [ctypes.POINTER(ctypes.c_float)]
    rows = []
    for ntask, per in ((1000, 1024), (4096, 65536)):
        n = ntask * per
        ms = ctypes.c_float()
        rc = lib.pktref_axpy_time(ntask, per, 0, 5, ctypes.byref(ms))
        x = torch.rand(n, device="cuda")
        y = torch.rand(n, device="cuda")
        pkt_b200.axpy(x.data_ptr(), y.data_ptr(), 0.5, n)
        torch.cuda.synchronize()
        best = None
        for _ in range(5):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            pkt_b200.axpy(x.data_ptr(), y.data_ptr(), 0.5, n)
            b.record()
            torch.cuda.synchronize()
            t = a.elapsed_time(b)
            best = t if best is None else min(best, t)
        rows.append({"elements": n, "pkt_ms": ms.value if rc == 0 else None,
                     "pkt_gbs": 12.0 * n / ms.value / 1e6 if rc == 0 and ms.value > 0 else None,
                     "b200_ms": best, "b200_gbs": 12.0 * n / best / 1e6})
        del x, y
    return rows


def train_rows():
    ours = os.path.join(ROOT, "tests", "cpp", "_build", "train_linear")
    subprocess.check_call(["make", "-s", "-C", os.path.join(ROOT, "tests", "cpp"), ours])
    rows = []
    for m, n, batch, steps in ((1024, 1024, 64, 20), (64, 128, 64, 100)):
        args = ["--m", str(m), "--n", str(n), "--batch", str(batch), "--steps", str(steps), "--lr", "0.001",
                "--skip-cpu"]
        row = {"m": m, "n": n, "batch": batch, "steps": steps}
        rc, out = run([os.path.join(REF, "train_linear")] + args)
        row["pkt_ms_per_step"] = _time_per_step(out) if rc == 0 else None
        for eng in ("tasks", "mlp"):
            rc, out = run([ours] + args + ["--engine", eng])
            row[f"b200_{eng}_ms_per_step"] = _time_per_step(out) if rc == 0 else None
        rows.append(row)
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--json", default=None)
    args = ap.parse_args()
    if not os.path.exists(os.path.join(REF, "train_linear")):
        print("pkt's build is missing (make -C oracle ref needs the reference tree)")
        return 1
    res = {"axpy": axpy_rows(), "train_linear": train_rows()}
    print("axpy (fastest of 5 launches, 12 B/element):")
    for r in res["axpy"]:
        print(f"  n={r['elements']:>11}: pkt {r['pkt_ms']:.4f} ms {r['pkt_gbs']:.0f} GB/s | "
              f"pkt_b200 {r['b200_ms']:.4f} ms {r['b200_gbs']:.0f} GB/s")
    print("train_linear (ms per step, --skip-cpu):")
    for r in res["train_linear"]:
        print(f"  m={r['m']} n={r['n']} batch={r['batch']} steps={r['steps']}: pkt {r['pkt_ms_per_step']} | "
              f"b200 tasks {r['b200_tasks_ms_per_step']} | b200 mlp {r['b200_mlp_ms_per_step']}")
    if args.json:
        with open(args.json, "w") as f:
            json.dump(res, f, indent=1)
    return 0


if __name__ == "__main__":
    sys.exit(main())
