"""Benchmark of the pkt MLP training step on B200.

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config cfg2]

Default workload (N=1): the 4-layer ReLU MLP 1024->4096->4096->4096->1024, bf16
weights/activations with fp32 accumulation and fp32 master weights, batch 8192,
MSE, SGD lr=1e-3 (the configuration the headline metric is quoted on). N>1:
data parallel, the same model with 8192 rows per GPU (weak scaling); by default
(--dp fused) one launch per step on every rank, the weight-gradient tiles
reduced inside it over peer memory (NVLink); --dp nccl: fp32 gradients
all-reduced with NCCL between the backward and the update launch; --dp
nccl-overlap: one NCCL all-reduce per layer on a side stream, each issued when
its layer's gradient is complete and overlapped with the rest of the backward
(the step in L launches, the grid leaving --reserve-sms SMs to NCCL).
One JSON line on rank 0.
"""
import argparse
import datetime
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    "cfg1": dict(dims=[128, 64], batch=256, dtype="tf32", lr=1e-2,
                 desc="train_linear: Linear 128->64, fp32/TF32, batch 256, bias, MSE, SGD lr=1e-2"),
    "cfg2": dict(dims=[1024, 4096, 4096, 4096, 1024], batch=8192, dtype="bf16", lr=1e-3,
                 desc="4-layer ReLU MLP 1024->4096->4096->4096->1024, bf16 weights/activations, "
                      "fp32 accumulate, fp32 master weights, batch 8192/GPU, MSE, SGD lr=1e-3"),
    "cfg3": dict(dims=[512] * 17, batch=2048, dtype="bf16", lr=1e-3,
                 desc="deep narrow MLP: 16 layers of width 512, ReLU, bf16/fp32-acc, batch 2048"),
    "cfg4": dict(dims=[8192] * 9, batch=8192, dtype="bf16", lr=1e-4, global_batch=65536,
                 desc="wide MLP: 8 layers of width 8192, ReLU, bf16/fp32-acc, batch 8192/GPU "
                      "(--scaling strong: global batch 65536 split over the GPUs)"),
    "cfg5": dict(dims=[1000, 3000, 777, 10], batch=4099, dtype="tf32", lr=5e-3,
                 desc="ragged MLP 1000->3000->777->10, fp32 storage with TF32 tensor cores, batch 4099"),
}


for _name, _cfg in CONFIGS.items():
    _cfg["name"] = _name


def flops_per_sample(dims):
    return sum(2.0 * dims[l] * dims[l + 1] * (3 if l > 0 else 2) for l in range(len(dims) - 1))


# DRAM bytes (read + write) of one pk_megakernel launch (= one training step),
# from one ncu capture of that config; the capture is summarised, with its
# command, in the named profile.
PROFILED_TRAFFIC = {
    "cfg2": {"bytes": (13.157e9 + 2.676e9) / 4,
             "source": "dram__bytes_read.sum + dram__bytes_write.sum of one 4-step pk_megakernel "
                       "launch in a separate ncu capture of this configuration, per step; a fixed "
                       "figure, not measured in this run"},
}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    except Exception:
        return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms; only samples whose
    timestamp falls inside the timed region (mark_begin / mark_end) are kept."""
    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.t0 = self.t1 = None

    def mark_begin(self):
        self.t0 = datetime.datetime.now()

    def mark_end(self):
        self.t1 = datetime.datetime.now()

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.Q,
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=5)
        rows = [r.split(",") for r in out.strip().splitlines() if r.strip()]
        sm, mx, reasons, power, kept = [], None, set(), [], 0
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [c.strip() for c in r]
            if len(r) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(r[0], "%Y/%m/%d %H:%M:%S.%f")
                if self.t0 and self.t1 and not (self.t0 <= ts <= self.t1):
                    continue
                sm.append(float(r[2]))
                mx = float(r[3])
                power.append(float(r[4]))
                kept += 1
            except ValueError:
                continue
            for n, v in zip(names, r[6:10]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": kept,
                "power_w_median": float(np.median(power)) if power else None}


def make_inputs(cfg, rank, seed=1234):
    dims, B = cfg["dims"], cfg["batch"]
    if cfg["name"] == "cfg1":
        # train_linear's own recipe: mt19937(0), W ~ U(+-1/sqrt(in)), b = 0, targets
        # from a fixed W*, b* ~ N(0, 1) plus N(0, 0.01^2) noise
        from pkt_b200.data import make_linear_task
        x, W, b, t = make_linear_task(dims[0], dims[1], B, seed=rank, noise=0.01)
        return x, t, [W], [b]
    rng = np.random.default_rng(seed + rank)
    x = rng.standard_normal((B, dims[0]), dtype=np.float32)
    if cfg["name"] == "cfg5":
        x = rng.uniform(-3, 3, (B, dims[0])).astype(np.float32)
        t = np.zeros((B, dims[-1]), np.float32)
        t[np.arange(B), rng.integers(0, dims[-1], B)] = 1.0
    else:
        t = rng.standard_normal((B, dims[-1]), dtype=np.float32)
    # Kaiming-uniform weights (bound sqrt(6/fan_in)), zero bias
    Ws = [(rng.uniform(-1, 1, (dims[l + 1], dims[l])) * np.sqrt(6.0 / dims[l])).astype(np.float32)
          for l in range(len(dims) - 1)]
    bs = [np.zeros(dims[l + 1], np.float32) for l in range(len(dims) - 1)]
    return x, t, Ws, bs


def cpu_full_batch(cfg, max_steps, budget_s, warmup=1):
    """The fp32 OpenMP restatement of pkt's host training loop extended to the MLP
    (oracle/cpu_mlp.cpp, built here with -O3 -march=native) on all host cores:
    `warmup` untimed full-batch steps, then full-batch steps until `max_steps` or
    `budget_s` seconds. Returns (result dict, description)."""
    from oracle import cpu_baseline as cb
    x, t, Ws, bs = make_inputs(cfg, 0)
    # every host CPU this process may run on (torchrun sets OMP_NUM_THREADS=1 for
    # its ranks; the baseline overrides it)
    try:
        threads = len(os.sched_getaffinity(0))
    except AttributeError:
        threads = os.cpu_count() or 1
    r = cb.time_mlp(cfg["dims"], x, t, Ws, bs, cfg["lr"], max_steps, budget_s, warmup=warmup,
                    threads=threads)
    desc = (f"{r['steps']} full-batch step(s) of {cfg['batch']} rows timed ({r['seconds']:.2f} s) "
            f"after {warmup} untimed; fp32 OpenMP restatement of pkt's host loop extended to the MLP "
            f"({cb.FLAGS}), {r['threads']} threads on {os.cpu_count()} logical CPUs, {cb.cpu_model()}")
    return r, desc


def init_dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def run_reference(args, cfg_name, cfg):
    ws, rank, _ = init_dist()
    if rank != 0:
        return
    # full-batch steps, as many of the requested K as fit in about a minute
    r, desc = cpu_full_batch(cfg, args.steps, 60.0, warmup=min(args.warmup, 1))
    v = r["samples_per_s"]
    line = {
        "impl": "reference", "metric": "MLP train samples/s & % dense BF16 TC peak at 1/2/4/8 B200",
        "value": v, "unit": "samples/s", "n_gpus": args.gpus, "steps": r["steps"],
        "steps_requested": args.steps, "warmup": min(args.warmup, 1),
        "ms_per_step": 1000.0 * cfg["batch"] / v,
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (the same seeded inputs and weights as the GPU arm)",
        "config": {"workload": cfg_name + ": " + cfg["desc"], "global_batch": cfg["batch"],
                   "parallelism": "host CPU, OpenMP"},
        "cpu_baseline": {"value": v, "unit": "samples/s", "cores": r["threads"], "kind": "port",
                         "sample": desc},
        "e2e": {"value": v, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "loss_first_last": [r["losses"][0], r["losses"][-1]],
    }
    if cfg_name == "cfg1":
        # pkt's own host loop (examples/train_linear.cu:101-151): single thread, no bias
        from oracle import cpu_baseline as cb
        x, t, Ws, _ = make_inputs(cfg, 0)
        sps, secs, last = cb.time_pkt_loop(Ws[0], x, t, 100, cfg["lr"])
        line["pkt_host_loop_1core"] = {"value": sps, "unit": "samples/s", "cores": 1,
                                       "sample": f"100 steps of pkt's loop (no bias) in {secs:.3f} s",
                                       "final_loss": last}
    print(json.dumps(line), flush=True)


def run_ours(args, cfg_name, cfg):
    import torch
    ws, rank, local = init_dist()
    torch.cuda.set_device(local)
    dist = None
    if ws > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    import pkt_b200
    from pkt_b200.mlp import to_bf16_bits

    dims, B = cfg["dims"], cfg["batch"]
    # fused data parallel needs bf16 weights; TF32 configs use the NCCL path
    nccl_dp = ws > 1 and (args.dp in ("nccl", "nccl-overlap") or cfg["dtype"] != "bf16")

    def make_engine(gm):
        return pkt_b200.MLP(dims, B, dtype=cfg["dtype"], lr=cfg["lr"], bias=True, grad_mode=gm,
                            device=local)

    eng = make_engine((1 if nccl_dp else 2) if ws > 1 else 0)
    if ws > 1 and not nccl_dp:
        # exchange the ranks' peer-memory handles once; if any rank cannot map its
        # peers, every rank falls back to the NCCL all-reduce path together
        ok, handle = 1, b""
        try:
            handle = eng.dp_handle()
        except Exception as e:  # noqa: BLE001
            print(f"rank {rank}: no exchange-region handle ({e})", file=sys.stderr)
            ok = 0
        handles = [None] * ws
        dist.all_gather_object(handles, (ok, handle))
        if all(h[0] for h in handles):
            try:
                eng.dp_connect(rank, ws, [h[1] for h in handles])
            except Exception as e:  # noqa: BLE001
                print(f"rank {rank}: cannot map the peers' exchange regions ({e})", file=sys.stderr)
                ok = 0
        else:
            ok = 0
        flag = torch.tensor([ok], device="cuda")
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        torch.cuda.synchronize()
        dist.barrier()
        if int(flag.item()) == 0:
            if rank == 0:
                print("fused data parallel unavailable: using the NCCL all-reduce path", file=sys.stderr)
            eng.close()
            nccl_dp = True
            eng = make_engine(1)
    if ws > 1:
        eng.set_grad_scale(1.0 / ws)
    x, t, Ws, bs = make_inputs(cfg, 0)  # same initial weights on every rank
    eng.set_params(Ws, bs)
    xs, ts = make_inputs(cfg, rank)[:2]  # per-rank data shard
    # two distinct pinned host batches, in the engine's storage type
    host_x, host_t = [], []
    for k in range(2):
        xa = eng.storage_array(np.roll(xs, k, axis=0))
        ta = eng.storage_array(np.roll(ts, k, axis=0))
        hx = torch.from_numpy(xa.view(np.int16) if xa.dtype == np.uint16 else xa).pin_memory()
        ht = torch.from_numpy(ta.view(np.int16) if ta.dtype == np.uint16 else ta).pin_memory()
        host_x.append(hx)
        host_t.append(ht)
    h2d_bytes = host_x[0].numel() * host_x[0].element_size() + host_t[0].numel() * host_t[0].element_size()

    stream = torch.cuda.Stream()
    copy_stream = torch.cuda.Stream()
    sp = stream.cuda_stream
    grad_t = None
    overlap = nccl_dp and args.dp == "nccl-overlap"
    L = len(dims) - 1
    if nccl_dp:
        gptr, gcount = eng.grad_buffer()
        grad_t = _wrap_device_f32(gptr, gcount, local)
    if overlap:
        # one all-reduce per layer on a side stream, issued as soon as the
        # segment that completes the layer's gradient has run, overlapped with the
        # following segments; the persistent grid leaves SMs free for NCCL
        eng.set_reserved_sms(args.reserve_sms)
        side = torch.cuda.Stream()
        seg_done = [torch.cuda.Event() for _ in range(L)]
        buckets = []
        for s_ in range(L):
            o, n = eng.grad_bucket(L - 1 - s_)
            buckets.append(grad_t[o:o + n])

    def step(s_ptr, n=1):
        if overlap:
            for s_ in range(L):
                eng.forward_backward_segment(s_, s_ptr)
                seg_done[s_].record(stream)
                side.wait_event(seg_done[s_])
                with torch.cuda.stream(side):
                    dist.all_reduce(buckets[s_])
            stream.wait_stream(side)
            eng.apply_update(s_ptr)
        elif nccl_dp:
            eng.forward_backward(s_ptr)
            with torch.cuda.stream(stream):
                dist.all_reduce(grad_t)
            eng.apply_update(s_ptr)
        else:
            eng.train(n, s_ptr)

    # Device-resident timing: on one GPU the engine runs MULTI steps per launch
    # (pkt_mlp_train with n >= 4 steps), the rest one launch per step.
    MULTI = 4
    group = MULTI if (ws == 1 and not nccl_dp and args.steps % MULTI == 0) else 1
    launches_per_step = (L + 1) if overlap else (2 if nccl_dp else 1)
    launches = (args.steps // group) * launches_per_step
    # ---------------- device-resident timing
    eng.load_batch_ptr(host_x[0].data_ptr(), host_t[0].data_ptr(), 0, sp)
    for _ in range(args.warmup):
        step(sp)
    torch.cuda.synchronize()
    eng.reset_losses()
    peaks, peak_kind = measured_peaks()
    sampler = ClockSampler(local)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)
    eng.clock_stats(reset=True)
    ncalls = args.steps // group
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(ncalls + 1)]
    sampler.mark_begin()
    wall0 = time.perf_counter()
    evs[0].record(stream)
    for i in range(ncalls):
        step(sp, group)
        evs[i + 1].record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall0
    sampler.mark_end()
    kcyc, kns, klaunches = eng.clock_stats()
    if dist:
        dist.barrier()
    clocks = sampler.stop()
    # effective SM clock of the timed launches: SM cycles / ns of CTA 0's lifetime,
    # summed over every launch (nvidia-smi's 50 ms polling sees few samples of a
    # short timed region)
    smi_mhz = clocks.get("sm_mhz")
    eff_mhz = kcyc * 1000.0 / kns if kns else None
    clocks = {"sm_mhz": eff_mhz,
              "sm_mhz_source": f"in-kernel clock64 / %globaltimer over CTA 0 of the {klaunches} timed launches",
              "sm_max_mhz": clocks.get("sm_max_mhz") or measured_peaks()[0].get("sm_max_mhz"),
              "reasons": clocks.get("reasons", []),
              "smi_sm_mhz_median": smi_mhz, "smi_samples": clocks.get("samples", 0),
              "power_w_median": clocks.get("power_w_median")}
    t_ms = evs[0].elapsed_time(evs[-1])
    per_call = [evs[i].elapsed_time(evs[i + 1]) for i in range(ncalls)]
    losses = eng.losses()
    if dist:
        tt = torch.tensor([t_ms], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_ms = float(tt.item())
    ms_per_step = t_ms / args.steps
    value = ws * B * args.steps / (t_ms / 1e3)
    F = flops_per_sample(dims) * B
    tflops = F / (ms_per_step / 1e3) / 1e12
    # per-launch kernel time (grad_mode 0: one launch per `group` steps) -> roofline
    # of the megakernel: the algorithmic FLOPs of one launch over its median time
    kern_ms = float(np.median(per_call)) if ws == 1 else ms_per_step * group
    achieved = F * group / (kern_ms / 1e3) / 1e12
    sustained = peaks.get("bf16_tflops_sustained", 1400.0)
    burst = peaks.get("bf16_tflops", 1590.0)

    # ---------------- end-to-end through the public API with host buffers
    eng.reset_losses()
    loss_host = torch.zeros(args.steps, dtype=torch.float32).pin_memory()
    done_ev = [torch.cuda.Event() for _ in range(args.steps)]
    copy_ev = [torch.cuda.Event() for _ in range(args.steps + 1)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(copy_stream)
    stream.wait_stream(copy_stream)
    cs = copy_stream.cuda_stream
    eng.load_batch_ptr(host_x[0].data_ptr(), host_t[0].data_ptr(), 0, cs)
    copy_ev[0].record(copy_stream)
    for i in range(args.steps):
        stream.wait_event(copy_ev[i])
        step(sp)
        done_ev[i].record(stream)
        # next batch into the other slot once the step that last read it (i-1) is done
        if i + 1 < args.steps:
            if i >= 1:
                copy_stream.wait_event(done_ev[i - 1])
            k = (i + 1) % 2
            eng.load_batch_ptr(host_x[k].data_ptr(), host_t[k].data_ptr(), 0, cs)
            copy_ev[i + 1].record(copy_stream)
        # device -> host read of this step's loss
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(done_ev[i])
            lp = eng.loss_ptr(i)
            loss_host[i:i + 1].copy_(_wrap_device_f32(lp, 1, local), non_blocking=True)
    copy_stream.wait_stream(stream)
    e1.record(copy_stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if dist:
        tt = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = float(tt.item())
    e2e_value = ws * B * args.steps / (e2e_ms / 1e3)
    e2e_losses = loss_host.numpy().copy()
    code = eng.status()[0]

    # Roofline denominator: the measured cuBLAS burst figure when the timed
    # region ran at (nearly) full SM clock, the sustained (power-capped) figure
    # when the clocks sampled during it show the power cap holding them down.
    sm, smax = clocks.get("sm_mhz"), clocks.get("sm_max_mhz")
    capped = bool(sm is not None and smax and sm < 0.93 * smax)
    peak = sustained if capped else burst
    traffic = PROFILED_TRAFFIC.get(cfg_name)
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak,
                "traffic": traffic["bytes"] * group if traffic else None,
                "traffic_source": traffic["source"] if traffic else None,
                "algorithmic_flop_per_launch": F * group, "steps_per_launch": group,
                "peak_kind": f"{peak_kind} " + ("bf16_tflops_sustained (effective SM clock of the timed "
                                                "launches below 93 % of max: power-capped)" if capped
                                                else "bf16_tflops burst (timed launches at full SM clock)"),
                "frac_of_burst": achieved / burst, "frac_of_sustained": achieved / sustained,
                "kernel": f"pk_megakernel (one launch = {group} training step{'s' if group > 1 else ''})"}
    if rank != 0:
        return
    line = {
        "metric": "MLP train samples/s & % dense BF16 TC peak at 1/2/4/8 B200",
        "value": value, "unit": "samples/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": cfg["dtype"],
        "data": "synthetic (seeded N(0,1) inputs/targets, Kaiming-uniform weights, zero bias)",
        "config": {"workload": cfg_name + ": " + cfg["desc"], "global_batch": B * ws,
                   "per_gpu_batch": B,
                   "parallelism": (f"dp{ws} ({('NCCL all-reduce per layer, overlapped' if overlap else 'NCCL all-reduce') if nccl_dp else 'fused peer-memory reduce'})"
                                   if ws > 1 else "single GPU"),
                   "l2": "no flush: every step streams > 126 MB (weights, activations, gradients "
                         "exceed L2)", "launches_per_step": launches / args.steps,
                   "steps_per_launch_device_resident": group,
                   "steps_per_launch_e2e": 1},
        "tflops": tflops, "pct_peak_measured_sustained": 100.0 * tflops / sustained,
        "pct_peak_measured_burst": 100.0 * tflops / burst,
        "pct_peak_spec_2250": 100.0 * tflops / 2250.0,
        "roofline": roofline,
        "e2e": {"value": e2e_value, "unit": "samples/s", "h2d_bytes_per_step": h2d_bytes,
                "d2h_bytes_per_step": 4,
                "method": "pkt_mlp_load_batch from pinned host memory (copy stream, next batch "
                          "overlapping the current step) + pkt_mlp_train + D2H loss read, every step"},
        "gpu_launches": launches,
        "clocks": clocks,
        "loss_first_last": [float(losses[0]), float(losses[-1])] if len(losses) else None,
        "e2e_loss_last": float(e2e_losses[-1]),
        "device_status": code,
        "wall_s_timed": wall,
    }
    if ws == 1 and not args.no_cpu:
        r, desc = cpu_full_batch(cfg, 2, 10.0, warmup=1)
        line["cpu_baseline"] = {"value": r["samples_per_s"], "unit": "samples/s",
                                "cores": r["threads"], "kind": "port", "sample": desc}
    print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


def _wrap_device_f32(ptr, count, device):
    import torch

    class _CAI:
        def __init__(self):
            self.__cuda_array_interface__ = {"shape": (count,), "typestr": "<f4",
                                             "data": (ptr, False), "version": 3, "strides": None}
    return torch.as_tensor(_CAI(), device=torch.device("cuda", device))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="cfg2", choices=sorted(CONFIGS))
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--reserve-sms", type=int, default=16,
                    help="--dp nccl-overlap: SMs the step's grid leaves to NCCL")
    ap.add_argument("--dp", default="fused", choices=["fused", "nccl", "nccl-overlap"],
                    help="N>1: weight gradients reduced inside the step launch over peer memory "
                         "(fused), by an NCCL all-reduce between two launches (nccl), or by one NCCL "
                         "all-reduce per layer overlapped with the backward (nccl-overlap)")
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                    help="weak: the configuration's batch on every GPU; strong: its global batch "
                         "(cfg4: 65536) split evenly over the GPUs")
    args = ap.parse_args()
    cfg = CONFIGS[args.config]
    if args.scaling == "strong":
        ws = int(os.environ.get("WORLD_SIZE", "1"))
        gb = cfg.get("global_batch", cfg["batch"])
        if gb % ws:
            sys.exit(f"global batch {gb} does not split over {ws} GPUs")
        cfg = dict(cfg, batch=gb // ws)
    if args.impl == "reference":
        run_reference(args, args.config, cfg)
    else:
        run_ours(args, args.config, cfg)


if __name__ == "__main__":
    main()
