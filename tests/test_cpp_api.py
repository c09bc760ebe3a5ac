"""The pkt-compatible C++ API (include/pk/*, pk::Runtime over the C-ABI) and the
C++ example programs, built with g++ against libpkt_b200.so.

Host-only programs (descriptor layout, slot ring constants) run on CPU; the
runtime programs and the examples need the GPU. The examples' printed lines
follow pkt's examples/train_linear.cu and examples/axpy_example.cu."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BUILD = os.path.join(ROOT, "tests", "cpp", "_build")


def _make(target):
    subprocess.check_call(["make", "-s", "-C", os.path.join(ROOT, "tests", "cpp"),
                           os.path.join(BUILD, target)])
    return os.path.join(BUILD, target)


def _run(binary, *args, timeout=300):
    r = subprocess.run([binary, *args], capture_output=True, text=True, timeout=timeout)
    return r.returncode, r.stdout + r.stderr


def test_headers_compile_and_descriptor_layout():
    rc, out = _run(_make("test_task"))
    assert rc == 0, out


def test_slot_ring_and_warp_roles():
    rc, out = _run(_make("test_pipeline"))
    assert rc == 0, out


def test_train_linear_cpu_line_matches_pkt():
    # the CPU part of the C++ example restates pkt's loop: same printed digits as
    # pkt's own binary (tests/golden/pkt_train_linear_cpu.txt)
    b = _make("train_linear")
    r = subprocess.run([b, "--m", "64", "--n", "128", "--batch", "256", "--steps", "100", "--lr",
                        "0.01"], capture_output=True, text=True, timeout=120)
    assert "CPU final loss: 9.80123e-05" in r.stdout
    assert "Initial host loss: 0.000100954" in r.stdout


@pytest.mark.gpu
def test_runtime_cases_on_gpu():
    rc, out = _run(_make("test_runtime"))
    assert rc == 0, out


@pytest.mark.gpu
def test_axpy_example_bit_exact():
    rc, out = _run(_make("axpy_example"))
    assert rc == 0 and "Status: PASSED" in out, out


@pytest.mark.gpu
@pytest.mark.parametrize("engine", ["tasks", "mlp"])
def test_train_linear_example_check_loss(engine):
    rc, out = _run(_make("train_linear"), "--m", "64", "--n", "128", "--batch", "64", "--steps", "50",
                   "--lr", "0.01", "--check-loss", "--check-tasks" if engine == "tasks" else "--skip-cpu",
                   "--engine", engine)
    assert rc == 0, out
    assert re.search(r"Time per step: [0-9.e-]+ ms", out), out


@pytest.mark.gpu
def test_train_linear_example_mlp_layers_bf16():
    rc, out = _run(_make("train_linear"), "--m", "64", "--n", "256", "--batch", "512", "--steps", "20",
                   "--lr", "0.01", "--engine", "mlp", "--layers", "256,512,64", "--dtype", "bf16",
                   "--bias", "--skip-cpu")
    assert rc == 0, out
    first = float(re.search(r"Device first step loss: ([0-9.e+-]+)", out).group(1))
    last = float(re.search(r"Device final loss: ([0-9.e+-]+)", out).group(1))
    assert last < first, out


@pytest.mark.gpu
@pytest.mark.parametrize("engine", ["tasks", "mlp"])
def test_train_linear_perf_json(engine, tmp_path):
    """--perf / --perf-json (pkt examples/train_linear.cu:724-935): per-role summary
    printed, JSON written with the per-CTA totals."""
    import json
    path = str(tmp_path / "perf.json")
    rc, out = _run(_make("train_linear"), "--m", "256", "--n", "512", "--batch", "64", "--steps", "8",
                   "--lr", "0.01", "--skip-cpu", "--engine", engine, "--perf-json", path)
    assert rc == 0, out
    assert "Per-role counters" in out and "controller.deps_wait" in out, out
    d = json.load(open(path))
    assert d["blocks"] > 0 and d["totals"]["tasks_issued"] > 0 and d["sm_mhz"] > 0
