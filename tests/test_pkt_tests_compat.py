"""pkt's own test programs (tests/test_task.cu, test_pipeline.cu, test_axpy.cu,
test_runtime.cu, test_paging.cu), compiled unchanged against this build's
headers (include/pkt_compat forwarding to include/pk, linked with
libpkt_b200.so) by `make -C oracle compat` where the reference tree is present;
the binaries travel in oracle/_ref/compat. pkt's tests return "pass" for their
device cases when no CUDA device is present, so the CPU run covers the host
cases (descriptor layout, constants) and the GPU run everything.

Also a program's own op through pkt's plugin point (tests/cpp/test_user_op.cu:
pk::OpTraits with load / compute / store, launched by pk::launch_with_ops)."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
COMPAT = os.path.join(ROOT, "oracle", "_ref", "compat")


def _run(name, timeout=300):
    path = os.path.join(COMPAT, name)
    if not os.path.exists(path):
        pytest.skip("pkt's tests were not built here (make -C oracle compat needs the reference tree)")
    r = subprocess.run([path], capture_output=True, text=True, timeout=timeout)
    return r.returncode, r.stdout + r.stderr


@pytest.mark.parametrize("name", ["test_task", "test_pipeline"])
def test_pkt_host_tests_unchanged(name):
    rc, out = _run(name)
    assert rc == 0 and "0 failed" in out, out


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["test_task", "test_pipeline", "test_axpy", "test_runtime", "test_paging"])
def test_pkt_tests_unchanged_on_gpu(name):
    rc, out = _run(name)
    assert rc == 0 and "0 failed" in out, out


def test_user_op_program_compiles():
    subprocess.check_call(["make", "-s", "-C", os.path.join(ROOT, "tests", "cpp"),
                           os.path.join(ROOT, "tests", "cpp", "_build", "test_user_op")])


@pytest.mark.gpu
def test_user_op_runs_in_the_megakernel():
    test_user_op_program_compiles()
    r = subprocess.run([os.path.join(ROOT, "tests", "cpp", "_build", "test_user_op")], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0 and "0 failed" in r.stdout, r.stdout + r.stderr
