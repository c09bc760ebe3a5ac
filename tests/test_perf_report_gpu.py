"""pkt_b200.perf_report: per-role counters of an MLP step on one GPU, with the
SGD fused into the gradient epilogue and with the fused data-parallel path at
world size 1."""
import pytest

from _gpu import require_gpu

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("grad_mode", ["0", "2"])
def test_perf_report_prints_counters(capsys, grad_mode):
    require_gpu()
    from pkt_b200 import perf_report
    perf_report.main(["--dims", "256,512,128", "--batch", "1024", "--steps", "2", "--warmup", "1",
                      "--grad-mode", grad_mode])
    out = capsys.readouterr().out
    assert "ms/step" in out
    for name in ("mma_issue", "kblocks", "epi_gemm", "ctrl_dep_wait"):
        assert name in out


@pytest.mark.parametrize("grad_mode", ["0", "1", "2"])
def test_trace_report_one_step(capsys, grad_mode):
    """pkt_b200.trace_report: the per-task trace of one step, its layer hops and
    (fused data parallel at world size 1) the reduce tasks' wait and work."""
    require_gpu()
    from pkt_b200 import trace_report
    trace_report.main(["--dims", "256x5", "--batch", "1024", "--warmup", "2", "--grad-mode", grad_mode])
    out = capsys.readouterr().out
    assert "MMA issuer" in out and "layer hops" in out
    assert "fwd:" in out and "dgrad:" in out
    if grad_mode == "2":
        assert "dp_reduce" in out and "wait" in out
