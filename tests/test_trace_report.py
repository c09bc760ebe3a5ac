"""pkt_b200.trace_report's analysis on a synthetic trace (no GPU): the per-GEMM
table, the layer-hop breakdown and the SIMT task table, including the fused
data-parallel reduce's wait / work split."""
import numpy as np

from pkt_b200 import trace_report as T


def record(cta, op, stamps, gemm=0, tm=0, tn=0):
    w0 = cta | (op << 16) | (gemm << 32) | (tm << 48) | (tn << 56)
    return [w0] + list(stamps)


def test_hops_and_simt_tables():
    dims = [64, 64, 64]  # GEMMs registered: fwd0 fwd1 dgrad1 wgrad1 wgrad0
    names = T.gemm_names(dims)
    assert names == ["fwd0", "fwd1", "dgrad1", "wgrad1", "wgrad0"]
    g = {n: i for i, n in enumerate(names)}
    base = 1_000_000
    us = lambda v: base + int(v * 1000)  # noqa: E731
    tr = []
    # row block 0: two fwd0 tiles end at 10 and 11 us; the fwd1 tile is ready at 12,
    # loads at 12.5, MMA 13 -> 15, epilogue 15.5 -> 17
    tr.append(record(0, 3, [us(0), us(1), us(1.5), us(2), us(8), us(8.5), us(10)], g["fwd0"], 0, 0))
    tr.append(record(1, 3, [us(0), us(1), us(1.5), us(2), us(9), us(9.5), us(11)], g["fwd0"], 0, 1))
    tr.append(record(2, 3, [us(5), us(12), us(12.5), us(13), us(15), us(15.5), us(17)], g["fwd1"], 0, 0))
    # a fused data-parallel reduce: starts at 20, its wait ends at 23, done at 30
    tr.append(record(3, 33, [us(18), us(19), us(23), 0, 0, us(20), us(30)]))
    tr.append(record(3, 21, [us(18), us(19), 0, 0, 0, us(31), us(32)]))
    rep = T.analyse(np.array(tr, dtype=np.uint64), dims)
    assert rep["gemm_tiles"] == 3 and rep["tasks"] == 5
    h = rep["hops"]["fwd"]
    assert abs(h["producer_spread"] - 1.0) < 1e-9
    assert abs(h["to_ready"] - 1.0) < 1e-9  # 11 -> 12
    assert abs(h["ready_to_load"] - 0.5) < 1e-9
    assert abs(h["load_to_mma"] - 0.5) < 1e-9
    assert abs(h["mma"] - 2.0) < 1e-9
    assert abs(h["epilogue"] - 1.5) < 1e-9
    assert abs(h["hop"] - 6.0) < 1e-9  # 11 -> 17
    r = rep["simt"]["dp_reduce"]
    assert r["tasks"] == 1 and abs(r["run_us_mean"] - 10.0) < 1e-9
    assert abs(r["wait_us_mean"] - 3.0) < 1e-9 and abs(r["work_us_mean"] - 7.0) < 1e-9
    assert rep["simt"]["loss_reduce"]["tasks"] == 1
    T.print_report(rep)  # formats without error
