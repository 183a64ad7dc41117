"""Host logic of bench.py that needs no GPU: the end-to-end pipeline's upload order, the operand
generator and config shared by both arms, and the reference arm's isolation from the product library."""
from __future__ import annotations

import os

import numpy as np
import pytest


@pytest.mark.parametrize("n_a,n_b,bytes_a,bytes_b", [(8, 4, 1024 * 6144, 2048 * 6144), (8, 1, 1, 8), (1, 1, 1, 1),
                                                     (8, 4, 512 * 6144, 7168 * 6144), (3, 5, 100, 100)])
def test_upload_order_sends_every_chunk_once(n_a, n_b, bytes_a, bytes_b):
    import bench
    order = bench.e2e_upload_order(n_a, n_b, bytes_a, bytes_b)
    assert sorted(order) == sorted([("A", i) for i in range(n_a)] + [("B", j) for j in range(n_b)])
    assert order[:2] == [("B", 0), ("A", 0)]
    for kind in "AB":  # each operand's chunks go up in order
        idx = [k for t, k in order if t == kind]
        assert idx == sorted(idx)


def test_upload_order_for_cfg2_keeps_bytes_balanced():
    """cfg2: 8 A chunks of 6.3 MB and 4 B chunks of 12.6 MB alternate two A per B."""
    import bench
    order = bench.e2e_upload_order(8, 4, 1024 * 6144, 2048 * 6144)
    assert [t for t, _ in order] == list("BAABAABAABAA")


def test_bench_generator_matches_package_synth():
    """bench.py's numpy generator (used by both arms) draws exactly the operands of the package's
    synth.make_operands(kind="codes"), which the parity tests use."""
    import bench
    from mxfp6_b200.synth import make_operands
    for M, N, K, er in [(256, 384, 512, (120, 134)), (128, 256, 1000, (118, 136))]:
        A, sA, Bt, sB = bench.synth_codes(M, N, K, 11, er)
        ops = make_operands(M, N, K, kind="codes", seed=11, exp_range=er)
        for a, b in ((A, ops.A), (sA, ops.sA), (Bt, ops.Bt), (sB, ops.sB)):
            assert a.dtype == b.dtype and np.array_equal(a, b)


def test_bench_config_is_shared_by_both_arms():
    import bench
    c = bench.bench_config("cfg2", 4, 1)
    assert c["N_per_gpu"] == 8192 and c["N_total"] == 4 * 8192
    s = bench.bench_config("cfg5", 1, 8)
    assert s["N_per_gpu"] == 3584 and s["N_total"] == 28672
    assert "route" not in c  # the route needs the product library; it is a separate key


def test_reference_arm_maps_no_product_library(tmp_path):
    """The reference arm times the reference's CPU GEMM on operands from bench.py's own numpy
    generator: neither the package nor libmxfp6gemm.so is loaded into its process."""
    import json
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = (
        "import sys, json, bench\n"
        "class A: pass\n"
        "a = A(); a.config = 'cfg1'; a.strong = False; a.shard_of = 1; a.steps = 1; a.warmup = 1\n"
        "a.ref_seconds = 0.2\n"
        "bench.run_reference_arm(a)\n"
        "maps = open('/proc/self/maps').read()\n"
        "print(json.dumps({'pkg': 'mxfp6_b200' in sys.modules, 'so': 'libmxfp6gemm' in maps}))\n")
    r = subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True, timeout=600,
                       env={**os.environ, "PYTHONPATH": root})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [json.loads(x) for x in r.stdout.strip().splitlines()]
    ref_line, probe = lines[0], lines[-1]
    assert probe == {"pkg": False, "so": False}
    assert ref_line["impl"] == "reference" and ref_line["config"] == __import__("bench").bench_config("cfg1", 1, 1)


def test_reference_sweep_table():
    """The reference's headline table as the sweep leg carries it (benchmark_results.md:23-74 of
    eeezio/mxfp6-gemm, its 36 measured rows): M = 2048, unique (N, K), every N a multiple of 128
    (a shape this library runs), and the count-weighted total of the published MI350X latencies
    that the leg's summary compares against."""
    import bench
    rows = bench.REF_SWEEP
    assert bench.REF_SWEEP_M == 2048 and len(rows) == 36
    assert len({(n, k) for n, k, _, _ in rows}) == 36
    assert all(n % 128 == 0 and k > 0 and c > 0 and ms > 0 for n, k, c, ms in rows)
    assert sum(c * ms for _, _, c, ms in rows) == pytest.approx(10.135534, abs=1e-6)
    assert sum(c for _, _, c, _ in rows) == 285
