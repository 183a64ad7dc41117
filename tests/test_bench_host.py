"""Host logic of bench.py that needs no GPU: the end-to-end pipeline's upload order."""
from __future__ import annotations

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
