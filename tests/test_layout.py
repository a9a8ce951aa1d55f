"""Stripe map and derivations: the Python restatements (package and oracle), the C
restatement and — where it was built in this container — the reference's own
common/kv_layout.h (oracle/_ref), all against fixtures recorded from test/kv_layout_ref.py
and the reference's KATs (test/test_layout.py:13-59, test/test_allocator.py:79-93)."""
import json
import os

import pytest

import oracle
from conftest import GOLDEN
from kv_offload_proto_b200 import offload, pool, workload

with open(os.path.join(GOLDEN, "layout.json")) as f:
    FX = json.load(f)


@pytest.mark.parametrize("g", FX["grid"], ids=lambda g: "S{}N{}".format(g["S"], g["N"]))
def test_node_and_seg_row(g):
    S, N = g["S"], g["N"]
    lib = oracle.lib()
    ref = oracle.ref_layout_lib()
    for row, node, sr in zip(g["rows"], g["node"], g["seg_row"]):
        assert pool.node_of(row, S, N) == node and oracle.node_of(row, S, N) == node
        assert pool.seg_row_of(row, S, N) == sr and oracle.seg_row_of(row, S, N) == sr
        assert lib.ko_node_of(row, S, N) == node and lib.ko_seg_row(row, S, N) == sr
        if ref is not None:
            assert ref.ref_node_of(row, S, N) == node and ref.ref_seg_row_of(row, S, N) == sr


def test_per_layer_seg_rows_and_offsets():
    ref = oracle.ref_layout_lib()
    for lr, n, want in FX["plsr"]:
        assert pool.per_layer_seg_rows(lr, n) == want
        if ref is not None and lr > 0:
            assert ref.ref_per_layer_seg_rows(lr, n) == want
    for layer, row, S, N, p, rb, off, addr in FX["seg_offset"]:
        assert oracle.seg_offset(layer, row, S, N, p, rb) == off
        assert 0x10000 + (layer * p + pool.seg_row_of(row, S, N)) * rb == addr
        if ref is not None:
            assert ref.ref_seg_offset(layer, row, S, N, p, rb) == off


def test_reference_layout_kats():
    # test/test_layout.py:31-37 and :46-52, restated.
    assert [pool.node_of(r, 1, 2) for r in range(6)] == [0, 1, 0, 1, 0, 1]
    assert [pool.node_of(r, 64, 2) for r in (0, 63, 64, 127, 128)] == [0, 0, 1, 1, 0]
    assert oracle.seg_offset(1, 3, 1, 2, 50, 128) == 6528
    assert [pool.seg_row_of(r, 1, 2) for r in range(8)] == [0, 0, 1, 1, 2, 2, 3, 3]


def test_stripe_map_collides_for_s_gt_1():
    """The reference map drops row % S: with S=16, N=8 and 32768 rows only 2048 distinct
    (node, segRow) pairs exist; the opt-in injective map is a bijection."""
    S, N, rows = 16, 8, 32768
    ref_pairs = {(pool.node_of(r, S, N), pool.seg_row_of(r, S, N)) for r in range(rows)}
    inj_pairs = {(pool.node_of(r, S, N), pool.seg_row_of(r, S, N, injective=True)) for r in range(rows)}
    assert len(ref_pairs) == 2048
    assert len(inj_pairs) == rows
    plsr = pool.per_layer_seg_rows_injective(rows, S, N)
    assert max(sr for _, sr in inj_pairs) < plsr
    for r in range(0, rows, 97):
        assert oracle.lib().ko_seg_row_injective(r, S, N) == pool.seg_row_of(r, S, N, injective=True)


def test_injective_equals_reference_at_s1():
    for N in (1, 2, 7):
        for r in range(500):
            assert pool.seg_row_of(r, 1, N, injective=True) == pool.seg_row_of(r, 1, N)


def test_validate_cases_reference_semantics():
    ref = oracle.ref_layout_lib()
    for (L, rows, rb, S, N), ok in FX["validate"]:
        mine = 1 <= N <= 64 and L >= 1 and rows >= 1 and rb > 0 and rb % 128 == 0 and S >= 1
        assert mine == ok
        if ref is not None:
            plsr = pool.per_layer_seg_rows(rows, N) if N > 0 else 0
            assert (ref.ref_validate(N, L, rows, plsr, rb, S) == 0) == ok


def test_ht_size_align_and_fingerprint():
    for p, k, want in FX["ht_size"]:
        assert offload.compute_ht_size(p, k) == want == oracle.ht_size(p, k)
    for v, a, want in FX["align"]:
        assert offload.align(v, a) == want
    for r, l, k, want in FX["row_word"]:
        assert workload.row_word(r, l, k) == want
        assert int(workload.fingerprint_rows([r], l, k + 1)[0, k]) == want
