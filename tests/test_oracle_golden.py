"""Pins the CPU oracle and the host bucketizer to the reference's own outputs.

- packing_kat.json: the reference's verify_packing pairs (preprocess_layer_fixed_gpu.py:336-361)
  run through its pack_fp16_with_index;
- bm_*.npz: layouts written by the reference's bucketize_fp16_packed, plus cutoff /
  selection / output expectations from an independent numpy restatement of
  bucketMul.cl (tests/golden/make_golden.py).
"""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN, GOLDEN_CASES, golden


def rel_err(a, ref):
    a, ref = np.asarray(a, np.float64), np.asarray(ref, np.float64)
    rms = np.sqrt(np.mean(ref * ref))
    return np.max(np.abs(a - ref)) / (rms if rms > 0 else 1.0)


def test_packing_kat(weights_mod):
    kat = json.load(open(os.path.join(GOLDEN, "packing_kat.json")))
    for (v, p), packed, (uv, up) in zip(kat["pairs"], kat["packed_u16"], kat["unpacked"]):
        assert weights_mod.pack_fp16_with_index(v, p) == packed
        val, pos = weights_mod.unpack_fp16_with_index(packed)
        assert pos == p == up
        assert val == uv
        assert abs(val - v) / (abs(v) + 1e-8) < 0.01  # the reference's own tolerance (:356-357)


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_host_bucketizer_matches_reference_layout(weights_mod, case):
    g = golden(case)
    W = g["W"].view(np.float16)
    bw = weights_mod.bucketize_fp16_packed(W)
    np.testing.assert_array_equal(bw.buckets, g["buckets"])
    np.testing.assert_array_equal(bw.stats[:, 3], g["stats3"])
    assert (bw.stats == bw.stats[:, :1]).all()
    np.testing.assert_array_equal(bw.probes, g["probes"])


def test_tie_order_is_stable_in_reference():
    t = json.load(open(os.path.join(GOLDEN, "tie_order.json")))
    assert t["reference_is_stable"] and t["reference_slots"] == t["stable_slots"]


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_oracle_cutoff_and_selection_match_fixture(ora, case):
    g = golden(case)
    k = 0
    for xi, kind in enumerate(g["x_kinds"]):
        x = g["x"][xi]
        for eff in g["efforts"]:
            P = min(len(x), 4096)
            assert ora.target_count(float(eff), P) == g["target"][k]
            cut, iters = ora.find_cutoff(x, g["probes"], float(eff))
            assert np.float32(cut).view(np.uint32) == g["cutoff"][k].view(np.uint32), (kind, eff)
            assert iters == g["iters"][k], (kind, eff)
            rows = ora.prepare_dispatch(x, g["stats3"], 1, cut)
            sel = np.unpackbits(g["sel_packed"][k])[: len(g["stats3"])].astype(bool)
            np.testing.assert_array_equal(rows, np.nonzero(sel)[0])
            out = ora.bucket_mul(g["buckets"], x, rows)
            assert rel_err(out, g["out"][k]) < 1e-5, (kind, eff)
            k += 1


def test_oracle_edge_semantics(ora):
    g = golden("bm_256x64.npz")
    zeros = np.zeros(64, np.float32)
    cut, _ = ora.find_cutoff(zeros, g["probes"], 0.25)
    assert cut == 0.0
    # 1e5*|0*s| = 0 >= 0: every row is selected for a zero input (bucketMul.cl:380 uses >=)
    assert len(ora.prepare_dispatch(zeros, g["stats3"], 1, cut)) == 16 * 64


def test_oracle_file_layout_stride(ora, weights_mod):
    """stats_stride=4 on the [R][4] file layout selects exactly what stride 1 selects."""
    g = golden("bm_128x512.npz")
    bw = weights_mod.bucketize_fp16_packed(g["W"].view(np.float16))
    x = g["x"][0]
    o4, n4, c4 = ora.bucketmul_full(x, bw.stats, 4, bw.probes, bw.buckets, 0.25)
    o1, n1, c1 = ora.bucketmul_full(x, bw.stats[:, 3].copy(), 1, bw.probes, bw.buckets, 0.25)
    assert n4 == n1 and c4 == c1
    np.testing.assert_array_equal(o4, o1)


def test_oracle_all_rows_close_to_dense(ora):
    """Accumulating every bucket row reproduces the dense GEMV up to the packing error
    (the 4 slot bits stay in the multiplicand, so ~1% per weight)."""
    g = golden("bm_128x512.npz")
    x = g["x"][0]
    R = g["buckets"].shape[0]
    out = ora.bucket_mul(g["buckets"], x, np.arange(R, dtype=np.int32))
    dense = ora.dense_gemv(g["W"], x)
    assert rel_err(out, dense) < 2e-2


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_oracle_all_rows_equal_the_packed_dense_matrix(ora, weights_mod, case):
    """The dense path's matrix: bucketMul over every bucket row (bucketMul.cl:392-497) is the
    fp64 product with W' = (bits(W) & 0xFFF0) | (row & 15) up to fp32 summation, on the
    reference's own bucket fixtures and every fixture input."""
    g = golden(case)
    R = g["buckets"].shape[0]
    wp = weights_mod.dense_packed(g["W"].view(np.float16))
    for x in g["x"]:
        out = ora.bucket_mul(g["buckets"], x, np.arange(R, dtype=np.int32))
        ref = ora.dense_gemv(wp, x)
        assert rel_err(out, ref) < 1e-5, case


def test_oracle_fp16_roundtrip(ora):
    L = ora.lib()
    for v in [0.0, -0.0, 1.0, -2.5, 65504.0, 1e-7, 6.1e-5, 3.14159, 70000.0]:
        h = L.ora_float_to_half(v)
        assert h == int(np.float16(v).view(np.uint16)), v
    for h in range(0, 65536, 97):
        f = L.ora_half_to_float(h)
        ref = np.uint16(h).view(np.float16).astype(np.float32)
        assert (np.isnan(f) and np.isnan(ref)) or np.float32(f) == ref
