#!/usr/bin/env python3
"""Write the golden fixtures in tests/golden/ (run in a container that has the reference).

Layout fixtures come from the reference itself: its preprocess_layer_fixed_gpu.py is
imported from the reference checkout and its bucketize_fp16_packed (preprocess_layer_fixed_
gpu.py:110-242) and pack_fp16_with_index (:40-66, the verify_packing pairs of :340-346) are
run on seeded inputs.  Cutoff / selection / output expectations are written by an
independent numpy restatement of bucketMul.cl:68-214 (cutoff), :351-386 (dispatch) and
:392-447 (accumulation): the reference's OpenCL cannot execute here, so those values are a
second restatement the C oracle is cross-checked against, not an executed reference.

Usage:  python tests/golden/make_golden.py --reference <reference checkout>
        (or IAM_REFERENCE_DIR=<reference checkout> python tests/golden/make_golden.py)
The fixtures are small .npz files; nothing here is needed at test time except them.
"""
import argparse
import importlib.util
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
EFFORTS = [0.05, 0.1, 0.25, 0.5, 1.0]
PROBES = 4096


def load_reference(ref_dir):
    path = os.path.join(ref_dir, "preprocess_layer_fixed_gpu.py")
    spec = importlib.util.spec_from_file_location("ref_preprocess", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


# ---------------------------------------------------------------- numpy restatement


def np_importance(x, s):
    x = np.asarray(x, np.float32)
    s = np.asarray(s, np.float32)
    return (np.float32(1e5) * np.abs(x * s)).astype(np.float32)


def np_cutoff(x, probes_u16, effort):
    """bucketMul.cl:68-214 + bucket_mul.hpp:164, vectorised."""
    P = min(len(x), PROBES)
    quantile = int((P - 1) * (1.0 - float(np.float32(effort))))
    target = P - quantile
    imp = np_importance(x[:P], probes_u16[:P].view(np.float16).astype(np.float32))
    lo, hi = np.float32(imp.min()), np.float32(imp.max())
    mid = np.float32((lo + hi) / np.float32(2))
    min_c, max_c = P, 0
    for it in range(20):
        cnt = int(np.count_nonzero(imp > mid))
        if cnt < target:
            hi, max_c = mid, cnt
        else:
            lo, min_c = mid, cnt
        nxt = np.float32((lo + hi) / np.float32(2))
        if cnt == target or np.float32(hi - lo) < np.float32(1e-5) or abs(max_c - min_c) < 3:
            return mid, it + 1, target
        mid = nxt
    return mid, 20, target


def np_select(x, stats3_u16, cutoff):
    """bucketMul.cl:351-386: row r selected iff 1e5*|x[r//16]*stats[r][3]| >= cutoff."""
    R = len(stats3_u16)
    xi = np.repeat(np.asarray(x, np.float32), 16)[:R]
    imp = np_importance(xi, stats3_u16.view(np.float16).astype(np.float32))
    return imp >= np.float32(cutoff)


def np_bucket_mul(buckets_u16, x, sel):
    """bucketMul.cl:392-447 + :453-497: unmasked packed weight times x into slot bits&15."""
    R, C = buckets_u16.shape
    rows = np.nonzero(sel)[0]
    out = np.zeros((C, 16), np.float64)
    w = buckets_u16[rows]  # (S, C)
    wf = w.view(np.float16).astype(np.float64)
    slot = (w & 15).astype(np.int64)
    xv = np.asarray(x, np.float64)[rows // 16][:, None]
    np.add.at(out, (np.broadcast_to(np.arange(C), w.shape), slot), xv * wf)
    return out.reshape(-1).astype(np.float32)


# ---------------------------------------------------------------- cases


def make_x(kind, n, rng):
    if kind == "gaussian":
        return rng.standard_normal(n).astype(np.float32)
    if kind == "uniform":
        return rng.uniform(-1.0, 1.0, n).astype(np.float32)
    if kind == "zeros":
        return np.zeros(n, np.float32)
    if kind == "ones":
        return np.ones(n, np.float32)
    if kind == "outliers":  # the outlier inputs: 1% of channels scaled x20
        x = rng.standard_normal(n).astype(np.float32)
        idx = rng.choice(n, max(1, n // 100), replace=False)
        x[idx] *= np.float32(20.0)
        return x
    raise ValueError(kind)


def bucketize_case(ref, name, out_dim, in_dim, seed, ties=False):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((out_dim, in_dim)) * 0.02).astype(np.float16)
    if ties:
        # few distinct magnitudes, both signs: forces equal |w| inside buckets
        W = (np.round(W.astype(np.float32) / np.float32(0.01)) * np.float32(0.01)).astype(np.float16)
    bm = ref.bucketize_fp16_packed(W, bsize=16)
    buckets = bm.buckets[0].view(np.uint16)
    stats = bm.stats[0].view(np.uint16)
    probes = bm.probes[0].view(np.uint16)
    assert (stats == stats[:, :1]).all(), "reference writes identical stats channels"
    case = dict(W=W.view(np.uint16), buckets=buckets, stats3=stats[:, 3].copy(),
                probes=probes.copy(), ties=np.int32(ties))
    kinds = ["gaussian", "uniform", "zeros", "ones", "outliers"]
    xs, exp_cut, exp_it, exp_tgt, exp_sel, exp_out = [], [], [], [], [], []
    for k, kind in enumerate(kinds):
        x = make_x(kind, in_dim, np.random.default_rng(1000 + seed * 10 + k))
        xs.append(x)
        for eff in EFFORTS:
            cut, it, tgt = np_cutoff(x, probes, eff)
            sel = np_select(x, case["stats3"], cut)
            exp_cut.append(np.float32(cut))
            exp_it.append(it)
            exp_tgt.append(tgt)
            exp_sel.append(np.packbits(sel))
            exp_out.append(np_bucket_mul(buckets, x, sel))
    case.update(x=np.stack(xs), x_kinds=np.array(kinds), efforts=np.array(EFFORTS, np.float32),
                cutoff=np.array(exp_cut, np.float32), iters=np.array(exp_it, np.int32),
                target=np.array(exp_tgt, np.int32), sel_packed=np.stack(exp_sel),
                out=np.stack(exp_out))
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **case)
    print(f"wrote {name}.npz  W={out_dim}x{in_dim} ties={ties}")


def packing_kat(ref):
    pairs = [(1.5, 0), (-0.5, 7), (0.0, 15), (3.14159, 8), (-2.71828, 3)]  # :340-346
    packed = [int(np.float16(ref.pack_fp16_with_index(v, p)).view(np.uint16)) for v, p in pairs]
    unpacked = [ref.unpack_fp16_with_index(np.uint16(b).view(np.float16)) for b in packed]
    with open(os.path.join(HERE, "packing_kat.json"), "w") as f:
        json.dump({"pairs": pairs, "packed_u16": packed,
                   "unpacked": [[float(v), int(p)] for v, p in unpacked]}, f, indent=1)
    print("wrote packing_kat.json")


def torch_tie_order(ref):
    """Record whether the reference's torch.argsort orders equal |w| like a stable sort."""
    W = np.array([[0.5], [-0.5], [0.25], [0.5]] * 4, np.float16)  # out=16, in=1, many ties
    bm = ref.bucketize_fp16_packed(W, bsize=16)
    slots = (bm.buckets[0].view(np.uint16)[:, 0] & 15).tolist()
    mags = np.abs(W[:, 0].astype(np.float32))
    stable = sorted(range(16), key=lambda s: (-mags[s], s))
    with open(os.path.join(HERE, "tie_order.json"), "w") as f:
        json.dump({"reference_slots": slots, "stable_slots": stable,
                   "reference_is_stable": slots == stable}, f, indent=1)
    print("tie order stable:", slots == stable)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("IAM_REFERENCE_DIR"),
                    help="the reference checkout (default: $IAM_REFERENCE_DIR)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set IAM_REFERENCE_DIR")
    ref = load_reference(args.reference)
    packing_kat(ref)
    torch_tie_order(ref)
    bucketize_case(ref, "bm_256x64", 256, 64, seed=0)
    bucketize_case(ref, "bm_128x512", 128, 512, seed=1)
    bucketize_case(ref, "bm_48x96_ties", 48, 96, seed=2, ties=True)
    bucketize_case(ref, "bm_16x4096", 16, 4096, seed=3)


if __name__ == "__main__":
    sys.exit(main())
