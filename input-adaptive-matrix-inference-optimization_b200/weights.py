"""Host-side weight utilities: the reference's bucket layout and its on-disk format.

bucketize_fp16_packed restates preprocess_layer_fixed_gpu.py:110-242 with numpy (the same
numpy calls for the two means, so the float32 summation order is numpy's own; |w| ties are
ordered by lower original slot, which is what the reference's torch.argsort produced on
the recorded tie fixture).  save_bucketmul_binary / load_bucketmul_binary follow
preprocess_layer_fixed_gpu.py:245-282 and binary_loader.hpp:59-193 (including its size
validation).  save_npy_fp16 / load_npy_fp16 follow model.hpp:54-81 (.npy, raw fp16 payload).
"""
import os
from dataclasses import dataclass

import numpy as np


@dataclass
class BucketWeight:
    buckets: np.ndarray  # uint16 [16*in_dim][out_dim/16]
    stats: np.ndarray    # uint16 [16*in_dim][4]
    probes: np.ndarray   # uint16 [in_dim]
    in_dim: int
    out_dim: int
    bsize: int = 16


def bucketize_fp16_packed(W, bsize=16):
    """W: float16 [out_dim][in_dim] -> BucketWeight (preprocess_layer_fixed_gpu.py:110-242)."""
    W = np.asarray(W, dtype=np.float16)
    out_dim, in_dim = W.shape
    if out_dim % bsize:
        raise ValueError(f"{out_dim} not divisible by {bsize}")
    C = out_dim // bsize
    W_T = W.T.astype(np.float32, copy=False)               # :145 (transposed layout kept)
    probes = np.mean(np.abs(W_T), axis=1).astype(np.float16)  # :154
    Wb = W_T.reshape(in_dim, C, bsize)
    order = np.argsort(-np.abs(Wb), axis=2, kind="stable")  # :170 (descending |w|)
    sv = np.take_along_axis(Wb, order, axis=2)              # :174
    vals = np.transpose(sv, (0, 2, 1)).reshape(in_dim * bsize, C)      # :183-188
    pos = np.transpose(order, (0, 2, 1)).reshape(in_dim * bsize, C)
    bits = vals.astype(np.float16).view(np.uint16)
    buckets = (bits & 0xFFF0) | (pos.astype(np.uint16) & 0x000F)       # :196
    avg = np.mean(np.abs(vals.astype(np.float32)), axis=1).astype(np.float16)  # :212-213
    stats = np.repeat(avg.view(np.uint16)[:, None], 4, axis=1)          # :217-221
    return BucketWeight(buckets.astype(np.uint16), np.ascontiguousarray(stats),
                        probes.view(np.uint16).copy(), in_dim, out_dim, bsize)


def dense_from_buckets(buckets):
    """Dense uint16 W'[16*C][in] from buckets[16*in][C]: each packed word returns to row
    16*c + slot (slot = its low 4 bits, preprocess_layer_fixed_gpu.py:196), column i.  bucketMul
    with every bucket row selected multiplies by exactly this matrix (bucketMul.cl:430-434)."""
    buckets = np.asarray(buckets, dtype=np.uint16)
    R, C = buckets.shape
    in_dim = R // 16
    b = buckets.reshape(in_dim, 16, C)                        # [i][rank][c]
    slot = (b & 0xF).astype(np.int64)
    dense = np.zeros((C, 16, in_dim), dtype=np.uint16)        # [c][slot][i]
    ii = np.broadcast_to(np.arange(in_dim)[:, None, None], b.shape)
    cc = np.broadcast_to(np.arange(C)[None, None, :], b.shape)
    dense[cc, slot, ii] = b
    return dense.reshape(C * 16, in_dim)


def dense_packed(W):
    """The same matrix straight from W (float16 [out][in]): (bits & 0xFFF0) | (row & 15)."""
    bits = np.asarray(W, dtype=np.float16).view(np.uint16)
    rows = np.arange(bits.shape[0], dtype=np.uint16)[:, None]
    return (bits & np.uint16(0xFFF0)) | (rows & np.uint16(0xF))


def pack_fp16_with_index(value, position):
    """preprocess_layer_fixed_gpu.py:40-66."""
    bits = int(np.float16(value).view(np.uint16))
    return (bits & 0xFFF0) | (position & 0xF)


def unpack_fp16_with_index(packed_u16):
    """preprocess_layer_fixed_gpu.py:69-89 -> (value, position)."""
    b = int(packed_u16)
    return float(np.uint16(b & 0xFFF0).view(np.float16)), b & 0xF


def save_bucketmul_binary(bw, path):
    """Writes {path}_buckets.bin / _stats.bin / _probes.bin / _meta.txt (:245-282)."""
    bw.buckets.astype(np.uint16).tofile(f"{path}_buckets.bin")
    bw.stats.astype(np.uint16).tofile(f"{path}_stats.bin")
    bw.probes.astype(np.uint16).tofile(f"{path}_probes.bin")
    R, C = bw.buckets.shape
    with open(f"{path}_meta.txt", "w") as f:
        f.write("# BucketMul Weight Metadata\n# All arrays are FP16 (2 bytes per element)\n\n")
        f.write(f"buckets_shape: 1 {R} {C}\n")
        f.write(f"stats_shape: 1 {R} 4\n")
        f.write(f"probes_shape: 1 {bw.in_dim}\n")
        f.write(f"in_dim: {bw.in_dim}\nout_dim: {bw.out_dim}\nbsize: {bw.bsize}\ndtype: float16\n")


class WeightFormatError(IOError):
    pass


def read_meta(meta_file):
    """binary_loader.hpp:59-102 (keys, comments, missing-dimension check)."""
    if not os.path.exists(meta_file):
        raise WeightFormatError(f"Cannot open metadata file: {meta_file}")
    meta = {}
    with open(meta_file) as f:
        for line in f:
            line = line.strip()
            if not line or line.startswith("#"):
                continue
            key, _, rest = line.partition(" ")
            meta[key.rstrip(":")] = [int(v) for v in rest.split()] if key != "dtype:" else rest.strip()
    if not meta.get("in_dim", [0])[0] or not meta.get("out_dim", [0])[0]:
        raise WeightFormatError("Invalid metadata - missing dimensions")
    return meta


def _read_exact(path, n_elems):
    """binary_loader.hpp:105-134: the file size must equal the metadata size."""
    if not os.path.exists(path):
        raise WeightFormatError(f"Cannot open binary file: {path}")
    size = os.path.getsize(path)
    if size != 2 * n_elems:
        raise WeightFormatError(f"File size mismatch: {path} has {size} bytes, expected {2 * n_elems}")
    return np.fromfile(path, dtype=np.uint16)


def load_bucketmul_binary(path):
    meta = read_meta(f"{path}_meta.txt")
    b0, b1, b2 = meta["buckets_shape"]
    s0, s1, s2 = meta["stats_shape"]
    p0, p1 = meta["probes_shape"]
    buckets = _read_exact(f"{path}_buckets.bin", b0 * b1 * b2).reshape(b0 * b1, b2)
    stats = _read_exact(f"{path}_stats.bin", s0 * s1 * s2).reshape(s0 * s1, s2)
    probes = _read_exact(f"{path}_probes.bin", p0 * p1)
    return BucketWeight(buckets, stats, probes, meta["in_dim"][0], meta["out_dim"][0], meta["bsize"][0])


def save_npy_fp16(path, arr):
    np.save(path, np.asarray(arr, dtype=np.float16))


def load_npy_fp16(path):
    """model.hpp:54-81: the payload after the .npy header, as raw fp16 bits."""
    if not os.path.exists(path):
        raise WeightFormatError(f"Cannot open: {path}")
    with open(path, "rb") as f:
        data = f.read()
    if data[:6] != b"\x93NUMPY":
        raise WeightFormatError(f"not a .npy file: {path}")
    hlen = int.from_bytes(data[8:10], "little")
    return np.frombuffer(data[10 + hlen:], dtype=np.uint16).copy()


MATRICES = ("q", "k", "v", "o", "gate", "up", "down")


def layer_weight_name(layer, short):
    """transformer layer file prefix (preprocess_layer_fixed_gpu.py:323)."""
    return f"layer{layer}_{short}_proj_bucketmul_fp16"
