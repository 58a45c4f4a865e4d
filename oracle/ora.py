"""ctypes binding of oracle/libiam_oracle.so -- TEST INFRASTRUCTURE ONLY.

Imported only by tests/, __graft_entry__.smoke() (as the checker) and bench.py's
cpu_baseline / --impl reference leg (as the timed CPU restatement).  Never by the product.
See iam_oracle.h for what each function restates and how parity is pinned.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libiam_oracle.so")

_vp = ctypes.c_void_p
_lib = None


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        L.ora_half_to_float.restype = ctypes.c_float
        L.ora_half_to_float.argtypes = [ctypes.c_uint16]
        L.ora_float_to_half.restype = ctypes.c_uint16
        L.ora_float_to_half.argtypes = [ctypes.c_float]
        L.ora_target_count.restype = ctypes.c_int
        L.ora_target_count.argtypes = [ctypes.c_float, ctypes.c_int]
        L.ora_find_cutoff.restype = ctypes.c_float
        L.ora_find_cutoff.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp]
        L.ora_prepare_dispatch.restype = ctypes.c_long
        L.ora_prepare_dispatch.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_long, ctypes.c_long, ctypes.c_int,
                                           ctypes.c_float, _vp]
        L.ora_bucket_mul.restype = None
        L.ora_bucket_mul.argtypes = [_vp, ctypes.c_int, _vp, ctypes.c_long, _vp, ctypes.c_long, _vp, ctypes.c_int]
        L.ora_bucketmul_full.restype = ctypes.c_long
        L.ora_bucketmul_full.argtypes = [_vp, _vp, ctypes.c_int, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_long, ctypes.c_float, _vp, _vp, _vp, ctypes.c_int]
        L.ora_dense_gemv.restype = None
        L.ora_dense_gemv.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp]
        L.ora_rmsnorm.restype = None
        L.ora_rmsnorm.argtypes = [_vp, ctypes.c_int, ctypes.c_float, _vp, _vp]
        L.ora_rope_table.restype = None
        L.ora_rope_table.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_double, _vp]
        L.ora_rope_apply.restype = None
        L.ora_rope_apply.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp]
        L.ora_silu_mul.restype = None
        L.ora_silu_mul.argtypes = [_vp, _vp, ctypes.c_int, _vp]
        L.ora_lm_head.restype = None
        L.ora_lm_head.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp, ctypes.c_int]
        L.ora_model_forward.restype = ctypes.c_int
        L.ora_model_forward.argtypes = [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_float, _vp, _vp, ctypes.c_int]
        L.ora_model_forward_dense.restype = ctypes.c_int
        L.ora_model_forward_dense.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int]
        L.ora_attention.restype = None
        L.ora_attention.argtypes = [_vp, _vp, _vp, _vp, ctypes.c_int, _vp]
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _u16(a):
    return np.ascontiguousarray(a, dtype=np.uint16)


def target_count(effort, P):
    return lib().ora_target_count(effort, P)


def find_cutoff(x, probes, effort):
    x, probes = _f32(x), _u16(probes)
    P = min(len(x), 4096)
    it = ctypes.c_int(0)
    c = lib().ora_find_cutoff(_p(x), _p(probes), P, target_count(effort, P), ctypes.byref(it))
    return np.float32(c), it.value


def prepare_dispatch(x, stats, stats_stride, cutoff, in_dim=None, row0=0, expert_size=None):
    x, stats = _f32(x), _u16(stats)
    in_dim = len(x) if in_dim is None else in_dim
    expert_size = (stats.size // stats_stride - row0) if expert_size is None else expert_size
    rows = np.empty(max(expert_size, 1), np.int32)
    n = lib().ora_prepare_dispatch(_p(x), _p(stats), stats_stride, row0, expert_size, in_dim, cutoff, _p(rows))
    return rows[:n].copy()


def bucket_mul(buckets, x, rows, row0=0, nthreads=1):
    buckets, x = _u16(buckets), _f32(x)
    rows = np.ascontiguousarray(rows, np.int32)
    cols = buckets.shape[1]
    out = np.empty(16 * cols, np.float32)
    lib().ora_bucket_mul(_p(buckets), cols, _p(x), row0, _p(rows), len(rows), _p(out), nthreads)
    return out


def bucketmul_full(x, stats, stats_stride, probes, buckets, effort, expert_no=0, in_dim=None, expert_size=None,
                   nthreads=1):
    """-> (out[16*C], selected_count, cutoff)"""
    x, stats, probes, buckets = _f32(x), _u16(stats), _u16(probes), _u16(buckets)
    in_dim = len(x) if in_dim is None else in_dim
    cols = buckets.shape[1]
    expert_size = 16 * in_dim if expert_size is None else expert_size
    out = np.empty(16 * cols, np.float32)
    rows = np.empty(max(expert_size, 1), np.int32)
    cut = ctypes.c_float(0)
    n = lib().ora_bucketmul_full(_p(x), _p(stats), stats_stride, _p(probes), _p(buckets), expert_no, in_dim, cols,
                                 expert_size, effort, _p(out), _p(rows), ctypes.byref(cut), nthreads)
    return out, int(n), np.float32(cut.value)


def dense_gemv(W_u16, x):
    W_u16, x = _u16(W_u16), _f32(x)
    M, N = W_u16.shape
    out = np.empty(M, np.float64)
    lib().ora_dense_gemv(_p(W_u16), M, N, _p(x), _p(out))
    return out


def rmsnorm(x, gain_u16, eps=1e-5):
    x = _f32(x)
    out = np.empty_like(x)
    lib().ora_rmsnorm(_p(x), len(x), eps, _p(_u16(gain_u16)) if gain_u16 is not None else None, _p(out))
    return out


def rope_table(pos, head_dim, theta=1e6):
    cs = np.empty(head_dim, np.float32)
    lib().ora_rope_table(pos, head_dim, theta, _p(cs))
    return cs


def rope_apply(x, n_heads, head_dim, cs):
    x = _f32(x)
    out = np.empty_like(x)
    lib().ora_rope_apply(_p(x), n_heads, head_dim, _p(_f32(cs)), _p(out))
    return out


def silu_mul(g, u):
    g, u = _f32(g), _f32(u)
    out = np.empty_like(g)
    lib().ora_silu_mul(_p(g), _p(u), len(g), _p(out))
    return out


def lm_head(W_u16, x, nthreads=1):
    W_u16, x = _u16(W_u16), _f32(x)
    rows, cols = W_u16.shape
    out = np.empty(rows, np.float32)
    lib().ora_lm_head(_p(W_u16), rows, cols, _p(x), _p(out), nthreads)
    return out


def attention(cfg, q_roped, k_layer, v_layer, n_tokens):
    """ora_attention (aux.cl:497-540, :204-225, :370-384): every query head over the first
    n_tokens of one layer's fp16 caches k/v [n_kv_heads][max_ctx][head_dim]; q post-RoPE."""
    c = _Config(cfg["dim"], cfg["n_layers"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"], cfg["ffn_dim"],
                cfg["vocab"], cfg["max_ctx"], cfg.get("norm_eps", 1e-5), cfg.get("rope_theta", 1e6))
    q = _f32(q_roped)
    out = np.empty(cfg["n_heads"] * cfg["head_dim"], np.float32)
    lib().ora_attention(ctypes.byref(c), _p(q), _p(_u16(k_layer)), _p(_u16(v_layer)), n_tokens, _p(out))
    return out


# ---------------------------------------------------------------- model (ctypes structs)

class _Config(ctypes.Structure):
    _fields_ = [("dim", ctypes.c_int), ("n_layers", ctypes.c_int), ("n_heads", ctypes.c_int),
                ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("ffn_dim", ctypes.c_int),
                ("vocab", ctypes.c_int), ("max_ctx", ctypes.c_int), ("norm_eps", ctypes.c_float),
                ("rope_theta", ctypes.c_double)]


class _BM(ctypes.Structure):
    _fields_ = [("buckets", _vp), ("stats", _vp), ("probes", _vp), ("in_dim", ctypes.c_int),
                ("out_dim", ctypes.c_int), ("stats_stride", ctypes.c_int)]


class _Layer(ctypes.Structure):
    _fields_ = [("attn_norm", _vp), ("ffn_norm", _vp)] + [(n, _BM) for n in ("wq", "wk", "wv", "wo", "w1", "w2", "w3")]


class _Model(ctypes.Structure):
    _fields_ = [("cfg", _Config), ("embed", _vp), ("final_norm", _vp), ("lm_head", _vp), ("layers", _vp),
                ("k_cache", _vp), ("v_cache", _vp)]


class OracleModel:
    """Decode-step oracle over host numpy weights (dict layout of iam_b200 model weights).

    cfg: dict(dim, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, max_ctx, norm_eps, rope_theta)
    weights: dict(embed [V][D] u16, final_norm [D] u16, lm_head [V][D] u16 (may be embed),
                  layers: list of dict(attn_norm, ffn_norm, q/k/v/o/gate/up/down -> BucketWeight))
    """

    _MAP = {"wq": "q", "wk": "k", "wv": "v", "wo": "o", "w1": "gate", "w2": "down", "w3": "up"}

    def __init__(self, cfg, weights):
        self.cfg = dict(cfg)
        self._keep = []
        c = _Config(cfg["dim"], cfg["n_layers"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"],
                    cfg["ffn_dim"], cfg["vocab"], cfg["max_ctx"], cfg.get("norm_eps", 1e-5),
                    cfg.get("rope_theta", 1e6))
        layers = (_Layer * cfg["n_layers"])()
        for li, lw in enumerate(weights["layers"]):
            L = layers[li]
            L.attn_norm = self._hold(_u16(lw["attn_norm"]))
            L.ffn_norm = self._hold(_u16(lw["ffn_norm"]))
            for field, short in self._MAP.items():
                bw = lw[short]
                stats = _u16(bw.stats)
                setattr(L, field, _BM(self._hold(_u16(bw.buckets)), self._hold(stats), self._hold(_u16(bw.probes)),
                                      bw.in_dim, bw.out_dim, stats.shape[1] if stats.ndim == 2 else 1))
        self._layers = layers
        kv = cfg["n_layers"] * cfg["n_kv_heads"] * cfg["max_ctx"] * cfg["head_dim"]
        self.k_cache = np.zeros(kv, np.uint16)
        self.v_cache = np.zeros(kv, np.uint16)
        embed = _u16(weights["embed"])
        lm = weights.get("lm_head")
        self.m = _Model(c, self._hold(embed), self._hold(_u16(weights["final_norm"])),
                        self._hold(embed if lm is None else _u16(lm)), ctypes.cast(layers, _vp),
                        _p(self.k_cache), _p(self.v_cache))

    def _hold(self, a):
        self._keep.append(a)
        return _p(a)

    def set_kv(self, k_cache, v_cache):
        """k/v: uint16 [n_layers][n_kv_heads][max_ctx][head_dim]."""
        self.k_cache[:] = np.ascontiguousarray(k_cache, np.uint16).reshape(-1)
        self.v_cache[:] = np.ascontiguousarray(v_cache, np.uint16).reshape(-1)

    def forward(self, token, pos, effort, nthreads=1):
        logits = np.empty(self.cfg["vocab"], np.float32)
        sel = ctypes.c_long(0)
        best = lib().ora_model_forward(ctypes.byref(self.m), token, pos, effort, _p(logits), ctypes.byref(sel),
                                       nthreads)
        return best, logits, sel.value

    def forward_dense(self, token, pos, nthreads=1):
        """One step with every bucket row selected (the dense path's product)."""
        logits = np.empty(self.cfg["vocab"], np.float32)
        best = lib().ora_model_forward_dense(ctypes.byref(self.m), token, pos, _p(logits), nthreads)
        return best, logits
