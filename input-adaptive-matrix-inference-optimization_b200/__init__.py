"""iam_b200 -- Python host mirror of the reference's C++ host API over libiamb200.so.

The product is the C ABI in include/iam_b200.h (and the C++ shim include/iam_b200.hpp);
this module binds it with ctypes for tests and bench.py.  Device memory and streams come
from torch (plumbing only).  There is no CPU path: if libiamb200.so is missing or the GPU
is not an sm_100 part, every call raises.

Load it by path (the directory name is not a Python identifier):

    spec = importlib.util.spec_from_file_location(
        "iam_b200", "<repo>/input-adaptive-matrix-inference-optimization_b200/__init__.py",
        submodule_search_locations=["<repo>/input-adaptive-matrix-inference-optimization_b200"])
"""
import ctypes
import os

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libiamb200.so")

IAM_OK, IAM_ERR_ARG, IAM_ERR_IO, IAM_ERR_CUDA, IAM_ERR_NCCL, IAM_ERR_TIMEOUT, IAM_ERR_UNSUPPORTED, \
    IAM_ERR_NOMEM = range(8)
PROBES_COUNT = 4096

_vp = ctypes.c_void_p
_i32 = ctypes.c_int
_i64 = ctypes.c_longlong
_f32 = ctypes.c_float

# name -> argtypes (all return int unless listed in _RESTYPES)
_SIGNATURES = {
    "iam_version": [],
    "iam_last_error": [],
    "iam_device_info": [_i32, _vp, _vp, _vp],
    "iam_bucketmul_plan_info": [_i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp],
    "iam_bucketmul_create": [_vp, _i32],
    "iam_bucketmul_destroy": [_vp],
    "iam_bucketmul_cutoff": [_vp, _vp, _vp, _i32, _i32, _f32, _vp, _vp, _vp],
    "iam_bucketmul_calc_dispatch": [_vp, _vp, _vp, _i32, _vp, _i32, _i32, _i32, _i32, _f32, _vp],
    "iam_bucketmul_read_dispatch": [_vp, _vp, _vp, _vp, _vp],
    "iam_bucketmul_mul": [_vp, _vp, _i32, _i32, _vp, _vp],
    "iam_bucketmul_full": [_vp, _vp, _vp, _i32, _vp, _vp, _i32, _i32, _i32, _i32, _f32, _vp, _vp, _vp, _vp],
    "iam_bucketmul_phase_times": [_vp, _vp],
    "iam_bucketmul_status": [_vp],
    "iam_bucketmul_trace": [_vp, _vp, ctypes.c_int],
    "iam_bucketmul_full_noalloc": [_vp, _vp, _i32, _vp, _vp, _i32, _i32, _i32, _i32, _f32, _vp, _vp, _vp, _vp],
    "iam_stats_pack": [_vp, _i64, _vp, _vp],
    "iam_bucketize": [_vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp],
    "iam_dense_create": [_i32, _i32, _i32, _i32, _vp],
    "iam_dense_destroy": [_vp],
    "iam_dense_gemm": [_vp, _vp, _i32, _i32, _vp, _i32, _vp, _vp, _i32, _i32, _vp],
    "iam_dense_status": [_vp],
    "iam_dense_unpack": [_vp, _i32, _i32, _vp, _vp],
}
_RESTYPES = {"iam_version": ctypes.c_char_p, "iam_last_error": ctypes.c_char_p}

_lib = None


class IamError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"iam error {code}: {msg}")
        self.code = code


def load_library(path=LIB_PATH):
    """Load libiamb200.so (fails loudly: there is no fallback path)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise IamError(IAM_ERR_UNSUPPORTED, f"{path} not built; run build.py")
    lib = ctypes.CDLL(path)
    for name, args in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPES.get(name, ctypes.c_int)
    _lib = lib
    return lib


def exported_symbols():
    return list(_SIGNATURES)


def check(rc):
    if rc != IAM_OK:
        raise IamError(rc, load_library().iam_last_error().decode(errors="replace"))
    return rc


def _ptr(t):
    if t is None:
        return None
    return ctypes.c_void_p(t.data_ptr())


def _stream(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


class BucketMul:
    """Mirror of BucketMul (bucket_mul.hpp:99-268) on one device; arguments are torch
    tensors on that device.  stats may be the file layout [R][4] (stats_stride=4) or the
    packed channel 3 [R] (stats_stride=1)."""

    def __init__(self, device=0):
        self.lib = load_library()
        self.h = ctypes.c_void_p()
        check(self.lib.iam_bucketmul_create(ctypes.byref(self.h), device))

    def close(self):
        if self.h:
            self.lib.iam_bucketmul_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def status(self):
        """Raises IamError(IAM_ERR_TIMEOUT) if a full_mul launch gave up at its grid barrier."""
        check(self.lib.iam_bucketmul_status(self.h))

    def phase_times(self, times):
        """Diagnostics: later full_mul launches write CTA 0's 16 int64 trace slots into `times`."""
        check(self.lib.iam_bucketmul_phase_times(self.h, _ptr(times)))

    def trace(self, stamps):
        """Diagnostics: later full_mul launches write 16 int64 per CTA into `stamps` (None: off)."""
        cap = 0 if stamps is None else int(stamps.numel()) // 16
        check(self.lib.iam_bucketmul_trace(self.h, _ptr(stamps), cap))

    def cutoff(self, x, probes, in_dim, effort, out, iters=None, expert_no=0, stream=None):
        check(self.lib.iam_bucketmul_cutoff(self.h, _ptr(x), _ptr(probes), expert_no, in_dim, effort,
                                            _ptr(out), _ptr(iters), _stream(stream)))

    def calc_dispatch(self, x, stats, probes, expert_no, in_size, bucket_cols, expert_size, effort,
                      stats_stride=4, stream=None):
        check(self.lib.iam_bucketmul_calc_dispatch(self.h, _ptr(x), _ptr(stats), stats_stride, _ptr(probes),
                                                   expert_no, in_size, bucket_cols, expert_size, effort,
                                                   _stream(stream)))

    def read_dispatch(self, rows=None, count=None, cutoff=None, stream=None):
        check(self.lib.iam_bucketmul_read_dispatch(self.h, _ptr(rows), _ptr(count), _ptr(cutoff),
                                                   _stream(stream)))

    def mul(self, buckets, out, bucket_rows=None, bucket_cols=None, stream=None):
        rows = buckets.shape[0] if bucket_rows is None else bucket_rows
        cols = buckets.shape[1] if bucket_cols is None else bucket_cols
        check(self.lib.iam_bucketmul_mul(self.h, _ptr(buckets), rows, cols, _ptr(out), _stream(stream)))

    def full_mul(self, x, stats, probes, buckets, expert_no, in_size, bucket_cols, expert_size, effort, out,
                 stats_stride=4, count=None, cutoff=None, stream=None):
        check(self.lib.iam_bucketmul_full(self.h, _ptr(x), _ptr(stats), stats_stride, _ptr(probes),
                                          _ptr(buckets), expert_no, in_size, bucket_cols, expert_size, effort,
                                          _ptr(out), _ptr(count), _ptr(cutoff), _stream(stream)))


def bucketmul_full_noalloc(x, stats, probes, buckets, expert_no, in_size, bucket_cols, expert_size, effort, out,
                           stats_stride=4, count=None, cutoff=None, stream=None):
    """iam_bucketmul_full_noalloc: fullMul with the library's built-in scratch (no device
    allocation; calls must not overlap on the GPU; bucket_cols <= 1024)."""
    check(load_library().iam_bucketmul_full_noalloc(_ptr(x), _ptr(stats), stats_stride, _ptr(probes), _ptr(buckets),
                                                    expert_no, in_size, bucket_cols, expert_size, effort, _ptr(out),
                                                    _ptr(count), _ptr(cutoff), _stream(stream)))


def plan_info(vec, cluster, bucket_cols, in_dim):
    """-> (max_active_clusters, log2_lanes_per_row, n_tiles, n_splits) of the fused bucketMul plan."""
    a, b, c, d = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    check(load_library().iam_bucketmul_plan_info(vec, cluster, bucket_cols, in_dim, ctypes.byref(a),
                                                 ctypes.byref(b), ctypes.byref(c), ctypes.byref(d)))
    return a.value, b.value, c.value, d.value


def stats_pack(stats4, stats1, stream=None):
    check(load_library().iam_stats_pack(_ptr(stats4), stats4.numel() // 4, _ptr(stats1), _stream(stream)))


def bucketize(w, buckets, stats4=None, stats1=None, probes=None, stream=None):
    """GPU bucketize of W[out][in] (torch uint16/int16/float16 tensor holding fp16 bits)."""
    out_dim, in_dim = w.shape
    check(load_library().iam_bucketize(_ptr(w), out_dim, in_dim, _ptr(buckets), _ptr(stats4), _ptr(stats1),
                                       _ptr(probes), _stream(stream)))


def dense_unpack(buckets, w_out, in_dim=None, bucket_cols=None, stream=None):
    """iam_dense_unpack: dense fp16 W'[16*cols][in] from buckets[16*in][cols] (every row selected)."""
    rows, cols = buckets.shape
    in_dim = rows // 16 if in_dim is None else in_dim
    cols = cols if bucket_cols is None else bucket_cols
    check(load_library().iam_dense_unpack(_ptr(buckets), in_dim, cols, _ptr(w_out), _stream(stream)))


class Dense:
    """Dense tensor-core products (iam_dense_*): y[t][o] = residual[t][o] + sum_i W[o][i] x[t][i],
    the reference's basicMul (matrix.cl:80-93) batched over tokens.  W is fp16 bits
    [out][in] (uint16/int16/float16 tensor), x / y / residual fp32 [tokens][...]."""

    def __init__(self, max_tokens, max_in_dim, max_out_dim, device=0):
        self.lib = load_library()
        self.h = ctypes.c_void_p()
        check(self.lib.iam_dense_create(max_tokens, max_in_dim, max_out_dim, device, ctypes.byref(self.h)))

    def close(self):
        if self.h:
            self.lib.iam_dense_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def gemm(self, w, x, y, residual=None, precision=0, split_k=0, stream=None):
        out_dim, in_dim = w.shape
        check(self.lib.iam_dense_gemm(self.h, _ptr(w), out_dim, in_dim, _ptr(x), x.shape[0], _ptr(residual),
                                      _ptr(y), precision, split_k, _stream(stream)))

    def status(self):
        check(self.lib.iam_dense_status(self.h))


# ---------------------------------------------------------------- decode model

class ModelConfig(ctypes.Structure):
    """iam_model_config (include/iam_b200.h)."""
    _fields_ = [("dim", _i32), ("n_layers", _i32), ("n_heads", _i32), ("n_kv_heads", _i32), ("head_dim", _i32),
                ("ffn_dim", _i32), ("vocab", _i32), ("max_ctx", _i32), ("norm_eps", _f32),
                ("rope_theta", ctypes.c_double), ("tied_embeddings", _i32)]

    @classmethod
    def make(cls, dim, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, max_ctx, norm_eps=1e-5,
             rope_theta=1e6, tied_embeddings=1):
        return cls(dim, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, max_ctx, norm_eps, rope_theta,
                   tied_embeddings)

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_}


MISTRAL_7B = dict(dim=4096, n_layers=32, n_heads=32, n_kv_heads=8, head_dim=128, ffn_dim=14336, vocab=32000)

W_EMBED, W_FINAL_NORM, W_LM_HEAD, W_ATTN_NORM, W_FFN_NORM, W_K_CACHE, W_V_CACHE, W_MATRIX = 0, 1, 2, 3, 4, 5, 6, 16
MATRIX_NAMES = ("q", "k", "v", "o", "gate", "up", "down")

_SIGNATURES.update({
    "iam_model_create_random": [_vp, _vp, ctypes.c_ulonglong, _i32],
    "iam_model_load": [_vp, ctypes.c_char_p, _vp, _i32],
    "iam_model_destroy": [_vp],
    "iam_model_reset": [_vp, _vp],
    "iam_model_forward": [_vp, _i32, _i32, _f32, _vp, _vp],
    "iam_layer_forward": [_vp, _i32, _vp, _i32, _f32, _vp, _vp],
    "iam_attention_forward": [_vp, _i32, _vp, _i32, _f32, _vp, _vp],
    "iam_feedforward_forward": [_vp, _i32, _vp, _f32, _vp, _vp],
    "iam_model_prefill": [_vp, _vp, _i32, _i32, _vp, _vp, _vp],
    "iam_model_generate": [_vp, _i32, _i32, _i32, _f32, _vp, _vp],
    "iam_model_set_kv": [_vp, _i32, _vp, _vp, _i32, _vp],
    "iam_model_fill_kv_random": [_vp, _i32, ctypes.c_ulonglong, _vp],
    "iam_model_read_weight": [_vp, _i32, _i32, _vp, ctypes.c_size_t, _vp],
    "iam_model_selected_rows": [_vp, _vp],
    "iam_model_step_bytes": [_vp, _i32, _vp],
    "iam_model_profile_steps": [_vp, _f32, _i32, _vp, _vp, _i32, _vp, _vp],
    "iam_tp_unique_id": [_vp],
    "iam_model_status": [_vp],
    "iam_model_save": [_vp, ctypes.c_char_p],
    "iam_model_selected_rows_by_matrix": [_vp, _vp, _i32],
    "iam_tp_shard_info": [_vp, _i32, _i32, _vp],
    "iam_tp_wait_selftest": [_i32, _i32, _i64, _vp, _vp, _vp],
    "iam_model_capture_floats": [_vp, _vp],
    "iam_model_capture": [_vp, _vp, ctypes.c_size_t],
    "iam_model_create_random_tp": [_vp, _vp, ctypes.c_ulonglong, _i32, _i32, _i32, _vp],
    "iam_model_load_tp": [_vp, ctypes.c_char_p, _vp, _i32, _i32, _i32, _vp],
})
KERNEL_KINDS = ("embed", "bucketmul", "attention", "lm_head", "other", "collective")
TP_ID_BYTES = 128


def tp_unique_id():
    """NCCL id for a tensor-parallel group (rank 0 makes it, every rank passes it in)."""
    buf = (ctypes.c_ubyte * TP_ID_BYTES)()
    check(load_library().iam_tp_unique_id(buf))
    return bytes(buf)


def tp_shard_info(cfg, rank, world):
    """Shards of rank `rank` of `world` (no GPU needed): {matrix: (col0, cols, in0, in1)}, plus
    'vocab': (row0, rows)."""
    out = (ctypes.c_int * (4 * len(MATRIX_NAMES) + 2))()
    check(load_library().iam_tp_shard_info(ctypes.byref(cfg), rank, world, out))
    res = {name: tuple(out[4 * i:4 * i + 4]) for i, name in enumerate(MATRIX_NAMES)}
    res["vocab"] = (out[4 * len(MATRIX_NAMES)], out[4 * len(MATRIX_NAMES) + 1])
    return res


def tp_wait_selftest(n=256, spin_limit=4096, device=0):
    """iam_tp_wait_selftest: -> (status code, error word, first call ms, second call ms)."""
    err, t1, t2 = ctypes.c_uint(), ctypes.c_float(), ctypes.c_float()
    rc = load_library().iam_tp_wait_selftest(device, n, spin_limit, ctypes.byref(err), ctypes.byref(t1),
                                             ctypes.byref(t2))
    return rc, err.value, t1.value, t2.value


def _tp_args(tp):
    rank, world, uid = tp
    if len(uid) != TP_ID_BYTES:
        raise IamError(IAM_ERR_ARG, "tensor parallel id must be 128 bytes")
    return rank, world, (ctypes.c_ubyte * TP_ID_BYTES).from_buffer_copy(uid)


class Model:
    """Mirror of MistralModel (model.hpp:84-237) on one device, or one rank of a
    tensor-parallel group (tp=(rank, world, tp_unique_id() of rank 0))."""

    def __init__(self, cfg, h, tp=None):
        self.cfg, self.h, self.lib = cfg, h, load_library()
        self.rank, self.world = (tp[0], tp[1]) if tp else (0, 1)

    @classmethod
    def random(cls, cfg, seed=0, device=0, tp=None):
        lib = load_library()
        h = ctypes.c_void_p()
        if tp:
            rank, world, uid = _tp_args(tp)
            check(lib.iam_model_create_random_tp(ctypes.byref(h), ctypes.byref(cfg), seed, device, rank, world, uid))
        else:
            check(lib.iam_model_create_random(ctypes.byref(h), ctypes.byref(cfg), seed, device))
        return cls(cfg, h, tp)

    @classmethod
    def load(cls, weights_dir, cfg, device=0, tp=None):
        lib = load_library()
        h = ctypes.c_void_p()
        if tp:
            rank, world, uid = _tp_args(tp)
            check(lib.iam_model_load_tp(ctypes.byref(h), os.fsencode(weights_dir), ctypes.byref(cfg), device, rank,
                                        world, uid))
        else:
            check(lib.iam_model_load(ctypes.byref(h), os.fsencode(weights_dir), ctypes.byref(cfg), device))
        return cls(cfg, h, tp)

    def close(self):
        if self.h:
            self.lib.iam_model_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def save(self, weights_dir):
        """Writes the model in the reference's on-disk layout (the directory must exist)."""
        check(self.lib.iam_model_save(self.h, os.fsencode(weights_dir)))

    def status(self):
        """Raises IamError(IAM_ERR_TIMEOUT) if a tensor-parallel exchange gave up on a peer."""
        check(self.lib.iam_model_status(self.h))

    def reset(self, stream=None):
        check(self.lib.iam_model_reset(self.h, _stream(stream)))

    def forward(self, token, pos, effort, logits=None, stream=None):
        check(self.lib.iam_model_forward(self.h, token, pos, effort, _ptr(logits), _stream(stream)))

    def layer_forward(self, layer, x, pos, effort, out, stream=None):
        """iam_layer_forward (TransformerLayer::forward): out = the decoder layer applied to x
        (device float tensors of dim) at pos, over the model's KV cache of that layer."""
        check(self.lib.iam_layer_forward(self.h, layer, _ptr(x), pos, effort, _ptr(out), _stream(stream)))

    def attention_forward(self, layer, h, pos, effort, out, stream=None):
        """iam_attention_forward (Attention::forward): q/k/v, attention at pos and o of a
        normalised input, no residual."""
        check(self.lib.iam_attention_forward(self.h, layer, _ptr(h), pos, effort, _ptr(out), _stream(stream)))

    def feedforward_forward(self, layer, h, effort, out, stream=None):
        """iam_feedforward_forward (FeedForward::forward): down(SiLU(gate(h)) * up(h)), no
        residual."""
        check(self.lib.iam_feedforward_forward(self.h, layer, _ptr(h), effort, _ptr(out), _stream(stream)))

    def prefill(self, tokens, start_pos=0, logits=None, stream=None):
        """iam_model_prefill: the prompt through the dense tensor-core path in one pass; returns
        the greedy next token."""
        arr = (ctypes.c_int * len(tokens))(*[int(t) for t in tokens])
        nxt = ctypes.c_int(-1)
        check(self.lib.iam_model_prefill(self.h, arr, len(tokens), start_pos, _ptr(logits), ctypes.byref(nxt),
                                         _stream(stream)))
        return nxt.value

    def generate(self, first_token, start_pos, n_tokens, effort, tokens, stream=None):
        check(self.lib.iam_model_generate(self.h, first_token, start_pos, n_tokens, effort, _ptr(tokens),
                                          _stream(stream)))

    def set_kv(self, layer, k, v, n_tokens, stream=None):
        check(self.lib.iam_model_set_kv(self.h, layer, _ptr(k), _ptr(v), n_tokens, _stream(stream)))

    def fill_kv_random(self, n_tokens, seed=0, stream=None):
        check(self.lib.iam_model_fill_kv_random(self.h, n_tokens, seed, _stream(stream)))

    def read_weight(self, which, layer=0):
        """-> numpy uint16 array with the weight's bits (blocking)."""
        import numpy as np
        n = ctypes.c_size_t()
        check(self.lib.iam_model_read_weight(self.h, layer, which, None, 0, ctypes.byref(n)))
        out = np.empty(n.value // 2, np.uint16)
        check(self.lib.iam_model_read_weight(self.h, layer, which, out.ctypes.data_as(ctypes.c_void_p), n.value,
                                             None))
        return out

    def selected_rows(self):
        t = ctypes.c_longlong()
        check(self.lib.iam_model_selected_rows(self.h, ctypes.byref(t)))
        return t.value

    def selected_rows_by_matrix(self):
        """-> int32 array [n_layers, 7] of the last step's selected rows (q, k, v, o, gate, up, down)."""
        import numpy as np
        n = self.cfg.n_layers * len(MATRIX_NAMES)
        out = np.zeros(n, np.int32)
        check(self.lib.iam_model_selected_rows_by_matrix(self.h, out.ctypes.data_as(ctypes.c_void_p), n))
        return out.reshape(self.cfg.n_layers, len(MATRIX_NAMES))

    def capture(self, buf):
        """iam_model_capture: later steps record every layer's bucketMul inputs, cutoffs and
        outputs into `buf` (fp32 device tensor of capture_floats() elements; None: off)."""
        check(self.lib.iam_model_capture(self.h, _ptr(buf), 0 if buf is None else buf.numel()))

    def capture_floats(self):
        n = ctypes.c_longlong()
        check(self.lib.iam_model_capture_floats(ctypes.byref(self.cfg), ctypes.byref(n)))
        return n.value

    def capture_records(self, buf):
        """Splits a capture buffer (copied to the host) into per-layer dicts of numpy arrays."""
        import numpy as np
        c = self.cfg
        d, a, kv, f = c.dim, c.n_heads * c.head_dim, c.n_kv_heads * c.head_dim, c.ffn_dim
        parts = [("x_qkv", d), ("q", a), ("k", kv), ("v", kv), ("x_o", a), ("res_o", d), ("out_o", d),
                 ("x_gu", d), ("gate", f), ("up", f), ("x_down", f), ("res_down", d), ("out_down", d),
                 ("cutoff", 8)]
        per = sum(n for _, n in parts)
        host = buf.detach().cpu().numpy().reshape(c.n_layers, per)
        recs = []
        for l in range(c.n_layers):
            off, rec = 0, {}
            for name, n in parts:
                rec[name] = host[l, off:off + n].copy()
                off += n
            recs.append(rec)
        return recs

    def step_bytes(self, context):
        t = ctypes.c_longlong()
        check(self.lib.iam_model_step_bytes(self.h, context, ctypes.byref(t)))
        return t.value

    def profile_steps(self, effort, steps, stream=None):
        """-> list of (kind, avg_ms) per launch of one decode step (diagnostics; advances pos)."""
        cap = 4096
        ms = (ctypes.c_float * cap)()
        kinds = (ctypes.c_int * cap)()
        n = ctypes.c_int()
        check(self.lib.iam_model_profile_steps(self.h, effort, steps, ms, kinds, cap, ctypes.byref(n),
                                               _stream(stream)))
        return [(KERNEL_KINDS[kinds[k]], ms[k]) for k in range(n.value)]

    def export_weights(self):
        """Host copy of every weight in the oracle's layout (tests use it as the checker's input)."""
        import importlib
        weights = importlib.import_module(__name__ + ".weights")
        c = self.cfg
        qn, kvn = c.n_heads * c.head_dim, c.n_kv_heads * c.head_dim
        shapes = {"q": (qn, c.dim), "k": (kvn, c.dim), "v": (kvn, c.dim), "o": (c.dim, qn),
                  "gate": (c.ffn_dim, c.dim), "up": (c.ffn_dim, c.dim), "down": (c.dim, c.ffn_dim)}
        layers = []
        for l in range(c.n_layers):
            lw = {"attn_norm": self.read_weight(W_ATTN_NORM, l), "ffn_norm": self.read_weight(W_FFN_NORM, l)}
            for mi, name in enumerate(MATRIX_NAMES):
                out_dim, in_dim = shapes[name]
                b = self.read_weight(W_MATRIX + 3 * mi, l).reshape(16 * in_dim, out_dim // 16)
                s1 = self.read_weight(W_MATRIX + 3 * mi + 1, l)
                p = self.read_weight(W_MATRIX + 3 * mi + 2, l)
                lw[name] = weights.BucketWeight(b, s1.reshape(-1, 1), p, in_dim, out_dim)
            layers.append(lw)
        embed = self.read_weight(W_EMBED).reshape(c.vocab, c.dim)
        lm = None if c.tied_embeddings else self.read_weight(W_LM_HEAD).reshape(c.vocab, c.dim)
        return {"embed": embed, "final_norm": self.read_weight(W_FINAL_NORM), "lm_head": lm, "layers": layers}
