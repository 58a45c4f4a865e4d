"""A C++ program written against include/iam_b200.hpp (tests/shim_program.cpp) runs on the GPU
and its outputs match the CPU oracle: BucketMul::fullMul and calcDispatch + mul on a reference
fixture, MistralModel::forward over a few tokens (test_generation.cpp:202-213), and the
block-level classes TransformerLayer / Attention / FeedForward (transformer_layer.hpp:75-122,
attention.hpp:135-202, feedforward.hpp:180) on a 2-layer model.

The block outputs are compared with the oracle's restatement of the same block on the same
input and the GPU's KV cache.  Each block's bucketMuls after the first see inputs whose last
bits differ from the oracle's (different fp32 summation orders), so a row on the cutoff can go
the other way; a block whose selected-row counts all equal the oracle's is held to
LOGIT_TOL x RMS, one with a moved row to FLIP_TOL (decode_parity)."""
import os
import shutil
import subprocess

import numpy as np
import pytest

from conftest import GOLDEN, ROOT
from decode_parity import FLIP_TOL, LOGIT_TOL, check_steps, rel_err

PKG_LIB = os.path.join(ROOT, "input-adaptive-matrix-inference-optimization_b200", "lib")
CUDA = "/usr/local/cuda"
SMALL = dict(dim=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn_dim=512, vocab=512, max_ctx=32)
SEED = 11
EFFORT = 0.5
TOKENS = [5, 17, 99, 3, 42, 7]


def build_program(out_path, link=True):
    """Compiles tests/shim_program.cpp against include/ (and links libiamb200.so)."""
    cxx = shutil.which("g++")
    if not cxx or not os.path.isdir(os.path.join(CUDA, "include")):
        pytest.skip("no host C++ compiler or CUDA headers")
    cmd = [cxx, "-std=c++17", "-O1", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), "-I",
           os.path.join(CUDA, "include"), os.path.join(ROOT, "tests", "shim_program.cpp")]
    if link:
        cmd += ["-o", str(out_path), "-L", PKG_LIB, "-liamb200", "-L", os.path.join(CUDA, "lib64"), "-lcudart",
                f"-Wl,-rpath,{PKG_LIB}", f"-Wl,-rpath,{os.path.join(CUDA, 'lib64')}"]
    else:
        cmd += ["-c", "-o", str(out_path)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return out_path


def test_shim_program_builds(tmp_path):
    """The program compiles and links against libiamb200.so without a GPU."""
    if not os.path.exists(os.path.join(PKG_LIB, "libiamb200.so")):
        pytest.skip("libiamb200.so not built")
    build_program(tmp_path / "shim_program")


def _write_inputs(d, cfg, fx):
    bm = np.load(os.path.join(GOLDEN, "bm_256x64.npz"))
    in_dim, out_dim = bm["probes"].shape[0], bm["W"].shape[0]
    x = bm["x"][2].astype(np.float32)
    with open(d / "bm_in.bin", "wb") as f:
        np.array([in_dim, out_dim], np.int32).tofile(f)
        np.array([EFFORT], np.float32).tofile(f)
        x.tofile(f)
        bm["stats3"].astype(np.uint16).tofile(f)
        bm["probes"].astype(np.uint16).tofile(f)
        bm["buckets"].astype(np.uint16).tofile(f)
    c = cfg.as_dict()
    with open(d / "model_in.bin", "wb") as f:
        np.array([c["dim"], c["n_layers"], c["n_heads"], c["n_kv_heads"], c["head_dim"], c["ffn_dim"], c["vocab"],
                  c["max_ctx"], int(c.get("tied_embeddings", 0))], np.int32).tofile(f)
        np.array([c["norm_eps"]], np.float32).tofile(f)
        np.array([c["rope_theta"]], np.float64).tofile(f)
        np.array([SEED], np.uint64).tofile(f)
        np.array([EFFORT], np.float32).tofile(f)
        np.array([len(TOKENS)] + TOKENS + [len(TOKENS)], np.int32).tofile(f)
        fx["x"].tofile(f)
        fx["h"].tofile(f)
    return bm, x


def _read(d, name, dtype):
    return np.fromfile(d / name, dtype)


def _block_err(got, ref, same):
    err = rel_err(got, ref)
    assert err < (LOGIT_TOL if same else FLIP_TOL), (err, same)
    return err


@pytest.mark.gpu
@pytest.mark.timeout(600)
def test_shim_program_matches_oracle(iam, ora, cuda, tmp_path):
    cfg = iam.ModelConfig.make(**SMALL)
    rng = np.random.default_rng(3)
    fx = {"x": rng.standard_normal(cfg.dim).astype(np.float32),
          "h": rng.standard_normal(cfg.dim).astype(np.float32)}
    bm, xb = _write_inputs(tmp_path, cfg, fx)
    prog = build_program(tmp_path / "shim_program")
    r = subprocess.run([str(prog), str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr

    # BucketMul: both entry styles against the oracle on the fixture
    ref, _, _ = ora.bucketmul_full(xb, bm["stats3"], 1, bm["probes"], bm["buckets"], EFFORT)
    for name in ("bm_full.bin", "bm_two_step.bin"):
        assert rel_err(_read(tmp_path, name, np.float32), ref) < 1e-3, name

    # MistralModel::forward, teacher forced on the same tokens (same seed -> same weights)
    m = iam.Model.random(cfg, seed=SEED)
    w = m.export_weights()
    m.close()
    c = cfg.as_dict()
    om = ora.OracleModel(c, w)
    logits = _read(tmp_path, "model_logits.bin", np.float32).reshape(len(TOKENS), cfg.vocab)
    sel = _read(tmp_path, "model_sel.bin", np.int64)
    steps = []
    for i, tok in enumerate(TOKENS):
        best, lref, osel = om.forward(tok, i, EFFORT)
        steps.append(dict(pos=i, err=rel_err(logits[i], lref), same=(int(sel[i]) == osel),
                          gpu=int(np.argmax(logits[i])), ref=best, ref_logits=lref,
                          rms=float(np.sqrt(np.mean(lref.astype(np.float64) ** 2)))))
    check_steps(steps, max_flip_frac=1.0)

    # the blocks, on the oracle's restatement over the GPU's cache
    P = len(TOKENS)
    hd, nh, nkv = c["head_dim"], c["n_heads"], c["n_kv_heads"]
    cs = ora.rope_table(P, hd, c["rope_theta"])

    def bmul(x, lw, name):
        b = lw[name]
        out, n, _ = ora.bucketmul_full(x, np.asarray(b.stats).reshape(-1), 1, b.probes, b.buckets, EFFORT,
                                       in_dim=b.in_dim)
        return out.astype(np.float32), n

    def attention_block(h, lw, kc, vc):
        q, nq = bmul(h, lw, "q")
        _, nk = bmul(h, lw, "k")
        _, nv = bmul(h, lw, "v")
        kc = kc.reshape(nkv, c["max_ctx"], hd)
        vc = vc.reshape(nkv, c["max_ctx"], hd)
        att = ora.attention(c, ora.rope_apply(q, nh, hd, cs), kc, vc, P + 1).astype(np.float32)
        o, no = bmul(att, lw, "o")
        return o, [nq, nk, nv, no]

    def ffn_block(h, lw):
        g, ng = bmul(h, lw, "gate")
        u, nu = bmul(h, lw, "up")
        d, nd = bmul(ora.silu_mul(g, u).astype(np.float32), lw, "down")
        return d, [ng, nu, nd]

    l0, l1 = w["layers"][0], w["layers"][1]
    # TransformerLayer(0): x + attn(norm(x)), then + ffn(norm(.))
    x = fx["x"]
    o, na = attention_block(ora.rmsnorm(x, l0["attn_norm"], c["norm_eps"]), l0,
                            _read(tmp_path, "layer_k.bin", np.uint16), _read(tmp_path, "layer_v.bin", np.uint16))
    x1 = (x + o).astype(np.float32)
    d, nf = ffn_block(ora.rmsnorm(x1, l0["ffn_norm"], c["norm_eps"]), l0)
    ref_layer = (x1 + d).astype(np.float32)
    cnt = _read(tmp_path, "layer_counts.bin", np.int32)
    e_layer = _block_err(_read(tmp_path, "layer_out.bin", np.float32), ref_layer, list(cnt) == na + nf)

    # Attention(1) and FeedForward(1) on the normalised input h
    o, na = attention_block(fx["h"], l1, _read(tmp_path, "attn_k.bin", np.uint16),
                            _read(tmp_path, "attn_v.bin", np.uint16))
    cnt = _read(tmp_path, "attn_counts.bin", np.int32)
    e_att = _block_err(_read(tmp_path, "attn_out.bin", np.float32), o, list(cnt[:4]) == na)
    d, nf = ffn_block(fx["h"], l1)
    cnt = _read(tmp_path, "ffn_counts.bin", np.int32)
    e_ffn = _block_err(_read(tmp_path, "ffn_out.bin", np.float32), d, list(cnt[4:]) == nf)
    print(f"shim program: layer {e_layer:.2e}, attention {e_att:.2e}, feedforward {e_ffn:.2e} x rms")
