"""Decode-model parity on the GPU against the CPU oracle's decode step (ora_model_forward,
which follows model.hpp:152-231 / transformer_layer.hpp:75-122 / attention.hpp:135-404).

Bar (decode_parity.py): every bucketMul on identical inputs selects exactly the oracle's rows
(cutoff bits, counts) with outputs within 1e-3 x RMS; whole steps, teacher forced over the
prompt and 32 greedy tokens: logits within 1e-3 x RMS and the same greedy token whenever the
step's selections equal the oracle's (fp32 summation order can move a row that sits on the
cutoff; such steps are reported and held to 5e-2).
"""
import os

import numpy as np
import pytest

from decode_parity import (LOGIT_TOL, check_captured_bucketmuls, check_captured_layers, check_steps, rel_err,
                           teacher_forced_steps)

pytestmark = pytest.mark.gpu

SMALL = dict(dim=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn_dim=512, vocab=512, max_ctx=96)


@pytest.fixture(scope="module")
def torch_mod(cuda):
    import torch
    return torch


@pytest.fixture(scope="module")
def small(iam, cuda):
    cfg = iam.ModelConfig.make(**SMALL)
    m = iam.Model.random(cfg, seed=7)
    w = m.export_weights()
    yield cfg, m, w
    m.close()


def oracle_for(ora, cfg, w):
    d = cfg.as_dict()
    return ora.OracleModel(d, w)


@pytest.mark.parametrize("effort", [0.25, 0.5, 1.0])
def test_decode_matches_oracle(small, ora, torch_mod, effort):
    """The prompt, then 32 greedy tokens, decoded by the GPU and (teacher forced) the oracle:
    logits within 1e-3 x RMS and the same greedy token on every step whose selections equal
    the oracle's; a step where a row on the cutoff went the other way is reported as such.
    Then the captured-graph generation decodes exactly the eager steps' greedy tokens."""
    torch = torch_mod
    cfg, m, w = small
    om = oracle_for(ora, cfg, w)
    prompt = np.random.default_rng(1).integers(3, cfg.vocab, 8).tolist()
    n_gen = 32
    m.reset()
    torch.cuda.synchronize()
    logits = torch.empty(cfg.vocab, dtype=torch.float32, device="cuda")
    steps, toks = teacher_forced_steps(m, om, prompt, 0, n_gen, effort, logits, torch)
    # near effort 1.0 the cutoff sits among the smallest importances, where rounding order
    # flips rows often: every flip step is held to FLIP_TOL, the others to LOGIT_TOL
    flips, worst = check_steps(steps, max_flip_frac=1.0)
    print(f"effort {effort}: {len(steps)} steps, flips at {flips}, worst equal-selection error {worst:.2e}")
    m.reset()
    for pos, tok in enumerate(prompt):
        m.forward(tok, pos, effort)
    gen = torch.empty(n_gen, dtype=torch.int32, device="cuda")
    m.generate(toks[len(prompt)], len(prompt), n_gen, effort, gen)
    torch.cuda.synchronize()
    assert gen.cpu().tolist() == toks[len(prompt) + 1:len(prompt) + 1 + n_gen]


@pytest.mark.parametrize("effort", [0.25, 1.0])
def test_captured_step_matches_oracle_op_by_op(small, iam, ora, torch_mod, effort):
    """Every operation of a decode step on the inputs the kernels actually used: each
    bucketMul selects exactly the oracle's rows (cutoff bits, counts) with outputs within
    1e-3 x RMS; RMSNorm, the RoPE'd fp16 K/V append and the residual stream bit for bit;
    attention, SiLU * up and the LM head within 1e-4 x RMS."""
    torch = torch_mod
    cfg, m, w = small
    buf = torch.zeros(m.capture_floats(), dtype=torch.float32, device="cuda")
    logits = torch.empty(cfg.vocab, dtype=torch.float32, device="cuda")
    m.capture(buf)
    try:
        m.reset()
        for pos, tok in enumerate([5, 77, 300, 11, 42]):
            m.forward(tok, pos, effort, logits)
            torch.cuda.synchronize()
            kv = [(m.read_weight(iam.W_K_CACHE, l), m.read_weight(iam.W_V_CACHE, l)) for l in range(cfg.n_layers)]
            check_captured_layers(ora, cfg, w, m.capture_records(buf), m.selected_rows_by_matrix(), kv, pos, effort,
                                  logits.cpu().numpy())
    finally:
        m.capture(None)


def test_decode_is_deterministic(small, torch_mod):
    torch = torch_mod
    cfg, m, _ = small
    outs = []
    for _ in range(2):
        m.reset()
        logits = torch.empty(cfg.vocab, dtype=torch.float32, device="cuda")
        for pos, tok in enumerate([5, 17, 99, 3]):
            m.forward(tok, pos, 0.25, logits)
        torch.cuda.synchronize()
        outs.append(logits.cpu().numpy().view(np.uint32).copy())
    assert (outs[0] == outs[1]).all()


def test_reference_file_layout_loads(small, iam, weights_mod, torch_mod, tmp_path):
    """Weights written in the reference's on-disk layout load through iam_model_load and
    give bit-identical logits (same weights, deterministic kernels)."""
    torch = torch_mod
    cfg, m, w = small
    d = str(tmp_path)
    for l, lw in enumerate(w["layers"]):
        for name in iam.MATRIX_NAMES:
            bw = lw[name]
            stats4 = np.repeat(np.asarray(bw.stats).reshape(-1, 1), 4, axis=1)
            weights_mod.save_bucketmul_binary(
                weights_mod.BucketWeight(bw.buckets, stats4, bw.probes, bw.in_dim, bw.out_dim),
                os.path.join(d, weights_mod.layer_weight_name(l, name)))
        np.save(os.path.join(d, f"layer{l}_input_layernorm.npy"), lw["attn_norm"].view(np.float16))
        np.save(os.path.join(d, f"layer{l}_post_attention_layernorm.npy"), lw["ffn_norm"].view(np.float16))
    np.save(os.path.join(d, "embed_tokens.npy"), w["embed"].view(np.float16))
    np.save(os.path.join(d, "norm_weight.npy"), w["final_norm"].view(np.float16))
    m2 = iam.Model.load(d, cfg)
    outs = []
    for mm in (m, m2):
        mm.reset()
        logits = torch.empty(cfg.vocab, dtype=torch.float32, device="cuda")
        for pos, tok in enumerate([11, 22, 33]):
            mm.forward(tok, pos, 0.5, logits)
        torch.cuda.synchronize()
        outs.append(logits.cpu().numpy().view(np.uint32).copy())
    m2.close()
    assert (outs[0] == outs[1]).all()
    # truncated file -> IAM_ERR_IO
    with open(os.path.join(d, weights_mod.layer_weight_name(1, "down") + "_stats.bin"), "r+b") as f:
        f.truncate(10)
    with pytest.raises(iam.IamError) as e:
        iam.Model.load(d, cfg)
    assert e.value.code == iam.IAM_ERR_IO


def test_model_save_writes_the_reference_layout(small, iam, weights_mod, torch_mod, tmp_path):
    """iam_model_save writes the reference's on-disk layout: the Python restatement of the
    reference's reader accepts every file, the bytes equal the model's weights, and a model
    loaded back from the directory gives bit-identical logits."""
    torch = torch_mod
    cfg, m, w = small
    d = str(tmp_path)
    m.save(d)
    for l, lw in enumerate(w["layers"]):
        for name in iam.MATRIX_NAMES:
            back = weights_mod.load_bucketmul_binary(os.path.join(d, weights_mod.layer_weight_name(l, name)))
            bw = lw[name]
            np.testing.assert_array_equal(back.buckets.reshape(-1), np.asarray(bw.buckets).reshape(-1))
            np.testing.assert_array_equal(back.stats.reshape(-1, 4)[:, 3], np.asarray(bw.stats).reshape(-1))
            assert (back.stats.reshape(-1, 4) == back.stats.reshape(-1, 4)[:, :1]).all()  # 4 identical channels
            np.testing.assert_array_equal(back.probes.reshape(-1), np.asarray(bw.probes).reshape(-1))
            assert (back.in_dim, back.out_dim) == (bw.in_dim, bw.out_dim)
        np.testing.assert_array_equal(weights_mod.load_npy_fp16(os.path.join(d, f"layer{l}_input_layernorm.npy")),
                                      lw["attn_norm"].reshape(-1))
    emb = np.load(os.path.join(d, "embed_tokens.npy"))
    assert emb.dtype == np.float16 and emb.shape == (cfg.vocab, cfg.dim)
    np.testing.assert_array_equal(emb.view(np.uint16).reshape(-1), w["embed"].reshape(-1))
    m2 = iam.Model.load(d, cfg)
    outs = []
    for mm in (m, m2):
        mm.reset()
        logits = torch.empty(cfg.vocab, dtype=torch.float32, device="cuda")
        for pos, tok in enumerate([11, 22, 33]):
            mm.forward(tok, pos, 0.25, logits)
        torch.cuda.synchronize()
        outs.append(logits.cpu().numpy().view(np.uint32).copy())
    m2.close()
    assert (outs[0] == outs[1]).all()


def test_model_rejects_bad_arguments(small, iam):
    cfg, m, _ = small
    for token, pos, effort in [(-1, 0, 0.5), (cfg.vocab, 0, 0.5), (1, cfg.max_ctx, 0.5), (1, 0, 0.0), (1, 0, 2.0)]:
        with pytest.raises(iam.IamError) as e:
            m.forward(token, pos, effort)
        assert e.value.code == iam.IAM_ERR_ARG
    bad = iam.ModelConfig.make(**dict(SMALL, n_kv_heads=3))
    with pytest.raises(iam.IamError):
        iam.Model.random(bad)


def test_positions_past_max_ctx_are_refused(iam, torch_mod):
    """Every entry point that moves the device position checks it on the host first: a
    continuing generate or a profile run that would decode at max_ctx or beyond is refused
    with IAM_ERR_ARG before anything is launched, and the model stays usable."""
    torch = torch_mod
    cfg = iam.ModelConfig.make(**dict(SMALL, max_ctx=24))
    m = iam.Model.random(cfg, seed=11)
    toks = torch.empty(32, dtype=torch.int32, device="cuda")
    m.generate(5, 0, 20, 0.5, toks)  # positions 0..19: fits
    for call in (lambda: m.generate(-1, 0, 5, 0.5, toks),       # 20..24: past the cache
                 lambda: m.generate(3, 20, 5, 0.5, toks),        # explicit start past it
                 lambda: m.profile_steps(0.5, 5)):               # 20..24 again
        with pytest.raises(iam.IamError) as e:
            call()
        assert e.value.code == iam.IAM_ERR_ARG
    m.generate(-1, 0, 4, 0.5, toks)  # 20..23: exactly fills the cache
    torch.cuda.synchronize()
    m.status()  # no step ran at or past max_ctx
    with pytest.raises(iam.IamError):
        m.generate(-1, 0, 1, 0.5, toks)
    m.forward(7, cfg.max_ctx - 1, 0.5)  # an explicit position inside the cache is fine
    m.reset()
    m.generate(-1, 0, 3, 0.5, toks)  # after a reset the position is 0 again
    torch.cuda.synchronize()
    m.status()
    m.close()


def test_config3_mistral_layer(iam, ora, torch_mod):
    """One Mistral-7B decoder layer (d 4096, 32/8 heads, ffn 14336), KV cache
    of 1024 random N(0,1) fp16 tokens, gains 1.0, effort 0.25; plus the tied 32000-row head."""
    torch = torch_mod
    cfg = iam.ModelConfig.make(**dict(iam.MISTRAL_7B, n_layers=1, max_ctx=1040))
    m = iam.Model.random(cfg, seed=3)
    m.fill_kv_random(1024, seed=5)
    torch.cuda.synchronize()
    w = m.export_weights()
    om = oracle_for(ora, cfg, w)
    om.set_kv(m.read_weight(iam.W_K_CACHE, 0), m.read_weight(iam.W_V_CACHE, 0))
    logits = torch.empty(cfg.vocab, dtype=torch.float32, device="cuda")
    buf = torch.zeros(m.capture_floats(), dtype=torch.float32, device="cuda")
    m.capture(buf)
    m.forward(1234, 1024, 0.25, logits)
    torch.cuda.synchronize()
    nthreads = os.cpu_count() or 1
    # the 7 bucketMuls of the layer on the inputs the kernels used: exact selection
    check_captured_bucketmuls(ora, w, m.capture_records(buf), m.selected_rows_by_matrix(), 0.25, nthreads)
    best, ref, sel = om.forward(1234, 1024, 0.25, nthreads=nthreads)
    got = logits.cpu().numpy()
    check_steps([dict(pos=1024, err=rel_err(got, ref), same=(m.selected_rows() == sel), gpu=int(np.argmax(got)),
                      ref=best, ref_logits=ref, rms=float(np.sqrt(np.mean(ref.astype(np.float64) ** 2))))],
                max_flip_frac=1.0)
    assert m.selected_rows() > 0
    m.close()
