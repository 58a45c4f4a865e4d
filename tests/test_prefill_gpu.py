"""Batched dense prefill (iam_model_prefill) against the oracle's dense decode step
(ora_model_forward_dense: every bucket row selected) run token by token.  The reference ingests
a prompt one forward() at a time (test_generation.cpp:202-213); the prefill ingests it in one
pass of tensor-core products, and causal attention makes the two the same computation.

Bar: logits within 1e-3 x RMS (the north star's floating-point bar), the same greedy next
token, and KV caches within one fp16 ulp plus 1e-3 x RMS of the oracle's."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3
DECODE_TOL = 5e-3  # a bucketMul decode step after the prefill (the model tests' bar)
SMALL = dict(dim=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn_dim=512, vocab=512, max_ctx=96)


def rel_err(a, ref):
    a, ref = np.asarray(a, np.float64), np.asarray(ref, np.float64)
    rms = np.sqrt(np.mean(ref * ref))
    return float(np.max(np.abs(a - ref)) / (rms if rms > 0 else 1.0))


def kv_close(iam, m, om, layers, n_kv, max_ctx, hd, n_tokens):
    for l in range(layers):
        for which, ref_all in ((iam.W_K_CACHE, om.k_cache), (iam.W_V_CACHE, om.v_cache)):
            got = m.read_weight(which, l).reshape(n_kv, max_ctx, hd)[:, :n_tokens].view(np.float16).astype(np.float32)
            ref = ref_all.reshape(layers, n_kv, max_ctx, hd)[l, :, :n_tokens].view(np.float16).astype(np.float32)
            # the fp32 values behind them differ by the products' error (relative to the RMS of
            # a projection, not to each element, and growing through the layers: 2.1e-4 x RMS
            # measured at layer 1 of the Mistral shape); rounding each to fp16 can then land on
            # neighbouring values, one ulp (<= |ref| 2^-10) apart
            rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
            err = np.abs(got - ref) - np.abs(ref) * 2.0 ** -10
            assert float(err.max()) <= LOGIT_TOL * rms, (l, which, float(err.max()) / rms)


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


def test_prefill_matches_dense_oracle(small, iam, ora, torch_mod):
    torch = torch_mod
    cfg, m, w = small
    om = ora.OracleModel(cfg.as_dict(), w)
    prompt = np.random.default_rng(1).integers(3, cfg.vocab, 20).tolist()
    m.reset()
    logits = torch.empty(cfg.vocab, dtype=torch.float32, device="cuda")
    nxt = m.prefill(prompt, 0, logits)
    for pos, tok in enumerate(prompt):
        best, ref = om.forward_dense(tok, pos)
    got = logits.cpu().numpy()
    assert rel_err(got, ref) < LOGIT_TOL, rel_err(got, ref)
    assert nxt == best == int(np.argmax(got))
    kv_close(iam, m, om, cfg.n_layers, cfg.n_kv_heads, cfg.max_ctx, cfg.head_dim, len(prompt))


def test_prefill_in_chunks_and_two_calls(iam, ora, torch_mod, monkeypatch):
    """Chunks of 7 tokens (IAM_PREFILL_CHUNK) and a prompt split over two calls at different
    start positions give the same logits as one pass."""
    torch = torch_mod
    monkeypatch.setenv("IAM_PREFILL_CHUNK", "7")
    cfg = iam.ModelConfig.make(**SMALL)
    m = iam.Model.random(cfg, seed=9)
    om = ora.OracleModel(cfg.as_dict(), m.export_weights())
    prompt = np.random.default_rng(2).integers(3, cfg.vocab, 30).tolist()
    logits = torch.empty(cfg.vocab, dtype=torch.float32, device="cuda")
    m.prefill(prompt[:12], 0)
    nxt = m.prefill(prompt[12:], 12, logits)
    for pos, tok in enumerate(prompt):
        best, ref = om.forward_dense(tok, pos)
    assert rel_err(logits.cpu().numpy(), ref) < LOGIT_TOL
    assert nxt == best
    m.close()


@pytest.mark.parametrize("effort", [0.25, 1.0])
def test_decode_continues_after_prefill(small, iam, ora, torch_mod, effort):
    """The bucketMul decode step reads the KV cache the prefill wrote."""
    torch = torch_mod
    cfg, m, w = small
    om = ora.OracleModel(cfg.as_dict(), w)
    prompt = np.random.default_rng(3).integers(3, cfg.vocab, 16).tolist()
    m.reset()
    nxt = m.prefill(prompt, 0)
    for pos, tok in enumerate(prompt):
        best, _ = om.forward_dense(tok, pos)
    assert nxt == best
    logits = torch.empty(cfg.vocab, dtype=torch.float32, device="cuda")
    tok = nxt
    for i in range(4):
        m.forward(tok, len(prompt) + i, effort, logits)
        torch.cuda.synchronize()
        ref_best, ref, _ = om.forward(tok, len(prompt) + i, effort)
        got = logits.cpu().numpy()
        assert rel_err(got, ref) < DECODE_TOL, (i, rel_err(got, ref))
        assert int(np.argmax(got)) == ref_best
        tok = ref_best


def test_prefill_rejects_bad_arguments(small, iam):
    cfg, m, _ = small
    with pytest.raises(iam.IamError):
        m.prefill([1, 2, cfg.vocab], 0)  # token out of range
    with pytest.raises(iam.IamError):
        m.prefill([1] * 10, cfg.max_ctx - 5)  # past max_ctx
    with pytest.raises(iam.IamError):
        m.prefill([], 0)


def test_prefill_mistral_layers(iam, ora, torch_mod):
    """Two Mistral-7B decoder layers (d 4096, 32/8 heads, head_dim 128, ffn 14336) with the tied
    32000-row head: a 24-token prompt in one pass against 24 dense oracle steps."""
    torch = torch_mod
    cfg = iam.ModelConfig.make(**dict(iam.MISTRAL_7B, n_layers=2, max_ctx=64))
    m = iam.Model.random(cfg, seed=4)
    om = ora.OracleModel(cfg.as_dict(), m.export_weights())
    prompt = np.random.default_rng(4).integers(3, cfg.vocab, 24).tolist()
    logits = torch.empty(cfg.vocab, dtype=torch.float32, device="cuda")
    nxt = m.prefill(prompt, 0, logits)
    for pos, tok in enumerate(prompt):
        best, ref = om.forward_dense(tok, pos, nthreads=os.cpu_count() or 1)
    got = logits.cpu().numpy()
    assert rel_err(got, ref) < LOGIT_TOL, rel_err(got, ref)
    assert nxt == best
    kv_close(iam, m, om, cfg.n_layers, cfg.n_kv_heads, cfg.max_ctx, cfg.head_dim, len(prompt))
    m.close()


def test_prefill_without_the_silu_epilogue(iam, ora, torch_mod):
    """ffn_dim 144 is not a multiple of 128: gate and up stay separate matrices and SiLU runs as
    its own pass (the other configs take the fused gate|up epilogue)."""
    torch = torch_mod
    cfg = iam.ModelConfig.make(**dict(SMALL, ffn_dim=144))
    m = iam.Model.random(cfg, seed=11)
    om = ora.OracleModel(cfg.as_dict(), m.export_weights())
    prompt = np.random.default_rng(5).integers(3, cfg.vocab, 18).tolist()
    logits = torch.empty(cfg.vocab, dtype=torch.float32, device="cuda")
    nxt = m.prefill(prompt, 0, logits)
    for pos, tok in enumerate(prompt):
        best, ref = om.forward_dense(tok, pos)
    assert rel_err(logits.cpu().numpy(), ref) < LOGIT_TOL
    assert nxt == best
    m.close()
