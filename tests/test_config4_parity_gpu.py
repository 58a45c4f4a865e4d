"""The full 32-layer Mistral-7B-shaped model (random N(0, 0.02) weights, tied 32000-token
embeddings, seed 0) against the CPU oracle at efforts 0.25, 0.5 and 1.0: the workload the
decode benchmark measures.

The 128-token prompt (seed 1, ids uniform in [3, 32000)) is ingested token by token
(test_generation.cpp:202-213), then 32 greedy decode steps (test_generation.cpp:239-291).
At four of them every operation of the step is checked on the inputs the GPU used, layer by
layer (decode_parity.check_captured_layers): the 224 bucketMuls select exactly the oracle's
rows (cutoff bits, counts) with outputs within 1e-3 x RMS; RMSNorm, the RoPE'd fp16 K/V
append and the residual stream are bit for bit the oracle's; attention, SiLU * up and the LM
head within 1e-4 x RMS; the greedy token is the oracle's (up to a near tie).  The
captured-graph generation then decodes exactly the eager steps' tokens.

Whole trajectories are not compared at this depth: the fp16 KV cache turns the last-bit
differences of two fp32 summation orders into whole fp16 ulps, which move later cutoffs by
a row now and then, and over 32 layers of a random-init network the two trajectories part.
"""
import os

import numpy as np
import pytest

from decode_parity import check_captured_layers

pytestmark = pytest.mark.gpu

PROMPT_LEN = 128
N_DECODE = 32
CHECK_STEPS = (0, 10, 20, N_DECODE - 1)


@pytest.fixture(scope="module")
def config4(iam, cuda):
    import torch
    cfg = iam.ModelConfig.make(**dict(iam.MISTRAL_7B, max_ctx=PROMPT_LEN + N_DECODE + 8))
    m = iam.Model.random(cfg, seed=0)
    w = m.export_weights()
    yield cfg, m, w, torch
    m.close()


@pytest.mark.timeout(1800)
@pytest.mark.parametrize("effort", [0.25, 0.5, 1.0])
def test_config4_every_op_matches_oracle(iam, ora, config4, effort):
    cfg, m, w, torch = config4
    nthreads = os.cpu_count() or 1
    prompt = np.random.default_rng(1).integers(3, cfg.vocab, PROMPT_LEN).tolist()
    logits = torch.empty(cfg.vocab, dtype=torch.float32, device="cuda")
    m.reset()
    for pos, tok in enumerate(prompt):
        m.forward(tok, pos, effort, logits)
    torch.cuda.synchronize()
    first = tok = int(torch.argmax(logits).item())

    buf = torch.zeros(m.capture_floats(), dtype=torch.float32, device="cuda")
    m.capture(buf)
    toks, worst = [], []
    try:
        for i in range(N_DECODE):
            pos = PROMPT_LEN + i
            m.forward(tok, pos, effort, logits)
            torch.cuda.synchronize()
            got = logits.cpu().numpy()
            if i in CHECK_STEPS:
                kv = [(m.read_weight(iam.W_K_CACHE, l), m.read_weight(iam.W_V_CACHE, l)) for l in range(cfg.n_layers)]
                worst.append(check_captured_layers(ora, cfg, w, m.capture_records(buf), m.selected_rows_by_matrix(), kv,
                                                   pos, effort, got, nthreads))
            tok = int(np.argmax(got))
            toks.append(tok)
    finally:
        m.capture(None)
    bm, att, lm = (max(x[j] for x in worst) for j in range(3))
    print(f"config 4, effort {effort}: {len(CHECK_STEPS)} steps x 32 layers checked; bucketMul worst {bm:.2e}, "
          f"attention {att:.2e}, LM head {lm:.2e} x rms")

    # the captured-graph path decodes the eager steps' greedy tokens bit for bit
    m.reset()
    for pos, t in enumerate(prompt):
        m.forward(t, pos, effort)
    gen = torch.empty(N_DECODE, dtype=torch.int32, device="cuda")
    m.generate(first, PROMPT_LEN, N_DECODE, effort, gen)
    torch.cuda.synchronize()
    assert gen.cpu().tolist() == toks
