"""Decode attention against the CPU oracle on both kernel layouts, at contexts on either side
of each switch between them.

Contexts of at most 256 tokens (kAttnLaneShortMax, one chunk per KV head) and of at least 2048
(kAttnLaneMinCtx) take the tensor-core layout, the others the half-warp layout; the choice is
made on the device from the position, so one captured step serves every context.  Two
Mistral-7B-shaped layers (d 4096, 32/8 heads, head_dim 128) over a random N(0, 1) fp16 KV
prefix; each case decodes two steps, and on each step every operation is checked on the inputs
the GPU used (decode_parity.check_captured_layers): attention over the GPU's own cache
(aux.cl:497-540, :204-225, :370-384) within 1e-4 x RMS, and the bucketMuls, norms, KV append
and LM head as in the other model tests.  Config 5's context (8192 tokens) is the last case.
"""
import os

import numpy as np
import pytest

from decode_parity import check_captured_layers

pytestmark = pytest.mark.gpu


@pytest.mark.timeout(900)
@pytest.mark.parametrize("ctx", [100, 255, 1000, 2046, 2500, 8192])
def test_long_context_attention_matches_oracle(iam, ora, cuda, ctx):
    import torch
    cfg = iam.ModelConfig.make(**dict(iam.MISTRAL_7B, n_layers=2, max_ctx=ctx + 8))
    m = iam.Model.random(cfg, seed=4)
    try:
        m.fill_kv_random(ctx, seed=6)
        torch.cuda.synchronize()
        w = m.export_weights()
        logits = torch.empty(cfg.vocab, dtype=torch.float32, device="cuda")
        buf = torch.zeros(m.capture_floats(), dtype=torch.float32, device="cuda")
        nthreads = os.cpu_count() or 1
        tok = 4321
        m.capture(buf)
        worst = 0.0
        for pos in (ctx, ctx + 1):  # contexts ctx + 1 and ctx + 2 tokens
            m.forward(tok, pos, 0.25, logits)
            torch.cuda.synchronize()
            got = logits.cpu().numpy()
            kv = [(m.read_weight(iam.W_K_CACHE, l), m.read_weight(iam.W_V_CACHE, l)) for l in range(cfg.n_layers)]
            _, att, _ = check_captured_layers(ora, cfg, w, m.capture_records(buf), m.selected_rows_by_matrix(), kv,
                                              pos, 0.25, got, nthreads)
            worst = max(worst, att)
            tok = int(np.argmax(got))
        m.capture(None)
        print(f"context {ctx + 1}..{ctx + 2}: attention worst {worst:.2e} x rms")
    finally:
        m.close()
