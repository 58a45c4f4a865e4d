"""Decode-step parity helpers shared by the model tests (GPU model against the CPU oracle).

Two checks, because the cutoff search is a discontinuous function of its input:

* bucketMul on identical inputs.  A capture (iam_model_capture) records, for one decode step,
  every layer's bucketMul inputs exactly as the kernels used them, their cutoffs and outputs.
  The oracle's bucketMul (bucketMul.cl:68-497 restated) runs on the same inputs: the cutoff
  bits and the selected-row count must be equal and the outputs within BM_TOL x RMS.
* whole steps, teacher forced.  GPU and oracle decode the same token sequence (the GPU's
  greedy tokens).  Their fp32 sums run in different orders, so a bucket row whose importance
  sits within rounding of the cutoff can go either way and move one matrix's selection by a
  row ("a flip", visible as a different selected-row total); such a step is reported as one and
  held to FLIP_TOL, every other step to LOGIT_TOL with the same greedy token (up to a near tie).
"""
import numpy as np

BM_TOL = 1e-3      # bucketMul output, max |gpu - oracle| / rms(oracle), identical inputs
LOGIT_TOL = 1e-3   # logits of a step whose selections equal the oracle's
FLIP_TOL = 5e-2    # logits of a step where a row on the cutoff went the other way

MATS = ("q", "k", "v", "o", "gate", "up", "down")


def rel_err(a, ref):
    a, ref = np.asarray(a, np.float64), np.asarray(ref, np.float64)
    rms = np.sqrt(np.mean(ref * ref))
    return float(np.max(np.abs(a - ref)) / (rms if rms > 0 else 1.0))


def check_captured_bucketmuls(ora, weights, recs, counts, effort, nthreads=1):
    """Every bucketMul of a captured step against the oracle on the captured inputs.
    weights: Model.export_weights(); recs: Model.capture_records(); counts: the step's
    selected_rows_by_matrix().  Returns the worst output error."""
    worst = 0.0
    for l, rec in enumerate(recs):
        lw = weights["layers"][l]
        xs = {"q": rec["x_qkv"], "k": rec["x_qkv"], "v": rec["x_qkv"], "o": rec["x_o"],
              "gate": rec["x_gu"], "up": rec["x_gu"], "down": rec["x_down"]}
        outs = {"q": rec["q"], "k": rec["k"], "v": rec["v"], "o": rec["out_o"], "gate": rec["gate"],
                "up": rec["up"], "down": rec["out_down"]}
        res = {"o": rec["res_o"], "down": rec["res_down"]}
        for mi, name in enumerate(MATS):
            bw = lw[name]
            x = xs[name]
            ref, n, cut = ora.bucketmul_full(x, np.asarray(bw.stats).reshape(-1), 1, bw.probes, bw.buckets, effort,
                                             in_dim=bw.in_dim, nthreads=nthreads)
            got_cut = np.float32(rec["cutoff"][mi])
            assert got_cut.view(np.uint32) == np.float32(cut).view(np.uint32), (l, name, got_cut, cut)
            assert int(counts[l, mi]) == n, (l, name, int(counts[l, mi]), n)
            if name in res:  # out = residual + bucketMul (add32, bucketMul.cl:517-520)
                full = (res[name].astype(np.float32) + ref.astype(np.float32)).astype(np.float32)
                err = float(np.max(np.abs(outs[name].astype(np.float64) - full)) /
                            max(np.sqrt(np.mean(ref.astype(np.float64) ** 2)), 1e-30))
            else:
                err = rel_err(outs[name], ref)
            assert err < BM_TOL, (l, name, err)
            worst = max(worst, err)
    return worst


GLUE_TOL = 1e-4    # attention, LM head on identical inputs (their fp32 orders and expf differ)


def check_captured_layers(ora, cfg, weights, recs, counts, kv, pos, effort, logits, nthreads=1):
    """Every operation of a captured decode step on the inputs the GPU used, layer by layer:
    RMSNorm * gain (aux.cl:156-196, bit for bit), the 7 bucketMuls (check_captured_bucketmuls),
    RoPE of k and its fp16 append together with v's (attention.hpp:207-309, bit for bit),
    attention over the GPU's cache (aux.cl:497-540, :204-225, :370-384), SiLU * up
    (matrix.cl:27-32), the residual stream from layer to layer (bit for bit) and the final
    RMSNorm + LM head (aux.cl:454-490) with its greedy token.  kv: [(k, v)] per layer, each
    [n_kv_heads][max_ctx][head_dim] fp16 bits as read after the step."""
    c = cfg.as_dict()
    hd, nh, nkv = c["head_dim"], c["n_heads"], c["n_kv_heads"]
    worst_bm = check_captured_bucketmuls(ora, weights, recs, counts, effort, nthreads)
    cs = ora.rope_table(pos, hd, c["rope_theta"])
    worst_att = 0.0
    for l, rec in enumerate(recs):
        lw = weights["layers"][l]
        if l > 0:
            assert np.array_equal(rec["res_o"].view(np.uint32), recs[l - 1]["out_down"].view(np.uint32)), l
        h = ora.rmsnorm(rec["res_o"], lw["attn_norm"], c["norm_eps"])
        assert np.array_equal(rec["x_qkv"].view(np.uint32), h.view(np.uint32)), l
        k16 = ora.rope_apply(rec["k"], nkv, hd, cs).astype(np.float16).view(np.uint16)
        v16 = rec["v"].astype(np.float16).view(np.uint16)
        kc, vc = (np.asarray(a).reshape(nkv, c["max_ctx"], hd) for a in kv[l])
        assert np.array_equal(kc[:, pos, :], k16.reshape(nkv, hd)), l
        assert np.array_equal(vc[:, pos, :], v16.reshape(nkv, hd)), l
        att = ora.attention(c, ora.rope_apply(rec["q"], nh, hd, cs), kc, vc, pos + 1)
        e = rel_err(rec["x_o"], att)
        assert e < GLUE_TOL, (l, e)
        worst_att = max(worst_att, e)
        h2 = ora.rmsnorm(rec["out_o"], lw["ffn_norm"], c["norm_eps"])
        assert np.array_equal(rec["x_gu"].view(np.uint32), h2.view(np.uint32)), l
        e = rel_err(rec["x_down"], ora.silu_mul(rec["gate"], rec["up"]))
        assert e < GLUE_TOL, (l, e)
    hf = ora.rmsnorm(recs[-1]["out_down"], weights["final_norm"], c["norm_eps"])
    lm = weights["lm_head"] if weights["lm_head"] is not None else weights["embed"]
    ref = ora.lm_head(lm, hf, nthreads)
    e = rel_err(logits, ref)
    assert e < GLUE_TOL, e
    g, r = int(np.argmax(logits)), int(np.argmax(ref))
    if g != r:  # only a near tie may change the greedy token
        assert abs(float(ref[g]) - float(ref[r])) <= 2 * e * np.sqrt(np.mean(ref.astype(np.float64) ** 2)), (g, r)
    return worst_bm, worst_att, e


def teacher_forced_steps(m, om, tokens, start_pos, n_free, effort, logits, torch, nthreads=1, on_step=None):
    """Decodes tokens[i] at start_pos + i on both sides, then n_free more steps, each on the
    GPU's greedy token of the step before (the reference driver's loop,
    test_generation.cpp:239-291).  Returns (one dict per step, every token decoded or chosen)."""
    steps = []
    toks = list(tokens)
    total = len(tokens) + n_free
    for i in range(total):
        pos = start_pos + i
        m.forward(toks[i], pos, effort, logits)
        torch.cuda.synchronize()
        if on_step:
            on_step(i)
        best, ref, sel = om.forward(toks[i], pos, effort, nthreads=nthreads)
        got = logits.cpu().numpy()
        steps.append(dict(pos=pos, err=rel_err(got, ref), same=(m.selected_rows() == sel), gpu=int(np.argmax(got)),
                          ref=best, ref_logits=ref, rms=float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))))
        if i >= len(tokens) - 1:
            toks.append(int(np.argmax(got)))
    return steps, toks


def check_steps(steps, max_flip_frac=0.5):
    """Asserts the per-step bar; returns (flip steps, worst equal-selection error)."""
    flips = [s["pos"] for s in steps if not s["same"]]
    worst = 0.0
    for s in steps:
        if s["same"]:
            assert s["err"] < LOGIT_TOL, (s["pos"], s["err"])
            worst = max(worst, s["err"])
            if s["gpu"] != s["ref"]:  # only a near tie may change the greedy token
                gap = abs(float(s["ref_logits"][s["gpu"]]) - float(s["ref_logits"][s["ref"]]))
                assert gap <= 2 * s["err"] * s["rms"], (s["pos"], s["gpu"], s["ref"], gap)
        else:
            assert s["err"] < FLIP_TOL, (s["pos"], s["err"])
    assert len(flips) <= max_flip_frac * len(steps), flips
    return flips, worst
