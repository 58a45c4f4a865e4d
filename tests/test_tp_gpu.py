"""Tensor-parallel decode on 2 GPUs (IAM_TP_TEST_WORLD=4 or 8 for more; one process per GPU,
the library's NVLink exchanges) against the single-GPU model built from the same seed: the
sharded weights are slices of the same bucketized matrices, so the selection is identical and
only the fp32 summation order of the row-parallel sums differs.  Skipped when the box has
fewer GPUs than ranks.
"""
import datetime
import os
import socket
import tempfile

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

# max |tp - single| / rms(single) of the logits.  Every layer after the first sees inputs that
# differ from the single-GPU run in the last bits (world partial sums added in another order),
# so a row at the cutoff can be selected on one side only; the gap grows with the number of
# ranks.  Greedy tokens and the argmax must still be identical.
LOGIT_TOL = 5e-3
LOGIT_TOL_WIDE = 2e-2  # more than 2 ranks
SEL_TOL = 5e-3         # relative difference of the selected-row totals
WORLD = int(os.environ.get("IAM_TP_TEST_WORLD", "2"))  # ranks of the group (one GPU each)
SMALL = dict(dim=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn_dim=512, vocab=512, max_ctx=96)
if WORLD > 2:  # heads, kv heads and bucket columns divisible by 4 and 8
    SMALL = dict(dim=256, n_layers=2, n_heads=8, n_kv_heads=8, head_dim=64, ffn_dim=512, vocab=512, max_ctx=96)
MISTRAL_1L = dict(dim=4096, n_layers=1, n_heads=32, n_kv_heads=8, head_dim=128, ffn_dim=14336, vocab=32000,
                  max_ctx=1152)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(model, torch, cfg_d, effort, kv_prefix):
    """forward logits at three positions after a random KV prefix of kv_prefix tokens, then 32
    greedy tokens from the same point (reset and prefix refilled in between)."""
    dev = torch.device("cuda", torch.cuda.current_device())
    model.reset()
    if kv_prefix:
        model.fill_kv_random(kv_prefix, seed=5)
    logits = torch.empty(cfg_d["vocab"], dtype=torch.float32, device=dev)
    outs = []
    for i, tok in enumerate([5, 17, 3]):
        model.forward(tok, kv_prefix + i, effort, logits)
        torch.cuda.synchronize()
        outs.append(logits.cpu().numpy().copy())
    sel = model.selected_rows()
    model.reset()
    if kv_prefix:
        model.fill_kv_random(kv_prefix, seed=5)
    toks = torch.zeros(32, dtype=torch.int32, device=dev)
    model.generate(7, kv_prefix, 32, effort, toks)
    torch.cuda.synchronize()
    model.status()  # raises if a tensor-parallel exchange gave up on a peer
    return outs, sel, toks.cpu().numpy().copy()


def _rank_main(rank, world, port, outdir):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import torch
    import torch.distributed as dist
    from conftest import load_pkg
    iam = load_pkg()
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    res = {}
    for name, cfg_d, seed, efforts, prefix in (("small", SMALL, 3, (0.25, 0.5, 1.0), 0),
                                               ("mistral1", MISTRAL_1L, 11, (0.25,), 1024)):
        uid = [iam.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        cfg = iam.ModelConfig.make(**cfg_d)
        tp = iam.Model.random(cfg, seed=seed, device=rank, tp=(rank, world, uid[0]))
        for eff in efforts:
            res[(name, "tp", eff)] = _run(tp, torch, cfg_d, eff, prefix)
        tp.close()
        if rank == 0:  # the unsharded model, same seed
            one = iam.Model.random(cfg, seed=seed, device=0)
            for eff in efforts:
                res[(name, "one", eff)] = _run(one, torch, cfg_d, eff, prefix)
            one.close()
        dist.barrier()
    np.save(os.path.join(outdir, f"rank{rank}.npy"), np.array([res], dtype=object), allow_pickle=True)
    dist.barrier()
    dist.destroy_process_group()


def rel_err(a, ref):
    a, ref = np.asarray(a, np.float64), np.asarray(ref, np.float64)
    return float(np.max(np.abs(a - ref)) / max(np.sqrt(np.mean(ref * ref)), 1e-30))


def test_tp_matches_single_gpu(iam, cuda):
    import torch
    import torch.multiprocessing as mp
    world = WORLD
    if torch.cuda.device_count() < world:
        pytest.skip(f"tensor-parallel test needs {world} GPUs")
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank_main, args=(world, _free_port(), d), nprocs=world, join=True, start_method="spawn")
        res = [np.load(os.path.join(d, f"rank{r}.npy"), allow_pickle=True)[0] for r in range(world)]
    r0 = res[0]
    tol = LOGIT_TOL if world <= 2 else LOGIT_TOL_WIDE
    for (name, kind, eff), (logits_tp, sel_tp, toks_tp) in r0.items():
        if kind != "tp":
            continue
        logits_1, sel_1, toks_1 = r0[(name, "one", eff)]
        errs = [rel_err(a, b) for a, b in zip(logits_tp, logits_1)]
        print(f"tp{world} {name} effort {eff}: logits rel err {max(errs):.2e}, selected {sel_tp} vs {sel_1}")
        for a, b, e in zip(logits_tp, logits_1, errs):
            assert e < tol, (name, eff, e)
            assert int(np.argmax(a)) == int(np.argmax(b)), (name, eff)
        assert abs(sel_tp - sel_1) <= SEL_TOL * sel_1, (name, eff, sel_tp, sel_1)
        assert np.array_equal(toks_tp, toks_1), (name, eff, toks_tp, toks_1)
        for rr in res[1:]:  # every rank holds the same gathered logits, count and tokens
            l_r, s_r, t_r = rr[(name, "tp", eff)]
            for a, c in zip(logits_tp, l_r):
                assert np.array_equal(a, c), (name, eff)
            assert s_r == sel_tp and np.array_equal(t_r, toks_tp), (name, eff)
