"""Tensor-parallel decode on 2 GPUs (one process per GPU, NCCL inside the library) against
the single-GPU model built from the same seed: the sharded weights are slices of the same
bucketized matrices, so the selection is identical and only the fp32 summation order of the
row-parallel all-reduces differs.  Needs two GPUs; skipped on a one-GPU box.
"""
import datetime
import os
import socket
import tempfile

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

LOGIT_TOL = 5e-3  # max |tp - single| / rms(single) of the logits
SMALL = dict(dim=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn_dim=512, vocab=512, max_ctx=96)
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


def test_tp2_matches_single_gpu(iam, cuda):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("tensor-parallel test needs 2 GPUs")
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank_main, args=(world, _free_port(), d), nprocs=world, join=True, start_method="spawn")
        r0 = np.load(os.path.join(d, "rank0.npy"), allow_pickle=True)[0]
        r1 = np.load(os.path.join(d, "rank1.npy"), allow_pickle=True)[0]
    for (name, kind, eff), (logits_tp, sel_tp, toks_tp) in r0.items():
        if kind != "tp":
            continue
        logits_1, sel_1, toks_1 = r0[(name, "one", eff)]
        l1, s1, t1 = r1[(name, "tp", eff)]
        for a, b, c in zip(logits_tp, logits_1, l1):
            assert np.array_equal(a, c), (name, eff)          # both ranks hold the same gathered logits
            assert rel_err(a, b) < LOGIT_TOL, (name, eff, rel_err(a, b))
            assert int(np.argmax(a)) == int(np.argmax(b)), (name, eff)
        assert sel_tp == s1 == sel_1, (name, eff, sel_tp, s1, sel_1)  # same selection, counted once
        assert np.array_equal(toks_tp, t1), (name, eff)
        assert np.array_equal(toks_tp, toks_1), (name, eff, toks_tp, toks_1)
