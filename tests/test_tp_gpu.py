"""Tensor-parallel decode on 2 GPUs (IAM_TP_TEST_WORLD=4 or 8 for more; one process per GPU,
the library's NVLink exchanges) against the single-GPU model built from the same seed: the
sharded weights are slices of the same bucketized matrices.  Skipped when the box has fewer
GPUs than ranks.  The default step exchanges everything inside its kernels; the second test
runs the small model with the exchange launches put back (IAM_TP_PUSH=0: all-gathers of the
heads and of gate/up; IAM_TP_FUSED=0: also the gather-reduce launches after o and down).
"""
import datetime
import os
import socket
import tempfile

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

# Tensor parallelism keeps every bit of the single-GPU decode: each bucketMul selects the same
# rows on every rank (replicated stats and probes, the same cutoff search on the same input),
# every output is summed over the same input ranges in the same order (the range decomposition
# follows from the whole matrix; the row-parallel o and down ranks exchange their ranges'
# partials and add them in range order), the attention chunks follow from the context alone,
# and the LM head rows do not depend on the vocabulary split.  So logits, selections and greedy
# tokens must be identical, step by step, to the unsharded model built from the same seed.
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


def _fill(model, kv_prefix):
    model.reset()
    if kv_prefix:
        model.fill_kv_random(kv_prefix, seed=5)


def _generate(model, torch, effort, kv_prefix, n=32):
    dev = torch.device("cuda", torch.cuda.current_device())
    _fill(model, kv_prefix)
    toks = torch.zeros(n, dtype=torch.int32, device=dev)
    model.generate(7, kv_prefix, n, effort, toks)
    torch.cuda.synchronize()
    model.status()  # raises if a tensor-parallel exchange gave up on a peer
    return toks.cpu().numpy().copy()


def _teacher_forced(model, torch, cfg_d, effort, kv_prefix, seq):
    """logits and per-bucketMul selected-row counts of every step when the model is fed 7,
    seq[0], seq[1], ... (the same tokens for both models)."""
    dev = torch.device("cuda", torch.cuda.current_device())
    _fill(model, kv_prefix)
    logits = torch.empty(cfg_d["vocab"], dtype=torch.float32, device=dev)
    outs, sels = [], []
    for i, tok in enumerate([7] + list(seq[:-1])):
        model.forward(int(tok), kv_prefix + i, effort, logits)
        torch.cuda.synchronize()
        outs.append(logits.cpu().numpy().copy())
        sels.append(model.selected_rows_by_matrix().copy())
    model.status()
    return np.stack(outs), np.stack(sels)  # logits [steps, vocab], counts [steps, layers, 7]


CASES = (("small", SMALL, 3, (0.25, 0.5, 1.0), 0), ("mistral1", MISTRAL_1L, 11, (0.25,), 1024))


def _rank_main(rank, world, port, outdir, env=None, cases=CASES):
    import sys
    os.environ.update(env or {})  # read when a model is created
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import torch
    import torch.distributed as dist
    from conftest import load_pkg
    iam = load_pkg()
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=180))
    res = {}
    for name, cfg_d, seed, efforts, prefix in cases:
        cfg = iam.ModelConfig.make(**cfg_d)
        seqs = {}
        if rank == 0:  # the unsharded model, same seed: its greedy tokens and logits
            one = iam.Model.random(cfg, seed=seed, device=0)
            for eff in efforts:
                seqs[eff] = _generate(one, torch, eff, prefix)
                res[(name, "one", eff)] = (seqs[eff],) + _teacher_forced(one, torch, cfg_d, eff, prefix, seqs[eff])
            one.close()
        box = [seqs]
        dist.broadcast_object_list(box, src=0)
        seqs = box[0]
        uid = [iam.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        tp = iam.Model.random(cfg, seed=seed, device=rank, tp=(rank, world, uid[0]))
        for eff in efforts:
            toks = _generate(tp, torch, eff, prefix)
            res[(name, "tp", eff)] = (toks,) + _teacher_forced(tp, torch, cfg_d, eff, prefix, seqs[eff])
        tp.close()
        dist.barrier()
    np.save(os.path.join(outdir, f"rank{rank}.npy"), np.array([res], dtype=object), allow_pickle=True)
    dist.barrier()
    dist.destroy_process_group()


def rel_err(a, ref):
    a, ref = np.asarray(a, np.float64), np.asarray(ref, np.float64)
    return float(np.max(np.abs(a - ref)) / max(np.sqrt(np.mean(ref * ref)), 1e-30))


def _check_identical(world, env=None, cases=CASES):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"tensor-parallel test needs {world} GPUs")
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank_main, args=(world, _free_port(), d, env, cases), nprocs=world, join=True,
                           start_method="spawn")
        res = [np.load(os.path.join(d, f"rank{r}.npy"), allow_pickle=True)[0] for r in range(world)]
    tag = " ".join(f"{k}={v}" for k, v in (env or {}).items())
    r0 = res[0]
    for (name, kind, eff), (toks_tp, logits_tp, sel_tp) in r0.items():
        if kind != "tp":
            continue
        toks_1, logits_1, sel_1 = r0[(name, "one", eff)]
        # o and down report each rank's share; q, k, v, gate, up the whole selection
        sel = sel_tp.copy()
        sel[:, :, [3, 6]] = sum(rr[(name, "tp", eff)][2][:, :, [3, 6]] for rr in res)
        ntok = int(np.argmax(toks_tp != toks_1)) if (toks_tp != toks_1).any() else len(toks_1)
        nsel = int(np.all(sel == sel_1, axis=(1, 2)).sum())
        nlog = int(sum(np.array_equal(a.view(np.uint32), b.view(np.uint32)) for a, b in zip(logits_tp, logits_1)))
        print(f"tp{world}{' ' + tag if tag else ''} {name} effort {eff}: {nlog}/{len(logits_1)} steps with bit-identical logits, "
              f"{nsel}/{len(sel_1)} with identical selections; free-running greedy tokens equal for "
              f"{ntok}/{len(toks_1)}")
        assert np.array_equal(toks_tp, toks_1), (name, eff, toks_tp, toks_1)
        assert np.array_equal(sel, sel_1), (name, eff)
        assert nlog == len(logits_1), (name, eff)
        assert np.all(np.isfinite(logits_tp)), (name, eff)
        for rr in res[1:]:  # every rank holds the same gathered logits and generated tokens
            t_r, l_r, s_r = rr[(name, "tp", eff)]
            assert np.array_equal(l_r, logits_tp), (name, eff)
            assert np.array_equal(t_r, toks_tp), (name, eff)
            assert np.array_equal(s_r[:, :, :3], sel_tp[:, :, :3]), (name, eff)


def test_tp_matches_single_gpu(iam, cuda):
    _check_identical(WORLD)


@pytest.mark.parametrize("env", [{"IAM_TP_PUSH": "0"}, {"IAM_TP_FUSED": "0"}], ids=["allgather", "gather_reduce"])
def test_tp_exchange_launches_match_single_gpu(iam, cuda, env):
    _check_identical(WORLD, env, cases=(("small", SMALL, 3, (0.25, 1.0), 0),))


def _mismatch_main(rank, world, port, outdir):
    import sys
    if rank == world - 1:
        os.environ["IAM_TP_PUSH"] = "0"  # this rank alone: the exchange launches put back
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import torch
    import torch.distributed as dist
    from conftest import load_pkg
    iam = load_pkg()
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=180))
    uid = [iam.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    try:
        iam.Model.random(iam.ModelConfig.make(**SMALL), seed=3, device=rank, tp=(rank, world, uid[0])).close()
        code = 0
    except iam.IamError as e:
        code = e.code
    with open(os.path.join(outdir, f"rank{rank}.txt"), "w") as f:
        f.write(str(code))
    dist.barrier()
    dist.destroy_process_group()


def test_tp_mismatched_settings_refused(iam, cuda):
    """Ranks started with different exchange settings would launch different exchange
    sequences and wait on each other; model creation refuses them on every rank instead."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"tensor-parallel test needs {WORLD} GPUs")
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_mismatch_main, args=(WORLD, _free_port(), d), nprocs=WORLD, join=True,
                           start_method="spawn")
        codes = [int(open(os.path.join(d, f"rank{r}.txt")).read()) for r in range(WORLD)]
    assert codes == [iam.IAM_ERR_ARG] * WORLD, codes
