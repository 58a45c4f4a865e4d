"""Tensor-parallel host logic on CPU: the shard layout the library reports (iam_tp_shard_info,
no GPU needed) and, on world_size-2 gloo ranks, the Megatron split of a bucketMul checked on
the oracle against the unsharded result.

Column-parallel (q, k, v, gate, up): every rank runs the same cutoff search and selection on
the replicated x and stats, and multiplies its own bucket columns; gathering the column slices
must give the unsharded output bit for bit.  Row-parallel (o, down): every rank runs the same
cutoff search on the full x[0:P] and keeps the selected rows of its own inputs; the selected
row sets partition the unsharded selection exactly and the summed partial outputs match the
unsharded output within the bucketMul tolerance (the fp32 summation order changes).
"""
import datetime
import os
import socket
import tempfile

import numpy as np
import pytest

from conftest import ROOT, golden

TOL = 1e-3  # max |sharded - unsharded| / rms(unsharded)
CASES = ["bm_256x64.npz", "bm_128x512.npz"]
EFFORTS = (0.1, 0.25, 1.0)


def _cfg(iam, **kw):
    base = dict(dim=256, n_layers=2, n_heads=8, n_kv_heads=4, head_dim=32, ffn_dim=512, vocab=512, max_ctx=64)
    base.update(kw)
    return iam.ModelConfig.make(**base)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_shard_info_partitions_every_matrix(iam, world):
    cfg = iam.ModelConfig.make(**iam.MISTRAL_7B, max_ctx=2048)
    full = iam.tp_shard_info(cfg, 0, 1)
    shards = [iam.tp_shard_info(cfg, r, world) for r in range(world)]
    for name in iam.MATRIX_NAMES:
        c0, C, i0, n_in = full[name]
        cols = sorted((s[name][0], s[name][0] + s[name][1]) for s in shards)
        ins = sorted((s[name][2], s[name][3]) for s in shards)
        if name in ("o", "down"):  # row-parallel: every rank all columns, a slice of inputs
            assert all(c == (0, C) for c in cols)
            assert ins[0][0] == 0 and ins[-1][1] == n_in
            assert all(a[1] == b[0] for a, b in zip(ins, ins[1:]))
            assert len({b - a for a, b in ins}) == 1
        else:  # column-parallel: a slice of columns, all inputs
            assert all(i == (0, n_in) for i in ins)
            assert cols[0][0] == 0 and cols[-1][1] == C
            assert all(a[1] == b[0] for a, b in zip(cols, cols[1:]))
    vocab = sorted((s["vocab"][0], s["vocab"][0] + s["vocab"][1]) for s in shards)
    assert vocab[0][0] == 0 and vocab[-1][1] == cfg.vocab
    # rank r's heads: q columns of heads [r*H/T, (r+1)*H/T), kv columns of its kv heads
    for r, s in enumerate(shards):
        assert s["q"][0] * 16 == r * (cfg.n_heads // world) * cfg.head_dim
        assert s["k"][0] * 16 == r * (cfg.n_kv_heads // world) * cfg.head_dim
        assert s["o"][2] == r * (cfg.n_heads // world) * cfg.head_dim      # o's inputs = this rank's heads
        assert s["down"][2] == s["gate"][0] * 16                            # down's inputs = its FFN slice


def test_shard_info_rejects_uneven_worlds(iam):
    cfg = iam.ModelConfig.make(**iam.MISTRAL_7B, max_ctx=2048)
    for world in (3, 5, 16):
        with pytest.raises(iam.IamError) as e:
            iam.tp_shard_info(cfg, 0, world)
        assert e.value.code in (iam.IAM_ERR_UNSUPPORTED, iam.IAM_ERR_ARG)
    with pytest.raises(iam.IamError):
        iam.tp_shard_info(cfg, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, outdir):
    import sys
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist
    from oracle import ora
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    report = []
    for case in CASES:
        g = golden(case)
        buckets, stats, probes = g["buckets"], g["stats3"], g["probes"]
        in_dim, C = probes.size, buckets.shape[1]
        for xi in range(g["x"].shape[0]):
            x = g["x"][xi]
            for eff in EFFORTS:
                full, n_full, cut_full = ora.bucketmul_full(x, stats, 1, probes, buckets, float(eff))
                cut, _ = ora.find_cutoff(x, probes, float(eff))  # same on every rank: replicated x, probes
                rows = ora.prepare_dispatch(x, stats, 1, cut)
                # column-parallel: own columns, gathered in rank order
                cl = C // world
                part = ora.bucket_mul(np.ascontiguousarray(buckets[:, rank * cl:(rank + 1) * cl]), x, rows)
                parts = [torch.zeros(16 * cl) for _ in range(world)]
                dist.all_gather(parts, torch.from_numpy(part))
                col_out = torch.cat(parts).numpy()
                # row-parallel: own inputs' selected rows, partial outputs summed
                il = in_dim // world
                mine = rows[(rows >= 16 * rank * il) & (rows < 16 * (rank + 1) * il)]
                partial = torch.from_numpy(ora.bucket_mul(buckets, x, mine))
                dist.all_reduce(partial)
                counts = torch.tensor([len(mine)])
                dist.all_reduce(counts)
                report.append(dict(case=case, xi=xi, eff=eff, cut_same=bool(cut.tobytes() == cut_full.tobytes()),
                                   n_full=n_full, n_sum=int(counts.item()),
                                   col_exact=bool(np.array_equal(col_out.view(np.uint32), full.view(np.uint32))),
                                   row_err=float(np.max(np.abs(partial.numpy().astype(np.float64) - full)) /
                                                 max(float(np.sqrt(np.mean(full.astype(np.float64) ** 2))), 1e-30))))
    np.save(os.path.join(outdir, f"rank{rank}.npy"), np.array(report, dtype=object), allow_pickle=True)
    dist.barrier()
    dist.destroy_process_group()


def test_bucketmul_split_on_gloo_ranks_matches_unsharded_oracle():
    import torch.multiprocessing as mp
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank_main, args=(world, _free_port(), d), nprocs=world, join=True, start_method="spawn")
        for r in range(world):
            report = np.load(os.path.join(d, f"rank{r}.npy"), allow_pickle=True)
            assert len(report) == len(CASES) * 5 * len(EFFORTS)
            for e in report:
                assert e["cut_same"], e          # identical cutoff on every rank
                assert e["n_sum"] == e["n_full"], e  # row shards partition the selection
                assert e["col_exact"], e         # column shards: bit-exact
                assert e["row_err"] < TOL, e     # row shards: summation order only
