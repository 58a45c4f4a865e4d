"""iam_bucketmul_full_noalloc: the bucketMul for callers that cannot allocate device memory
(allocator or memory-pool callbacks, plug-ins whose host framework owns every device
allocation).  Its scratch is a built-in __device__ array, so it must give what the
allocating iam_bucketmul_full gives, call after call, and refuse shapes beyond that
array's size.  Collected last on purpose (file name) so a failure here comes after every
other test has run.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-3  # max |noalloc - full| / rms(full), the bucketMul parity tolerance


def rel_err(a, ref):
    a, ref = np.asarray(a, np.float64), np.asarray(ref, np.float64)
    rms = np.sqrt(np.mean(ref * ref))
    return float(np.max(np.abs(a - ref)) / (rms if rms > 0 else 1.0))


def _weights(iam, torch, out_dim, in_dim, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    W = (torch.randn((out_dim, in_dim), generator=gen, device="cuda") * 0.02).half().view(torch.int16)
    buckets = torch.empty((16 * in_dim, out_dim // 16), dtype=torch.int16, device="cuda")
    s4 = torch.empty((16 * in_dim, 4), dtype=torch.int16, device="cuda")
    probes = torch.empty(in_dim, dtype=torch.int16, device="cuda")
    iam.bucketize(W, buckets, s4, None, probes)
    x = torch.randn(in_dim, generator=gen, device="cuda")
    return buckets, s4, probes, x


@pytest.mark.parametrize("shape", [(4096, 4096), (4096, 14336), (1024, 512)])
def test_noalloc_matches_full_on_consecutive_calls(iam, cuda, shape):
    import torch
    out_dim, in_dim = shape
    C, R = out_dim // 16, 16 * in_dim
    bm = iam.BucketMul(0)
    for call, (seed, effort) in enumerate([(1, 0.25), (2, 0.6)]):  # two calls in a row
        buckets, s4, probes, x = _weights(iam, torch, out_dim, in_dim, seed + 10 * out_dim)
        ref = torch.empty(out_dim, dtype=torch.float32, device="cuda")
        got = torch.full((out_dim,), float("nan"), dtype=torch.float32, device="cuda")
        cnt_ref = torch.zeros(1, dtype=torch.int32, device="cuda")
        cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
        cut_ref = torch.zeros(1, dtype=torch.float32, device="cuda")
        cut = torch.zeros(1, dtype=torch.float32, device="cuda")
        bm.full_mul(x, s4, probes, buckets, 0, in_dim, C, R, effort, ref, stats_stride=4, count=cnt_ref,
                    cutoff=cut_ref)
        iam.bucketmul_full_noalloc(x, s4, probes, buckets, 0, in_dim, C, R, effort, got, stats_stride=4,
                                   count=cnt, cutoff=cut)
        torch.cuda.synchronize()
        assert int(cnt.item()) == int(cnt_ref.item()) > 0, call
        assert cut.cpu().numpy().view(np.uint32)[0] == cut_ref.cpu().numpy().view(np.uint32)[0], call
        assert rel_err(got.cpu().numpy(), ref.cpu().numpy()) < TOL, call
    bm.close()


def test_noalloc_rejects_shapes_beyond_its_scratch(iam, cuda):
    import torch
    in_dim, cols = 16, 1025  # out_dim 16400 > 16384
    buckets = torch.zeros((16 * in_dim, cols), dtype=torch.int16, device="cuda")
    s1 = torch.zeros(16 * in_dim, dtype=torch.int16, device="cuda")
    probes = torch.zeros(in_dim, dtype=torch.int16, device="cuda")
    x = torch.zeros(in_dim, dtype=torch.float32, device="cuda")
    out = torch.zeros(16 * cols, dtype=torch.float32, device="cuda")
    with pytest.raises(iam.IamError) as e:
        iam.bucketmul_full_noalloc(x, s1, probes, buckets, 0, in_dim, cols, 16 * in_dim, 0.5, out, stats_stride=1)
    assert e.value.code == iam.IAM_ERR_ARG
    assert "1024" in str(e.value)
