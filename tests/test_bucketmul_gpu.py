"""GPU parity of the bucketMul operator (C ABI via ctypes) against the CPU oracle.

Bar: cutoff bit-exact, selected bucket-row SET identical, outputs
within max-abs 1e-3 x output RMS for fp16 weights with fp32 accumulation.
"""
import numpy as np
import pytest

from conftest import GOLDEN_CASES, golden

pytestmark = pytest.mark.gpu

TOL = 1e-3  # max |gpu - oracle| / rms(oracle)


def rel_err(a, ref):
    a, ref = np.asarray(a, np.float64), np.asarray(ref, np.float64)
    rms = np.sqrt(np.mean(ref * ref))
    return float(np.max(np.abs(a - ref)) / (rms if rms > 0 else 1.0))


def dev(a, torch):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(a).cuda()


def host(t, dtype):
    return t.cpu().numpy().view(dtype)


@pytest.fixture(scope="module")
def torch_mod(cuda):
    import torch
    return torch


@pytest.fixture(scope="module")
def bm(iam, cuda):
    b = iam.BucketMul(0)
    yield b
    b.close()


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_cutoff_bit_exact(bm, torch_mod, case):
    torch = torch_mod
    g = golden(case)
    probes = dev(g["probes"], torch)
    out = torch.empty(1, dtype=torch.float32, device="cuda")
    iters = torch.empty(1, dtype=torch.int32, device="cuda")
    k = 0
    for xi in range(len(g["x_kinds"])):
        x = g["x"][xi]
        xd = dev(x, torch)
        for eff in g["efforts"]:
            bm.cutoff(xd, probes, len(x), float(eff), out, iters)
            torch.cuda.synchronize()
            assert host(out, np.uint32)[0] == g["cutoff"][k].view(np.uint32), (case, g["x_kinds"][xi], eff)
            assert int(iters.item()) == int(g["iters"][k])
            k += 1


@pytest.mark.parametrize("case", GOLDEN_CASES)
@pytest.mark.parametrize("stride", [4, 1])
def test_dispatch_set_and_mul(bm, torch_mod, ora, case, stride):
    """calcDispatch + mul (bucket_mul.hpp:147-252): selected rows identical, output within tol."""
    torch = torch_mod
    g = golden(case)
    stats = np.repeat(g["stats3"][:, None], 4, axis=1) if stride == 4 else g["stats3"]
    R, C = g["buckets"].shape
    d_stats, d_probes, d_buckets = dev(stats, torch), dev(g["probes"], torch), dev(g["buckets"], torch)
    rows = torch.empty(R, dtype=torch.int32, device="cuda")
    cnt = torch.empty(1, dtype=torch.int32, device="cuda")
    cut = torch.empty(1, dtype=torch.float32, device="cuda")
    out = torch.empty(16 * C, dtype=torch.float32, device="cuda")
    k = 0
    for xi in range(len(g["x_kinds"])):
        x = g["x"][xi]
        xd = dev(x, torch)
        for eff in g["efforts"]:
            bm.calc_dispatch(xd, d_stats, d_probes, 0, len(x), C, R, float(eff), stats_stride=stride)
            bm.read_dispatch(rows, cnt, cut)
            bm.mul(d_buckets, out)
            torch.cuda.synchronize()
            n = int(cnt.item())
            sel = np.unpackbits(g["sel_packed"][k])[:R].astype(bool)
            np.testing.assert_array_equal(rows[:n].cpu().numpy(), np.nonzero(sel)[0])
            assert host(cut, np.uint32)[0] == g["cutoff"][k].view(np.uint32)
            ref = ora.bucket_mul(g["buckets"], x, np.nonzero(sel)[0].astype(np.int32))
            assert rel_err(out.cpu().numpy(), ref) < TOL, (case, eff)
            k += 1


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_full_fused(bm, torch_mod, ora, case):
    """fullMul as one fused launch: count, cutoff, output."""
    torch = torch_mod
    g = golden(case)
    R, C = g["buckets"].shape
    d_stats, d_probes, d_buckets = dev(g["stats3"], torch), dev(g["probes"], torch), dev(g["buckets"], torch)
    cnt = torch.empty(1, dtype=torch.int32, device="cuda")
    cut = torch.empty(1, dtype=torch.float32, device="cuda")
    out = torch.empty(16 * C, dtype=torch.float32, device="cuda")
    for xi in range(len(g["x_kinds"])):
        x = g["x"][xi]
        xd = dev(x, torch)
        for eff in g["efforts"]:
            bm.full_mul(xd, d_stats, d_probes, d_buckets, 0, len(x), C, R, float(eff), out, stats_stride=1,
                        count=cnt, cutoff=cut)
            torch.cuda.synchronize()
            ref, n, c = ora.bucketmul_full(x, g["stats3"], 1, g["probes"], g["buckets"], float(eff))
            assert int(cnt.item()) == n
            assert host(cut, np.uint32)[0] == np.float32(c).view(np.uint32)
            assert rel_err(out.cpu().numpy(), ref) < TOL, (case, eff)


def test_deterministic(bm, torch_mod):
    torch = torch_mod
    g = golden("bm_128x512.npz")
    R, C = g["buckets"].shape
    d = [dev(a, torch) for a in (g["x"][4], g["stats3"], g["probes"], g["buckets"])]
    outs = []
    for _ in range(3):
        out = torch.empty(16 * C, dtype=torch.float32, device="cuda")
        bm.full_mul(d[0], d[1], d[2], d[3], 0, 512, C, R, 0.25, out, stats_stride=1)
        torch.cuda.synchronize()
        outs.append(out.cpu().numpy().view(np.uint32))
    assert (outs[0] == outs[1]).all() and (outs[1] == outs[2]).all()


def test_expert_offset(bm, torch_mod, ora, weights_mod):
    """expertNo > 0 offsets probes by 4096*expertNo and rows by expertSize*expertNo."""
    torch = torch_mod
    rng = np.random.default_rng(7)
    ws = [weights_mod.bucketize_fp16_packed((rng.standard_normal((64, 4096)) * 0.02).astype(np.float16))
          for _ in range(2)]
    buckets = np.concatenate([w.buckets for w in ws])
    stats = np.concatenate([w.stats for w in ws])
    probes = np.concatenate([w.probes for w in ws])
    x = rng.standard_normal(4096).astype(np.float32)
    R, C = ws[0].buckets.shape
    out = torch.empty(16 * C, dtype=torch.float32, device="cuda")
    cnt = torch.empty(1, dtype=torch.int32, device="cuda")
    bm.full_mul(dev(x, torch), dev(stats, torch), dev(probes, torch), dev(buckets, torch), 1, 4096, C, R, 0.3,
                out, stats_stride=4, count=cnt)
    torch.cuda.synchronize()
    ref, n, _ = ora.bucketmul_full(x, stats, 4, probes, buckets, 0.3, expert_no=1, expert_size=R)
    ref1, n1, _ = ora.bucketmul_full(x, ws[1].stats, 4, ws[1].probes, ws[1].buckets, 0.3)
    assert n == n1 == int(cnt.item())
    np.testing.assert_array_equal(ref, ref1)
    assert rel_err(out.cpu().numpy(), ref) < TOL


@pytest.mark.parametrize("bad", ["effort0", "effort_big", "effort_nan", "stride", "null", "dims"])
def test_invalid_arguments(bm, torch_mod, iam, bad):
    torch = torch_mod
    g = golden("bm_256x64.npz")
    R, C = g["buckets"].shape
    x, s, p, b = (dev(a, torch) for a in (g["x"][0], g["stats3"], g["probes"], g["buckets"]))
    out = torch.empty(16 * C, dtype=torch.float32, device="cuda")
    kw = dict(x=x, stats=s, probes=p, buckets=b, expert_no=0, in_size=64, bucket_cols=C, expert_size=R,
              effort=0.25, out=out, stats_stride=1)
    if bad == "effort0":
        kw["effort"] = 0.0
    elif bad == "effort_big":
        kw["effort"] = 1.5
    elif bad == "effort_nan":
        kw["effort"] = float("nan")
    elif bad == "stride":
        kw["stats_stride"] = 2
    elif bad == "null":
        kw["stats"] = None
    elif bad == "dims":
        kw["in_size"] = 0
    with pytest.raises(iam.IamError) as e:
        bm.full_mul(**kw)
    assert e.value.code == iam.IAM_ERR_ARG


def test_mul_without_dispatch_fails(iam, cuda):
    import torch
    b = iam.BucketMul(0)
    out = torch.empty(256, dtype=torch.float32, device="cuda")
    buckets = torch.zeros((1024, 16), dtype=torch.int16, device="cuda")
    with pytest.raises(iam.IamError):
        b.mul(buckets, out)
    b.close()


def test_gpu_bucketize_matches_reference_layout(iam, torch_mod):
    torch = torch_mod
    for case in GOLDEN_CASES:
        g = golden(case)
        out_dim, in_dim = g["W"].shape
        W = dev(g["W"], torch)
        buckets = torch.empty((16 * in_dim, out_dim // 16), dtype=torch.int16, device="cuda")
        s4 = torch.empty((16 * in_dim, 4), dtype=torch.int16, device="cuda")
        s1 = torch.empty(16 * in_dim, dtype=torch.int16, device="cuda")
        pr = torch.empty(in_dim, dtype=torch.int16, device="cuda")
        iam.bucketize(W, buckets, s4, s1, pr)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(host(buckets, np.uint16), g["buckets"])
        np.testing.assert_array_equal(host(s1, np.uint16), g["stats3"])
        np.testing.assert_array_equal(host(s4, np.uint16)[:, 0], g["stats3"])
        np.testing.assert_array_equal(host(pr, np.uint16), g["probes"])


SHAPES = {"wq": (4096, 4096), "wk": (1024, 4096), "w1": (14336, 4096), "w2": (4096, 14336)}


@pytest.fixture(scope="module")
def big_weights(iam, torch_mod, weights_mod):
    """Config-2 shapes: W ~ N(0, 0.02) fp16 from a seeded CUDA generator, bucketized on the GPU,
    checked against the host (numpy) bucketizer on a slice."""
    torch = torch_mod
    gen = torch.Generator(device="cuda").manual_seed(0)
    res = {}
    for name, (o, i) in SHAPES.items():
        W = (torch.randn((o, i), generator=gen, device="cuda") * 0.02).half().view(torch.int16)
        buckets = torch.empty((16 * i, o // 16), dtype=torch.int16, device="cuda")
        s1 = torch.empty(16 * i, dtype=torch.int16, device="cuda")
        pr = torch.empty(i, dtype=torch.int16, device="cuda")
        iam.bucketize(W, buckets, None, s1, pr)
        torch.cuda.synchronize()
        res[name] = (W, buckets, s1, pr)
    # layout spot check vs the numpy restatement on a 256-output slice
    W, buckets, s1, pr = res["wk"]
    Wn = host(W, np.uint16)[:256].view(np.float16)
    ref = weights_mod.bucketize_fp16_packed(Wn)
    Wsl = torch.from_numpy(Wn.view(np.int16).copy()).cuda()
    b2 = torch.empty((16 * 4096, 16), dtype=torch.int16, device="cuda")
    s2 = torch.empty(16 * 4096, dtype=torch.int16, device="cuda")
    p2 = torch.empty(4096, dtype=torch.int16, device="cuda")
    iam.bucketize(Wsl, b2, None, s2, p2)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host(b2, np.uint16), ref.buckets)
    np.testing.assert_array_equal(host(s2, np.uint16), ref.stats[:, 3])
    np.testing.assert_array_equal(host(p2, np.uint16), ref.probes)
    return res


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("xkind", ["gaussian", "outliers"])
def test_config2_shapes(bm, torch_mod, ora, big_weights, name, xkind):
    """Mistral attention/FFN shapes (x with 1% outliers x20) at every effort."""
    torch = torch_mod
    W, buckets, s1, pr = big_weights[name]
    o, i = SHAPES[name]
    rng = np.random.default_rng(11)
    x = rng.standard_normal(i).astype(np.float32)
    if xkind == "outliers":
        idx = rng.choice(i, i // 100, replace=False)
        x[idx] *= 20.0
    hb, hs, hp = host(buckets, np.uint16), host(s1, np.uint16), host(pr, np.uint16)
    xd = dev(x, torch)
    R, C = hb.shape
    out = torch.empty(16 * C, dtype=torch.float32, device="cuda")
    cnt = torch.empty(1, dtype=torch.int32, device="cuda")
    cut = torch.empty(1, dtype=torch.float32, device="cuda")
    for eff in [0.05, 0.1, 0.25, 0.5, 1.0]:
        bm.full_mul(xd, s1, pr, buckets, 0, i, C, R, eff, out, stats_stride=1, count=cnt, cutoff=cut)
        torch.cuda.synchronize()
        ref, n, c = ora.bucketmul_full(x, hs, 1, hp, hb, eff, nthreads=8)
        assert host(cut, np.uint32)[0] == np.float32(c).view(np.uint32), (name, eff)
        assert int(cnt.item()) == n, (name, eff)
        assert rel_err(out.cpu().numpy(), ref) < TOL, (name, eff)
