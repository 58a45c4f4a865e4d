"""Dense tensor-core path (iam_dense_*, tcgen05): the GEMM against an fp64 product of the same
fp16 matrix, the unpack kernel against its host restatement (itself pinned to the reference's
bucket fixtures), and the dense product of an unpacked matrix against the oracle's bucketMul
with every bucket row selected (bucketMul.cl:392-497).

Tolerances: the north star's floating-point bar is max-abs <= 1e-3 x RMS of the output.
precision 0 (activations as fp16 hi + lo, fp32 accumulation) is held to 1e-4 x RMS.
precision 1 (fp16 activations) does NOT meet the bar: rounding x to 11 bits alone measured
1.03e-3 x RMS on N(0,1) inputs (K = 4096) and 1.3e-3 with outlier channels, so it is checked
against 3e-3 and never used where parity is claimed."""
import numpy as np
import pytest
import torch

from conftest import GOLDEN_CASES, golden

pytestmark = pytest.mark.gpu

TOL_SPLIT = 1e-4
TOL_FP16 = 3e-3


def _w16(m, k, seed, dev):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(m, k, generator=g) * 0.02).half().to(dev)


def _x(n, k, seed, dev, outliers=True):
    g = torch.Generator().manual_seed(seed + 1)
    x = torch.randn(n, k, generator=g)
    if outliers:  # 1% of channels x20, as in the sweep config
        idx = torch.randperm(k, generator=g)[: max(1, k // 100)]
        x[:, idx] *= 20.0
    return x.to(dev)


def _rel_err(y, ref):
    ref = ref.double()
    rms = ref.pow(2).mean().sqrt().clamp_min(1e-30)
    return ((y.double() - ref).abs().max() / rms).item()


def _ref(w16, x, residual=None):
    y = x.double() @ w16.double().T
    return y if residual is None else y + residual.double()


@pytest.fixture(scope="module")
def dense(iam, cuda):
    d = iam.Dense(max_tokens=512, max_in_dim=16384, max_out_dim=16384)
    yield d
    d.close()


@pytest.mark.parametrize("m,k,n", [(4096, 4096, 1), (4096, 4096, 16), (4096, 4096, 128), (4096, 4096, 200),
                                   (1024, 4096, 300), (14336, 4096, 64), (4096, 14336, 128)])
def test_gemm_matches_fp64(iam, cuda, dense, m, k, n):
    w = _w16(m, k, m + k, cuda)
    x = _x(n, k, n, cuda)
    y = torch.empty(n, m, device=cuda)
    dense.gemm(w, x, y)
    dense.status()
    err = _rel_err(y, _ref(w, x))
    assert err <= TOL_SPLIT, err


@pytest.mark.parametrize("m,k,n", [(200, 72, 17), (130, 4104, 65), (16, 8, 1), (300, 1000, 129)])
def test_gemm_ragged_edges(iam, cuda, dense, m, k, n):
    """M, K and token counts off every tile multiple: the TMA boxes read zeros outside the
    matrices and the epilogue stores only inside."""
    w = _w16(m, k, 7, cuda)
    x = _x(n, k, 8, cuda, outliers=False)
    y = torch.full((n + 1, m), 123.0, device=cuda)  # one guard row after the output
    dense.gemm(w, x, y[:n])
    dense.status()
    assert _rel_err(y[:n], _ref(w, x)) <= TOL_SPLIT
    assert torch.all(y[n] == 123.0)


def test_gemm_fp16_activations(iam, cuda, dense):
    """precision 1 rounds every activation to fp16 (2^-11 relative), which alone costs ~1e-3 x
    RMS; the hi + lo split (precision 0, the default) is more exact by over an order of
    magnitude on the same inputs."""
    w = _w16(4096, 4096, 3, cuda)
    x = _x(64, 4096, 4, cuda, outliers=False)
    y = torch.empty(64, 4096, device=cuda)
    dense.gemm(w, x, y, precision=1)
    dense.status()
    err = _rel_err(y, _ref(w, x))
    assert err <= TOL_FP16, err
    xo = _x(64, 4096, 4, cuda, outliers=True)
    y1, y0 = torch.empty_like(y), torch.empty_like(y)
    dense.gemm(w, xo, y1, precision=1)
    dense.gemm(w, xo, y0, precision=0)
    e1, e0 = _rel_err(y1, _ref(w, xo)), _rel_err(y0, _ref(w, xo))
    assert e0 <= TOL_SPLIT and e0 < e1 / 10, (e0, e1)


def test_gemm_split_k_deterministic_and_residual_in_place(iam, cuda, dense):
    m, k, n = 4096, 14336, 32
    w = _w16(m, k, 11, cuda)
    x = _x(n, k, 12, cuda)
    r = torch.randn(n, m, device=cuda)
    ref = _ref(w, x, r)
    outs = []
    for split in (1, 3, 8, 3):
        y = r.clone()
        dense.gemm(w, x, y, residual=y, split_k=split)  # y := y + W x, in place
        dense.status()
        assert _rel_err(y, ref) <= TOL_SPLIT, split
        outs.append(y)
    assert torch.equal(outs[1], outs[3])  # the same split twice: the same bits


def test_gemm_rejects_bad_shapes(iam, cuda, dense):
    w = _w16(64, 12, 1, cuda)  # in_dim % 8 != 0: the TMA row stride would not be 16-byte aligned
    x = torch.randn(4, 12, device=cuda)
    y = torch.empty(4, 64, device=cuda)
    with pytest.raises(iam.IamError) as e:
        dense.gemm(w, x, y)
    assert e.value.code == iam.IAM_ERR_ARG
    w = _w16(64, 64, 1, cuda)
    with pytest.raises(iam.IamError):
        dense.gemm(w, torch.randn(513, 64, device=cuda), torch.empty(513, 64, device=cuda))  # > max_tokens


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_unpack_matches_restatement_on_reference_buckets(iam, cuda, weights_mod, case):
    g = golden(case)
    b = torch.from_numpy(g["buckets"].view(np.int16)).to(cuda)
    out_dim, in_dim = g["W"].shape
    w = torch.empty(out_dim, in_dim, dtype=torch.int16, device=cuda)
    if in_dim % 8:
        pytest.skip("dense rows must be 16-byte aligned")
    iam.dense_unpack(b, w)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(w.cpu().numpy().view(np.uint16), weights_mod.dense_packed(g["W"].view(np.float16)))


def test_unpack_of_gpu_bucketized_mistral_shape(iam, cuda, weights_mod):
    m, k = 1024, 4096  # wk / wv: 64 bucket columns
    w = _w16(m, k, 5, cuda)
    R, C = 16 * k, m // 16
    buckets = torch.empty(R, C, dtype=torch.int16, device=cuda)
    iam.bucketize(w.view(torch.int16), buckets)
    dense_w = torch.empty(m, k, dtype=torch.int16, device=cuda)
    iam.dense_unpack(buckets, dense_w)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dense_w.cpu().numpy().view(np.uint16), weights_mod.dense_packed(w.cpu().numpy()))


def test_dense_equals_bucketmul_with_every_row_selected(iam, cuda, ora, dense):
    """The oracle's bucketMul (bucketMul.cl:392-497) over ALL bucket rows and the tensor-core
    GEMM over the unpacked matrix compute the same product."""
    g = golden("bm_128x512.npz")
    b = torch.from_numpy(g["buckets"].view(np.int16)).to(cuda)
    out_dim, in_dim = g["W"].shape
    w = torch.empty(out_dim, in_dim, dtype=torch.int16, device=cuda)
    iam.dense_unpack(b, w)
    xs = g["x"]  # [5][512] fp32, the fixture's inputs
    y = torch.empty(xs.shape[0], out_dim, device=cuda)
    dense.gemm(w, torch.from_numpy(xs).to(cuda), y)
    dense.status()
    rows = np.arange(16 * in_dim, dtype=np.int32)
    for t in range(xs.shape[0]):
        ref = ora.bucket_mul(g["buckets"], xs[t], rows)
        rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
        assert float(np.max(np.abs(y[t].cpu().numpy() - ref))) <= TOL_SPLIT * rms, t
