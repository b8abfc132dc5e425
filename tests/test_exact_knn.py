"""gann_exact_knn (brute-force ground truth) against a torch int64/float64
brute force on the same data."""
import numpy as np
import pytest
import torch

from gustann_b200.index import datagen


def _ref_u8(X, Q, k, ip):
    # exact integer arithmetic on the CPU (no int64 matmul on CUDA)
    x = X.cpu().to(torch.int64)
    q = Q.cpu().to(torch.int64)
    dot = q @ x.T
    d = -dot if ip else (q * q).sum(1)[:, None] + (x * x).sum(1)[None, :] - 2 * dot
    # ascending by (distance, id)
    key = d * (1 << 32) + torch.arange(x.shape[0], device=x.device)[None, :]
    v, i = torch.topk(key, k, dim=1, largest=False)
    return i.to(torch.int32), (v >> 32).to(torch.float32)


@pytest.mark.gpu
@pytest.mark.parametrize("n,dim,nq,k,ip", [(5000, 128, 333, 10, False), (4099, 64, 65, 100, False),
                                           (3000, 128, 40, 1, True), (777, 48, 31, 128, False)])
def test_u8_exact_ids_and_distances(n, dim, nq, k, ip):
    from gustann_b200.api import exact_knn, METRIC_IP, METRIC_L2
    g = torch.Generator(device="cuda").manual_seed(n + dim)
    X = torch.randint(0, 256, (n, dim), generator=g, device="cuda", dtype=torch.uint8)
    Q = torch.randint(0, 256, (nq, dim), generator=g, device="cuda", dtype=torch.uint8)
    ids, d = exact_knn(X, Q, k, METRIC_IP if ip else METRIC_L2)
    ri, rd = _ref_u8(X, Q, k, ip)
    assert torch.equal(d.cpu(), rd)
    assert torch.equal(ids.cpu(), ri)


@pytest.mark.gpu
@pytest.mark.parametrize("n,dim,nq,k,ip", [(6000, 96, 100, 10, False), (2500, 768, 37, 100, True),
                                           (1000, 42, 50, 16, False)])
def test_f32_matches_float64(n, dim, nq, k, ip):
    from gustann_b200.api import exact_knn, METRIC_IP, METRIC_L2
    spec = datagen.MixtureSpec("deep", n, dim, 20, 0.1, center_scale=dim ** -0.5)
    X = datagen.base_vectors(spec, device="cuda")
    Q = datagen.query_vectors(spec, nq, device="cuda")
    if dim * 4 % 16:
        # rows must be 16-byte aligned: pad the row stride, keep `dim` columns
        pad = (dim + 3) // 4 * 4
        Xp = torch.zeros((n, pad), device="cuda")
        Xp[:, :dim] = X
        Qp = torch.zeros((nq, pad), device="cuda")
        Qp[:, :dim] = Q
        X, Q = Xp[:, :dim], Qp[:, :dim]
    ids, d = exact_knn(X, Q, k, METRIC_IP if ip else METRIC_L2)
    x, q = X.double(), Q.double()
    dd = -(q @ x.T) if ip else torch.cdist(q, x) ** 2
    rv, ri = torch.topk(dd, k, dim=1, largest=False)
    # identical ids except near-ties; distances within fp32 rounding
    hit = sum(len(set(a.tolist()) & set(b.tolist())) for a, b in zip(ids.cpu(), ri.cpu()))
    assert hit >= 0.999 * nq * k
    assert torch.allclose(d.double(), rv, rtol=1e-4, atol=1e-4)
    assert bool((d[:, 1:] >= d[:, :-1]).all())


@pytest.mark.gpu
def test_bad_arguments():
    from gustann_b200.api import exact_knn, GustANNError
    X = torch.zeros((100, 16), dtype=torch.uint8, device="cuda")
    with pytest.raises(GustANNError):
        exact_knn(X, X.float(), 5)
    with pytest.raises(GustANNError):
        exact_knn(X, X, 129)
    ids, d = exact_knn(X, X[:0], 5)
    assert ids.shape == (0, 5)
