"""The index builder's CUDA RobustPrune (gann_robust_prune) against the torch
restatement in gustann_b200.index.graph.robust_prune on the same candidates."""
import pytest
import torch

from gustann_b200.index import datagen
from gustann_b200.index.graph import robust_prune


def _candidates(X, b, k, seed):
    g = torch.Generator(device=X.device).manual_seed(seed)
    n = X.shape[0]
    pts = torch.randperm(n, generator=g, device=X.device)[:b]
    ci = torch.randint(0, n, (b, k), generator=g, device=X.device)
    ci[:, 0] = pts                                   # the point itself is never kept
    ci[:, -3:] = -1                                  # empty slots
    x = X.double()
    d = ((x[ci.clamp_min(0)] - x[pts][:, None, :]) ** 2).sum(-1).float()
    d = torch.where(ci >= 0, d, torch.full_like(d, float("inf")))
    # nearest-first with distinct ids (duplicates blanked)
    srt, o = torch.sort(ci, dim=1)
    dup = torch.zeros_like(srt, dtype=torch.bool)
    dup[:, 1:] = (srt[:, 1:] == srt[:, :-1]) & (srt[:, 1:] >= 0)
    ci = torch.where(dup.scatter(1, o, dup), torch.full_like(ci, -1), ci)
    d = torch.where(ci >= 0, d, torch.full_like(d, float("inf")))
    o = torch.argsort(d, dim=1, stable=True)
    return pts, torch.gather(ci, 1, o), torch.gather(d, 1, o)


@pytest.mark.gpu
@pytest.mark.parametrize("alpha", [1.0, 1.2])
def test_u8_prune_equals_torch(alpha):
    from gustann_b200.api import robust_prune as gpu_prune
    torch.backends.cuda.matmul.allow_tf32 = False
    spec = datagen.MixtureSpec("sift", 20000, 128, 20, 20.0)
    X = datagen.base_vectors(spec, device="cuda")
    pts, ci, cd = _candidates(X, 3000, 164, 7)
    got, gd = gpu_prune(X, pts, ci, cd, 64, alpha)
    # uint8 distances are exact integers on both sides (fp32 sums < 2^24)
    ref, rd = robust_prune(X, pts, ci, cd, 64, alpha, return_dist=True)
    assert torch.equal(got.long(), ref)
    assert torch.equal(gd, rd)


@pytest.mark.gpu
@pytest.mark.parametrize("dim", [96, 768])
def test_f32_prune_matches_torch(dim):
    from gustann_b200.api import robust_prune as gpu_prune
    torch.backends.cuda.matmul.allow_tf32 = False
    spec = datagen.MixtureSpec("deep", 8000, dim, 20, 0.1, center_scale=dim ** -0.5)
    X = datagen.base_vectors(spec, device="cuda")
    pts, ci, cd = _candidates(X, 1000, 128, 11)
    got, _ = gpu_prune(X, pts, ci, cd, 32, 1.2)
    ref = robust_prune(X, pts, ci, cd, 32, 1.2)
    # float32 distances are summed differently (direct vs norm expansion):
    # only borderline decisions may differ
    same = (got.long() == ref).all(1).float().mean().item()
    assert same > 0.97
    assert bool(((got >= 0).sum(1) > 0).all())


@pytest.mark.gpu
def test_prune_rejects_bad_arguments():
    from gustann_b200.api import GustANNError, robust_prune as gpu_prune
    X = torch.zeros((10, 16), dtype=torch.uint8, device="cuda")
    p = torch.zeros(2, dtype=torch.int32, device="cuda")
    c = torch.zeros((2, 300), dtype=torch.int32, device="cuda")
    with pytest.raises(GustANNError):
        gpu_prune(X, p, c, c.float(), 4, 1.2)           # k > 256
    with pytest.raises(GustANNError):
        gpu_prune(X, p, c[:, :8], c[:, :8].float(), 4, 0.5)   # alpha < 1


@pytest.mark.gpu
def test_sort_unique_rows_equals_torch():
    """gann_sort_unique_rows against the torch restatement (graph._dedup_sorted_rows)
    on rows with repeated ids at equal distances and empty slots."""
    from gustann_b200.api import sort_unique_rows
    from gustann_b200.index.graph import _dedup_sorted_rows
    g = torch.Generator(device="cuda").manual_seed(3)
    rows, k = 5000, 164
    ids = torch.randint(0, 400, (rows, k), generator=g, device="cuda")
    ids[torch.rand((rows, k), generator=g, device="cuda") < 0.1] = -1
    base = torch.rand(400, generator=g, device="cuda")
    d = torch.where(ids >= 0, base[ids.clamp_min(0)], torch.full_like(base[:1].expand(rows, k), float("inf")))
    ri, rd = _dedup_sorted_rows(ids, d)
    oi, od = sort_unique_rows(ids, d)
    assert torch.equal(oi.long(), ri)
    assert torch.equal(od, rd)
    # the nearest copy of a repeated id stays
    i2 = torch.tensor([[5, 7, 5, -1]], device="cuda")
    d2 = torch.tensor([[0.5, 0.2, 0.1, 0.0]], device="cuda")
    oi, od = sort_unique_rows(i2, d2)
    assert oi.tolist() == [[5, 7, -1, -1]] and od[0, :2].tolist() == [0.10000000149011612, 0.20000000298023224]
