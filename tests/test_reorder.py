"""Record order grouped by coarse partition (gustann_b200/index/reorder.py).

The permutation must be a permutation, and along it the rows' nearest sampled
centers (exact squared L2, ties to the lower center index) must be
non-decreasing, with input order kept inside a center. Integer-valued rows
keep every distance exact in both the kernel and the check.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", ["u8", "f32"])
def test_partition_order_groups_rows_by_nearest_center(dtype):
    import torch
    from gustann_b200.index.reorder import partition_order
    g = torch.Generator().manual_seed(3)
    n, d, parts = 20000, 32, 64
    X = torch.randint(0, 256 if dtype == "u8" else 16, (n, d), generator=g, dtype=torch.uint8)
    if dtype == "f32":
        X = X.to(torch.float32)
    perm = partition_order(X.cuda(), parts=parts, seed=5, block=4096).cpu()
    assert torch.equal(torch.sort(perm).values, torch.arange(n))
    # the centers the function samples, and every row's nearest one (float64)
    pick = torch.randperm(n, generator=torch.Generator().manual_seed(5))[:parts].sort().values
    Xd = X.to(torch.float64)
    C = Xd[pick]
    dist = torch.cat([((Xd[s:s + 2000, None, :] - C[None]) ** 2).sum(-1) for s in range(0, n, 2000)])
    label = dist.argmin(1)          # exact integers; argmin takes the first index among ties
    lab = label[perm].numpy()
    assert (np.diff(lab) >= 0).all()
    for c in np.unique(lab)[:8]:
        rows = perm.numpy()[lab == c]
        assert (np.diff(rows) > 0).all()
