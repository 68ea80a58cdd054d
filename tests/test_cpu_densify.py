"""Densification statistics (blitzgs_b200.densify) against the reference's
masked updates restated in the oracle, over several seeded cameras."""
import torch

from blitzgs_b200 import densify as DZ
from oracle import rasterizer_oracle as O


def test_stats_equal_reference_updates_over_cameras():
    gen = torch.Generator().manual_seed(5)
    P = 5000
    st = DZ.DensificationStats(P, "cpu")
    mr, acc, den = torch.zeros(P), torch.zeros(P, 1), torch.zeros(P, 1)
    for _ in range(6):
        radii = torch.randint(-1, 40, (P,), generator=gen).clamp(min=0).to(torch.int32)
        grad = torch.randn(P, 2, generator=gen) * 1e-3
        O.densification_stats(mr, acc, den, radii, grad)
        # the fused steps pass the visible rows only, in list order (not sorted)
        rows = torch.nonzero(radii > 0).flatten()
        rows = rows[torch.randperm(rows.numel(), generator=gen)]
        DZ.update_max_radii(st, radii)
        DZ.accumulate_grad(st, rows, grad[rows])
    assert torch.equal(st.max_radii2D, mr)
    assert torch.equal(st.xyz_gradient_accum, acc)
    assert torch.equal(st.denom, den)
    avg = st.average_grad()
    assert torch.all(avg[den.flatten() == 0] == 0)
    seen = den.flatten() > 0
    assert torch.equal(avg[seen], acc[seen] / den[seen])


def test_empty_camera_and_reset():
    st = DZ.DensificationStats(10, "cpu")
    DZ.accumulate_grad(st, torch.zeros(0, dtype=torch.int64), torch.zeros(0, 2))
    DZ.update_max_radii(st, torch.zeros(10, dtype=torch.int32))
    assert not st.denom.any() and not st.max_radii2D.any()
    DZ.update_max_radii(st, torch.arange(10, dtype=torch.int32))
    DZ.accumulate_grad(st, torch.tensor([3, 7]), torch.tensor([[3.0, 4.0], [0.0, 1.0]]))
    assert st.max_radii2D[9] == 9 and st.xyz_gradient_accum[3, 0] == 5.0 and st.denom[7, 0] == 1
    st.reset()
    assert not st.xyz_gradient_accum.any() and not st.denom.any() and not st.max_radii2D.any()
