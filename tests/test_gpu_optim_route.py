"""Sparse Adam (the reference's _C.adamUpdate / SparseGaussianAdam) and the
rectangle routing op (_C.get_local2j_ids_bool_adjust_mode6) against golden
vectors the reference CUDA module produced (tests/golden/make_golden_optim.py),
against the CPU oracle, and the compact-row Adam against the dense one."""
import os
import sys

import numpy as np
import pytest
import torch

from blitzgs_b200 import ops, rasterizer as RZ, scene as S, step as ST
from oracle import rasterizer_oracle as O
from tests.helpers import scene_params

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_golden_optim as G  # noqa: E402


@pytest.fixture(scope="module")
def golden():
    g = np.load(os.path.join(HERE, "golden", "golden_optim.npz"))
    adam, route = G.inputs()
    assert str(g["input_sha256"]) == G.checksum(adam, route)
    return g, adam, route


def _run_adam(param, grads, vis, dev, rows_form=False):
    N, M = param.shape
    p = param.clone().to(dev)
    m = torch.zeros_like(p)
    v = torch.zeros_like(p)
    rows = torch.nonzero(vis).flatten().to(dev)
    for t, gr in enumerate(grads, start=1):
        if rows_form:
            ops.adam_update_rows(p, gr.to(dev)[rows].contiguous(), m, v, rows, G.lr_at(t), 0.9, 0.999, G.EPS, N, M)
        else:
            RZ._C.adamUpdate(p, gr.to(dev), m, v, vis.to(dev), G.lr_at(t), 0.9, 0.999, G.EPS, N, M)
    torch.cuda.synchronize()
    return p.cpu(), m.cpu(), v.cpu()


def test_adam_bit_exact_against_reference(golden, cuda_device):
    g, adam, _ = golden
    for (M, N), (param, grads, vis) in zip(G.ADAM_CASES, adam):
        p, m, v = _run_adam(param, grads, vis, cuda_device)
        assert np.array_equal(p[vis].numpy().view(np.uint32), g[f"adam{M}_param"].view(np.uint32))
        assert np.array_equal(m[vis].numpy().view(np.uint32), g[f"adam{M}_exp_avg"].view(np.uint32))
        assert np.array_equal(v[vis].numpy().view(np.uint32), g[f"adam{M}_exp_avg_sq"].view(np.uint32))
        # invisible Gaussians keep their parameters and zero moments
        assert torch.equal(p[~vis], param[~vis]) and not m[~vis].any() and not v[~vis].any()


def test_adam_rows_form_equals_dense_form(golden, cuda_device):
    _, adam, _ = golden
    for param, grads, vis in adam:
        a = _run_adam(param, grads, vis, cuda_device)
        b = _run_adam(param, grads, vis, cuda_device, rows_form=True)
        for x, y in zip(a, b):
            assert torch.equal(x, y)


def test_adam_matches_oracle_on_a_longer_run(cuda_device):
    """Twenty steps on new seeded data with a visibility mask that changes
    every step: all rows, bit for bit, against the CPU restatement."""
    gen = torch.Generator().manual_seed(77)
    N, M = 30_000, 4
    param = torch.randn(N, M, generator=gen)
    p, m, v = param.clone().to(cuda_device), torch.zeros(N, M, device=cuda_device), torch.zeros(N, M,
                                                                                                 device=cuda_device)
    po, mo, vo = param.clone(), torch.zeros(N, M), torch.zeros(N, M)
    for t in range(1, 21):
        gr = torch.randn(N, M, generator=gen) * 10 ** (-1 - t % 4)
        vis = torch.rand(N, generator=gen) < 0.5
        RZ._C.adamUpdate(p, gr.to(cuda_device), m, v, vis.to(cuda_device), G.lr_at(t), 0.9, 0.999, G.EPS, N, M)
        O.adam_update(po, gr, mo, vo, vis, G.lr_at(t), 0.9, 0.999, G.EPS)
    for x, y in ((p, po), (m, mo), (v, vo)):
        assert torch.equal(x.cpu(), y)


@pytest.mark.parametrize("avoid", [False, True])
def test_mode6_routing_bit_exact(golden, cuda_device, avoid):
    g, _, (means2D, radii, rects) = golden
    ca = {"avoid_pixel_all2all": avoid}
    mask = RZ._C.get_local2j_ids_bool_adjust_mode6(G.H, G.W, 0, G.WS, means2D.to(cuda_device), radii.to(cuda_device),
                                                    rects.to(cuda_device), ca).cpu().numpy()
    assert np.array_equal(mask, g[f"mode6_avoid{int(avoid)}"])
    assert np.array_equal(mask, O.route_rect_bool(means2D.numpy(), radii.numpy(), G.H, G.W, rects.numpy(), avoid))


def test_sparse_gaussian_adam_sparse_and_dense_gradients_agree(cuda_device):
    """One SparseGaussianAdam step from the fused step's sparse gradients
    equals the reference's way -- the same gradient made dense, with the
    radius > 0 visibility -- bit for bit."""
    sc = S.mid(seed=6, P=300_000, n_cams=1)
    cam = sc.cameras[0].to(cuda_device)
    gt = S.target_image(6, cam.image_height, cam.image_width).to(cuda_device)
    rs = S.raster_settings(cam, device=cuda_device)
    model = [t.to(cuda_device).clone().requires_grad_(True) for t in scene_params(sc)]
    loss, l1, ss, radii, *_ = ST.view_loss(model, rs, gt, sparse_grad=True)
    loss.backward()
    grads = [p.grad for p in model]
    results = []
    for sparse in (True, False):
        params = [p.detach().clone().requires_grad_(True) for p in model]
        for p, g in zip(params, grads):
            p.grad = g if sparse else g.to_dense()
        opt = RZ.SparseGaussianAdam([{"params": [p], "lr": 1e-3} for p in params], lr=1e-3, eps=1e-15)
        opt.step(radii > 0, params[0].shape[0])
        results.append([p.detach().cpu() for p in params])
    for a, b in zip(*results):
        assert torch.equal(a, b)
    changed = (results[0][0] != model[0].detach().cpu()).any(dim=1)
    assert changed.any() and not changed.all()


@pytest.mark.parametrize("bsz", [3, 4, 7])
def test_adam_rows_fuse_the_batch_gradient_scaling(golden, cuda_device, bsz):
    """The trainer's `param.grad /= bsz` before the step (train_internal.py:
    504-515), fused into the rows update, gives the same bits as dividing
    with PyTorch first."""
    _, adam, _ = golden
    for param, grads, vis in adam:
        N, M = param.shape
        rows = torch.nonzero(vis).flatten().to(cuda_device)
        outs = []
        for fused in (False, True):
            p = param.clone().to(cuda_device)
            m = torch.zeros_like(p)
            v = torch.zeros_like(p)
            for t, gr in enumerate(grads, start=1):
                g = gr.to(cuda_device)
                if not fused:
                    g /= bsz
                scale = float(np.float32(1.0) / np.float32(bsz)) if fused else 1.0
                ops.adam_update_rows(p, g[rows].contiguous(), m, v, rows, G.lr_at(t), 0.9, 0.999, G.EPS, N, M,
                                     grad_scale=scale)
            outs.append((p.cpu(), m.cpu(), v.cpu()))
        for a, b in zip(*outs):
            assert torch.equal(a.view(torch.int32), b.view(torch.int32))


def test_densification_stats_from_the_fused_step_match_reference(cuda_device):
    """view_loss(densify=...) accumulates max_radii2D, the viewspace gradient
    norm and the count of the visible Gaussians (train_internal.py:340-371,
    gaussian_model.py:792-794) from its render-backward record; compared with
    the same updates applied to the reference's own radii and means2D
    gradient of config 1 (golden_tiny.npz)."""
    from blitzgs_b200 import densify as DZ
    from tests.conftest import golden_path
    gp = golden_path("golden_tiny.npz")
    g = np.load(gp)
    if "g_means2D" not in g:
        pytest.skip("golden_tiny.npz predates the full gradient rows")
    sc = S.tiny()
    cam = sc.cameras[0].to(cuda_device)
    gt = S.target_image(0, cam.image_height, cam.image_width).to(cuda_device)
    model = [t.to(cuda_device).requires_grad_(True) for t in scene_params(sc)]
    rs = S.raster_settings(cam, device=cuda_device)
    stats = DZ.DensificationStats(sc.P, cuda_device)
    for sparse in (False, True):  # two steps: the statistics accumulate
        for p in model:
            p.grad = None
        loss, *_ = ST.view_loss(model, rs, gt, scale_reg_weight=0.0, sparse_grad=sparse, densify=stats)
        loss.backward()
    torch.cuda.synchronize()
    radii = torch.from_numpy(g["radii"])
    vis = radii > 0
    gm = torch.from_numpy(g["g_means2D"]).reshape(-1, 2)
    mr, acc, den = torch.zeros(sc.P), torch.zeros(sc.P, 1), torch.zeros(sc.P, 1)
    for _ in range(2):
        O.densification_stats(mr, acc, den, radii, gm)
    assert torch.equal(stats.max_radii2D.cpu(), mr)
    assert torch.equal(stats.denom.cpu(), den)
    assert not stats.xyz_gradient_accum.cpu()[~vis].any()
    from tests.helpers import normwise_rel
    assert normwise_rel(stats.xyz_gradient_accum.cpu(), acc) <= 1e-4
