"""The fused step writes dense parameter gradients straight into ``.grad``
(blitzgs_b200.step._GradBuffers): only the rows of the Gaussians a view sees
are written, into the existing gradient or into a reused buffer whose rows
from earlier views are zeroed again.  Checked against the gradients the same
step returns through ``torch.autograd.grad`` (which never writes in place), up
to the order of the render backward's float atomics (normwise 1e-6; a row
left over from an earlier view would be off by its whole value): one view, two views accumulated in one backward, a reused buffer
after ``.grad = None`` with a different view, after an in-place change of the
gradient, and while another reference to the old gradient is alive."""
import pytest
import torch

from blitzgs_b200 import scene as S, step as ST
from tests.helpers import normwise_rel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def case(cuda_device):
    sc = S.tiny(seed=3, P=20000)
    sc.cameras.append(S.look_at_camera([2.0, -1.0, -2.2], [0, 0, 0], [0, -1, 0], 256, 256, 1.0, uid=1))
    dev = cuda_device
    model = [t.to(dev).contiguous().requires_grad_(True) for t in
             (sc.xyz, sc.scaling, sc.rotation, sc.opacity, sc.features_dc, sc.features_rest)]
    rasters = [S.raster_settings(c.to(dev), device=dev) for c in sc.cameras]
    gts = [S.target_image(k, 256, 256).to(dev) for k in range(2)]
    return model, rasters, gts


def _loss(model, rasters, gts, views):
    total = None
    for v in views:
        loss = ST.view_loss(model, rasters[v], gts[v])[0]
        total = loss if total is None else total + loss
    return total


def _expected(model, rasters, gts, views):
    return torch.autograd.grad(_loss(model, rasters, gts, views), model)


def _close(a, e):
    return normwise_rel(a, e) <= 1e-6


def _check(model, expected):
    for p, e in zip(model, expected):
        assert p.grad is not None and p.grad.shape == p.shape
        assert _close(p.grad, e), normwise_rel(p.grad, e)


def test_in_place_gradients_equal_the_returned_ones(case):
    model, rasters, gts = case
    for p in model:
        p.grad = None
    _loss(model, rasters, gts, [0]).backward()
    _check(model, _expected(model, rasters, gts, [0]))
    first = [p.grad for p in model]
    # two views in one backward: the second adds into the first's rows
    for p in model:
        p.grad = None
    del first
    _loss(model, rasters, gts, [0, 1]).backward()
    _check(model, _expected(model, rasters, gts, [0, 1]))
    # a reused buffer after .grad = None, with only the other view: the first
    # view's rows must be zero again
    for p in model:
        p.grad = None
    _loss(model, rasters, gts, [1]).backward()
    _check(model, _expected(model, rasters, gts, [1]))
    # an in-place change of the gradient outside the step: the buffer is
    # zeroed in full before it is used again
    for p in model:
        p.grad.add_(1.0)
        p.grad = None
    _loss(model, rasters, gts, [0]).backward()
    _check(model, _expected(model, rasters, gts, [0]))
    # someone still holds the old gradient: it is left alone
    held = [p.grad for p in model]
    snapshot = [g.clone() for g in held]
    for p in model:
        p.grad = None
    _loss(model, rasters, gts, [1]).backward()
    _check(model, _expected(model, rasters, gts, [1]))
    for g, s in zip(held, snapshot):
        assert torch.equal(g, s)
    # an existing gradient of the caller's own is accumulated into
    for p in model:
        p.grad = torch.full_like(p, 0.5)
    _loss(model, rasters, gts, [0]).backward()
    exp = _expected(model, rasters, gts, [0])
    for p, e in zip(model, exp):
        assert _close(p.grad, e + 0.5)
