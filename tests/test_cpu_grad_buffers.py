"""The in-place gradient buffers of the fused steps (step._GradBuffers), on the
CPU: the host logic that decides where a view's gradient rows go.

A toy autograd node follows the fused step's protocol: its backward asks
_GradBuffers.targets() for buffers, writes only its listed rows (set on a
fresh buffer, added when accumulating), reports them with written() and
returns no gradient; when targets() declines it returns dense gradients the
usual way.  Every scenario must leave .grad exactly where plain autograd
leaves it: a fresh buffer, a reused buffer whose earlier rows are zeroed, two
views in one backward, a buffer the caller still holds, a gradient changed in
place, a gradient the caller created, torch.autograd.grad, and a parameter
with a hook."""
import pytest
import torch
from torch.autograd.graph import get_gradient_edge

from blitzgs_b200 import ops
from blitzgs_b200 import step as ST

P = 50


class _Rows(torch.autograd.Function):
    """loss = sum over listed rows r of <w_r, a[r]> + <v_r, b[r]>."""

    @staticmethod
    def forward(ctx, a, b, rows, w, v, bufs):
        ctx.save_for_backward(rows, w, v)
        ctx.bufs = bufs
        ctx.params = (a, b)
        ctx.nodes = [get_gradient_edge(t).node for t in (a, b)]
        return (a[rows] * w).sum() + (b[rows] * v).sum()

    @staticmethod
    def backward(ctx, g):
        rows, w, v = ctx.saved_tensors
        inplace = ctx.bufs.targets(ctx.params, ctx.nodes)
        if inplace is not None:
            entries, accumulate = inplace
            for e, val in zip(entries, (g * w, g * v)):
                t = e["t"]
                if accumulate:
                    t[rows] += val
                else:
                    t[rows] = val
            ctx.bufs.written(ctx.params, entries, (rows, rows.numel()), fresh=not accumulate)
            return None, None, None, None, None, None
        ga = torch.zeros_like(ctx.params[0])
        gb = torch.zeros_like(ctx.params[1])
        ga[rows] = g * w
        gb[rows] = g * v
        return ga, gb, None, None, None, None


def _view(seed):
    g = torch.Generator().manual_seed(seed)
    rows = torch.randperm(P, generator=g)[: 5 + seed % 7]
    return rows, torch.randn(rows.numel(), 3, generator=g), torch.randn(rows.numel(), 1, generator=g)


def _expected(views):
    a = torch.zeros(P, 3)
    b = torch.zeros(P, 1)
    for rows, w, v in views:
        a[rows] += w
        b[rows] += v
    return a, b


@pytest.fixture
def bufs(monkeypatch):
    def zero_rows(ts, rows, n):
        for t in ts:
            t.view(t.shape[0], -1)[rows[:n].long()] = 0.0
    monkeypatch.setattr(ops, "zero_rows", zero_rows)
    return ST._GradBuffers()


def _params():
    return torch.randn(P, 3).requires_grad_(True), torch.randn(P, 1).requires_grad_(True)


def _loss(a, b, bufs, *seeds):
    views = [_view(s) for s in seeds]
    return sum(_Rows.apply(a, b, r, w, v, bufs) for r, w, v in views), views


def _check(a, b, views):
    ea, eb = _expected(views)
    assert torch.equal(a.grad, ea) and torch.equal(b.grad, eb)


def test_fresh_then_reused_buffer(bufs):
    a, b = _params()
    loss, views = _loss(a, b, bufs, 1)
    loss.backward()
    _check(a, b, views)
    assert len(bufs._entries) == 2, "the rows went into buffers kept by the step"
    first = a.grad.data_ptr()
    a.grad = b.grad = None
    loss, views = _loss(a, b, bufs, 2)  # different rows: the first view's rows must read zero
    loss.backward()
    _check(a, b, views)
    assert a.grad.data_ptr() == first, "an unshared buffer is reused"


def test_two_views_in_one_backward_accumulate(bufs):
    a, b = _params()
    loss, views = _loss(a, b, bufs, 3, 4)
    loss.backward()
    _check(a, b, views)
    # and a further backward without clearing adds to .grad, as autograd does
    loss2, views2 = _loss(a, b, bufs, 5)
    loss2.backward()
    _check(a, b, views + views2)


def test_held_buffer_is_not_reused(bufs):
    a, b = _params()
    loss, views = _loss(a, b, bufs, 6)
    loss.backward()
    held = a.grad
    kept = held.clone()
    a.grad = b.grad = None
    loss, views2 = _loss(a, b, bufs, 7)
    loss.backward()
    _check(a, b, views2)
    assert a.grad is not held and torch.equal(held, kept), "a gradient the caller holds is left alone"


def test_gradient_changed_in_place(bufs):
    a, b = _params()
    loss, views = _loss(a, b, bufs, 8)
    loss.backward()
    a.grad.mul_(0.5)  # e.g. the trainer's division by the batch size
    b.grad.mul_(0.5)
    ea, eb = _expected(views)
    loss, views2 = _loss(a, b, bufs, 9)
    loss.backward()  # accumulates into the changed gradient
    ea2, eb2 = _expected(views2)
    assert torch.allclose(a.grad, 0.5 * ea + ea2) and torch.allclose(b.grad, 0.5 * eb + eb2)
    a.grad = b.grad = None
    loss, views3 = _loss(a, b, bufs, 10)  # reuse after an in-place change: zeroed in full
    loss.backward()
    _check(a, b, views3)


def test_gradient_created_by_the_caller(bufs):
    a, b = _params()
    a.grad = torch.ones(P, 3)
    b.grad = torch.ones(P, 1)
    loss, views = _loss(a, b, bufs, 11)
    loss.backward()
    ea, eb = _expected(views)
    assert torch.equal(a.grad, 1 + ea) and torch.equal(b.grad, 1 + eb)


def test_autograd_grad_and_hooks_take_the_usual_path(bufs):
    a, b = _params()
    loss, views = _loss(a, b, bufs, 12)
    ga, gb = torch.autograd.grad(loss, (a, b))
    ea, eb = _expected(views)
    assert torch.equal(ga, ea) and torch.equal(gb, eb) and a.grad is None
    seen = []
    a.register_hook(lambda g: seen.append(g.clone()))
    loss, views = _loss(a, b, bufs, 13)
    loss.backward()
    _check(a, b, views)
    assert len(seen) == 1 and torch.equal(seen[0], _expected(views)[0]), "the hook sees the gradient"
    assert not bufs._entries, "neither case writes into kept buffers"
