"""The render's capacity-sized issue (ops.render_forward), on the CPU.

The first view of an image size reads its binning totals back before it
bins.  Later views are binned and blended with buffers 25% above the
largest totals seen so far, before the totals arrive on the host.  A view
that needs more than those capacities is binned and blended again with its
exact totals.  Its observation counts are cleared before the second pass.
The native calls are replaced by recorders here: the test checks the host
decisions (which sizes each binning is issued with, when it is redone, the
capacities kept, the state handed to the backward), not the kernels."""
import ctypes

import numpy as np
import pytest
import torch

from blitzgs_b200 import _lib, ops

H, W = 64, 96  # 4 x 6 tiles


class _Ev:
    def __init__(self, *a, **k):
        pass

    def record(self, *a):
        pass

    def synchronize(self):
        pass


@pytest.fixture
def calls(monkeypatch):
    log = []

    def fake_call(name, *args):
        if name == "blitz_read_totals":
            # (totals, vis_count, status, host_totals, host_n, host_status, stream): copy {R, n_vis}
            ctypes.memmove(args[3], args[0], 16)
        elif name == "blitz_render_bin":
            log.append(("bin", int(args[2]), int(args[1])))  # (R, n_vis) the binning was issued with
        elif name == "blitz_render_blend":
            log.append(("blend",))
            # the blend adds each Gaussian's observations: one per pass here
            obs = np.ctypeslib.as_array((ctypes.c_int32 * int(args[0])).from_address(args[16]))
            obs += 1
        return 0

    def pinned(dev, n, dtype, tag=""):
        key = (dev.index, n, dtype, tag, "cpu")
        t = ops._PINNED.get(key)
        if t is None:
            buf = torch.zeros(n, dtype=dtype)
            t = ops._PINNED[key] = (buf, buf.numpy())
        return t

    monkeypatch.setattr(_lib, "call", fake_call)
    monkeypatch.setattr(_lib, "stream_ptr", lambda *a: 0)
    monkeypatch.setattr(ops, "_pinned", pinned)
    monkeypatch.setattr(ops, "_require_cuda", lambda *a: None)
    monkeypatch.setattr(torch.cuda, "Event", _Ev)
    monkeypatch.setattr(ops, "_RENDER_CAPS", {})
    return log


def _view(P, R, V):
    g = torch.Generator().manual_seed(P + R)
    m2 = torch.rand(P, 2, generator=g) * torch.tensor([W, H])
    inputs = (m2, torch.rand(P, generator=g), torch.ones(P, dtype=torch.int32), torch.rand(P, 4, generator=g),
              torch.rand(P, 3, generator=g), torch.zeros(3))
    counts = torch.ones(P, dtype=torch.int32)
    totals = torch.tensor([R, V], dtype=torch.int64)
    return inputs, counts, totals


def _render(P, R, V):
    inputs, counts, totals = _view(P, R, V)
    color, _, _, _, out_observe, state = ops.render_forward(*inputs, None, H, W, counts=counts, totals=totals)
    return state, out_observe


def test_first_view_reads_totals_then_later_views_use_capacities(calls):
    st, _ = _render(200, 400, 80)
    assert calls == [("bin", 400, 80), ("blend",)]  # exact sizes, read back first
    key = (None, (W + 15) // 16 * ((H + 15) // 16))
    assert ops._RENDER_CAPS[key] == (500, 100)  # 25% above, rounded up
    assert (st.R, st.n_vis, st.point_list.numel()) == (400, 80, 400)
    del calls[:]
    st, _ = _render(200, 350, 70)  # within the capacities: one pass, issued with them
    assert calls == [("bin", 500, 100), ("blend",)]
    assert (st.R, st.n_vis) == (350, 70) and st.point_list.numel() == 500
    assert ops._RENDER_CAPS[key] == (500, 100)


def test_a_view_beyond_the_capacities_is_binned_again_with_its_totals(calls):
    _render(200, 400, 80)
    del calls[:]
    st, out_observe = _render(200, 700, 90)  # more instances than the 500 the buffers hold
    assert calls == [("bin", 500, 100), ("blend",), ("bin", 700, 90), ("blend",)]
    assert (st.R, st.n_vis) == (700, 90) and st.point_list.numel() == 700
    assert st.strip_ids.numel() == 8 * 700 and st.strip_pos.numel() == 8 * 700
    # cleared before the second pass: the counts are that pass's alone
    assert torch.equal(out_observe, torch.ones(200, dtype=torch.int32))
    key = (None, (W + 15) // 16 * ((H + 15) // 16))
    assert ops._RENDER_CAPS[key] == (875, 113)
    del calls[:]
    _render(200, 100, 120)  # more visible Gaussians than the capacity: redone too
    assert calls == [("bin", 875, 113), ("blend",), ("bin", 100, 120), ("blend",)]


def test_capacities_never_exceed_the_gaussian_count_for_visible(calls):
    _render(50, 40, 48)  # capacity for visible Gaussians would be 60 > P = 50
    del calls[:]
    _render(50, 30, 45)
    assert calls == [("bin", 50, 50), ("blend",)]


def test_caller_read_totals_bins_once_with_them(calls):
    inputs, counts, totals = _view(120, 300, 60)
    _, _, _, _, _, st = ops.render_forward(*inputs, None, H, W, counts=counts, totals=totals,
                                           totals_host=(300, 60), caps_update=True)
    assert calls == [("bin", 300, 60), ("blend",)]
    assert np.array_equal([st.R, st.n_vis], [300, 60])
