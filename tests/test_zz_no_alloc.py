"""blitz_render_bin_noalloc: binning for callers that cannot allocate device
memory when they call us (for example a host whose memory pool owns the whole
GPU, or a plain-C host with no device allocator).  It must give exactly what
blitz_render_bin gives with a caller-provided scratch buffer, call after call,
even though every call reuses the same fixed scratch array.

This file is collected last on purpose (pytest orders files by name), so a
failure here never hides the results of the other tests."""
import ctypes

import numpy as np
import pytest
import torch

from blitzgs_b200 import _lib, ops, scene as S
from blitzgs_b200._lib import ptr


def _binning_inputs(sc, dev):
    cam = sc.cameras[0]
    rs = S.raster_settings(cam, device=dev)
    xyz, s, q, o = sc.xyz.to(dev), torch.exp(sc.scaling).to(dev), torch.nn.functional.normalize(sc.rotation).to(dev), \
        torch.sigmoid(sc.opacity).to(dev)
    shs = torch.cat((sc.features_dc, sc.features_rest), 1).to(dev)
    m2, d, r, co, rgb, _, _ = ops.preprocess_forward(xyz, s, q, o.reshape(-1), ops.sh_layout(shs=shs), rs)
    H, W = cam.image_height, cam.image_width
    P = m2.shape[0]
    counts = torch.empty((P,), dtype=torch.int32, device=dev)
    totals = torch.empty((2,), dtype=torch.int64, device=dev)
    st = _lib.stream_ptr()
    _lib.call("blitz_render_count", P, H, W, ptr(m2), ptr(r), None, ptr(counts), ptr(totals), st)
    R, n_vis = [int(v) for v in totals.cpu()]
    return dict(P=P, H=H, W=W, m2=m2, d=d, r=r, counts=counts, R=R, n_vis=n_vis)


def _bin_with_caller_scratch(x, dev):
    gx, gy = (x["W"] + 15) // 16, (x["H"] + 15) // 16
    pl = torch.empty((max(x["R"], 1),), dtype=torch.int32, device=dev)
    ranges = torch.empty((gx * gy, 2), dtype=torch.int32, device=dev)
    nbytes = _lib.load().blitz_render_scratch_bytes(x["P"], x["n_vis"], x["R"], x["H"], x["W"])
    scratch = torch.empty((nbytes,), dtype=torch.uint8, device=dev)
    _lib.call("blitz_render_bin", x["P"], x["n_vis"], x["R"], x["H"], x["W"], ptr(x["m2"]), ptr(x["d"]), ptr(x["r"]),
              None, ptr(x["counts"]), ptr(scratch), nbytes, ptr(pl), ptr(ranges), _lib.stream_ptr())
    return pl[: x["R"]].cpu().numpy(), ranges.cpu().numpy()


def _bin_without_allocation(x, dev):
    gx, gy = (x["W"] + 15) // 16, (x["H"] + 15) // 16
    # the caller still owns inputs and outputs; only the scratch is gone
    pl = torch.full((max(x["R"], 1),), -1, dtype=torch.int32, device=dev)
    ranges = torch.full((gx * gy, 2), -1, dtype=torch.int32, device=dev)
    _lib.call("blitz_render_bin_noalloc", x["P"], x["n_vis"], x["R"], x["H"], x["W"], ptr(x["m2"]), ptr(x["d"]),
              ptr(x["r"]), None, ptr(x["counts"]), ptr(pl), ptr(ranges), _lib.stream_ptr())
    return pl[: x["R"]].cpu().numpy(), ranges.cpu().numpy()


@pytest.mark.gpu
def test_noalloc_binning_matches_caller_scratch_twice(cuda_device):
    # two different scenes in a row: the second call must not see anything the
    # first one left in the shared scratch array
    for sc in (S.tiny(seed=41, P=12000, H=200, W=264), S.tiny(seed=42, P=5000, H=96, W=120)):
        x = _binning_inputs(sc, cuda_device)
        assert x["R"] > 0
        a_pl, a_rg = _bin_with_caller_scratch(x, cuda_device)
        b_pl, b_rg = _bin_without_allocation(x, cuda_device)
        torch.cuda.synchronize()
        # integer outputs: identical, element for element
        assert np.array_equal(a_pl, b_pl)
        assert np.array_equal(a_rg, b_rg)


@pytest.mark.gpu
def test_noalloc_call_allocates_no_device_memory(cuda_device):
    """The promise itself: once the library is loaded, a call takes no device
    memory from the driver (free memory unchanged) and none from PyTorch's
    allocator."""
    x = _binning_inputs(S.tiny(seed=43, P=8000, H=160, W=208), cuda_device)
    gx, gy = (x["W"] + 15) // 16, (x["H"] + 15) // 16
    pl = torch.empty((max(x["R"], 1),), dtype=torch.int32, device=cuda_device)
    ranges = torch.empty((gx * gy, 2), dtype=torch.int32, device=cuda_device)
    args = (x["P"], x["n_vis"], x["R"], x["H"], x["W"], ptr(x["m2"]), ptr(x["d"]), ptr(x["r"]), None,
            ptr(x["counts"]), ptr(pl), ptr(ranges), _lib.stream_ptr())
    _lib.call("blitz_render_bin_noalloc", *args)  # first call on the device: resolves the array's address
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(cuda_device)
    stats0 = torch.cuda.memory_stats(cuda_device)
    for _ in range(3):
        _lib.call("blitz_render_bin_noalloc", *args)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(cuda_device)
    stats1 = torch.cuda.memory_stats(cuda_device)
    assert free1 == free0, f"device free memory changed by {free0 - free1} bytes"
    for k in ("allocated_bytes.all.current", "num_alloc_retries", "num_device_alloc"):
        assert stats1.get(k, 0) == stats0.get(k, 0), k


def test_noalloc_rejects_requests_beyond_its_fixed_scratch():
    """Checked on the host before any launch, so no GPU is needed."""
    lib = _lib.load()
    big_R = 40_000_000
    assert lib.blitz_render_scratch_bytes(10_000_000, 5_000_000, big_R, 864, 1152) > (64 << 20)
    rc = lib.blitz_render_bin_noalloc(10_000_000, 5_000_000, big_R, 864, 1152, None, None, None, None, None, None,
                                      None, None)
    assert rc == 10002
    assert b"fixed" in lib.blitz_last_error()
    rc = lib.blitz_render_bin_noalloc(-1, 0, 0, 864, 1152, None, None, None, None, None, None, None, None)
    assert rc == 10001
