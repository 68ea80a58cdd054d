"""Shared helpers for the parity tests (tolerances are stated here)."""
import numpy as np
import torch

# Rendered images: within 1e-5 absolute in fp32.
IMG_ATOL = 1e-5
# Gradients: within 1e-4 relative (normwise per tensor: ||a-b|| <= 1e-4 ||b||),
# allowing for the reordering of floating-point sums that replaces atomics.
GRAD_RTOL = 1e-4


def normwise_rel(a, b):
    a = torch.as_tensor(a, dtype=torch.float64).reshape(-1)
    b = torch.as_tensor(b, dtype=torch.float64).reshape(-1)
    den = b.norm().item()
    return (a - b).norm().item() / (den if den > 0 else 1.0)


def assert_grad_close(a, b, rtol=GRAD_RTOL, name=""):
    r = normwise_rel(a, b)
    assert r <= rtol, f"{name}: normwise relative error {r:.3e} > {rtol:.1e}"


def scene_params(sc, device=None):
    ts = (sc.xyz, sc.scaling, sc.rotation, sc.opacity, sc.features_dc, sc.features_rest)
    return tuple(t.to(device) if device is not None else t for t in ts)


def activated(sc, device=None):
    xyz, s, q, o, dc, rest = scene_params(sc, device)
    return (xyz, torch.exp(s), torch.nn.functional.normalize(q), torch.cat((dc, rest), 1), torch.sigmoid(o))
