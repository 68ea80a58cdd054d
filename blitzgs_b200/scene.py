"""Seeded synthetic scenes and cameras standing in for Mill-19 / UrbanScene3D /
MatrixCity (absent here).  All generation runs on the CPU with a
``torch.Generator`` so every machine produces bit-identical inputs.

Parameters are produced in the reference's raw (pre-activation) layout of
``GaussianModel`` (scene/gaussian_model.py:44-58, 248-276): ``_xyz [P,3]``,
``_scaling [P,3]`` log-scales, ``_rotation [P,4]`` unnormalised quaternions,
``_opacity [P,1]`` logits, ``_features_dc [P,1,3]`` and ``_features_rest
[P,15,3]``.  Cameras follow scene/cameras.py:111-133 and
utils/graphics_utils.py:42-76: ``world_view_transform`` is the transposed
world-to-view matrix, ``full_proj_transform = world_view_transform @
projection^T``, znear 0.01, zfar 100, camera looking down +z in view space,
y down in the image.
"""
import math
from dataclasses import dataclass, field

import numpy as np
import torch


@dataclass
class Camera:
    image_height: int
    image_width: int
    FoVx: float
    FoVy: float
    world_view_transform: torch.Tensor  # [4,4] float32
    full_proj_transform: torch.Tensor   # [4,4] float32
    camera_center: torch.Tensor         # [3] float32
    uid: int = 0

    def to(self, device):
        return Camera(self.image_height, self.image_width, self.FoVx, self.FoVy,
                      self.world_view_transform.to(device), self.full_proj_transform.to(device),
                      self.camera_center.to(device), self.uid)

    @property
    def tanfovx(self):
        return math.tan(self.FoVx * 0.5)

    @property
    def tanfovy(self):
        return math.tan(self.FoVy * 0.5)


def projection_matrix(znear, zfar, fovX, fovY):
    """Perspective projection, as utils/graphics_utils.py:56-76."""
    tan_y = math.tan(fovY / 2)
    tan_x = math.tan(fovX / 2)
    top = tan_y * znear
    bottom = -top
    right = tan_x * znear
    left = -right
    P = torch.zeros(4, 4)
    P[0, 0] = 2.0 * znear / (right - left)
    P[1, 1] = 2.0 * znear / (top - bottom)
    P[0, 2] = (right + left) / (right - left)
    P[1, 2] = (top + bottom) / (top - bottom)
    P[3, 2] = 1.0
    P[2, 2] = zfar / (zfar - znear)
    P[2, 3] = -(zfar * znear) / (zfar - znear)
    return P


def look_at_camera(position, target, up, W, H, fovx, uid=0, znear=0.01, zfar=100.0):
    """Camera at ``position`` looking at ``target``; ``fovx`` in radians."""
    pos = np.asarray(position, np.float64)
    fwd = np.asarray(target, np.float64) - pos
    fwd /= np.linalg.norm(fwd)
    upv = np.asarray(up, np.float64)
    right = np.cross(fwd, upv)
    if np.linalg.norm(right) < 1e-8:
        right = np.cross(fwd, np.array([0.0, 1.0, 0.0]))
    right /= np.linalg.norm(right)
    down = np.cross(fwd, right)
    Rw2c = np.stack([right, down, fwd], 0)  # rows: camera x (right), y (down), z (forward)
    t = -Rw2c @ pos
    W2C = np.eye(4)
    W2C[:3, :3] = Rw2c
    W2C[:3, 3] = t
    fovy = 2 * math.atan(math.tan(fovx / 2) * H / W)
    wv = torch.tensor(np.float32(W2C)).transpose(0, 1).contiguous()
    proj = projection_matrix(znear, zfar, fovx, fovy).transpose(0, 1)
    full = (wv.unsqueeze(0).bmm(proj.unsqueeze(0))).squeeze(0).contiguous()
    center = wv.inverse()[3, :3].contiguous()
    return Camera(H, W, fovx, fovy, wv, full, center, uid)


@dataclass
class Scene:
    name: str
    xyz: torch.Tensor
    scaling: torch.Tensor
    rotation: torch.Tensor
    opacity: torch.Tensor
    features_dc: torch.Tensor
    features_rest: torch.Tensor
    cameras: list = field(default_factory=list)
    sh_degree: int = 3

    @property
    def P(self):
        return self.xyz.shape[0]

    def to(self, device):
        return Scene(self.name, *(t.to(device) for t in (self.xyz, self.scaling, self.rotation, self.opacity,
                                                          self.features_dc, self.features_rest)),
                     [c.to(device) for c in self.cameras], self.sh_degree)

    def activated(self):
        """(means3D, scales, rotations, shs [P,16,3], opacities) as the reference getters produce."""
        return (self.xyz, torch.exp(self.scaling), torch.nn.functional.normalize(self.rotation),
                torch.cat((self.features_dc, self.features_rest), dim=1), torch.sigmoid(self.opacity))


def _params(g, P, log_scale_mu, log_scale_sigma):
    scaling = torch.randn(P, 3, generator=g) * log_scale_sigma + log_scale_mu
    rotation = torch.randn(P, 4, generator=g)
    opacity = torch.randn(P, 1, generator=g)
    dc = torch.randn(P, 1, 3, generator=g) * 0.5
    rest = torch.randn(P, 15, 3, generator=g) * 0.05
    return scaling, rotation, opacity, dc, rest


def tiny(seed=0, P=16384, H=256, W=256):
    """Config 1: U[-1,1]^3 means, log-scale N(-4,0.3), one camera at distance 3, FoV 60 deg."""
    g = torch.Generator().manual_seed(seed)
    xyz = torch.rand(P, 3, generator=g) * 2 - 1
    s, r, o, dc, rest = _params(g, P, -4.0, 0.3)
    cam = look_at_camera([0.0, 0.0, -3.0], [0, 0, 0], [0, -1, 0], W, H, math.radians(60))
    return Scene("tiny", xyz, s, r, o, dc, rest, [cam])


def aerial_cameras(g, n, W, H, fovx_deg, center_xy, span, alt_lo, alt_hi, pitch_lo_deg, pitch_hi_deg,
                   uid0=0):
    cams = []
    for k in range(n):
        u = torch.rand(5, generator=g, dtype=torch.float64).tolist()
        cx = center_xy[0] + (u[0] - 0.5) * span
        cy = center_xy[1] + (u[1] - 0.5) * span
        alt = alt_lo + (alt_hi - alt_lo) * u[2]
        yaw = 2 * math.pi * u[3]
        pitch = math.radians(pitch_lo_deg + (pitch_hi_deg - pitch_lo_deg) * u[4])
        pos = np.array([cx, cy, alt])
        horiz = np.array([math.cos(yaw), math.sin(yaw), 0.0])
        fwd = horiz * math.cos(pitch) + np.array([0, 0, -1.0]) * math.sin(pitch)
        up = np.array([0, 0, 1.0]) if pitch < math.radians(89.9) else horiz
        cams.append(look_at_camera(pos, pos + fwd, up, W, H, math.radians(fovx_deg), uid=uid0 + k))
    return cams


def mid(seed=0, P=1_000_000, n_cams=4, H=864, W=1152):
    """Config 2: 1M Gaussians in a 200x200x20 box, log-scale N(-1.5,0.5), nadir
    cameras (FoV 70 deg, altitude U[80,120], random yaw)."""
    g = torch.Generator().manual_seed(seed)
    xyz = torch.rand(P, 3, generator=g) * torch.tensor([200.0, 200.0, 20.0]) - torch.tensor([100.0, 100.0, 0.0])
    s, r, o, dc, rest = _params(g, P, -1.5, 0.5)
    cams = aerial_cameras(g, n_cams, W, H, 70.0, (0.0, 0.0), 60.0, 80.0, 120.0, 90.0, 90.0)
    return Scene("mid", xyz, s, r, o, dc, rest, cams)


def city(seed=0, P=8_000_000, n_cams=16, H=864, W=1152):
    """Config 3: 8M Gaussians from a Gaussian mixture (centres on a 40x40 grid
    over 1000x1000, sigma 3, centre heights U[0,40]) clamped to the
    1000x1000x40 box; log-scale N(-1.5,0.5); 1152x864 cameras with pitch
    U[45,90] deg, altitude U[80,120], FoV 70 deg."""
    g = torch.Generator().manual_seed(seed)
    gx = torch.linspace(-500 + 12.5, 500 - 12.5, 40)
    cx, cy = torch.meshgrid(gx, gx, indexing="ij")
    centres = torch.stack([cx.reshape(-1), cy.reshape(-1), torch.rand(1600, generator=g) * 40], 1)
    which = torch.randint(0, 1600, (P,), generator=g)
    xyz = centres[which] + torch.randn(P, 3, generator=g) * 3.0
    lo = torch.tensor([-500.0, -500.0, 0.0])
    hi = torch.tensor([500.0, 500.0, 40.0])
    xyz = torch.maximum(torch.minimum(xyz, hi), lo)
    s, r, o, dc, rest = _params(g, P, -1.5, 0.5)
    cams = aerial_cameras(g, n_cams, W, H, 70.0, (0.0, 0.0), 600.0, 80.0, 120.0, 45.0, 90.0)
    return Scene("city", xyz, s, r, o, dc, rest, cams)


def large(seed=0, P=20_000_000, n_cams=8, H=1080, W=1920):
    """Config 4: 20M Gaussians in 2000x2000x60, 1920x1080 FoV 60 deg cameras."""
    g = torch.Generator().manual_seed(seed)
    xyz = torch.rand(P, 3, generator=g) * torch.tensor([2000.0, 2000.0, 60.0]) - torch.tensor([1000.0, 1000.0, 0.0])
    s, r, o, dc, rest = _params(g, P, -1.5, 0.5)
    cams = aerial_cameras(g, n_cams, W, H, 60.0, (0.0, 0.0), 1200.0, 80.0, 120.0, 45.0, 90.0)
    return Scene("large", xyz, s, r, o, dc, rest, cams)


def skew(seed=0, P=8_000_000, n_cams=8, H=864, W=1152):
    """Config 5: 8M Gaussians, 90% in 10% of the 10x10-m cells (log-normal
    cell densities over a 1000x1000 area)."""
    g = torch.Generator().manual_seed(seed)
    ncell = 100 * 100
    dens = torch.exp(torch.randn(ncell, generator=g) * 1.0)
    hot = torch.randperm(ncell, generator=g)[: ncell // 10]
    w = torch.full((ncell,), 0.1 / (ncell - ncell // 10))
    w[hot] = 0.9 * dens[hot] / dens[hot].sum()
    cell = torch.multinomial(w, P, replacement=True, generator=g)
    cxy = torch.stack([(cell % 100).float(), (cell // 100).float()], 1) * 10.0 - 500.0
    xy = cxy + torch.rand(P, 2, generator=g) * 10.0
    z = torch.rand(P, 1, generator=g) * 40.0
    xyz = torch.cat([xy, z], 1)
    s, r, o, dc, rest = _params(g, P, -1.5, 0.5)
    cams = aerial_cameras(g, n_cams, W, H, 70.0, (0.0, 0.0), 600.0, 80.0, 120.0, 45.0, 90.0)
    return Scene("skew", xyz, s, r, o, dc, rest, cams)


CONFIGS = {"tiny": tiny, "mid": mid, "city": city, "large": large, "skew": skew}


def target_image(seed, H, W):
    """Seeded uniform uint8 target [3,H,W] (the reference divides GT by 255)."""
    g = torch.Generator().manual_seed(1000 + seed)
    return torch.randint(0, 256, (3, H, W), generator=g, dtype=torch.uint8)


def raster_settings(cam, sh_degree=3, bg=None, device=None):
    """Reference GaussianRasterizationSettings fields for a camera
    (gaussian_renderer/__init__.py:309-318)."""
    from .rasterizer import GaussianRasterizationSettings
    dev = device or cam.world_view_transform.device
    if bg is None:
        bg = torch.zeros(3, dtype=torch.float32, device=dev)
    return GaussianRasterizationSettings(
        image_height=int(cam.image_height), image_width=int(cam.image_width), tanfovx=cam.tanfovx,
        tanfovy=cam.tanfovy, bg=bg, scale_modifier=1.0, viewmatrix=cam.world_view_transform.to(dev),
        projmatrix=cam.full_proj_transform.to(dev), sh_degree=sh_degree, campos=cam.camera_center.to(dev),
        prefiltered=False, debug=False)
