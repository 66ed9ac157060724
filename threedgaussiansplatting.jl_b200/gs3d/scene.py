"""Scenes: the reference's 4-Gaussian test scene (scene.jl:123-188), scene radius
(scene.jl:49-73) and the seeded synthetic workloads that stand in for real captures.

Synthetic conventions (numpy PCG64, ``default_rng(seed)``): quaternions N(0,1)^4 (left
unnormalised, as stored by the reference), SH DC ~ N(0, 0.3), higher orders ~ N(0, 0.05),
degree 3; cameras look at the origin with +y as world up.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from .structs import GaussiansVector, PinholeCamera, fov_deg_to_focal_length, look_at_camera

F32 = np.float32
SH_C0 = 0.28209479177387814


def logit_np(x):
    x = np.asarray(x, dtype=F32)
    return (-np.log(F32(1) / x - F32(1))).astype(F32)


def color_to_sh_coeffs_dc(color) -> np.ndarray:
    """sh.jl:157-160"""
    return ((np.asarray(color, dtype=F32) - F32(0.5)) / F32(SH_C0)).astype(F32)


def create_test_scene(sh_degree: int = 0, two_cameras: bool = False, device="cpu"):
    """The reference's 'Julia logo' scene (scene.jl:123-188): 4 Gaussians (red, white behind
    the camera, green, purple), a 320 x 240 camera with 90 degrees horizontal FOV at the
    origin. Returns (gaussians, cameras)."""
    w, h = 320, 240
    f = F32(fov_deg_to_focal_length(90.0, w))
    cam = PinholeCamera.simple(w, h, f, np.eye(3, dtype=F32), np.zeros(3, dtype=F32))
    K_inv = np.linalg.inv(cam.intrinsic_matrix.astype(np.float64))
    means2d = np.array([[w / 3, w / 2 - 0.1, w / 2 + 0.1, 2 * w / 3],
                        [2 * h / 3, h / 2 + 0.1, h / 3, 2 * h / 3]], dtype=F32)
    depths = np.array([1, -1, 2, 3], dtype=F32)
    means = (K_inv @ np.concatenate([means2d * depths[None, :], depths[None, :]], 0)).astype(F32)
    opacity_features = logit_np([0.75, 0.99, 0.5, 0.99])
    scaling = np.log(np.array([[0.25, 10, 0.5, 1.0], [0.25, 20, 0.5, 0.75], [0.25, 30, 0.5, 0.5]],
                              dtype=F32)).astype(F32)
    rotation = np.array([[math.sqrt(2) / 2, 1, 1, math.sqrt(3)], [0, 0, 0, 1], [0, 0, 0, 0],
                         [math.sqrt(2) / 2, 0, 0, 0]], dtype=F32)
    order = (sh_degree + 1) ** 2
    colors = [(0.796, 0.235, 0.2), (1.0, 1.0, 1.0), (0.22, 0.596, 0.149), (0.584, 0.345, 0.698)]
    rest = [0.01, -0.01, 0.01, 0.01]
    sh = np.zeros((4, 3, order), dtype=F32)
    for g in range(4):
        sh[g, :, 0] = color_to_sh_coeffs_dc(colors[g])
        sh[g, :, 1:] = F32(rest[g])
    mo = np.concatenate([means.T, opacity_features[:, None]], 1).astype(F32)
    gv = GaussiansVector(torch.from_numpy(np.ascontiguousarray(mo)).to(device),
                         torch.from_numpy(np.ascontiguousarray(scaling.T)).to(device),
                         torch.from_numpy(np.ascontiguousarray(rotation.T)).to(device),
                         torch.from_numpy(sh).to(device))
    cams = [cam]
    if two_cameras:
        cams.append(PinholeCamera.simple(w, h, f, np.eye(3, dtype=F32), np.array([1, 0, 0], F32)))
    return gv, cams


def gaussians_from_point_cloud(points, rgb_colors, device="cpu") -> GaussiansVector:
    """The trainable Gaussians a coloured point cloud starts as (gaussians.jl:597-639): means
    at the points, opacity features logit(0.1), SH degree 0 with DC = (colour - 0.5) / C0 (the
    inverse of the degree-0 colour), identity rotations (1, 0, 0, 0), and all three log-scales
    = log of the mean Euclidean distance to the 3 nearest other points (the 4 nearest
    neighbours including the point itself, summed and divided by 3, as the reference does)."""
    from scipy.spatial import cKDTree
    pts = np.asarray(points, dtype=F32).reshape(-1, 3)
    cols = np.asarray(rgb_colors, dtype=F32).reshape(-1, 3)
    n = pts.shape[0]
    k = min(4, n)
    d, _ = cKDTree(pts.astype(np.float64)).query(pts.astype(np.float64), k=k)
    d = np.asarray(d, dtype=np.float64).reshape(n, k).astype(F32)
    mean_d = d.sum(axis=1, dtype=F32) / F32(3)
    with np.errstate(divide="ignore"):
        log_s = np.log(mean_d).astype(F32)
    mo = np.empty((n, 4), F32)
    mo[:, :3] = pts
    mo[:, 3] = logit_np(np.full(n, 0.1, F32))
    sf = np.repeat(log_s[:, None], 3, axis=1)
    rf = np.zeros((n, 4), F32)
    rf[:, 0] = 1
    c0 = F32(0.28209479177387814)
    sh = ((cols - F32(0.5)) / c0).astype(F32).reshape(n, 3, 1)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)
    return GaussiansVector(t(mo), t(sf), t(rf), t(sh))


def scene_radius(cameras, enlargement_factor: float = 1.1) -> float:
    """_compute_scene_radius (scene.jl:49-73): 1.1 x max distance to the camera centroid."""
    pos = np.stack([c.position.astype(np.float64) for c in cameras])
    center = pos.mean(0)
    return float(enlargement_factor * np.max(np.linalg.norm(pos - center, axis=1)))


@dataclass
class SceneSpec:
    n: int
    means: str            # "uniform:a" (U[-a,a]^3) or "normal:s" (N(0, s^2 I))
    log_scale_mu: float
    log_scale_sigma: float
    opacity_mu: float = 0.0
    opacity_sigma: float = 1.0
    sh_degree: int = 3


def synthetic_gaussians(spec: SceneSpec, seed: int, device="cpu") -> GaussiansVector:
    rng = np.random.default_rng(seed)
    n = spec.n
    kind, p = spec.means.split(":")
    p = float(p)
    if kind == "uniform":
        means = rng.uniform(-p, p, size=(n, 3))
    else:
        means = rng.normal(0.0, p, size=(n, 3))
    opac = rng.normal(spec.opacity_mu, spec.opacity_sigma, size=(n, 1))
    scal = rng.normal(spec.log_scale_mu, spec.log_scale_sigma, size=(n, 3))
    rot = rng.normal(0.0, 1.0, size=(n, 4))
    order = (spec.sh_degree + 1) ** 2
    sh = rng.normal(0.0, 0.05, size=(n, 3, order))
    sh[:, :, 0] = rng.normal(0.0, 0.3, size=(n, 3))
    mo = np.concatenate([means, opac], 1)
    f = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=F32)).to(device)
    return GaussiansVector(f(mo), f(scal), f(rot), f(sh))


def ring_cameras(k: int, width: int, height: int, fov_deg: float, radius: float, height_y: float):
    cams = []
    for i in range(k):
        a = 2 * math.pi * i / k
        cams.append(look_at_camera(width, height, fov_deg,
                                   (radius * math.cos(a), height_y, radius * math.sin(a))))
    return cams


def hemisphere_cameras(k: int, width: int, height: int, fov_deg: float, radius: float):
    """Fibonacci hemisphere (y >= 0) looking at the origin."""
    cams = []
    golden = math.pi * (3 - math.sqrt(5))
    for i in range(k):
        y = 0.05 + 0.95 * (i + 0.5) / k
        r = math.sqrt(max(0.0, 1 - y * y))
        a = golden * i
        cams.append(look_at_camera(width, height, fov_deg,
                                   (radius * r * math.cos(a), radius * y, radius * r * math.sin(a))))
    return cams


# BASELINE.json configs (synthetic stand-ins with the stated shapes and distributions)
CONFIGS = {
    0: dict(spec=SceneSpec(16_384, "uniform:1", -4.0, 0.5), seed=0,
            cameras=lambda: [look_at_camera(256, 256, 60.0, (0, 0, 3))]),
    1: dict(spec=SceneSpec(500_000, "uniform:3", -5.0, 0.5), seed=1,
            cameras=lambda: ring_cameras(32, 1280, 720, 50.0, 6.0, 1.5)),
    2: dict(spec=SceneSpec(300_000, "normal:1.5", -4.0, 0.5), seed=2,
            cameras=lambda: hemisphere_cameras(100, 1920, 1080, 50.0, 5.0)),
    3: dict(spec=SceneSpec(6_000_000, "normal:2", -5.5, 0.6, 1.0, 1.5), seed=3,
            cameras=lambda: ring_cameras(64, 3840, 2160, 45.0, 7.0, 0.0)),
    4: dict(spec=SceneSpec(3_000_000, "normal:2", -5.5, 0.6, 1.0, 1.5), seed=4,
            cameras=lambda: hemisphere_cameras(256, 1920, 1080, 50.0, 5.0)),
}


def target_image(width: int, height: int, seed: int, device="cpu") -> torch.Tensor:
    """Seeded uniform [0, 1] target in the 3 x h x w layout ((w, h, 3) tensor)."""
    rng = np.random.default_rng(seed)
    return torch.from_numpy(rng.uniform(0, 1, size=(width, height, 3)).astype(F32)).to(device)
