"""Host-side data model mirroring ThreeDGaussianSplatting.jl's types.

Layouts: a Julia column-major ``k x n`` array is a C-contiguous torch tensor of shape
``(n, k)``; ``3 x h x w`` images are ``(w, h, 3)`` tensors (u slowest, c fastest). All index
values stored in arrays are 1-based, as in the reference.

    PinholeCamera ........ cameras.jl:50-106, :345-380, :534-542
    RenderOptions ........ forward_structs.jl:579-719 (image_coordinates.jl for clip bounds)
    Tiling ............... forward_structs.jl:340-424
    GaussiansVector ...... gaussians.jl:30-52 (TrainableGaussiansVector)
    RenderBuffers ........ forward_structs.jl:1541-1600, :762-786
    RenderOutputs ........ forward_structs.jl:1-65
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _abi

F32 = np.float32
CLAMP = 0   # CovarianceBoundaryClamp
FILTER = 1  # BoundaryFilter

DEFAULT_MIN_ALPHA = 1 / 255
DEFAULT_MAX_ALPHA = 0.99
DEFAULT_MIN_TRANSMITTANCE = 0.0001
DEFAULT_DILATION_PX = 0.3
DEFAULT_CLIPPING_MARGIN_NC = 0.3
DEFAULT_MIN_AA_FACTOR = 0.0005
DEFAULT_NEAR = 0.2
DEFAULT_FAR = math.inf


def fov_to_focal_length(fov_rad: float, axis_size: float) -> float:
    """cameras.jl:534-537"""
    return axis_size / (2 * math.tan(fov_rad / 2))


def fov_deg_to_focal_length(fov_deg: float, axis_size: float) -> float:
    return fov_to_focal_length(math.radians(fov_deg), axis_size)


def check_sh_degree(d: int) -> None:
    """_check_sh_degree (gaussians.jl:243-252): SH degrees are 0, 1, 2 or 3."""
    if not 0 <= int(d) <= 3:
        raise ValueError(f"spherical harmonics degree {d} is not in 0..3")


@dataclass
class PinholeCamera:
    """PinholeCamera (cameras.jl:50-106). R_c2w / t_c2w are camera-to-world."""

    width: int
    height: int
    fx: float
    fy: float
    skew: float
    cx: float
    cy: float
    R_c2w: np.ndarray
    t_c2w: np.ndarray
    near_z: float = DEFAULT_NEAR
    far_z: float = DEFAULT_FAR

    @classmethod
    def simple(cls, width: int, height: int, focal_length: float, R_c2w, t_c2w) -> "PinholeCamera":
        """PinholeCamera(width, height, focal_length, rotation, translation) (cameras.jl:366-380):
        no skew, principal point at the image centre, 3DGS near/far planes."""
        return cls(int(width), int(height), float(F32(focal_length)), float(F32(focal_length)), 0.0,
                   float(F32(width) / F32(2)), float(F32(height) / F32(2)),
                   np.asarray(R_c2w, dtype=F32).reshape(3, 3), np.asarray(t_c2w, dtype=F32).reshape(3))

    @property
    def intrinsic_matrix(self) -> np.ndarray:
        return np.array([[self.fx, self.skew, self.cx], [0, self.fy, self.cy], [0, 0, 1]], dtype=F32)

    @property
    def projection_matrix_3x4(self) -> np.ndarray:
        """K [R' | -R' t] (cameras.jl:141-181), rounded to Float32."""
        R = self.R_c2w.astype(np.float64)
        t = self.t_c2w.astype(np.float64)
        Rw = R.T
        W = np.concatenate([Rw, (-Rw @ t)[:, None]], axis=1)
        return (self.intrinsic_matrix.astype(np.float64) @ W).astype(F32)

    @property
    def position(self) -> np.ndarray:
        return self.t_c2w.astype(F32)

    def to_c(self) -> _abi.Camera:
        c = _abi.Camera()
        c.width, c.height = self.width, self.height
        c.fx, c.fy, c.skew, c.cx, c.cy = self.fx, self.fy, self.skew, self.cx, self.cy
        c.near_z, c.far_z = self.near_z, self.far_z
        P = self.projection_matrix_3x4
        for j in range(4):
            for i in range(3):
                c.P[i + 3 * j] = float(P[i, j])
        for i in range(3):
            c.position[i] = float(self.position[i])
        return c

    def project(self, points: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
        """project_with_depth for an (N, 3) array (float64; for test helpers)."""
        P = self.projection_matrix_3x4.astype(np.float64)
        h = points.astype(np.float64) @ P[:, :3].T + P[:, 3]
        return h[:, :2] / h[:, 2:3], h[:, 2]


def look_at_camera(width: int, height: int, fov_deg_h: float, position, target=(0, 0, 0),
                   world_up=(0, 1, 0)) -> PinholeCamera:
    """Camera at `position` looking at `target`: z_cam = normalize(target - pos),
    x_cam = normalize(z_cam x up), y_cam = z_cam x x_cam (y points down)."""
    pos = np.asarray(position, dtype=np.float64)
    z = np.asarray(target, dtype=np.float64) - pos
    z /= np.linalg.norm(z)
    x = np.cross(z, np.asarray(world_up, dtype=np.float64))
    if np.linalg.norm(x) < 1e-9:
        x = np.cross(z, np.array([0.0, 0.0, 1.0]))
    x /= np.linalg.norm(x)
    y = np.cross(z, x)
    R = np.stack([x, y, z], axis=1)
    f = fov_deg_to_focal_length(fov_deg_h, width)
    return PinholeCamera.simple(width, height, f, R, pos)


@dataclass
class RenderOptions:
    """RenderOptions (forward_structs.jl:579-719). Clip values are stored in pixels."""

    sh_degree: int
    clipping_mode: int = CLAMP
    background: tuple = (0.0, 0.0, 0.0)
    use_antialiasing: bool = False
    min_alpha: float = float(F32(DEFAULT_MIN_ALPHA))
    max_alpha: float = float(F32(DEFAULT_MAX_ALPHA))
    min_transmittance: float = float(F32(DEFAULT_MIN_TRANSMITTANCE))
    dilation_x: float = float(F32(DEFAULT_DILATION_PX))
    dilation_y: float = float(F32(DEFAULT_DILATION_PX))
    clip_x_min: float = 0.0
    clip_x_max: float = 0.0
    clip_y_min: float = 0.0
    clip_y_max: float = 0.0
    antialiasing_min_factor: float = float(F32(DEFAULT_MIN_AA_FACTOR))

    @classmethod
    def create(cls, width: int, height: int, sh_degree: int, clipping_mode: int = CLAMP,
               background=(0.0, 0.0, 0.0), use_antialiasing: bool = False,
               clip_margin_nc: float = DEFAULT_CLIPPING_MARGIN_NC, **kw) -> "RenderOptions":
        """RenderOptions(width, height, sh_degree, mode; ...) with the NDC -> pixel clip
        conversion F(F(size) / 2 * (c + 1)) (image_coordinates.jl)."""
        def n2p(size, c):
            return float(F32(F32(size) / F32(2)) * (F32(c) + F32(1)))
        lo, hi = F32(-1 - clip_margin_nc), F32(1 + clip_margin_nc)
        return cls(sh_degree=int(sh_degree), clipping_mode=clipping_mode,
                   background=tuple(float(F32(b)) for b in background),
                   use_antialiasing=bool(use_antialiasing),
                   clip_x_min=n2p(width, lo), clip_x_max=n2p(width, hi),
                   clip_y_min=n2p(height, lo), clip_y_max=n2p(height, hi), **kw)

    @classmethod
    def for_camera(cls, camera: PinholeCamera, sh_degree: int, clipping_mode: int = CLAMP, **kw):
        return cls.create(camera.width, camera.height, sh_degree, clipping_mode, **kw)

    def with_sh_degree(self, d: int) -> "RenderOptions":
        o = RenderOptions(**self.__dict__)
        o.sh_degree = int(d)
        return o

    def to_c(self) -> _abi.RenderOptionsC:
        o = _abi.RenderOptionsC()
        for i in range(3):
            o.background[i] = self.background[i]
        o.antialiasing_min_factor = self.antialiasing_min_factor
        o.min_alpha, o.max_alpha = self.min_alpha, self.max_alpha
        o.min_transmittance = self.min_transmittance
        o.dilation_x, o.dilation_y = self.dilation_x, self.dilation_y
        o.clip_x_min, o.clip_x_max = self.clip_x_min, self.clip_x_max
        o.clip_y_min, o.clip_y_max = self.clip_y_min, self.clip_y_max
        o.sh_degree, o.clipping_mode = self.sh_degree, self.clipping_mode
        o.use_antialiasing = int(self.use_antialiasing)
        return o


def default_tile_size(width: int, height: int) -> tuple[int, int]:
    """get_default_tile_size (forward_structs.jl:419-424)."""
    return 16, (32 if width * height > 1_500_000 else 16)


@dataclass
class Tiling:
    """Tiling (forward_structs.jl:340-424)."""

    tile_width: int
    tile_height: int
    nb_tiles_x: int
    nb_tiles_y: int

    @classmethod
    def create(cls, width: int, height: int, tile_width: int | None = None,
               tile_height: int | None = None) -> "Tiling":
        if tile_width is None or tile_height is None:
            tile_width, tile_height = default_tile_size(width, height)
        return cls(tile_width, tile_height, -(-width // tile_width), -(-height // tile_height))

    @classmethod
    def for_camera(cls, camera: PinholeCamera, tile_width=None, tile_height=None) -> "Tiling":
        return cls.create(camera.width, camera.height, tile_width, tile_height)

    @property
    def nb_tiles(self) -> int:
        return self.nb_tiles_x * self.nb_tiles_y

    @property
    def highest_key_bit(self) -> int:
        """33 + floor(log2(nb_tiles)) (forward_core.jl:623)."""
        return 33 + (self.nb_tiles.bit_length() - 1)

    def to_c(self) -> _abi.TilingC:
        t = _abi.TilingC()
        t.tile_width, t.tile_height = self.tile_width, self.tile_height
        t.nb_tiles_x, t.nb_tiles_y = self.nb_tiles_x, self.nb_tiles_y
        return t


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


@dataclass
class GaussiansVector:
    """TrainableGaussiansVector: (n, 4) means+opacity logits, (n, 3) log-scales, (n, 4)
    quaternions (r, x, y, z), (n, 3, (d+1)^2) SH coefficients."""

    means_opacity_features: torch.Tensor
    scaling_features: torch.Tensor
    rotation_features: torch.Tensor
    sh_coeffs: torch.Tensor

    def __post_init__(self):
        n = self.means_opacity_features.shape[0]
        assert self.means_opacity_features.shape == (n, 4)
        assert self.scaling_features.shape == (n, 3)
        assert self.rotation_features.shape == (n, 4)
        assert self.sh_coeffs.shape[:2] == (n, 3)
        order = self.sh_coeffs.shape[2]
        assert int(round(math.sqrt(order))) ** 2 == order and order <= 16
        for t in (self.means_opacity_features, self.scaling_features, self.rotation_features,
                  self.sh_coeffs):
            assert t.dtype == torch.float32 and t.is_contiguous()

    @property
    def n(self) -> int:
        return self.means_opacity_features.shape[0]

    def __len__(self) -> int:
        return self.n

    @property
    def sh_degree(self) -> int:
        return int(round(math.sqrt(self.sh_coeffs.shape[2]))) - 1

    @property
    def device(self) -> torch.device:
        return self.means_opacity_features.device

    def to(self, device) -> "GaussiansVector":
        return GaussiansVector(*(t.to(device).contiguous() for t in self.tensors()))

    def clone(self) -> "GaussiansVector":
        return GaussiansVector(*(t.clone() for t in self.tensors()))

    def tensors(self):
        return (self.means_opacity_features, self.scaling_features, self.rotation_features,
                self.sh_coeffs)

    def set_sh_degree(self, d: int) -> None:
        """set_sh_degree! (gaussians.jl:1070-1080): grow or shrink the SH axis; new coefficients
        are 0."""
        check_sh_degree(d)
        old = self.sh_coeffs
        new = torch.zeros((old.shape[0], 3, (d + 1) ** 2), dtype=old.dtype, device=old.device)
        k = min(old.shape[2], new.shape[2])
        new[:, :, :k] = old[:, :, :k]
        self.sh_coeffs = new

    def replace(self, other: "GaussiansVector") -> None:
        """Take over `other`'s arrays (after densification)."""
        (self.means_opacity_features, self.scaling_features, self.rotation_features,
         self.sh_coeffs) = other.tensors()

    def to_c(self) -> _abi.GaussiansC:
        g = _abi.GaussiansC()
        g.n, g.sh_degree = self.n, self.sh_degree
        g.means_opacity_features = _ptr(self.means_opacity_features)
        g.scaling_features = _ptr(self.scaling_features)
        g.rotation_features = _ptr(self.rotation_features)
        g.sh_coeffs = _ptr(self.sh_coeffs)
        return g


@dataclass
class RenderOnlyGaussiansVector:
    """RenderOnlyGaussiansVector (gaussians.jl:342-392): (n, 4) means + opacities (after the
    sigmoid), (n, 6) lower 3D covariances (11, 21, 31, 22, 32, 33), (n, 3, (d+1)^2) SH
    coefficients. Rendered by gs3d_render_forward_render_only; not trainable."""

    means_opacities: torch.Tensor
    covariances: torch.Tensor
    sh_coeffs: torch.Tensor

    def __post_init__(self):
        n = self.means_opacities.shape[0]
        assert self.means_opacities.shape == (n, 4) and self.covariances.shape == (n, 6)
        assert self.sh_coeffs.shape[:2] == (n, 3)
        for t in (self.means_opacities, self.covariances, self.sh_coeffs):
            assert t.dtype == torch.float32 and t.is_contiguous()

    @property
    def n(self) -> int:
        return self.means_opacities.shape[0]

    @property
    def sh_degree(self) -> int:
        return int(round(math.sqrt(self.sh_coeffs.shape[2]))) - 1

    @property
    def device(self):
        return self.means_opacities.device

    def tensors(self):
        return (self.means_opacities, self.covariances, self.sh_coeffs)

    def to(self, device) -> "RenderOnlyGaussiansVector":
        return RenderOnlyGaussiansVector(*(t.to(device).contiguous() for t in self.tensors()))

    @classmethod
    def from_trainable(cls, g: "GaussiansVector") -> "RenderOnlyGaussiansVector":
        """The conversion of RenderOnlyGaussiansVector(ply_path) (gaussians.jl:741-762):
        opacities = sigmoid(opacity features), covariances = lower((R S)(R S)^T) with R the
        rotation of the normalised quaternion and S = diag(exp(scaling features))
        (`_scaling_rotation_features_to_covariances`, gaussians.jl:467-482), in float32."""
        mo = g.means_opacity_features.detach().cpu().numpy().astype(F32)
        s = np.exp(g.scaling_features.detach().cpu().numpy().astype(F32)).astype(F32)
        q = g.rotation_features.detach().cpu().numpy().astype(F32)
        qss = (q * q).sum(axis=1, dtype=F32)
        qs = np.sqrt(F32(2) * (F32(1) / qss)).astype(F32)
        r, x, y, z = (q[:, i] * qs for i in range(4))
        R = np.empty((q.shape[0], 3, 3), F32)
        R[:, 0, 0] = 1 - (y * y + z * z); R[:, 0, 1] = x * y - r * z; R[:, 0, 2] = x * z + r * y
        R[:, 1, 0] = x * y + r * z; R[:, 1, 1] = 1 - (x * x + z * z); R[:, 1, 2] = y * z - r * x
        R[:, 2, 0] = x * z - r * y; R[:, 2, 1] = y * z + r * x; R[:, 2, 2] = 1 - (x * x + y * y)
        RS = (R * s[:, None, :]).astype(F32)
        cov = np.einsum("nik,njk->nij", RS, RS).astype(F32)
        lower = np.stack([cov[:, 0, 0], cov[:, 1, 0], cov[:, 2, 0], cov[:, 1, 1], cov[:, 2, 1],
                          cov[:, 2, 2]], axis=1).astype(F32)
        mo_ro = mo.copy()
        mo_ro[:, 3] = (F32(1) / (F32(1) + np.exp(-mo[:, 3]))).astype(F32)
        dev = g.means_opacity_features.device
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        return cls(t(mo_ro), t(lower), g.sh_coeffs.detach().clone())

    def to_c(self) -> _abi.RenderOnlyGaussiansC:
        g = _abi.RenderOnlyGaussiansC()
        g.n, g.sh_degree = self.n, self.sh_degree
        g.means_opacities = _ptr(self.means_opacities)
        g.covariances = _ptr(self.covariances)
        g.sh_coeffs = _ptr(self.sh_coeffs)
        return g


@dataclass
class RenderOutputs:
    """RenderOutputs: rgb (w, h, 3), transmittance / depth / last index (w, h)."""

    rgb: torch.Tensor | None
    transmittance: torch.Tensor | None = None
    depth: torch.Tensor | None = None
    last_contributing_sdfgids: torch.Tensor | None = None

    @classmethod
    def create(cls, width: int, height: int, device, include_rgb=True, include_transmittance=True,
               include_depth=False, include_last_contributing_indices=True) -> "RenderOutputs":
        f = dict(dtype=torch.float32, device=device)
        return cls(
            torch.empty((width, height, 3), **f) if include_rgb else None,
            torch.empty((width, height), **f) if include_transmittance else None,
            torch.empty((width, height), **f) if include_depth else None,
            torch.empty((width, height), dtype=torch.int32, device=device)
            if include_last_contributing_indices else None)

    def image_hwc(self) -> torch.Tensor:
        """The RGB image as (h, w, 3)."""
        return self.rgb.permute(1, 0, 2)

    def to_c(self) -> _abi.RenderOutputsC:
        o = _abi.RenderOutputsC()
        o.rgb = _ptr(self.rgb)
        o.transmittance = _ptr(self.transmittance)
        o.depth = _ptr(self.depth)
        o.last_contributing_sdfgids = _ptr(self.last_contributing_sdfgids)
        return o


MAX_TILE_PIXELS = 512  # the rasterisers' CTA size bound (one thread per pixel of a tile)


@dataclass
class RenderBuffers:
    """RenderBuffers + Filtered2DGaussiansVector, capacity-allocated on `device`."""

    capacity_n: int
    capacity_dup: int
    nb_tiles: int
    keep_gaussians: torch.Tensor
    keep_gaussians_cs: torch.Tensor
    fgidx_to_gidx: torch.Tensor
    depths: torch.Tensor
    f2d: torch.Tensor  # (n, 9): mean2d(2) opacity(1) inverse covariance lower(3) colour(3)
    intersected_tile_ranges: torch.Tensor  # (n, 4): xmin ymin xmax ymax
    nb_overlapped_tiles: torch.Tensor
    nb_overlapped_tiles_cs: torch.Tensor
    df2dgs_codes: torch.Tensor
    dfgidx_to_fgidx: torch.Tensor
    sdf2dgs_codes: torch.Tensor
    sdfgidx_to_fgidx: torch.Tensor
    tiles_end_sdfgidx: torch.Tensor
    device_counts: torch.Tensor
    workspace: torch.Tensor
    host_counts: torch.Tensor = field(default=None)
    # contribution masks (one word per warp and 32 entries) written by the forward blend for the
    # backward blend
    # (gs3d_render_buffers.contrib_masks); None: not used
    contrib_masks: torch.Tensor = field(default=None)
    # tiles by descending duplicate count, filled by the forward blend and taken in that order by
    # both blends (gs3d_render_buffers.tile_order); None: row-major order
    tile_order: torch.Tensor = field(default=None)

    @classmethod
    def create(cls, capacity_n: int, nb_tiles: int, device, capacity_dup: int | None = None,
               keep_cs: bool = True, mask_dup: int | None = -1,
               tile_order: bool = True) -> "RenderBuffers":
        """`mask_dup`: duplicated entries the contribution masks can describe (-1: the smaller
        of capacity_dup and 2 capacity_n + 65536; None or 0: no masks). Renders with more
        duplicates than that run the backward blend without masks. `tile_order`: the blends
        take the longest tiles first."""
        if capacity_dup is None:
            capacity_dup = max(4 * capacity_n, 1 << 16)
        dev = torch.device(device)
        i32 = dict(dtype=torch.int32, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        cn = max(capacity_n, 1)
        ws = _workspace_bytes(cn, capacity_dup, nb_tiles)
        b = cls(capacity_n, capacity_dup, nb_tiles,
                torch.empty(cn, dtype=torch.uint8, device=dev),
                torch.empty(cn, **i32) if keep_cs else None,
                torch.empty(cn, **i32), torch.empty(cn, **f32), torch.empty((cn, 9), **f32),
                torch.empty((cn, 4), **i32), torch.empty(cn, **i32), torch.empty(cn, **i32),
                torch.empty(capacity_dup, dtype=torch.int64, device=dev),
                torch.empty(capacity_dup, **i32),
                torch.empty(capacity_dup, dtype=torch.int64, device=dev),
                torch.empty(capacity_dup, **i32), torch.empty(max(nb_tiles, 1), **i32),
                torch.zeros(4, **i32), torch.empty(ws, dtype=torch.uint8, device=dev))
        if dev.type == "cuda":
            b.host_counts = torch.zeros(4, dtype=torch.int32, pin_memory=True)
        if mask_dup == -1:
            mask_dup = min(capacity_dup, 2 * max(capacity_n, 1) + 65536)
        if mask_dup:
            words = (mask_dup // 32 + max(nb_tiles, 1) + 1) * (MAX_TILE_PIXELS // 32)
            b.contrib_masks = torch.empty(words, dtype=torch.int32, device=dev)
        if tile_order:
            b.tile_order = torch.empty(max(nb_tiles, 1), **i32)
        return b

    def grow_dup(self, needed: int) -> None:
        """set_nb_dfgaussians! growth (forward_structs.jl:1794-1805)."""
        cap = max(needed + needed // 2, self.capacity_dup * 2)
        dev = self.df2dgs_codes.device
        self.capacity_dup = cap
        self.df2dgs_codes = torch.empty(cap, dtype=torch.int64, device=dev)
        self.dfgidx_to_fgidx = torch.empty(cap, dtype=torch.int32, device=dev)
        self.sdf2dgs_codes = torch.empty(cap, dtype=torch.int64, device=dev)
        self.sdfgidx_to_fgidx = torch.empty(cap, dtype=torch.int32, device=dev)
        self.workspace = torch.empty(_workspace_bytes(max(self.capacity_n, 1), cap, self.nb_tiles),
                                     dtype=torch.uint8, device=dev)

    def to_c(self) -> _abi.RenderBuffersC:
        b = _abi.RenderBuffersC()
        b.capacity_n, b.capacity_dup = self.capacity_n, self.capacity_dup
        b.keep_gaussians = _ptr(self.keep_gaussians)
        b.keep_gaussians_cs = _ptr(self.keep_gaussians_cs)
        b.fgidx_to_gidx = _ptr(self.fgidx_to_gidx)
        b.depths = _ptr(self.depths)
        b.means2d_opacities_inverse_covariances_colors = _ptr(self.f2d)
        b.intersected_tile_ranges = _ptr(self.intersected_tile_ranges)
        b.nb_overlapped_tiles = _ptr(self.nb_overlapped_tiles)
        b.nb_overlapped_tiles_cs = _ptr(self.nb_overlapped_tiles_cs)
        b.df2dgs_codes = _ptr(self.df2dgs_codes)
        b.dfgidx_to_fgidx = _ptr(self.dfgidx_to_fgidx)
        b.sdf2dgs_codes = _ptr(self.sdf2dgs_codes)
        b.sdfgidx_to_fgidx = _ptr(self.sdfgidx_to_fgidx)
        b.tiles_end_sdfgidx = _ptr(self.tiles_end_sdfgidx)
        b.device_counts = _ptr(self.device_counts)
        b.workspace = _ptr(self.workspace)
        b.workspace_bytes = self.workspace.numel()
        if self.contrib_masks is not None:
            b.contrib_masks = _ptr(self.contrib_masks)
            b.contrib_mask_words = self.contrib_masks.numel()
        if self.tile_order is not None:
            b.tile_order = _ptr(self.tile_order)
        return b


def _workspace_bytes(capacity_n: int, capacity_dup: int, nb_tiles: int) -> int:
    import ctypes
    out = ctypes.c_size_t(0)
    _abi.check(_abi.lib().gs3d_render_forward_workspace_size(capacity_n, capacity_dup, nb_tiles,
                                                              ctypes.byref(out)))
    return max(int(out.value), 256)
