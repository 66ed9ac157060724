"""On-disk formats either side of the training path.

* The 3DGS PLY model: `save_ply` writes what the reference's `save_to_ply` writes
  (gaussians.jl:839-968): one binary little-endian `vertex` element with the float properties
  x y z [nx ny nz] f_dc_0..2 f_rest_* opacity scale_0..2 rot_0..3 in that order (the order the
  SIBR viewer needs), the rest coefficients channel by channel (f_rest_(c (h - 1) + k - 1) is
  coefficient k >= 1 of channel c, h = (degree + 1)^2), property type names float32 (or float
  with `use_float_double`, for readers such as SuperSplat), optional zero normals, optional zero
  padding to degree 3. `load_ply` reads it back like `_read_3DGS_ply` (gaussians.jl:553-592):
  the f_rest properties in numeric order, the degree from their count. Binary (either byte
  order) and ASCII files with scalar properties are read.
* cameras.json: `load_cameras_json` follows `load_cameras_from_json` /
  `json_camera_entry_to_pinhole_camera` (cameras.jl:403-506): width/height (optionally rescaled
  or forced), fx/fy scaled with them, optional skew/ppx/ppy (the principal point defaults to the
  image centre; the reference scales ppy by the x factor, kept here), optional near_z/far_z
  (default 0.2 / inf), `rotation` = camera-to-world rotation as a list of rows, `position` = the
  camera centre. `save_cameras_json` writes the reference's `JSON.lower` fields
  (cameras.jl:508-522), plus `path` per camera when image paths are given (:1182-1190).
* Training checkpoints (the reference has none): parameters, Adam moments and update count,
  ADC accumulators, iteration number, render SH degree and the camera-order state, so that a
  resumed `Trainer` takes the same views and steps as the uninterrupted run (the backward's
  float-atomic sums make any two runs differ in the last bits).
"""
from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np
import torch

from .structs import DEFAULT_FAR, DEFAULT_NEAR, F32, GaussiansVector, PinholeCamera

_PLY_TYPES = {
    "char": "i1", "int8": "i1", "uchar": "u1", "uint8": "u1", "short": "i2", "int16": "i2",
    "ushort": "u2", "uint16": "u2", "int": "i4", "int32": "i4", "uint": "u4", "uint32": "u4",
    "float": "f4", "float32": "f4", "double": "f8", "float64": "f8",
}


# -- PLY --------------------------------------------------------------------------------------
def _ply_property_names(sh_degree: int, force_sh_degree_3: bool, include_normals: bool) -> list[str]:
    h = 16 if force_sh_degree_3 else (sh_degree + 1) ** 2
    names = ["x", "y", "z"]
    if include_normals:
        names += ["nx", "ny", "nz"]
    names += [f"f_dc_{c}" for c in range(3)]
    names += [f"f_rest_{c * (h - 1) + k - 1}" for c in range(3) for k in range(1, h)]
    names += ["opacity"] + [f"scale_{i}" for i in range(3)] + [f"rot_{i}" for i in range(4)]
    return names


def save_ply(path, gaussians: GaussiansVector, force_sh_degree_3: bool = False,
             include_normals: bool = False, use_float_double: bool = False) -> None:
    """Write `gaussians` as a 3DGS PLY model (binary little endian, float32 values)."""
    mo = gaussians.means_opacity_features.detach().cpu().numpy().astype(F32)
    sf = gaussians.scaling_features.detach().cpu().numpy().astype(F32)
    rf = gaussians.rotation_features.detach().cpu().numpy().astype(F32)
    sh = gaussians.sh_coeffs.detach().cpu().numpy().astype(F32)  # (n, 3, h)
    n, h = mo.shape[0], sh.shape[2]
    hh = 16 if force_sh_degree_3 else h
    cols = [mo[:, 0], mo[:, 1], mo[:, 2]]
    if include_normals:
        cols += [np.zeros(n, F32)] * 3
    cols += [sh[:, c, 0] for c in range(3)]
    for c in range(3):
        for k in range(1, hh):
            cols.append(sh[:, c, k] if k < h else np.zeros(n, F32))
    cols += [mo[:, 3]] + [sf[:, i] for i in range(3)] + [rf[:, i] for i in range(4)]
    names = _ply_property_names(gaussians.sh_degree, force_sh_degree_3, include_normals)
    assert len(names) == len(cols)
    tname = "float" if use_float_double else "float32"
    header = ["ply", "format binary_little_endian 1.0", f"element vertex {n}"]
    header += [f"property {tname} {nm}" for nm in names]
    header.append("end_header")
    data = np.stack(cols, axis=1).astype("<f4") if n else np.zeros((0, len(cols)), "<f4")
    with open(path, "wb") as f:
        f.write(("\n".join(header) + "\n").encode("ascii"))
        f.write(np.ascontiguousarray(data).tobytes())


def _read_ply(path) -> dict[str, np.ndarray]:
    """The `vertex` element of a PLY file as {property: values}."""
    raw = Path(path).read_bytes()
    end = raw.find(b"end_header")
    if not raw.startswith(b"ply") or end < 0:
        raise ValueError(f"{path}: not a PLY file")
    body_start = raw.index(b"\n", end) + 1
    lines = raw[:end].decode("ascii").splitlines()
    fmt = None
    elements = []  # (name, count, [(prop, dtype)])
    for line in lines[1:]:
        parts = line.split()
        if not parts or parts[0] in ("comment", "obj_info"):
            continue
        if parts[0] == "format":
            fmt = parts[1]
        elif parts[0] == "element":
            elements.append((parts[1], int(parts[2]), []))
        elif parts[0] == "property":
            if parts[1] == "list":
                raise ValueError(f"{path}: list properties are not supported")
            if parts[1] not in _PLY_TYPES:
                raise ValueError(f"{path}: unknown property type {parts[1]}")
            elements[-1][2].append((parts[2], _PLY_TYPES[parts[1]]))
    if fmt not in ("binary_little_endian", "binary_big_endian", "ascii"):
        raise ValueError(f"{path}: unsupported format {fmt}")
    offset = body_start
    text_rows = raw[body_start:].decode("ascii").split("\n") if fmt == "ascii" else None
    row = 0
    for name, count, props in elements:
        if fmt == "ascii":
            rows = [r.split() for r in text_rows[row:row + count]]
            row += count
            values = {p: np.array([float(r[i]) for r in rows], dtype=dt) for i, (p, dt) in enumerate(props)}
        else:
            order = "<" if fmt == "binary_little_endian" else ">"
            dtype = np.dtype([(p, order + dt) for p, dt in props])
            arr = np.frombuffer(raw, dtype=dtype, count=count, offset=offset)
            offset += count * dtype.itemsize
            values = {p: arr[p] for p, _ in props}
        if name == "vertex":
            return values
    raise ValueError(f"{path}: no vertex element")


def load_ply(path, device="cpu") -> GaussiansVector:
    """Read a 3DGS PLY model (as `_read_3DGS_ply`): means, opacity logits, log-scales,
    quaternions (r, x, y, z) and SH coefficients of the degree the f_rest count implies."""
    v = _read_ply(path)
    n = len(v["x"])
    rest = sorted((k for k in v if k.startswith("f_rest_")), key=lambda k: int(k.rsplit("_", 1)[1]))
    if len(rest) % 3:
        raise ValueError(f"{path}: {len(rest)} f_rest properties is not a multiple of 3")
    h = len(rest) // 3 + 1
    if int(round(math.sqrt(h))) ** 2 != h or h > 16:
        raise ValueError(f"{path}: {len(rest)} f_rest properties match no SH degree <= 3")
    sh = np.zeros((n, 3, h), F32)
    for c in range(3):
        sh[:, c, 0] = v[f"f_dc_{c}"]
    for j, k in enumerate(rest):  # f_rest_j: coefficient j mod (h - 1) + 1 of channel j div (h - 1)
        sh[:, j // (h - 1), j % (h - 1) + 1] = v[k]
    mo = np.stack([v["x"], v["y"], v["z"], v["opacity"]], axis=1).astype(F32)
    sf = np.stack([v[f"scale_{i}"] for i in range(3)], axis=1).astype(F32)
    rf = np.stack([v[f"rot_{i}"] for i in range(4)], axis=1).astype(F32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)
    return GaussiansVector(t(mo), t(sf), t(rf), t(sh))


def load_ply_render_only(path, device="cpu"):
    """RenderOnlyGaussiansVector(ply_path) (gaussians.jl:741-762): a 3DGS PLY model with the
    opacities after the sigmoid and the 3D covariances precomputed."""
    from .structs import RenderOnlyGaussiansVector
    return RenderOnlyGaussiansVector.from_trainable(load_ply(path, device=device))


def read_point_cloud(path) -> tuple[np.ndarray, np.ndarray]:
    """A coloured point cloud PLY (x y z and red green blue, as COLMAP exports its points):
    ((n, 3) float32 points, (n, 3) float32 colours in [0, 1]; 8-bit colours are divided by 255)."""
    v = _read_ply(path)
    pts = np.stack([v["x"], v["y"], v["z"]], axis=1).astype(F32)
    cols = np.stack([v["red"], v["green"], v["blue"]], axis=1)
    if cols.dtype == np.uint8:
        cols = cols.astype(F32) / F32(255)
    return pts, cols.astype(F32)


def load_model_or_point_cloud(path, device="cpu") -> GaussiansVector:
    """A 3DGS model PLY as is, or a coloured point cloud PLY through
    `gaussians_from_point_cloud` (the script's first model)."""
    from .scene import gaussians_from_point_cloud
    props = _read_ply(path)
    if "f_dc_0" in props:
        return load_ply(path, device=device)
    pts, cols = read_point_cloud(path)
    return gaussians_from_point_cloud(pts, cols, device=device)


# -- cameras.json -----------------------------------------------------------------------------
def _f32(x) -> float:
    return float(F32(x))


def load_cameras_json(path, rescale_factor=None, forced_width=None, forced_height=None):
    """cameras.json entries (3DGS or the reference's own) as PinholeCameras."""
    cams = []
    for e in json.loads(Path(path).read_text()):
        if forced_width is not None:
            w = int(forced_width)
        elif rescale_factor is not None:
            w = int(np.rint(e["width"] * rescale_factor))
        else:
            w = int(e["width"])
        if forced_height is not None:
            h = int(forced_height)
        elif rescale_factor is not None:
            h = int(np.rint(e["height"] * rescale_factor))
        else:
            h = int(e["height"])
        sx = F32(w) / F32(e["width"])
        sy = F32(h) / F32(e["height"])
        fx = _f32(F32(e["fx"]) * sx)
        fy = _f32(F32(e["fy"]) * sy)
        skew = _f32(F32(e["skew"]) * sx) if "skew" in e else 0.0
        cx = _f32(F32(e["ppx"]) * sx) if "ppx" in e else _f32(F32(w) / F32(2))
        # the reference scales ppy by the x factor (cameras.jl:482-486)
        cy = _f32(F32(e["ppy"]) * sx) if "ppy" in e else _f32(F32(h) / F32(2))
        near = _f32(e.get("near_z", DEFAULT_NEAR))
        far = float(e["far_z"]) if "far_z" in e else DEFAULT_FAR
        R = np.asarray(e["rotation"], dtype=F32).reshape(3, 3)  # rows of the camera-to-world rotation
        t = np.asarray(e["position"], dtype=F32).reshape(3)
        cams.append(PinholeCamera(w, h, fx, fy, skew, cx, cy, R, t, near, far))
    return cams


def save_cameras_json(path, cameras, image_paths=None) -> None:
    """Write cameras as the reference's save_json does (readable by `load_cameras_json`)."""
    out = []
    for i, cam in enumerate(cameras):
        e = {"width": int(cam.width), "height": int(cam.height), "fx": float(cam.fx),
             "fy": float(cam.fy), "skew": float(cam.skew), "ppx": float(cam.cx),
             "ppy": float(cam.cy), "position": [float(x) for x in np.asarray(cam.t_c2w).reshape(3)],
             "rotation": [[float(x) for x in row] for row in np.asarray(cam.R_c2w).reshape(3, 3)]}
        if image_paths is not None:
            e["path"] = str(image_paths[i])
        out.append(e)
    Path(path).write_text(json.dumps(out, indent=2))


# -- training checkpoints ---------------------------------------------------------------------
def save_checkpoint(path, trainer) -> None:
    """Everything a Trainer needs to continue: parameters, Adam moments and update count, ADC
    accumulators, iteration number, render SH degree, camera-order state."""
    if trainer.device.type == "cuda":
        torch.cuda.synchronize(trainer.device)
    if hasattr(trainer, "sync_parameters"):  # data-parallel: all-gathers still in flight
        trainer.sync_parameters()
    g, m, a = trainer.gaussians, trainer.optimizer.moments, trainer.adc_buffers
    state = {
        "format": "gs3d-checkpoint-1",
        "gaussians": [t.detach().cpu() for t in g.tensors()],
        "moments": [t.detach().cpu() for t in m.tensors()],
        "update_count": int(trainer.optimizer.update_count),
        "adc_norms": a.accumulated_mean2d_grad_norms_ndc[: g.n].detach().cpu(),
        "adc_counts": a.rendering_contribution_counts[: g.n].detach().cpu(),
        "iteration_nb": int(trainer.iteration_nb),
        "render_sh_degree": int(trainer.render_options.sh_degree),
        "cameras_order": np.asarray(trainer.cameras_order).tolist(),
        "cameras_order_idx": int(trainer.cameras_order_idx),
        "next_orders": [np.asarray(o).tolist() for o in getattr(trainer, "_next_orders", [])],
        "rng_state": trainer.rng.bit_generator.state,
        "adc_seed": int(trainer.adc_seed),
    }
    if hasattr(trainer, "step_index"):  # data-parallel trainer: its view schedule
        state["step_index"] = int(trainer.step_index)
        state["perm"] = np.asarray(trainer.perm).tolist()
    torch.save(state, path)


def load_checkpoint(path, trainer) -> None:
    """Restore `save_checkpoint`'s state into `trainer` (built for the same cameras and
    options); its buffers are resized to the checkpoint's Gaussian count."""
    from . import adc as adc_mod
    from .optimizer import AdamMoments

    state = torch.load(path, map_location="cpu", weights_only=False)
    if state.get("format") != "gs3d-checkpoint-1":
        raise ValueError(f"{path}: not a gs3d checkpoint")
    dev = trainer.device
    g = GaussiansVector(*[t.to(dev).contiguous() for t in state["gaussians"]])
    trainer.gaussians.replace(g)
    trainer.optimizer.moments = AdamMoments(*[t.to(dev).contiguous() for t in state["moments"]])
    trainer.optimizer.update_count = int(state["update_count"])
    n = trainer.gaussians.n
    trainer.adc_buffers = adc_mod.AdcBuffers.create(n, dev)
    trainer.adc_buffers.accumulated_mean2d_grad_norms_ndc[:n].copy_(state["adc_norms"].to(dev))
    trainer.adc_buffers.rendering_contribution_counts[:n].copy_(state["adc_counts"].to(dev))
    trainer.iteration_nb = int(state["iteration_nb"])
    trainer.render_options = trainer.render_options.with_sh_degree(int(state["render_sh_degree"]))
    trainer.fgradients = type(trainer.fgradients).create(n, trainer.gaussians.sh_degree, dev)
    trainer.complete_adc_step()
    trainer.cameras_order = np.asarray(state["cameras_order"])
    trainer.cameras_order_idx = int(state["cameras_order_idx"])
    trainer.rng.bit_generator.state = state["rng_state"]
    trainer._next_orders = [np.asarray(o) for o in state.get("next_orders", [])]
    trainer._prefetched = None
    trainer.adc_seed = int(state["adc_seed"])
    if "step_index" in state and hasattr(trainer, "step_index"):
        trainer.step_index = int(state["step_index"])
        trainer.perm = np.asarray(state["perm"])
    if hasattr(trainer, "_ensure_padded"):
        trainer._ensure_padded()
