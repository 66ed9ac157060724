"""Headless entry points: `train` mirrors Scripts.train (scripts/train.jl:43-197) with
`show_gui = false`, `render` replaces the GUI loop of Scripts.render (scripts/render.jl:17-57)
with a loop over cameras that writes images.

train(input_dir, output_dir) differs from the reference only where the reference calls out of
the training path: instead of running COLMAP on a directory of images and building the first
model from its points (`process_colmap`, `processed_colmap_to_cameras_with_images_and_gaussians_model`),
`input_dir` holds `cameras.json` (entries with a `path` to each training image, relative to
`input_dir` or absolute) and `point_cloud.ply`: a 3DGS model, or a coloured point cloud (x y z red
green blue, e.g. exported from an SfM run) that starts as the reference's first model
(`gaussians_from_point_cloud`). Everything else follows the
script: validation cameras (`validation_ratio`, equidistant or random), `TrainingOptions` from the
training scene, the loop `while iteration_nb <= nb_iterations: maybe_eval_losses; training_step;
maybe_save` (so the last step brings iteration_nb to nb_iterations + 1, as there), the MSE / MAE /
DSSIM evaluation on the training and validation sets at `evaluation_iterations` (a period or a
collection), and the output layout `cameras.json` + `point_cloud/iteration_<n>/point_cloud.ply`.
Images are read from `.npy` ((height, width, 3) or (height, width), float in [0, 1] or uint8) or
binary `.ppm` / `.pgm` files (no image library in this image); renders are written the same way.
"""
from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import torch

from . import io
from .render import render as gs_render
from .scene import scene_radius
from .structs import (PinholeCamera, RenderBuffers, RenderOptions, RenderOutputs, Tiling,
                      fov_deg_to_focal_length)

# -- images -----------------------------------------------------------------------------------
def read_image(path) -> torch.Tensor:
    """An image file as a float32 (width, height, 3) tensor (the renderer's 3 x h x w layout)."""
    p = Path(path)
    if p.suffix == ".npy":
        a = np.load(p)
    elif p.suffix in (".ppm", ".pgm"):
        raw = p.read_bytes()
        fields, pos = [], 0
        while len(fields) < 4:  # magic, width, height, maxval; '#' comments between them
            while raw[pos:pos + 1].isspace():
                pos += 1
            if raw[pos:pos + 1] == b"#":
                pos = raw.index(b"\n", pos) + 1
                continue
            end = pos
            while not raw[end:end + 1].isspace():
                end += 1
            fields.append(raw[pos:end].decode("ascii"))
            pos = end
        pos += 1
        magic, w, h, maxval = fields[0], int(fields[1]), int(fields[2]), int(fields[3])
        ch = {"P6": 3, "P5": 1}.get(magic)
        if ch is None:
            raise ValueError(f"{p}: only binary PPM (P6) / PGM (P5) files are read")
        dt = np.dtype(">u2") if maxval > 255 else np.dtype("u1")
        a = np.frombuffer(raw, dtype=dt, count=w * h * ch, offset=pos).reshape(h, w, ch)
        a = a.astype(np.float32) / np.float32(maxval)
    else:
        raise ValueError(f"{p}: unsupported image format (use .npy, .ppm or .pgm)")
    if a.dtype == np.uint8:
        a = a.astype(np.float32) / np.float32(255)
    a = np.asarray(a, dtype=np.float32)
    if a.ndim == 2:
        a = a[:, :, None]
    if a.shape[2] == 1:
        a = np.repeat(a, 3, axis=2)
    return torch.from_numpy(np.ascontiguousarray(a[:, :, :3].transpose(1, 0, 2)))


def write_image(path, rgb: torch.Tensor) -> None:
    """Write a (width, height, 3) image as `.npy` ((height, width, 3) float32) or binary `.ppm`
    (8 bits, values clamped to [0, 1] and rounded)."""
    p = Path(path)
    a = rgb.detach().cpu().numpy().transpose(1, 0, 2)
    if p.suffix == ".npy":
        np.save(p, np.ascontiguousarray(a.astype(np.float32)))
    elif p.suffix == ".ppm":
        h, w = a.shape[:2]
        b = np.rint(np.clip(a, 0.0, 1.0) * 255.0).astype(np.uint8)
        p.write_bytes(f"P6\n{w} {h}\n255\n".encode("ascii") + np.ascontiguousarray(b).tobytes())
    else:
        raise ValueError(f"{p}: unsupported image format (use .npy or .ppm)")


# -- train ------------------------------------------------------------------------------------
def validation_camera_ids(nb_cameras: int, validation_ratio: float, random: bool, rng) -> list[int]:
    """0-based validation cameras as the script picks them: floor(n * ratio) cameras, either a
    random selection or every ceil(n / k)-th camera (1-based step:step:n)."""
    k = int(math.floor(nb_cameras * validation_ratio))
    if k == 0:
        return []
    if random:
        return sorted(int(i) for i in rng.permutation(nb_cameras)[:k])
    step = -(-nb_cameras // k)
    return [i - 1 for i in range(step, nb_cameras + 1, step)]


def _due(iteration_nb: int, spec) -> bool:
    if isinstance(spec, (int, np.integer)):
        return iteration_nb % int(spec) == 0
    return iteration_nb in set(spec)


def evaluate(trainer, cameras, images, device) -> dict[str, float] | None:
    """Mean MSE, MAE (L1) and DSSIM of `trainer`'s current model over (camera, image) pairs (the
    script's compute_losses)."""
    if not cameras:
        return None
    from .loss import LossComputer
    w, h = trainer.width, trainer.height
    lc = LossComputer(w, h, device, trainer.options.loss_dssim_vs_L1_weight)
    scratch = torch.empty((w, h, 3), dtype=torch.float32, device=device)
    mse = mae = dssim = 0.0
    for cam, img in zip(cameras, images):
        gt = img.to(device)
        gs_render(trainer.render_outputs, trainer.gaussians, cam, trainer.tiling,
                  trainer.render_options, trainer.render_buffers, contrib_masks=False)
        rgb = trainer.render_outputs.rgb
        v = lc(rgb, gt, scratch).clone()
        mse += float(((rgb - gt) ** 2).mean())
        mae += float(v[1])
        dssim += float(v[2])
    k = len(cameras)
    return {"mse": mse / k, "mae": mae / k, "dssim": dssim / k}


def train(input_dir, output_dir, *, render_options_from_camera=None, training_options_from_scene=None,
          evaluation_iterations=1000, save_iterations=(7000, 30_000), validation_ratio: float = 0.0,
          random_validation_cameras: bool = False, device="cuda", seed: int = 0, log=print):
    """Train the model `input_dir/point_cloud.ply` on the cameras and images of
    `input_dir/cameras.json`; write `output_dir/cameras.json` and the models of
    `save_iterations`. Returns (trainer, evaluations) with evaluations a list of
    (iteration_nb, {"training": {...}, "validation": {...} or None})."""
    from .training import Trainer, TrainingOptions

    input_dir, output_dir = Path(input_dir), Path(output_dir)
    device = torch.device(device)
    json_path = input_dir / "cameras.json"
    cameras = io.load_cameras_json(json_path)
    import json as _json
    entries = _json.loads(json_path.read_text())
    paths = [Path(e["path"]) if Path(e["path"]).is_absolute() else input_dir / e["path"] for e in entries]
    images = [read_image(p) for p in paths]
    for cam, img in zip(cameras, images):
        if img.shape != (cam.width, cam.height, 3):
            raise ValueError(f"image of size {tuple(img.shape[:2])} for a {cam.width}x{cam.height} camera")
    gaussians = io.load_model_or_point_cloud(input_dir / "point_cloud.ply", device=device)
    output_dir.mkdir(parents=True, exist_ok=True)
    io.save_cameras_json(output_dir / "cameras.json", cameras, image_paths=[str(p) for p in paths])

    rng = np.random.default_rng(seed)
    val_ids = validation_camera_ids(len(cameras), validation_ratio, random_validation_cameras, rng)
    train_ids = [i for i in range(len(cameras)) if i not in set(val_ids)]
    if not train_ids:
        raise ValueError(f"validation_ratio {validation_ratio} leaves no training camera")
    train_cams = [cameras[i] for i in train_ids]
    train_imgs = [images[i].pin_memory() if device.type == "cuda" else images[i] for i in train_ids]
    val_cams = [cameras[i] for i in val_ids]
    val_imgs = [images[i] for i in val_ids]

    first = train_cams[0]
    ro = (render_options_from_camera(first) if render_options_from_camera
          else RenderOptions.for_camera(first, gaussians.sh_degree))
    opts = (training_options_from_scene(train_cams) if training_options_from_scene
            else TrainingOptions(scene_radius=scene_radius(train_cams)))
    trainer = Trainer(gaussians, train_cams, train_imgs, ro, Tiling.for_camera(first), opts, seed=seed)

    evaluations = []
    while trainer.iteration_nb <= opts.nb_iterations:
        if _due(trainer.iteration_nb, evaluation_iterations):
            res = {"training": evaluate(trainer, train_cams, train_imgs, device),
                   "validation": evaluate(trainer, val_cams, val_imgs, device)}
            evaluations.append((trainer.iteration_nb, res))
            log(f"Losses after iteration {trainer.iteration_nb}:")
            for name, r in (("Training", res["training"]), ("Validation", res["validation"])):
                if r is not None:
                    log(f"  {name}:\n    MSE (L2): {r['mse']}\n    MAE (L1): {r['mae']}\n"
                        f"    DSSIM:    {r['dssim']}")
        trainer.training_step()
        if _due(trainer.iteration_nb, save_iterations):
            d = output_dir / "point_cloud" / f"iteration_{trainer.iteration_nb}"
            d.mkdir(parents=True, exist_ok=True)
            io.save_ply(d / "point_cloud.ply", trainer.gaussians)
            log(f"Saved Gaussians model after {trainer.iteration_nb} iterations to {d / 'point_cloud.ply'}")
    if device.type == "cuda":
        torch.cuda.synchronize(device)
    return trainer, evaluations


# -- render -----------------------------------------------------------------------------------
def default_camera() -> PinholeCamera:
    """The script's camera for a bare .ply: 1280 x 720, 90 degree horizontal field of view,
    identity rotation at the origin."""
    w, h = 1280, 720
    return PinholeCamera.simple(w, h, fov_deg_to_focal_length(90.0, w), np.eye(3), np.zeros(3))


def model_path(path, iterations=None) -> Path:
    """The script's model choice: a .ply as given, or in a training output directory
    point_cloud/iteration_<n>/point_cloud.ply for the largest (or the given) n."""
    p = Path(path)
    if not p.is_dir():
        return p
    if iterations is None:
        its = [int(d.name[len("iteration_"):]) for d in (p / "point_cloud").iterdir()
               if d.name.startswith("iteration_")]
        iterations = max(its)
    return p / "point_cloud" / f"iteration_{iterations}" / "point_cloud.ply"


def render(path, out_dir=None, *, iterations=None, cameras=None, sh_degree=None,
           image_format: str = "ppm", device="cuda") -> list[torch.Tensor]:
    """Render the model at `path` (a .ply, or a training output directory), loaded as a
    RenderOnlyGaussiansVector like the script does, for each camera (by
    default the output directory's cameras.json, else `default_camera()`); write
    `out_dir/render_<i>.<image_format>` when `out_dir` is given. Returns the (width, height, 3)
    images on the device."""
    device = torch.device(device)
    p = Path(path)
    g = io.load_ply_render_only(model_path(p, iterations), device=device)  # as the script loads it
    if cameras is None:
        cameras = (io.load_cameras_json(p / "cameras.json")
                   if p.is_dir() and (p / "cameras.json").exists() else [default_camera()])
    deg = g.sh_degree if sh_degree is None else int(sh_degree)
    if out_dir is not None:
        Path(out_dir).mkdir(parents=True, exist_ok=True)
    images, out, buf, key = [], None, None, None
    for i, cam in enumerate(cameras):
        til = Tiling.for_camera(cam)
        if key != (cam.width, cam.height, til.nb_tiles):
            out = RenderOutputs.create(cam.width, cam.height, device)
            buf = RenderBuffers.create(g.n, til.nb_tiles, device, mask_dup=None)
            key = (cam.width, cam.height, til.nb_tiles)
        gs_render(out, g, cam, til, RenderOptions.for_camera(cam, deg), buf, contrib_masks=False)
        img = out.rgb.clone()
        images.append(img)
        if out_dir is not None:
            write_image(Path(out_dir) / f"render_{i:05d}.{image_format}", img)
    return images
