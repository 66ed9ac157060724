"""Headless Scripts.train / Scripts.render (gs3d/scripts.py) end to end on the GPU: a small
synthetic scene written to disk as the script's inputs (cameras.json with image paths, the
initial point_cloud.ply), trained with validation cameras, evaluation and save iterations; the
saved models and cameras read back and rendered."""
import json

import numpy as np
import pytest
import torch

import gs3d
from gs3d import RenderBuffers, RenderOptions, RenderOutputs, Tiling, io, scripts
from gs3d.scene import SceneSpec, look_at_camera, synthetic_gaussians
from gs3d.training import TrainingOptions

pytestmark = pytest.mark.gpu


def _write_point_cloud(path, n, seed):
    rng = np.random.default_rng(seed)
    rec = np.zeros(n, dtype=[("x", "<f4"), ("y", "<f4"), ("z", "<f4"),
                             ("red", "u1"), ("green", "u1"), ("blue", "u1")])
    for k in ("x", "y", "z"):
        rec[k] = rng.uniform(-1, 1, n)
    for k in ("red", "green", "blue"):
        rec[k] = rng.integers(0, 256, n)
    head = (f"ply\nformat binary_little_endian 1.0\nelement vertex {n}\nproperty float x\n"
            "property float y\nproperty float z\nproperty uchar red\nproperty uchar green\n"
            "property uchar blue\nend_header\n").encode()
    path.write_bytes(head + rec.tobytes())


@pytest.mark.parametrize("start", ["model", "point_cloud"])
def test_headless_train_then_render(cuda, tmp_path, start):
    w, h = 96, 64
    cams = [look_at_camera(w, h, 60.0, (np.cos(a) * 3, 0.8, np.sin(a) * 3))
            for a in np.linspace(0, 2 * np.pi, 5, endpoint=False)]
    # targets: renders of a different scene, so the loss can go down
    truth = synthetic_gaussians(SceneSpec(3_000, "uniform:1", -3.5, 0.5), 21).to(cuda)
    inp = tmp_path / "input"
    inp.mkdir()
    entries = []
    for i, cam in enumerate(cams):
        out = RenderOutputs.create(w, h, cuda)
        til = Tiling.for_camera(cam)
        gs3d.render(out, truth, cam, til, RenderOptions.for_camera(cam, 3),
                    RenderBuffers.create(truth.n, til.nb_tiles, cuda))
        name = f"img{i}.npy" if i % 2 else f"img{i}.ppm"
        scripts.write_image(inp / name, out.rgb)
        entries.append(name)
    io.save_cameras_json(inp / "cameras.json", cams, image_paths=entries)
    if start == "model":
        io.save_ply(inp / "point_cloud.ply", synthetic_gaussians(SceneSpec(2_000, "uniform:1", -4.0, 0.5), 5))
    else:  # a coloured point cloud starts as the reference's first model (SH degree 0)
        _write_point_cloud(inp / "point_cloud.ply", 2_000, 5)

    logs = []
    outd = tmp_path / "output"
    trainer, evals = scripts.train(
        inp, outd, training_options_from_scene=lambda c: TrainingOptions(scene_radius=3.3, nb_iterations=40),
        evaluation_iterations=20, save_iterations=(20, 41), validation_ratio=0.4, log=logs.append)
    assert trainer.iteration_nb == 41  # the loop's last step takes iteration_nb past nb_iterations
    assert [it for it, _ in evals] == [0, 20, 40]
    assert all(r["validation"] is not None for _, r in evals)
    assert evals[-1][1]["training"]["mae"] < evals[0][1]["training"]["mae"]
    assert any("Saved Gaussians model after 41" in s for s in logs)
    saved = json.loads((outd / "cameras.json").read_text())
    assert len(saved) == 5 and all("path" in e for e in saved)
    for it in (20, 41):
        assert (outd / "point_cloud" / f"iteration_{it}" / "point_cloud.ply").exists()
    final = io.load_ply(outd / "point_cloud" / "iteration_41" / "point_cloud.ply", device=cuda)
    for a, b in zip(final.tensors(), trainer.gaussians.tensors()):
        assert torch.equal(a, b)

    # render: the directory's latest model for its cameras, written as images
    imgs = scripts.render(outd, tmp_path / "renders", image_format="npy", device=cuda)
    assert len(imgs) == 5 and len(list((tmp_path / "renders").glob("render_*.npy"))) == 5
    # the script renders the model as a RenderOnlyGaussiansVector, as the reference's does
    out = RenderOutputs.create(w, h, cuda)
    til = Tiling.for_camera(cams[2])
    gs3d.render(out, gs3d.RenderOnlyGaussiansVector.from_trainable(final), cams[2], til,
                RenderOptions.for_camera(cams[2], final.sh_degree),
                RenderBuffers.create(final.n, til.nb_tiles, cuda))
    assert torch.equal(imgs[2], out.rgb)
    assert torch.equal(scripts.read_image(tmp_path / "renders" / "render_00002.npy").to(cuda), out.rgb)
    # a bare .ply renders with the script's default camera
    one = scripts.render(outd / "point_cloud" / "iteration_20" / "point_cloud.ply", device=cuda)
    assert len(one) == 1 and one[0].shape == (1280, 720, 3)
