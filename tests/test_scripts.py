"""Host logic of the headless entry points (gs3d/scripts.py) on the CPU: image files, the
validation-camera choice and the model choice of scripts/train.jl and scripts/render.jl."""
import math

import numpy as np
import pytest
import torch

from gs3d import scripts


def test_image_files_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    img = torch.from_numpy(rng.uniform(0, 1, size=(7, 5, 3)).astype(np.float32))  # (w, h, 3)
    scripts.write_image(tmp_path / "a.npy", img)
    assert torch.equal(scripts.read_image(tmp_path / "a.npy"), img)
    assert np.load(tmp_path / "a.npy").shape == (5, 7, 3)  # stored as (h, w, 3)
    scripts.write_image(tmp_path / "a.ppm", img)
    back = scripts.read_image(tmp_path / "a.ppm")
    assert back.shape == (7, 5, 3)
    assert torch.equal(back, torch.from_numpy(np.rint(img.numpy() * 255).astype(np.float32) / 255))


def test_ppm_pgm_headers_and_uint8_npy(tmp_path):
    w, h = 3, 2
    px = bytes(range(w * h * 3))
    (tmp_path / "c.ppm").write_bytes(b"P6\n# comment\n3 2\n255\n" + px)
    a = scripts.read_image(tmp_path / "c.ppm")
    want = np.frombuffer(px, np.uint8).reshape(h, w, 3).astype(np.float32) / 255
    assert torch.equal(a, torch.from_numpy(want.transpose(1, 0, 2).copy()))
    (tmp_path / "g.pgm").write_bytes(b"P5 3 2 255\n" + bytes(range(6)))
    g = scripts.read_image(tmp_path / "g.pgm")
    assert g.shape == (3, 2, 3) and torch.equal(g[..., 0], g[..., 2])
    np.save(tmp_path / "u.npy", np.full((h, w, 3), 51, np.uint8))
    assert torch.allclose(scripts.read_image(tmp_path / "u.npy"), torch.full((w, h, 3), 0.2))
    (tmp_path / "x.png").write_bytes(b"")
    with pytest.raises(ValueError):
        scripts.read_image(tmp_path / "x.png")


def test_validation_cameras_as_the_script_picks_them():
    rng = np.random.default_rng(0)
    assert scripts.validation_camera_ids(10, 0.0, False, rng) == []
    assert scripts.validation_camera_ids(10, 0.2, False, rng) == [4, 9]      # 1-based 5:5:10
    assert scripts.validation_camera_ids(11, 0.2, False, rng) == [5]         # k = 2, step 6: 6:6:11
    ids = scripts.validation_camera_ids(20, 0.25, True, rng)
    assert len(ids) == 5 and len(set(ids)) == 5 and all(0 <= i < 20 for i in ids)


def test_evaluation_and_save_schedules():
    assert scripts._due(0, 1000) and scripts._due(2000, 1000) and not scripts._due(999, 1000)
    assert scripts._due(7000, (7000, 30_000)) and not scripts._due(7001, (7000, 30_000))


def test_model_choice(tmp_path):
    for n in (10, 300, 30):
        d = tmp_path / "out" / "point_cloud" / f"iteration_{n}"
        d.mkdir(parents=True)
        (d / "point_cloud.ply").write_bytes(b"")
    assert scripts.model_path(tmp_path / "out").parent.name == "iteration_300"
    assert scripts.model_path(tmp_path / "out", 30).parent.name == "iteration_30"
    assert scripts.model_path(tmp_path / "m.ply") == tmp_path / "m.ply"
    cam = scripts.default_camera()
    assert (cam.width, cam.height) == (1280, 720) and cam.fx == pytest.approx(640.0)


def test_train_rejects_inputs_before_touching_the_gpu(tmp_path):
    """A cameras.json whose image does not match its camera, or a split that leaves no training
    camera, is an error raised while reading the inputs."""
    from gs3d import io
    from gs3d.scene import look_at_camera
    cam = look_at_camera(8, 6, 60.0, (0, 0, 3))
    scripts.write_image(tmp_path / "a.npy", torch.zeros((7, 6, 3)))
    io.save_cameras_json(tmp_path / "cameras.json", [cam], image_paths=["a.npy"])
    with pytest.raises(ValueError, match="image of size"):
        scripts.train(tmp_path, tmp_path / "out", device="cpu")


# ---- learning-rate annealing (training.jl:287-302) -------------------------------------
def test_annealed_means_lr_schedule():
    from gs3d.training import TrainingOptions, annealed_means_lr

    o = TrainingOptions(scene_radius=2.5, nb_iterations=30_000)
    a, b = o.initial_means_lr, o.final_means_lr
    lrs = [annealed_means_lr(it, o) for it in (1, 2, 100, 15_000, 29_999, 30_000, 40_000)]
    # iteration 1 uses the initial rate, the last annealing iteration and later the final one
    # (each through one Float32 log and exp, as the reference evaluates them: log(lr) ~ -9
    # rounded to Float32 moves exp by up to ~2^-21 relative)
    assert lrs[0] == pytest.approx(a, rel=1e-6)
    assert lrs[-2] == lrs[-1] and lrs[-1] == pytest.approx(b, rel=1e-6)
    assert all(x > y for x, y in zip(lrs, lrs[1:-1]))
    # log-linear in between: the midpoint is the geometric mean
    mid = annealed_means_lr(1 + (30_000 - 1) // 2, o)
    assert mid == pytest.approx(math.sqrt(a * b), rel=1e-4)
    for it in (1, 7, 1234, 29_000):
        x = (it - 1) / (30_000 - 1)
        want = math.exp((1 - x) * math.log(a) + x * math.log(b))
        assert annealed_means_lr(it, o) == pytest.approx(want, rel=2e-6)
        assert isinstance(annealed_means_lr(it, o), float)
        assert annealed_means_lr(it, o) == float(np.float32(annealed_means_lr(it, o)))


def test_annealed_means_lr_degenerate_step_counts():
    from gs3d.training import TrainingOptions, annealed_means_lr

    two = TrainingOptions(scene_radius=1.0, nb_lr_annealing_steps=2)
    assert annealed_means_lr(1, two) == pytest.approx(two.initial_means_lr, rel=1e-6)
    assert annealed_means_lr(2, two) == pytest.approx(two.final_means_lr, rel=1e-6)
    one = TrainingOptions(scene_radius=1.0, nb_lr_annealing_steps=1)
    with pytest.raises(ValueError):
        annealed_means_lr(1, one)
    assert annealed_means_lr(5, one) == pytest.approx(one.final_means_lr, rel=1e-6)
    zero = TrainingOptions(scene_radius=1.0, nb_lr_annealing_steps=0)   # x clamps to 0
    assert annealed_means_lr(9, zero) == pytest.approx(zero.initial_means_lr, rel=1e-6)
