"""On-disk formats (gs3d/io.py) on the CPU: the 3DGS PLY model and cameras.json as the
reference writes and reads them (gaussians.jl:553-592, :839-968; cameras.jl:403-522)."""
import json
import math
import struct

import numpy as np
import pytest
import torch

from gs3d import io
from gs3d.scene import SceneSpec, look_at_camera, synthetic_gaussians


def random_gaussians(n, degree, seed=0):
    g = synthetic_gaussians(SceneSpec(n, "uniform:1", -4.0, 0.5), seed)
    g.set_sh_degree(degree)
    rng = np.random.default_rng(seed + 1)
    g.sh_coeffs.copy_(torch.from_numpy(rng.normal(0, 0.3, size=g.sh_coeffs.shape).astype(np.float32)))
    return g


@pytest.mark.parametrize("degree", [0, 1, 2, 3])
def test_ply_round_trip_is_exact(tmp_path, degree):
    g = random_gaussians(257, degree)
    p = tmp_path / "g.ply"
    io.save_ply(p, g)
    back = io.load_ply(p)
    assert back.sh_degree == degree
    for a, b in zip(g.tensors(), back.tensors()):
        assert torch.equal(a, b)


def test_ply_layout_matches_the_reference_writer(tmp_path):
    """Header (property order x y z f_dc_* f_rest_* opacity scale_* rot_*, type names) and the
    binary records: f_rest_(c (h-1) + k - 1) is coefficient k of channel c (gaussians.jl:885-902)."""
    g = random_gaussians(5, 2)
    p = tmp_path / "g.ply"
    io.save_ply(p, g)
    raw = p.read_bytes()
    head, body = raw.split(b"end_header\n", 1)
    lines = head.decode().splitlines()
    assert lines[:3] == ["ply", "format binary_little_endian 1.0", "element vertex 5"]
    props = [ln.split()[2] for ln in lines[3:]]
    assert all(ln.split()[1] == "float32" for ln in lines[3:])
    h = 9
    want = (["x", "y", "z", "f_dc_0", "f_dc_1", "f_dc_2"] +
            [f"f_rest_{i}" for i in range(3 * (h - 1))] +
            ["opacity", "scale_0", "scale_1", "scale_2", "rot_0", "rot_1", "rot_2", "rot_3"])
    assert props == want
    rec = np.frombuffer(body, dtype="<f4").reshape(5, len(want))
    sh = g.sh_coeffs.numpy()
    mo = g.means_opacity_features.numpy()
    i = 3
    assert np.array_equal(rec[i, :3], mo[i, :3])
    for c in range(3):
        assert rec[i, 3 + c] == sh[i, c, 0]
        for k in range(1, h):
            assert rec[i, 6 + c * (h - 1) + k - 1] == sh[i, c, k]
    assert rec[i, 6 + 3 * (h - 1)] == mo[i, 3]
    assert np.array_equal(rec[i, -7:-4], g.scaling_features.numpy()[i])
    assert np.array_equal(rec[i, -4:], g.rotation_features.numpy()[i])


def test_ply_options_normals_degree3_padding_float_names(tmp_path):
    g = random_gaussians(11, 1)
    p = tmp_path / "g.ply"
    io.save_ply(p, g, force_sh_degree_3=True, include_normals=True, use_float_double=True)
    head = p.read_bytes().split(b"end_header\n", 1)[0].decode().splitlines()
    props = [ln.split()[2] for ln in head[3:]]
    assert props[3:6] == ["nx", "ny", "nz"] and "f_rest_44" in props
    assert all(ln.split()[1] == "float" for ln in head[3:])
    back = io.load_ply(p)
    assert back.sh_degree == 3
    assert torch.equal(back.sh_coeffs[:, :, :4], g.sh_coeffs)
    assert torch.all(back.sh_coeffs[:, :, 4:] == 0)
    for a, b in zip(g.tensors()[:3], back.tensors()[:3]):
        assert torch.equal(a, b)


def _handmade_ply(fmt: str, rows):
    names = ["x", "y", "z", "f_dc_0", "f_dc_1", "f_dc_2", "f_rest_2", "f_rest_0", "f_rest_1",
             "f_rest_5", "f_rest_3", "f_rest_4", "f_rest_8", "f_rest_6", "f_rest_7", "opacity",
             "scale_0", "scale_1", "scale_2", "rot_0", "rot_1", "rot_2", "rot_3", "red"]
    types = ["float"] * 23 + ["uchar"]
    head = ["ply", f"format {fmt} 1.0", "comment hand made", f"element vertex {len(rows)}"]
    head += [f"property {t} {n}" for t, n in zip(types, names)]
    head += ["element face 0", "property float dummy", "end_header"]
    text = "\n".join(head) + "\n"
    if fmt == "ascii":
        return text.encode() + "".join(" ".join(str(v) for v in r) + "\n" for r in rows).encode()
    e = "<" if fmt == "binary_little_endian" else ">"
    body = b"".join(struct.pack(e + "23fB", *r) for r in rows)
    return text.encode() + body


@pytest.mark.parametrize("fmt", ["ascii", "binary_little_endian", "binary_big_endian"])
def test_ply_reader_follows_names_not_positions(tmp_path, fmt):
    """f_rest properties in any order are read in numeric order (as _read_3DGS_ply sorts them);
    extra properties and elements are ignored; degree 1 from 9 f_rest values."""
    rows = []
    for i in range(3):
        rest = {f"f_rest_{j}": 10.0 * i + j for j in range(9)}
        order = [2, 0, 1, 5, 3, 4, 8, 6, 7]
        rows.append([1.0 + i, 2.0, 3.0, 0.5, 0.25, -0.5] + [rest[f"f_rest_{j}"] for j in order] +
                    [0.75, -1.0, -2.0, -3.0, 1.0, 0.0, 0.0, 0.0, 7])
    p = tmp_path / f"h_{fmt}.ply"
    p.write_bytes(_handmade_ply(fmt, rows))
    g = io.load_ply(p)
    assert g.n == 3 and g.sh_degree == 1
    for i in range(3):
        assert g.means_opacity_features[i].tolist() == [1.0 + i, 2.0, 3.0, 0.75]
        assert g.sh_coeffs[i, :, 0].tolist() == [0.5, 0.25, -0.5]
        for c in range(3):
            for k in range(1, 4):
                assert g.sh_coeffs[i, c, k].item() == 10.0 * i + c * 3 + k - 1
    assert g.scaling_features[0].tolist() == [-1.0, -2.0, -3.0]
    assert g.rotation_features[0].tolist() == [1.0, 0.0, 0.0, 0.0]


def test_ply_reader_rejects_bad_files(tmp_path):
    p = tmp_path / "bad.ply"
    p.write_bytes(b"not a ply")
    with pytest.raises(ValueError):
        io.load_ply(p)
    p.write_bytes(b"ply\nformat binary_little_endian 1.0\nelement vertex 1\nproperty list uchar int idx\nend_header\n")
    with pytest.raises(ValueError):
        io.load_ply(p)


def test_cameras_json_round_trip(tmp_path):
    cams = [look_at_camera(640, 360, 50.0, (1.0, 2.0, 5.0)), look_at_camera(320, 200, 70.0, (-3, 1, 2))]
    cams[1].near_z = 0.2
    p = tmp_path / "cameras.json"
    io.save_cameras_json(p, cams, image_paths=["a.png", "b.png"])
    entries = json.loads(p.read_text())
    assert set(entries[0]) == {"width", "height", "fx", "fy", "skew", "ppx", "ppy", "position",
                               "rotation", "path"}
    back = io.load_cameras_json(p)
    for a, b in zip(cams, back):
        assert (a.width, a.height) == (b.width, b.height)
        for f in ("fx", "fy", "skew", "cx", "cy"):
            assert np.float32(getattr(a, f)) == np.float32(getattr(b, f))
        assert np.array_equal(np.asarray(a.R_c2w, np.float32), b.R_c2w)
        assert np.array_equal(np.asarray(a.t_c2w, np.float32), b.t_c2w)
        assert np.array_equal(a.projection_matrix_3x4, b.projection_matrix_3x4)


def test_cameras_json_3dgs_entries_and_rescaling(tmp_path):
    """An original-3DGS entry (no skew / principal point / clip planes): centred principal point,
    near 0.2, far inf; rescale_factor rounds the size and scales the focal lengths with it; a
    given ppy is scaled by the x factor, as the reference does."""
    R = [[1.0, 0.0, 0.0], [0.0, 0.0, -1.0], [0.0, 1.0, 0.0]]
    e = {"id": 0, "img_name": "img0", "width": 1000, "height": 750, "position": [0.5, -1.0, 2.0],
         "rotation": R, "fy": 900.0, "fx": 910.0}
    e2 = dict(e, ppx=510.0, ppy=370.0, near_z=0.5, far_z=100.0)
    p = tmp_path / "cameras.json"
    p.write_text(json.dumps([e, e2]))
    c, c2 = io.load_cameras_json(p)
    assert (c.width, c.height, c.fx, c.fy, c.skew, c.cx, c.cy) == (1000, 750, 910.0, 900.0, 0.0, 500.0, 375.0)
    assert c.near_z == np.float32(0.2) and math.isinf(c.far_z)
    assert np.array_equal(c.R_c2w, np.asarray(R, np.float32))
    assert np.array_equal(c.t_c2w, np.asarray([0.5, -1.0, 2.0], np.float32))
    assert (c2.cx, c2.cy, c2.near_z, c2.far_z) == (510.0, 370.0, 0.5, 100.0)
    r, r2 = io.load_cameras_json(p, rescale_factor=0.5)
    assert (r.width, r.height) == (500, 375)
    assert r.fx == np.float32(np.float32(910.0) * (np.float32(500) / np.float32(1000)))
    sx = np.float32(500) / np.float32(1000)
    assert r2.cy == float(np.float32(np.float32(370.0) * sx))
    f, _ = io.load_cameras_json(p, forced_width=800, forced_height=600)
    assert (f.width, f.height) == (800, 600)
    assert f.fy == float(np.float32(np.float32(900.0) * (np.float32(600) / np.float32(750))))


def test_gaussians_from_point_cloud_as_the_reference_initialises(tmp_path):
    """gaussians.jl:597-639: means at the points, logit(0.1) opacity features, degree-0 SH from
    the colours, identity rotations, log-scales = log(sum of the 4 nearest distances incl. the
    point itself / 3); a coloured point-cloud PLY (uchar colours) goes through it."""
    from gs3d.scene import gaussians_from_point_cloud
    rng = np.random.default_rng(2)
    pts = rng.uniform(-1, 1, size=(50, 3)).astype(np.float32)
    cols = rng.uniform(0, 1, size=(50, 3)).astype(np.float32)
    g = gaussians_from_point_cloud(pts, cols)
    assert g.n == 50 and g.sh_degree == 0
    mo = g.means_opacity_features.numpy()
    assert np.array_equal(mo[:, :3], pts)
    assert np.allclose(1 / (1 + np.exp(-mo[:, 3].astype(np.float64))), 0.1, rtol=1e-6)
    assert np.allclose(g.sh_coeffs.numpy()[:, :, 0] * 0.28209479177387814 + 0.5, cols, atol=1e-6)
    assert np.array_equal(g.rotation_features.numpy(), np.tile([1, 0, 0, 0], (50, 1)).astype(np.float32))
    d = np.sqrt(((pts[:, None, :].astype(np.float64) - pts[None, :, :]) ** 2).sum(-1))
    want = np.log(np.sort(d, axis=1)[:, :4].sum(1) / 3)
    sf = g.scaling_features.numpy()
    assert np.allclose(sf[:, 0], want, rtol=1e-5) and np.array_equal(sf[:, 0], sf[:, 2])

    header = ("ply\nformat binary_little_endian 1.0\nelement vertex 50\nproperty float x\n"
              "property float y\nproperty float z\nproperty uchar red\nproperty uchar green\n"
              "property uchar blue\nend_header\n").encode()
    u8 = (cols * 255).astype(np.uint8)
    rec = np.zeros(50, dtype=[("x", "<f4"), ("y", "<f4"), ("z", "<f4"), ("r", "u1"), ("g", "u1"), ("b", "u1")])
    rec["x"], rec["y"], rec["z"] = pts[:, 0], pts[:, 1], pts[:, 2]
    rec["r"], rec["g"], rec["b"] = u8[:, 0], u8[:, 1], u8[:, 2]
    p = tmp_path / "points.ply"
    p.write_bytes(header + rec.tobytes())
    pc = io.load_model_or_point_cloud(p)
    assert pc.sh_degree == 0 and np.array_equal(pc.means_opacity_features.numpy()[:, :3], pts)
    assert np.allclose(pc.sh_coeffs.numpy()[:, :, 0] * 0.28209479177387814 + 0.5, u8 / 255.0, atol=1e-6)
    m = tmp_path / "model.ply"
    io.save_ply(m, g)
    assert torch.equal(io.load_model_or_point_cloud(m).sh_coeffs, g.sh_coeffs)
