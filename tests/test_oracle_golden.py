"""Pin the CPU oracle to the reference's own golden data (no GPU needed).

Fixtures come from tests/golden/reference_golden.json, extracted from
ThreeDGaussianSplatting.jl's test files by tests/golden/extract_golden.py. Tolerances are the
reference's own: atol 1e-3 on rendered pixels (test/forward_core.jl:122-141), rtol 1e-2 (atol
1e-3 where the golden value is zero) on gradients (test/backward_core.jl:178-185), exact on
integer/index data.
"""
import math

import numpy as np
import pytest

from gs3d import RenderOptions, Tiling
from gs3d.scene import create_test_scene
from oracle import oracle as O


def _scene(deg):
    gv, cams = create_test_scene(deg)
    cam = cams[0]
    return O.NpGaussians.from_vector(gv), cam, RenderOptions.for_camera(cam, deg), Tiling.for_camera(cam, 16, 16)


# ---- exp / log of the oracle (published-method implementations) -----------------------
def _ulp_err(got, want):
    want32 = np.float32(want)
    spacing = np.spacing(np.abs(want32)) if want32 != 0 else np.float32(1e-45)
    return abs(float(got) - want) / float(spacing)


def test_oracle_exp_log_accuracy():
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.uniform(-87, 88, 2000), rng.uniform(-8, 1, 2000), [0.0, -1e-8, 1e-8]])
    worst = max(_ulp_err(O.expf(float(np.float32(x))), math.exp(float(np.float32(x)))) for x in xs)
    assert worst <= 2.0, worst
    ys = np.concatenate([10 ** rng.uniform(-37, 38, 2000), rng.uniform(0.5, 2, 2000), [1.0, 2.0]])
    worst = max(_ulp_err(O.logf(float(np.float32(y))), math.log(float(np.float32(y)))) for y in ys
                if abs(math.log(float(np.float32(y)))) > 1e-3)
    assert worst <= 2.0, worst
    assert O.expf(-200.0) == 0.0 and math.isinf(O.expf(100.0)) and math.isnan(O.expf(float("nan")))
    assert O.logf(0.0) == -math.inf and math.isnan(O.logf(-1.0))


# ---- RenderHelpers (test/forward_core.jl:1-76) ------------------------------------------
def test_render_helpers_golden(golden):
    fc = golden["forward_core"]
    keep = np.array(fc["keep_gaussians"], np.uint8)
    cs, f2g = O.compact(keep)
    assert cs[-1] == keep.sum() == 3
    assert f2g.tolist() == [int(x) for x in fc["fgidx_to_gidx"]]
    ntiles = np.array(fc["nb_overlapped_tiles"], np.int32)
    ranges = np.array(fc["intersected_tile_ranges"], np.int32).reshape(-1, 4)
    depths = np.array(fc["depths"], np.float32)
    tiling = Tiling.create(2, 2, 1, 1)
    codes, dfg = O.dup_keys(ntiles, ranges, depths, tiling.nb_tiles_x)
    assert dfg.tolist() == [int(x) for x in fc["dfgidx_to_fgidx"]]
    assert tiling.highest_key_bit == 35
    scodes, sfg = O.sort_pairs(codes, dfg, tiling.highest_key_bit)
    assert sfg.tolist() == [int(x) for x in fc["sdfgidx_to_fgidx"]]
    assert O.tiles_end(scodes, tiling.nb_tiles).tolist() == [int(x) for x in fc["tiles_end_sdfgidx"]]


# ---- RenderConsistency golden pixels (test/forward_core.jl:143-164) ----------------------
@pytest.mark.parametrize("deg", [0, 3])
def test_render_golden_pixels(golden, deg):
    g, cam, opt, til = _scene(deg)
    r = O.render(g, cam, til, opt)
    assert r["F"] == 3  # the white Gaussian is behind the camera
    for px in golden["forward_core"]["rgb_pixels"][str(deg)]:
        got = r["rgb"][px["u"] - 1, px["v"] - 1]
        np.testing.assert_allclose(got, px["rgb"], atol=1e-3)


@pytest.mark.parametrize("deg", [0, 1, 2, 3])
def test_cpu_render_matches_gpu_path(deg):
    """The reference's CPU/GPU consistency test (test/forward_core.jl:78-141), here between the
    two oracle restatements: same pixels at atol 1e-3, and the empty pixels coincide."""
    g, cam, opt, til = _scene(deg)
    r = O.render(g, cam, til, opt)
    c = O.cpu_render(g, cam, opt)
    np.testing.assert_allclose(r["rgb"], c["rgb"], atol=1e-3)
    np.testing.assert_allclose(r["trans"], c["trans"], atol=1e-3)
    np.testing.assert_allclose(r["depth"], c["depth"], atol=1e-3)
    assert r["last"][0, 0] == 0
    assert np.array_equal(r["last"] == 0, r["trans"] == 1.0)
    c4 = O.cpu_render(g, cam, opt, nthreads=4)
    assert np.array_equal(c4["rgb"], c["rgb"])


# ---- BackwardConsistency (test/backward_core.jl) ------------------------------------------
def _approx(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    if np.all(b == 0):
        return np.allclose(a, b, atol=1e-3)
    return np.allclose(a, b, rtol=1e-2, atol=0)


@pytest.mark.parametrize("deg", [0, 3])
@pytest.mark.parametrize("flags", [0, 1])
def test_backward_golden(golden, deg, flags):
    g, cam, opt, til = _scene(deg)
    r = O.render(g, cam, til, opt)
    N = r["rgb"].size
    grad = (np.where(r["rgb"] > golden["backward_core"]["gt_gray"], 1.0, -1.0) / N).astype(np.float32)
    b = O.backward(g, cam, til, opt, r, grad, flags=flags)
    ref = golden["backward_core"]["gradients"][str(deg)]
    order = (deg + 1) ** 2
    for i in range(3):
        assert _approx(b["mean2d"][i], ref["means2d"][i])
        assert _approx(b["opacity_feature"][i], ref["opacity_features"][i])
        assert _approx(b["scaling"][i], ref["scaling_features"][i])
        assert _approx(b["rotation"][i], ref["rotation_features"][i])
        # reference SH literal is (order x 3), row-major in the text; ours is (3, order)
        sh_ref = np.array(ref["sh_coeffs"][i]).reshape(order, 3).T
        assert _approx(b["sh"][i], sh_ref)
        # the reference leaves its mean3d check commented out; the original 3DGS values agree
        assert _approx(b["mean3d"][i], ref["means3d"][i])


def test_sort_pairs_stable_and_masked():
    rng = np.random.default_rng(3)
    keys = rng.integers(0, 1 << 40, 5000, dtype=np.int64) | (rng.integers(0, 4, 5000, dtype=np.int64) << 50)
    vals = np.arange(5000, dtype=np.int32)
    ko, vo = O.sort_pairs(keys, vals, 36)
    masked = keys & ((1 << 36) - 1)
    order = np.argsort(masked, kind="stable")
    assert np.array_equal(vo, vals[order]) and np.array_equal(ko, keys[order])


def test_oracle_work_counts_match_a_direct_loop():
    """oracle_work_counts (the bench's roofline numerators) against a plain Python walk of the
    reference's blend loop (forward_core.jl:928-968) over the same render, on a small scene."""
    from gs3d.scene import SceneSpec, look_at_camera, synthetic_gaussians
    gv = synthetic_gaussians(SceneSpec(300, "uniform:1", -3.0, 0.5), 3)
    cam = look_at_camera(48, 40, 60.0, (0, 0, 3))
    opt = RenderOptions.for_camera(cam, 3)
    til = Tiling.for_camera(cam, 16, 8)
    f = O.render(O.NpGaussians.from_vector(gv), cam, til, opt)
    f32 = np.float32
    blends = contrib = 0
    for ty in range(til.nb_tiles_y):
        for tx in range(til.nb_tiles_x):
            tile = tx + ty * til.nb_tiles_x + 1
            start = 0 if tile == 1 else int(f["tiles_end"][tile - 2])
            end = int(f["tiles_end"][tile - 1])
            u0, v0 = tx * til.tile_width, ty * til.tile_height
            for pv in range(1, til.tile_height + 1):
                for pu in range(1, til.tile_width + 1):
                    if pu + u0 > cam.width or pv + v0 > cam.height:
                        continue
                    cu, cv = f32(pu) - f32(0.5), f32(pv) - f32(0.5)
                    T = f32(1)
                    for s in range(start, end):
                        r = f["f2d"][f["sfg"][s] - 1]
                        du, dv = r[0] - f32(u0), r[1] - f32(v0)
                        p4 = r[3] * du + r[4] * dv
                        p5 = r[4] * du + r[5] * dv
                        p6 = (f32(-0.5) * (r[3] * du * du + r[5] * dv * dv) - r[4] * du * dv
                              + f32(O.logf(float(r[2]))))
                        q = (f32(-0.5) * r[3] * (cu * cu) + f32(-0.5) * r[5] * (cv * cv)
                             - r[4] * (cu * cv) + p4 * cu + p5 * cv + p6)
                        blends += 1
                        alpha = min(f32(opt.max_alpha), f32(O.expf(float(q))))
                        if alpha < f32(opt.min_alpha):
                            continue
                        nT = T * (f32(1) - alpha)
                        if nT < f32(opt.min_transmittance):
                            break
                        T = nT
                        contrib += 1
    assert O.work_counts(f, cam, til, opt) == (blends, contrib)
    assert contrib > 0 and blends > contrib
