"""backward! and update! on the GPU against the CPU oracle.

Bar: per-Gaussian gradients within 1e-3 relative L2 of the oracle (whose per-pair sums are
exact doubles; the GPU sums float atomics in a different order), the reference's golden
gradients at its own tolerance, and the Adam step bit-exact given identical gradients.
"""
import numpy as np
import pytest
import torch

import gs3d
from gs3d import RenderBuffers, RenderOptions, RenderOutputs, Tiling
from gs3d.backward import FilteredGaussiansGradients, backward
from gs3d.optimizer import AdamOptimizer, LearningRates, bias_corrections
from gs3d.scene import SceneSpec, create_test_scene, look_at_camera, synthetic_gaussians
from oracle import oracle as O

pytestmark = pytest.mark.gpu

KEYS = ["mean2d", "opacity", "licov", "color", "mean3d", "opacity_feature", "scaling", "rotation", "sh"]


def run_gpu(gv, cam, til, opt, rgb_grad, device, fix16=False, masks=True, tile_order=True):
    """masks: the forward writes contribution masks and the backward blend walks them
    (k_bwd_raster_masks); without, the backward blend tests every entry (k_bwd_raster).
    tile_order: both blends take the tiles longest first; without, in row-major order."""
    g = gv.to(device)
    out = RenderOutputs.create(cam.width, cam.height, device)
    buf = RenderBuffers.create(g.n, til.nb_tiles, device, mask_dup=-1 if masks else None,
                               tile_order=tile_order)
    gs3d.render(out, g, cam, til, opt, buf)
    assert int(buf.device_counts[3]) == (1 if masks else 0)
    fg = FilteredGaussiansGradients.create(g.n, g.sh_degree, device)
    backward(fg, torch.from_numpy(rgb_grad).to(device), out, g, cam, til, opt, buf, fix_sh16=fix16)
    torch.cuda.synchronize()
    F, _ = gs3d.counts(buf)
    cpu = lambda t: t[:F].cpu().numpy()
    grads = dict(mean2d=cpu(fg.mean2d_grads), opacity=cpu(fg.opacity_grads),
                 licov=cpu(fg.licov2d_grads), color=cpu(fg.color_grads),
                 mean3d=cpu(fg.mean3d_grads), opacity_feature=cpu(fg.opacity_feature_grads),
                 scaling=cpu(fg.scaling_features_grads), rotation=cpu(fg.rotation_features_grads),
                 sh=cpu(fg.sh_coeffs_grads))
    return grads, (g, out, buf, fg)


def rel_l2(a, b):
    a = np.asarray(a, np.float64).reshape(len(a), -1)
    b = np.asarray(b, np.float64).reshape(len(b), -1)
    total = np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)
    per = np.linalg.norm(a - b, axis=1) / np.maximum(np.linalg.norm(b, axis=1), 1e-30)
    return total, per


def check_grads(gpu, ref, tol=1e-3, every_gaussian=True):
    """Each gradient array within `tol` relative L2 of the oracle's; per Gaussian, at least
    99.9% within `tol` and (every_gaussian) all within the reference test's rtol 1e-2. The GPU
    sums the per-pixel contributions with float atomics (as the reference does), so a Gaussian
    whose contributions cancel can carry a larger relative error than the array as a whole; the
    oracle sums in double. Scenes with millions of Gaussians check the individual Gaussians
    against the size of their terms instead (check_grads_2d_terms)."""
    for k in KEYS:
        total, per = rel_l2(gpu[k], ref[k])
        assert total <= tol, (k, total)
        norms = np.linalg.norm(np.asarray(ref[k], np.float64).reshape(len(per), -1), axis=1)
        big = norms > 1e-3 * norms.max()
        bad = np.count_nonzero(per[big] > tol)
        assert bad <= max(1, 1e-3 * np.count_nonzero(big)), (k, per[big].max(), bad)
        if every_gaussian:
            assert np.all(per[big] <= 1e-2), (k, per[big].max())


KEYS_2D = [("mean2d", 0, 2), ("opacity", 2, 3), ("licov", 3, 6), ("color", 6, 9)]


def check_grads_2d_terms(gpu, ref, mag, rel=1e-3, cancel=1e-3):
    """Every Gaussian's 2D gradients (the float-atomic sums) against the oracle's double sums:
    |gpu - ref| <= rel |ref| + cancel * mag, componentwise, with mag the oracle's sum of the
    per-pixel terms evaluated on absolute values (O.backward(with_magnitudes=True)). The second
    term bounds what float arithmetic can lose where values cancel: in the sum over pixels (any
    order) and inside each term (the colour difference T c - (colour behind) of
    backward_core.jl:253-262 cancels where a Gaussian matches what lies behind it)."""
    for k, lo, hi in KEYS_2D:
        g = np.asarray(gpu[k], np.float64).reshape(len(mag), -1)
        r = np.asarray(ref[k], np.float64).reshape(len(mag), -1)
        m = np.asarray(mag, np.float64)[:, lo:hi]
        err = np.abs(g - r)
        bound = rel * np.abs(r) + cancel * m
        worst = np.argmax(err - bound)
        assert np.all(err <= bound), (k, np.count_nonzero(err > bound), err.ravel()[worst],
                                      bound.ravel()[worst])


@pytest.mark.parametrize("deg", [0, 3])
def test_backward_test_scene_golden(cuda, golden, deg):
    gv, cams = create_test_scene(deg)
    cam = cams[0]
    opt = RenderOptions.for_camera(cam, deg)
    til = Tiling.for_camera(cam, 16, 16)
    ref_f = O.render(O.NpGaussians.from_vector(gv), cam, til, opt)
    N = ref_f["rgb"].size
    grad = (np.where(ref_f["rgb"] > 0.5, 1.0, -1.0) / N).astype(np.float32)
    gpu, _ = run_gpu(gv, cam, til, opt, grad, cuda)
    ref = O.backward(O.NpGaussians.from_vector(gv), cam, til, opt, ref_f, grad)
    check_grads(gpu, ref)
    gold = golden["backward_core"]["gradients"][str(deg)]
    order = (deg + 1) ** 2
    for i in range(3):
        for mine, theirs in ((gpu["mean2d"][i], gold["means2d"][i]),
                             (gpu["scaling"][i], gold["scaling_features"][i]),
                             (gpu["opacity_feature"][i], gold["opacity_features"][i]),
                             (gpu["sh"][i], np.array(gold["sh_coeffs"][i]).reshape(order, 3).T)):
            theirs = np.asarray(theirs, np.float64)
            if np.all(theirs == 0):
                assert np.allclose(mine, theirs, atol=1e-3)
            else:
                assert np.allclose(mine, theirs, rtol=1e-2, atol=0)


CASES = [
    ("cfg0", SceneSpec(16_384, "uniform:1", -4.0, 0.5), 0, (256, 256, 60.0, (0, 0, 3)), None, {}, 3),
    ("aa_bg", SceneSpec(16_384, "uniform:1", -4.0, 0.5), 5, (256, 256, 60.0, (0.3, 0.2, 2.5)), None,
     dict(use_antialiasing=True, background=(0.2, 0.5, 0.9)), 3),
    ("filter", SceneSpec(16_384, "uniform:1", -4.0, 0.5), 11, (256, 192, 60.0, (0, 0, 2.5)), None,
     dict(clipping_mode=gs3d.FILTER), 2),
    ("deg1_of3", SceneSpec(20_000, "uniform:1.5", -4.5, 0.5), 6, (320, 200, 70.0, (0, 1, 3)), None, {}, 1),
    ("p720", SceneSpec(40_000, "uniform:3", -4.0, 0.6), 7, (1280, 720, 50.0, (0, 1.5, 6)), None, {}, 3),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("fix16, masks, tile_order",
                         [(False, True, True), (True, True, True), (False, False, True), (False, True, False)],
                         ids=["masks", "masks_fix16", "no_masks", "masks_row_major"])
def test_backward_random(cuda, case, fix16, masks, tile_order):
    _, spec, seed, (w, h, fov, pos), tile, kw, deg = case
    gv = synthetic_gaussians(spec, seed)
    cam = look_at_camera(w, h, fov, pos)
    opt = RenderOptions.for_camera(cam, deg, **kw)
    til = Tiling.for_camera(cam, *(tile or (None, None)))
    rng = np.random.default_rng(seed)
    grad = rng.normal(0, 1e-5, size=(w, h, 3)).astype(np.float32)
    gpu, _ = run_gpu(gv, cam, til, opt, grad, cuda, fix16, masks, tile_order)
    g = O.NpGaussians.from_vector(gv)
    ref_f = O.render(g, cam, til, opt)
    ref = O.backward(g, cam, til, opt, ref_f, grad, flags=1 if fix16 else 0)
    check_grads(gpu, ref)


@pytest.mark.parametrize("deg", [0, 1, 2, 3])
def test_adam_bit_exact(cuda, deg):
    """Storage degree 3 with render degree deg: coefficients >= (deg + 1)^2 stay untouched."""
    spec = SceneSpec(16_384, "uniform:1", -4.0, 0.5)
    gv = synthetic_gaussians(spec, 0)
    cam = look_at_camera(256, 256, 60.0, (0, 0, 3))
    opt = RenderOptions.for_camera(cam, 3)
    til = Tiling.for_camera(cam)
    grad = np.random.default_rng(1).normal(0, 1e-4, size=(256, 256, 3)).astype(np.float32)
    gpu, (g, out, buf, fg) = run_gpu(gv, cam, til, opt, grad, cuda)
    F, _ = gs3d.counts(buf)
    # skip some filtered Gaussians, as ADC does (fgidx_to_gidx <= 0)
    buf.fgidx_to_gidx[: F : 7] = 0
    adam = AdamOptimizer(g, LearningRates(means=0.00016 * 3.3))
    rng = np.random.default_rng(2)
    for t in adam.moments.tensors():
        t.copy_(torch.from_numpy(np.abs(rng.normal(0, 1e-4, size=tuple(t.shape))).astype(np.float32)))
    adam.update_count = 5
    before_g = O.NpGaussians.from_vector(g)
    before_m = O.NpMoments.from_moments(adam.moments)
    params = adam.params_c(deg)
    adam.update(fg, buf.fgidx_to_gidx, buf.device_counts, deg)
    torch.cuda.synchronize()
    bc1, bc2 = bias_corrections(adam.beta1, adam.beta2, 5)
    O.adam(before_g, before_m, gpu, buf.fgidx_to_gidx[:F].cpu().numpy(), params, bc1, bc2)
    after_g = O.NpGaussians.from_vector(g)
    after_m = O.NpMoments.from_moments(adam.moments)
    for a, b in zip((after_g.mo, after_g.sf, after_g.rf, after_g.sh),
                    (before_g.mo, before_g.sf, before_g.rf, before_g.sh)):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    for a, b in zip((after_m.mm, after_m.om, after_m.sm, after_m.rm, after_m.shm),
                    (before_m.mm, before_m.om, before_m.sm, before_m.rm, before_m.shm)):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert adam.update_count == 6


def test_dense_adam_equals_sparse_adam(cuda):
    """One view: scatter + dense Adam (the data-parallel path) == the sparse update! bit for bit."""
    import ctypes as C
    from gs3d import _abi
    spec = SceneSpec(16_384, "uniform:1", -4.0, 0.5)
    gv = synthetic_gaussians(spec, 0)
    cam = look_at_camera(256, 256, 60.0, (0, 0, 3))
    opt = RenderOptions.for_camera(cam, 3)
    til = Tiling.for_camera(cam)
    grad = np.random.default_rng(1).normal(0, 1e-4, size=(256, 256, 3)).astype(np.float32)
    _, (g, out, buf, fg) = run_gpu(gv, cam, til, opt, grad, cuda)
    F, _ = gs3d.counts(buf)
    buf.fgidx_to_gidx[: F : 5] = 0
    g2 = g.clone()
    a1 = AdamOptimizer(g, LearningRates(means=0.001))
    a2 = AdamOptimizer(g2, LearningRates(means=0.001))
    a1.update(fg, buf.fgidx_to_gidx, buf.device_counts, 3)
    dense = torch.empty((g2.n, 60), dtype=torch.float32, device=cuda)
    lib = _abi.lib()
    fc = fg.to_c()
    _abi.check(lib.gs3d_scatter_dense_grads(C.byref(fc), C.c_void_p(buf.fgidx_to_gidx.data_ptr()),
                                            C.c_void_p(buf.device_counts.data_ptr()), 3,
                                            C.c_void_p(dense.data_ptr()), g2.n, None))
    gc, mc, pc = g2.to_c(), a2.moments.to_c(), a2.params_c(3)
    _abi.check(lib.gs3d_adam_step_dense(C.byref(gc), C.byref(mc), C.c_void_p(dense.data_ptr()),
                                        C.byref(pc), None))
    torch.cuda.synchronize()
    for x, y in zip(g.tensors(), g2.tensors()):
        assert torch.equal(x, y)
    for x, y in zip(a1.moments.tensors(), a2.moments.tensors()):
        assert torch.equal(x, y)


def test_adam_reference_golden(cuda, golden):
    """test/training.jl:181-257: beta1 = beta2 = 0.5, eps = 0, lr 1 (SH rest 10), t = 1,
    parameters and moments of Gaussian k equal to k, gradients of filtered index k equal to k."""
    tr = golden["training"]
    n = 10
    d = 1
    f32 = dict(dtype=torch.float32, device=cuda)
    # state after the reference's ADC step: Gaussian i holds the value of the old Gaussian it
    # came from (ngidx_to_gidx), moments as the reference asserts them (zeros for splits and
    # second clones)
    k = torch.tensor(tr["ngidx_to_gidx"], **f32)
    km = torch.tensor(tr["moments_after_adc"], **f32)
    g = gs3d.GaussiansVector(k[:, None].repeat(1, 4).contiguous(), k[:, None].repeat(1, 3).contiguous(),
                             k[:, None].repeat(1, 4).contiguous(),
                             k[:, None, None].repeat(1, 3, (d + 1) ** 2).contiguous())
    adam = AdamOptimizer(g, LearningRates(1.0, 1.0, 1.0, 1.0, 1.0, 10.0), beta1=0.5, beta2=0.5, epsilon=0.0)
    for t in adam.moments.tensors():
        t.copy_(km.view(-1, *([1] * (t.dim() - 1))).expand_as(t))
    before = g.means_opacity_features.clone()
    f2g = torch.tensor([int(x) for x in tr["adjusted_fgidx_to_gidx"]], dtype=torch.int32, device=cuda)
    F = f2g.numel()
    fg = FilteredGaussiansGradients.create(F, d, cuda)
    kf = torch.arange(1, F + 1, **f32)
    fg.mean3d_grads.copy_(kf[:, None].expand(F, 3))
    fg.opacity_feature_grads.copy_(kf)
    fg.scaling_features_grads.copy_(kf[:, None].expand(F, 3))
    fg.rotation_features_grads.copy_(kf[:, None].expand(F, 4))
    fg.sh_coeffs_grads.copy_(kf[:, None, None].expand(F, 3, 4))
    counts = torch.tensor([F, 0, 0, 0], dtype=torch.int32, device=cuda)
    adam.update(fg, f2g, counts, d)
    torch.cuda.synchronize()

    def expect(gidx, fgidx, lr=1.0):
        m1h, m2h = gidx + fgidx, gidx + fgidx ** 2
        return gidx - lr * m1h / np.sqrt(m2h), m1h / 2, m2h / 2

    for ngidx, gidx, fgidx in tr["adam"]["checked"]:
        i = ngidx - 1
        p, m, v = expect(gidx, fgidx)
        assert np.allclose(g.means_opacity_features[i].cpu().numpy(), p, rtol=1e-6)
        assert np.allclose(adam.moments.means_moments[i].cpu().numpy(), np.array([[m, v]] * 3), rtol=1e-6)
        assert np.allclose(adam.moments.opacity_features_moments[i].cpu().numpy(), [m, v], rtol=1e-6)
        assert np.allclose(g.scaling_features[i].cpu().numpy(), p, rtol=1e-6)
        assert np.allclose(g.rotation_features[i].cpu().numpy(), p, rtol=1e-6)
        assert np.allclose(g.sh_coeffs[i, :, 0].cpu().numpy(), p, rtol=1e-6)
        pr, mr, vr = expect(gidx, fgidx, 10.0)
        assert np.allclose(g.sh_coeffs[i, :, 1:].cpu().numpy(), pr, rtol=1e-6)
        assert np.allclose(adam.moments.sh_coeffs_moments[i, :, 1:].cpu().numpy()[..., 0], mr, rtol=1e-6)
    for i in [int(x) for x in tr["splits_second_copies_ids"]]:
        assert torch.equal(g.means_opacity_features[i - 1], before[i - 1])


def _scatter_rows(fg, buf, n, deg, device):
    import ctypes as C
    from gs3d import _abi
    dense = torch.empty((n, 60), dtype=torch.float32, device=device)
    fc = fg.to_c()
    _abi.check(_abi.lib().gs3d_scatter_dense_grads(
        C.byref(fc), C.c_void_p(buf.fgidx_to_gidx.data_ptr()), C.c_void_p(buf.device_counts.data_ptr()),
        deg, C.c_void_p(dense.data_ptr()), n, None))
    return dense


@pytest.mark.parametrize("deg", [1, 3])
def test_backward_dense_rows_match_scattered_gradients(cuda, deg):
    """gs3d_backward_dense writes each filtered Gaussian's 3D gradients into its dense row (and
    the touched flag); scattering gs3d_backward's F-compact gradients gives the same rows (the
    float-atomic 2D sums differ in the last bits between the two runs)."""
    from gs3d.backward import backward_dense
    spec = SceneSpec(16_384, "uniform:1", -4.0, 0.5)
    gv = synthetic_gaussians(spec, 4)
    cam = look_at_camera(256, 256, 60.0, (0, 0, 3))
    opt = RenderOptions.for_camera(cam, deg)
    til = Tiling.for_camera(cam)
    grad = np.random.default_rng(3).normal(0, 1e-4, size=(256, 256, 3)).astype(np.float32)
    _, (g, out, buf, fg) = run_gpu(gv, cam, til, opt, grad, cuda)
    want = _scatter_rows(fg, buf, g.n, deg, cuda)
    dense = torch.full((g.n + 5, 60), 7.0, dtype=torch.float32, device=cuda)  # zeroed by the call
    backward_dense(fg, torch.from_numpy(grad).to(cuda), out, g, cam, til, opt, buf, dense)
    torch.cuda.synchronize()
    got = dense[: g.n]
    assert torch.equal(got[:, 59], want[:, 59]) and torch.all(dense[g.n:] == 0)
    d = (got - want).abs()
    assert d.max() <= 1e-5 * want.abs().max() + 1e-12, d.max()
    assert torch.linalg.norm(got - want) <= 1e-5 * torch.linalg.norm(want)


def test_dense_adam_range_split_equals_full(cuda):
    """Two calls over [0, k) and [k, n) with the matching row slices == one call over [0, n)."""
    import ctypes as C
    from gs3d import _abi
    spec = SceneSpec(16_384, "uniform:1", -4.0, 0.5)
    gv = synthetic_gaussians(spec, 0)
    cam = look_at_camera(256, 256, 60.0, (0, 0, 3))
    opt = RenderOptions.for_camera(cam, 3)
    til = Tiling.for_camera(cam)
    grad = np.random.default_rng(1).normal(0, 1e-4, size=(256, 256, 3)).astype(np.float32)
    _, (g, out, buf, fg) = run_gpu(gv, cam, til, opt, grad, cuda)
    dense = _scatter_rows(fg, buf, g.n, 3, cuda)
    g2 = g.clone()
    a1 = AdamOptimizer(g, LearningRates(means=0.001))
    a2 = AdamOptimizer(g2, LearningRates(means=0.001))
    lib = _abi.lib()
    gc, mc, pc = g.to_c(), a1.moments.to_c(), a1.params_c(3)
    _abi.check(lib.gs3d_adam_step_dense(C.byref(gc), C.byref(mc), C.c_void_p(dense.data_ptr()),
                                        C.byref(pc), None))
    gc2, mc2, pc2 = g2.to_c(), a2.moments.to_c(), a2.params_c(3)
    k = 5001
    for lo, hi in ((0, k), (k, g2.n)):
        part = dense[lo:hi].contiguous()
        _abi.check(lib.gs3d_adam_step_dense_range(C.byref(gc2), C.byref(mc2), C.c_void_p(part.data_ptr()),
                                                  lo, hi, C.byref(pc2), None))
    torch.cuda.synchronize()
    for x, y in zip(g.tensors(), g2.tensors()):
        assert torch.equal(x, y)
    for x, y in zip(a1.moments.tensors(), a2.moments.tensors()):
        assert torch.equal(x, y)


def test_dense_adam_equals_sparse_adam_storage_degree_1(cuda):
    """The generic dense kernel (storage degree below 3) against the sparse update!, bit for bit."""
    import ctypes as C
    from gs3d import _abi
    spec = SceneSpec(16_384, "uniform:1", -4.0, 0.5, sh_degree=1)
    gv = synthetic_gaussians(spec, 2)
    cam = look_at_camera(256, 256, 60.0, (0, 0, 3))
    opt = RenderOptions.for_camera(cam, 1)
    til = Tiling.for_camera(cam)
    grad = np.random.default_rng(5).normal(0, 1e-4, size=(256, 256, 3)).astype(np.float32)
    _, (g, out, buf, fg) = run_gpu(gv, cam, til, opt, grad, cuda)
    dense = _scatter_rows(fg, buf, g.n, 1, cuda)
    g2 = g.clone()
    a1 = AdamOptimizer(g, LearningRates(means=0.001))
    a2 = AdamOptimizer(g2, LearningRates(means=0.001))
    a1.update(fg, buf.fgidx_to_gidx, buf.device_counts, 1)
    gc, mc, pc = g2.to_c(), a2.moments.to_c(), a2.params_c(1)
    _abi.check(_abi.lib().gs3d_adam_step_dense(C.byref(gc), C.byref(mc), C.c_void_p(dense.data_ptr()),
                                               C.byref(pc), None))
    torch.cuda.synchronize()
    for x, y in zip(g.tensors(), g2.tensors()):
        assert torch.equal(x, y)
    for x, y in zip(a1.moments.tensors(), a2.moments.tensors()):
        assert torch.equal(x, y)


def test_factored_rows_rebuild_dense_rows_over_views(cuda):
    """Three views of one scene. Per view, the factored rows (gs3d_backward_project_factored)
    hold the dense rows' geometry part bit for bit and the colour gradients with their live
    flags; the update from the views' summed geometry rows and their colour rows
    (gs3d_adam_step_factored_range, SH gradients rebuilt from the camera positions) equals the
    dense update from the summed dense rows, bit for bit, over two Gaussian ranges."""
    import ctypes as C
    from gs3d import _abi
    from gs3d.backward import backward_project_dense, backward_project_factored, backward_raster
    spec = SceneSpec(16_384, "uniform:1", -4.0, 0.5)
    g = synthetic_gaussians(spec, 5).to(cuda)
    n = g.n
    k = 6007
    dsum = gsum = None
    colours = []
    positions = []
    for v, pos in enumerate([(0, 0, 3), (2.0, 0.5, 2.2), (-1.5, 1.0, 2.5)]):
        cam = look_at_camera(256, 256, 60.0, pos)
        opt = RenderOptions.for_camera(cam, 3)
        til = Tiling.for_camera(cam)
        out = RenderOutputs.create(cam.width, cam.height, cuda)
        buf = RenderBuffers.create(n, til.nb_tiles, cuda)
        gs3d.render(out, g, cam, til, opt, buf)
        fg = FilteredGaussiansGradients.create(n, 3, cuda)
        grad = np.random.default_rng(10 + v).normal(0, 1e-4, size=(256, 256, 3)).astype(np.float32)
        backward_raster(fg, torch.from_numpy(grad).to(cuda), out, g, cam, til, opt, buf)
        dense = torch.zeros((n, 60), dtype=torch.float32, device=cuda)
        geom = torch.zeros((n, 12), dtype=torch.float32, device=cuda)
        colour = torch.zeros((n, 4), dtype=torch.float32, device=cuda)
        for lo, hi in ((0, k), (k, n)):
            backward_project_dense(fg, g, cam, til, opt, buf, dense[lo:], lo, hi)
            backward_project_factored(fg, g, cam, til, opt, buf, geom[lo:], colour[lo:], lo, hi)
        torch.cuda.synchronize()
        assert torch.equal(geom, dense[:, 48:60])
        touched = dense[:, 59] > 0
        assert int(touched.sum()) > n // 4
        assert torch.equal(colour[:, 3] > 0, touched)
        fl = colour[touched, 3].to(torch.int32)
        assert torch.all((fl & 1) == 1) and torch.all(fl <= 127)
        # positive colour implies live (colour >= 0)
        assert torch.all(((fl >> 4) & ~(fl >> 1) & 7) == 0)
        # a colour row reproduces its dense row's SH gradients: cg * basis(k = 1) on live channels
        c0 = (float(np.float32(0.28209479177387814)) * colour[touched, :3].double()).float()
        live = torch.stack([(fl >> (1 + c)) & 1 for c in range(3)], 1).bool()
        assert torch.equal(torch.where(live, c0, torch.zeros_like(c0)), dense[touched][:, [0, 16, 32]])
        dsum = dense if dsum is None else dsum + dense
        gsum = geom if gsum is None else gsum + geom
        colours.append(colour)
        positions.append(cam.position)
    g2 = g.clone()
    a1 = AdamOptimizer(g, LearningRates(means=0.001))
    a2 = AdamOptimizer(g2, LearningRates(means=0.001))
    a1.update_count = a2.update_count = 4
    lib = _abi.lib()
    gc, mc, pc = g.to_c(), a1.moments.to_c(), a1.params_c(3)
    _abi.check(lib.gs3d_adam_step_dense(C.byref(gc), C.byref(mc), C.c_void_p(dsum.data_ptr()),
                                        C.byref(pc), None))
    views = torch.stack(colours).contiguous()  # (3, n, 4): view stride n rows
    pos = np.ascontiguousarray(np.stack(positions).astype(np.float32))
    gc2, mc2, pc2 = g2.to_c(), a2.moments.to_c(), a2.params_c(3)
    for lo, hi in ((0, k), (k, n)):
        vpart = views[:, lo:hi].contiguous()
        _abi.check(lib.gs3d_adam_step_factored_range(
            C.byref(gc2), C.byref(mc2), C.c_void_p(gsum[lo:].data_ptr()), C.c_void_p(vpart.data_ptr()),
            3, hi - lo, pos.ctypes.data_as(C.POINTER(C.c_float)), lo, hi, C.byref(pc2), None))
    torch.cuda.synchronize()
    for x, y in zip(g.tensors(), g2.tensors()):
        assert torch.equal(x, y)
    for x, y in zip(a1.moments.tensors(), a2.moments.tensors()):
        assert torch.equal(x, y)


@pytest.mark.parametrize("deg, fix16", [(3, False), (3, True), (2, False), (0, False)])
def test_owner_colour_direction_rows(cuda, deg, fix16):
    """shard_sh's split of the mean gradient: gs3d_backward_project_factored with
    GS3D_BACKWARD_NO_COLOUR_DIRECTION leaves the colour -> direction term out (the colour rows
    and the other geometry columns unchanged), and gs3d_factored_colour_direction_range adds it
    back: with one view the rows equal the full projection backward's bit for bit (render degree
    `deg`, storage degree 3, two Gaussian ranges); over three views accumulated, the non-mean
    columns are equal and the means within float rounding of the per-view sums."""
    from gs3d.backward import backward_project_factored, backward_raster, colour_direction_rows
    spec = SceneSpec(16_384, "uniform:1", -4.0, 0.5)
    g = synthetic_gaussians(spec, 5).to(cuda)
    n = g.n
    k = 6007
    f32 = dict(dtype=torch.float32, device=cuda)
    acc_full = torch.zeros((n, 12), **f32)
    acc_own = torch.zeros((n, 12), **f32)
    colours = torch.zeros((3, n, 4), **f32)
    positions = []
    for v, pos in enumerate([(0, 0, 3), (2.0, 0.5, 2.2), (-1.5, 1.0, 2.5)]):
        cam = look_at_camera(256, 256, 60.0, pos)
        opt = RenderOptions.for_camera(cam, deg)
        til = Tiling.for_camera(cam)
        out = RenderOutputs.create(cam.width, cam.height, cuda)
        buf = RenderBuffers.create(n, til.nb_tiles, cuda)
        gs3d.render(out, g, cam, til, opt, buf)
        fg = FilteredGaussiansGradients.create(n, 3, cuda)
        grad = np.random.default_rng(20 + v).normal(0, 1e-4, size=(256, 256, 3)).astype(np.float32)
        backward_raster(fg, torch.from_numpy(grad).to(cuda), out, g, cam, til, opt, buf)
        full = torch.zeros((n, 12), **f32)
        own = torch.zeros((n, 12), **f32)
        col_full = torch.zeros((n, 4), **f32)
        for lo, hi in ((0, k), (k, n)):
            backward_project_factored(fg, g, cam, til, opt, buf, full[lo:], col_full[lo:], lo, hi,
                                      fix_sh16=fix16)
            backward_project_factored(fg, g, cam, til, opt, buf, own[lo:], colours[v, lo:], lo, hi,
                                      fix_sh16=fix16, colour_direction=False)
            backward_project_factored(fg, g, cam, til, opt, buf, acc_full[lo:], col_full[lo:], lo, hi,
                                      fix_sh16=fix16, accumulate=True)
            backward_project_factored(fg, g, cam, til, opt, buf, acc_own[lo:], colours[v, lo:], lo, hi,
                                      fix_sh16=fix16, accumulate=True, colour_direction=False)
        p = np.array([cam.position], dtype=np.float32)
        positions.append(cam.position)
        torch.cuda.synchronize()
        assert torch.equal(colours[v], col_full)
        assert torch.equal(own[:, 3:], full[:, 3:])
        if deg > 0:
            assert not torch.equal(own[:, :3], full[:, :3])
        for lo, hi in ((0, k), (k, n)):
            colour_direction_rows(g, own[lo:], colours[v, lo:], 1, hi - lo, p, lo, hi, deg, fix16)
        torch.cuda.synchronize()
        assert torch.equal(own, full), v
    pos3 = np.array(positions, dtype=np.float32)
    # colour rows of the three views at rows v * n + g (view stride n)
    flat = colours.reshape(3 * n, 4)
    for lo, hi in ((0, k), (k, n)):
        colour_direction_rows(g, acc_own[lo:], flat[lo:], 3, n, pos3, lo, hi, deg, fix16)
    torch.cuda.synchronize()
    assert torch.equal(acc_own[:, 3:], acc_full[:, 3:])
    scale = acc_full[:, :3].abs().max()
    assert torch.allclose(acc_own[:, :3], acc_full[:, :3], rtol=1e-5, atol=1e-6 * float(scale))


def test_factored_adam_rejects_bad_arguments(cuda):
    import ctypes as C
    from gs3d import _abi
    g = synthetic_gaussians(SceneSpec(1024, "uniform:1", -4.0, 0.5), 0).to(cuda)
    a = AdamOptimizer(g, LearningRates(means=0.001))
    geom = torch.zeros((g.n, 12), dtype=torch.float32, device=cuda)
    col = torch.zeros((g.n, 4), dtype=torch.float32, device=cuda)
    pos = (C.c_float * 3)(0.0, 0.0, 3.0)
    gc, mc, pc = g.to_c(), a.moments.to_c(), a.params_c(3)
    lib = _abi.lib()
    call = lambda nv, stride, lo, hi: lib.gs3d_adam_step_factored_range(
        C.byref(gc), C.byref(mc), C.c_void_p(geom.data_ptr()), C.c_void_p(col.data_ptr()), nv, stride,
        pos, lo, hi, C.byref(pc), None)
    assert call(0, g.n, 0, g.n) == _abi.GS3D_ERR_INVALID_ARGUMENT
    assert call(_abi.GS3D_MAX_FACTORED_VIEWS + 1, g.n, 0, g.n) == _abi.GS3D_ERR_INVALID_ARGUMENT
    assert call(1, g.n - 1, 0, g.n) == _abi.GS3D_ERR_INVALID_ARGUMENT
    assert call(1, g.n, 0, g.n + 1) == _abi.GS3D_ERR_INVALID_ARGUMENT
    assert call(1, g.n, 0, g.n) == _abi.GS3D_OK
    torch.cuda.synchronize()


@pytest.mark.parametrize("deg", [0, 1, 2, 3])
def test_rebuilt_sh_update_equals_sparse_update(cuda, deg):
    """gs3d_backward with GS3D_BACKWARD_SKIP_SH_GRADS leaves the SH gradients untouched and
    gs3d_adam_step_rebuild_sh, recomputing them from the colour gradients, the projected colours
    and the camera position, gives gs3d_adam_step's update bit for bit (render degree `deg`,
    storage degree 3, some filtered Gaussians skipped)."""
    spec = SceneSpec(16_384, "uniform:1", -4.0, 0.5)
    gv = synthetic_gaussians(spec, 6)
    cam = look_at_camera(256, 256, 60.0, (0.4, -0.3, 3))
    opt = RenderOptions.for_camera(cam, deg)
    til = Tiling.for_camera(cam)
    grad = np.random.default_rng(7).normal(0, 1e-4, size=(256, 256, 3)).astype(np.float32)
    _, (g, out, buf, fg) = run_gpu(gv, cam, til, opt, grad, cuda)
    F, _ = gs3d.counts(buf)
    buf.fgidx_to_gidx[: F : 7] = 0
    fg2 = FilteredGaussiansGradients.create(g.n, 3, cuda)
    fg2.sh_coeffs_grads.fill_(3.0)
    backward(fg2, torch.from_numpy(grad).to(cuda), out, g, cam, til, opt, buf, skip_sh_grads=True)
    torch.cuda.synchronize()
    assert torch.all(fg2.sh_coeffs_grads == 3.0)
    g2 = g.clone()
    a1 = AdamOptimizer(g, LearningRates(means=0.001))
    a2 = AdamOptimizer(g2, LearningRates(means=0.001))
    a1.update_count = a2.update_count = 2
    a1.update(fg, buf.fgidx_to_gidx, buf.device_counts, deg)
    # the same colour gradients as the first backward (the 2D sums of the second run may differ
    # in the last bits): the rebuilt update reads fg
    a2.update_rebuild_sh(fg, buf.fgidx_to_gidx, buf.device_counts, buf.f2d, cam.position, deg)
    torch.cuda.synchronize()
    for x, y in zip(g.tensors(), g2.tensors()):
        assert torch.equal(x, y)
    for x, y in zip(a1.moments.tensors(), a2.moments.tensors()):
        assert torch.equal(x, y)
