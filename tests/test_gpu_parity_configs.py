"""The CUDA path against the CPU oracle at the full sizes of the BASELINE configurations:

* config 4, the bench workload (3M Gaussians, 1920x1080, 16x32 tiles, 44 key bits), hemisphere
  cameras 0 and 131: one training step (render, L1 + DSSIM loss, backward, Adam);
* config 1 (500K Gaussians, 1280x720, ring camera 0): one training step;
* config 3 (6M Gaussians, 3840x2160, 16,320 tiles, 46 key bits): the forward render.

Bars: compaction, depths, 2D records, tile rectangles, duplicate counts, sorted keys and
values, tile ends, images and last contributors bit-exact (images also asserted within 1e-4);
the rasterisers' work counts exact; the loss within the loss test's tolerance; the nine gradient
arrays within 1e-3 relative L2 with >= 99.9% of the Gaussians within 1e-3
(test_gpu_backward_adam.check_grads). Per Gaussian, with millions of them some sums cancel to far
below their terms, where float atomics (the reference's summation too) lose digits that the
oracle's double sums keep: each Gaussian's 2D gradients are held to 1e-3 of their value plus 1e-3
of the sum of their terms' magnitudes, and the projection backward to 1e-3 per Gaussian on the
GPU's own 2D gradients. One Adam step is bit-exact given the same gradients, through both the
written-SH-gradient update and the trainer's rebuilt-SH update. The oracle runs on all host
threads (a few seconds per frame here).

Also `update_adc_stats_kernel!` (training.jl:472-497): the ADC accumulators after three views,
bit-exact against the oracle's accumulation of the same 2D gradients.
"""
import os

import numpy as np
import pytest
import torch

import gs3d
from gs3d import RenderBuffers, RenderOptions, RenderOutputs, Tiling
from gs3d import adc as adc_mod
from gs3d.backward import FilteredGaussiansGradients, backward
from gs3d.loss import LossComputer
from gs3d.optimizer import AdamOptimizer, LearningRates, bias_corrections
from gs3d.scene import CONFIGS, scene_radius, synthetic_gaussians, target_image
from oracle import oracle as O

from test_gpu_backward_adam import check_grads, check_grads_2d_terms, rel_l2
from test_gpu_forward import compare

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def oracle_threads():
    O.lib().oracle_set_threads(os.cpu_count() or 1)
    yield
    O.lib().oracle_set_threads(1)


_SCENE = {}


def scene(cfg_id):
    """(CPU GaussiansVector, NpGaussians, cameras) of a config, one config resident at a time."""
    if cfg_id not in _SCENE:
        _SCENE.clear()
        cfg = CONFIGS[cfg_id]
        gv = synthetic_gaussians(cfg["spec"], cfg["seed"])
        _SCENE[cfg_id] = (gv, O.NpGaussians.from_vector(gv), cfg["cameras"]())
    return _SCENE[cfg_id]


def gpu_forward(g, cam, til, opt, device):
    out = RenderOutputs.create(cam.width, cam.height, device, include_depth=True)
    buf = RenderBuffers.create(g.n, til.nb_tiles, device, capacity_dup=8 * g.n)
    gs3d.render(out, g, cam, til, opt, buf)
    torch.cuda.synchronize()
    F, D = gs3d.counts(buf)
    cpu = lambda t: t.cpu().numpy()
    r = dict(F=F, D=D, keep=cpu(buf.keep_gaussians[: g.n]), keep_cs=cpu(buf.keep_gaussians_cs[: g.n]),
             fgidx_to_gidx=cpu(buf.fgidx_to_gidx[:F]), depths=cpu(buf.depths[:F]),
             f2d=cpu(buf.f2d[:F]), ranges=cpu(buf.intersected_tile_ranges[:F]),
             ntiles=cpu(buf.nb_overlapped_tiles[:F]), scodes=cpu(buf.sdf2dgs_codes[:D]),
             sfg=cpu(buf.sdfgidx_to_fgidx[:D]), tiles_end=cpu(buf.tiles_end_sdfgidx[: til.nb_tiles]),
             rgb=cpu(out.rgb), trans=cpu(out.transmittance), depth=cpu(out.depth),
             last=cpu(out.last_contributing_sdfgids), reference_order=False)
    assert int(buf.device_counts[2]) == 0
    return r, out, buf


@pytest.mark.parametrize("cfg_id, cam_index", [(3, 0)], ids=["cfg3_4k_cam0"])
def test_full_size_forward_vs_oracle(cuda, cfg_id, cam_index):
    gv, npg, cams = scene(cfg_id)
    cam = cams[cam_index]
    opt = RenderOptions.for_camera(cam, 3)
    til = Tiling.for_camera(cam)
    g = gv.to(cuda)
    gpu, _, _ = gpu_forward(g, cam, til, opt, cuda)
    ref = O.render(npg, cam, til, opt, dup_capacity=gpu["D"] + 16)
    assert ref["F"] > 0.5 * gv.n and ref["D"] > 0
    compare(gpu, ref)


@pytest.mark.parametrize("cfg_id, cam_index", [(4, 0), (4, 131), (1, 0)],
                         ids=["cfg4_cam0", "cfg4_cam131", "cfg1_cam0"])
def test_full_size_training_step_vs_oracle(cuda, cfg_id, cam_index):
    gv, npg, cams = scene(cfg_id)
    cam = cams[cam_index]
    opt = RenderOptions.for_camera(cam, 3)
    til = Tiling.for_camera(cam)
    g = gv.to(cuda)
    n = g.n

    # render!
    gpu, out, buf = gpu_forward(g, cam, til, opt, cuda)
    ref_f = O.render(npg, cam, til, opt, dup_capacity=gpu["D"] + 16)
    compare(gpu, ref_f)
    F = gpu["F"]
    if cam_index == 0:  # the rasterisers' work counts (the bench's roofline numerators)
        from gs3d.render import work_counts
        assert work_counts(cam, til, opt, buf) == O.work_counts(ref_f, cam, til, opt)

    # loss against a seeded target; the same gradient image then drives both backward passes
    target = target_image(cam.width, cam.height, 1000 + cam_index)
    lc = LossComputer(cam.width, cam.height, cuda, 0.2)
    grad = torch.empty((cam.width, cam.height, 3), dtype=torch.float32, device=cuda)
    val = lc(out.rgb, target.to(cuda), grad).cpu().numpy()
    ref_loss, ref_grad = O.loss(ref_f["rgb"], target.numpy(), 0.2)
    np.testing.assert_allclose(val[:3], ref_loss, rtol=2e-5, atol=1e-6)
    grad_np = grad.cpu().numpy()
    assert np.abs(grad_np - ref_grad).max() <= 1e-3 * np.abs(ref_grad).max()

    # backward!
    fg = FilteredGaussiansGradients.create(n, 3, cuda)
    backward(fg, grad, out, g, cam, til, opt, buf)
    torch.cuda.synchronize()
    cpu = lambda t: t[:F].cpu().numpy()
    gpu_g = dict(mean2d=cpu(fg.mean2d_grads), opacity=cpu(fg.opacity_grads),
                 licov=cpu(fg.licov2d_grads), color=cpu(fg.color_grads),
                 mean3d=cpu(fg.mean3d_grads), opacity_feature=cpu(fg.opacity_feature_grads),
                 scaling=cpu(fg.scaling_features_grads), rotation=cpu(fg.rotation_features_grads),
                 sh=cpu(fg.sh_coeffs_grads))
    ref_g = O.backward(npg, cam, til, opt, ref_f, grad_np, with_magnitudes=True)
    # arrays within 1e-3 relative L2, >= 99.9% of the Gaussians within 1e-3; every Gaussian's 2D
    # gradients within 1e-3 of its value plus 1e-3 of the size of its per-pixel terms
    check_grads(gpu_g, ref_g, every_gaussian=False)
    check_grads_2d_terms(gpu_g, ref_g, ref_g["mag"])
    # the projection backward on the GPU's own 2D gradients (no summation-order effects):
    # every Gaussian with a gradient above 1e-3 of the largest within 1e-3 relative L2
    ref_p = O.backward(npg, cam, til, opt, ref_f, grad_np, grads_2d=gpu_g)
    for k in ("mean3d", "opacity_feature", "scaling", "rotation", "sh"):
        total, per = rel_l2(gpu_g[k], ref_p[k])
        norms = np.linalg.norm(np.asarray(ref_p[k], np.float64).reshape(len(per), -1), axis=1)
        big = norms > 1e-3 * norms.max()
        assert total <= 1e-5, (k, total)
        assert np.all(per[big] <= 1e-3), (k, per[big].max(), np.count_nonzero(per[big] > 1e-3))

    # update!: the GPU step from written SH gradients and the trainer's rebuilt-SH step both
    # equal the oracle's step on the GPU's gradients, bit for bit
    lr = LearningRates(means=0.00016 * scene_radius(cams))
    g2 = g.clone()
    a1, a2 = AdamOptimizer(g, lr), AdamOptimizer(g2, lr)
    rng = np.random.default_rng(cfg_id * 1000 + cam_index)
    for t1, t2 in zip(a1.moments.tensors(), a2.moments.tensors()):
        m = torch.from_numpy(np.abs(rng.normal(0, 1e-4, size=tuple(t1.shape))).astype(np.float32))
        t1.copy_(m)
        t2.copy_(m)
    a1.update_count = a2.update_count = 3000
    before_m = O.NpMoments.from_moments(a1.moments)
    params = a1.params_c(3)
    a1.update(fg, buf.fgidx_to_gidx, buf.device_counts, 3)
    a2.update_rebuild_sh(fg, buf.fgidx_to_gidx, buf.device_counts, buf.f2d, cam.position, 3)
    torch.cuda.synchronize()
    ref_g_after = npg.copy()
    bc1, bc2 = bias_corrections(a1.beta1, a1.beta2, 3000)
    O.adam(ref_g_after, before_m, gpu_g, gpu["fgidx_to_gidx"], params, bc1, bc2)
    for gg, aa in ((g, a1), (g2, a2)):
        after_g = O.NpGaussians.from_vector(gg)
        after_m = O.NpMoments.from_moments(aa.moments)
        for x, y in zip((after_g.mo, after_g.sf, after_g.rf, after_g.sh),
                        (ref_g_after.mo, ref_g_after.sf, ref_g_after.rf, ref_g_after.sh)):
            assert np.array_equal(x.view(np.uint32), y.view(np.uint32))
        for x, y in zip((after_m.mm, after_m.om, after_m.sm, after_m.rm, after_m.shm),
                        (before_m.mm, before_m.om, before_m.sm, before_m.rm, before_m.shm)):
            assert np.array_equal(x.view(np.uint32), y.view(np.uint32))


@pytest.mark.parametrize("cfg_id, n_views", [(1, 3), (4, 3)], ids=["cfg1_3views", "cfg4_3views"])
def test_adc_stats_accumulate_vs_oracle(cuda, cfg_id, n_views):
    """gs3d_adc_stats (k_adc_stats) over several views: each view adds
    sqrt((gx w/2)^2 + (gy h/2)^2) to acc and 1 to cnt for every filtered Gaussian with a nonzero
    2D mean gradient; compared bit for bit with the oracle's accumulation of the same 2D
    gradients, starting from nonzero accumulators."""
    gv, _, cams = scene(cfg_id)
    g = gv.to(cuda)
    n = g.n
    adc = adc_mod.AdcBuffers.create(n, cuda)
    rng = np.random.default_rng(17)
    acc0 = np.abs(rng.normal(0, 1e-3, n)).astype(np.float32)
    cnt0 = rng.integers(0, 5, n).astype(np.int32)
    adc.accumulated_mean2d_grad_norms_ndc.copy_(torch.from_numpy(acc0))
    adc.rendering_contribution_counts.copy_(torch.from_numpy(cnt0))
    acc, cnt = acc0.copy(), cnt0.copy()
    for v in range(n_views):
        cam = cams[(v * 37) % len(cams)]
        opt = RenderOptions.for_camera(cam, 3)
        til = Tiling.for_camera(cam)
        out = RenderOutputs.create(cam.width, cam.height, cuda)
        buf = RenderBuffers.create(n, til.nb_tiles, cuda, capacity_dup=8 * n)
        gs3d.render(out, g, cam, til, opt, buf)
        grad = torch.from_numpy(np.random.default_rng(v).normal(0, 1e-6, (cam.width, cam.height, 3))
                                .astype(np.float32)).to(cuda)
        fg = FilteredGaussiansGradients.create(n, 3, cuda)
        backward(fg, grad, out, g, cam, til, opt, buf)
        adc_mod.adc_stats(adc, fg, buf.fgidx_to_gidx, buf.device_counts, cam.width, cam.height)
        torch.cuda.synchronize()
        F, _ = gs3d.counts(buf)
        m2 = fg.mean2d_grads[:F].cpu().numpy()
        assert np.count_nonzero(np.all(m2 == 0, axis=1)) > 0  # some filtered Gaussians get no gradient
        O.adc_stats(acc, cnt, m2, buf.fgidx_to_gidx[:F].cpu().numpy(), cam.width, cam.height)
    got_acc = adc.accumulated_mean2d_grad_norms_ndc[:n].cpu().numpy()
    got_cnt = adc.rendering_contribution_counts[:n].cpu().numpy()
    assert np.array_equal(got_cnt, cnt)
    assert np.array_equal(got_acc.view(np.uint32), acc.view(np.uint32))
    assert np.count_nonzero(cnt != cnt0) > 0.1 * n
