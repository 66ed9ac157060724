"""Loss, densification and a whole training step on the GPU against the CPU oracle."""
import numpy as np
import pytest
import torch

import gs3d
from gs3d import RenderBuffers, RenderOptions, RenderOutputs, Tiling, _abi
from gs3d import adc as adc_mod
from gs3d.loss import LossComputer
from gs3d.optimizer import AdamMoments, bias_corrections
from gs3d.scene import SceneSpec, look_at_camera, synthetic_gaussians, target_image
from gs3d.training import Trainer, TrainingOptions
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("w,h,weight", [(64, 48, 0.2), (256, 256, 0.2), (333, 171, 0.5), (100, 80, 0.0),
                                        (1920, 1080, 0.2), (9, 7, 0.2)])
def test_loss_matches_oracle(cuda, w, h, weight):
    rng = np.random.default_rng(w * h)
    K = rng.uniform(0, 1, (w, h, 3)).astype(np.float32)
    K[: w // 2] = np.clip(K[: w // 2] * 0.3 + 0.2, 0, 1)  # some structure
    I = rng.uniform(0, 1, (w, h, 3)).astype(np.float32)
    I[5, 5] = K[5, 5]  # ties take the negative L1 branch
    lc = LossComputer(w, h, cuda, weight)
    grad = torch.empty((w, h, 3), dtype=torch.float32, device=cuda)
    val = lc(torch.from_numpy(K).to(cuda), torch.from_numpy(I).to(cuda), grad).cpu().numpy()
    ref, ref_grad = O.loss(K, I, weight)
    np.testing.assert_allclose(val[:3], ref, rtol=2e-5, atol=1e-6)
    g = grad.cpu().numpy()
    assert np.abs(g - ref_grad).max() <= 1e-3 * np.abs(ref_grad).max()


def _golden_adc_gpu(cuda, tr, prune, dens, clone):
    n = 8
    k = torch.arange(1, n + 1, dtype=torch.float32, device=cuda)
    mo = k[:, None].repeat(1, 4).contiguous()
    mo[:, 3] = torch.from_numpy(np.where(prune == 1, -10.0, 5.0).astype(np.float32)).to(cuda)
    sf = torch.from_numpy(np.where(clone[:, None] == 1, -6.0, 0.0).repeat(3, 1).astype(np.float32)).to(cuda)
    g = gs3d.GaussiansVector(mo, sf, k[:, None].repeat(1, 4).contiguous(),
                             k[:, None, None].repeat(1, 3, 4).contiguous())
    a = adc_mod.AdcBuffers.create(n, cuda)
    a.accumulated_mean2d_grad_norms_ndc.copy_(torch.from_numpy((dens == 1).astype(np.float32)))
    a.rendering_contribution_counts.fill_(1)
    return g, a


def test_adc_plan_apply_golden(cuda, golden):
    tr = golden["training"]
    prune = np.array(tr["should_prune"], np.uint8)
    dens = np.array(tr["should_densify"], np.uint8)
    clone = np.array(tr["should_clone"], np.uint8)
    g, a = _golden_adc_gpu(cuda, tr, prune, dens, clone)
    new_n = adc_mod.densify_prune_plan(a, g, 0.0002, 0.01, 0.005, 1e6, False)
    assert new_n == 10
    assert a.should_prune.cpu().numpy().tolist() == prune.tolist()
    assert a.should_densify.cpu().numpy().tolist() == dens.tolist()
    assert a.should_clone.cpu().numpy().tolist() == clone.tolist()
    assert a.ngidx_to_gidx[:10].cpu().numpy().tolist() == [int(x) for x in tr["ngidx_to_gidx"]]
    # the reference's apply test uses plain k-valued features; reuse its values here
    k = torch.arange(1, 9, dtype=torch.float32, device=cuda)
    g2 = gs3d.GaussiansVector(k[:, None].repeat(1, 4).contiguous(), k[:, None].repeat(1, 3).contiguous(),
                              k[:, None].repeat(1, 4).contiguous(), k[:, None, None].repeat(1, 3, 4).contiguous())
    m = AdamMoments.zeros(8, 1, cuda)
    for t in m.tensors():
        t.copy_(k.view(-1, *([1] * (t.dim() - 1))).expand_as(t))
    f2g = torch.tensor([int(x) for x in tr["original_fgidx_to_gidx"]], dtype=torch.int32, device=cuda)
    counts = torch.tensor([3, 0, 0, 0], dtype=torch.int32, device=cuda)
    ng, nm = adc_mod.densify_apply(a, g2, m, 10, float(np.exp(np.float32(10.0))), 7, f2g, counts)
    torch.cuda.synchronize()
    assert f2g.cpu().numpy().tolist() == [int(x) for x in tr["adjusted_fgidx_to_gidx"]]
    ids = [int(x) - 1 for x in tr["means_after_adc_ids"]]
    assert np.array_equal(ng.means_opacity_features[ids, :3].cpu().numpy(),
                          np.repeat(np.array(tr["means_after_adc"], np.float32)[:, None], 3, 1))
    np.testing.assert_allclose(ng.scaling_features.cpu().numpy(),
                               np.repeat(np.array(tr["scaling_after_adc"], np.float32)[:, None], 3, 1), rtol=1e-6)
    want = np.array(tr["moments_after_adc"], np.float32)
    for t in nm.tensors():
        arr = t.cpu().numpy().reshape(10, -1)
        assert np.array_equal(arr, np.repeat(want[:, None], arr.shape[1], 1))
    # bit-exact against the oracle, split means included
    go = O.NpGaussians.from_vector(g2)
    mo_ = O.NpMoments.from_moments(m)
    plan = dict(prune=prune, densify=dens, clone=clone,
                counts_cs=np.cumsum((1 - prune) + dens).astype(np.int32), new_n=10)
    ong, onm, of2g = O.adc_apply(go, mo_, plan, np.array(tr["original_fgidx_to_gidx"], np.int32),
                                 float(np.log(np.float32(np.exp(np.float32(10.0))))), 7)
    for a_, b_ in zip([t.cpu().numpy() for t in ng.tensors()], (ong.mo, ong.sf, ong.rf, ong.sh)):
        assert np.array_equal(a_.view(np.uint32), b_.view(np.uint32))


def test_adc_random_vs_oracle(cuda):
    n = 50_000
    gv = synthetic_gaussians(SceneSpec(n, "uniform:1", -4.0, 1.0), 3)
    g = gv.to(cuda)
    rng = np.random.default_rng(4)
    a = adc_mod.AdcBuffers.create(n, cuda)
    acc = rng.exponential(2e-4, n).astype(np.float32)
    cnt = rng.integers(0, 4, n).astype(np.int32)
    a.accumulated_mean2d_grad_norms_ndc.copy_(torch.from_numpy(acc))
    a.rendering_contribution_counts.copy_(torch.from_numpy(cnt))
    R = 3.3
    new_n = adc_mod.densify_prune_plan(a, g, 0.0002, 0.01 * R, 0.005, 0.1 * R, True)
    p = _abi.AdcParamsC()
    p.densification_mean2d_grad_norm_threshold_ndc = 0.0002
    p.densification_size_threshold = float(np.float32(0.01 * R))
    p.pruning_min_opacity = 0.005
    p.pruning_3d_max_scale = float(np.float32(0.1 * R))
    p.use_max_scale_pruning = 1
    go = O.NpGaussians.from_vector(gv)
    plan = O.adc_plan(go, acc, cnt, p)
    assert new_n == plan["new_n"]
    for k, t in (("prune", a.should_prune), ("densify", a.should_densify), ("clone", a.should_clone),
                 ("counts_cs", a.new_gaussian_counts_cs)):
        assert np.array_equal(t.cpu().numpy(), plan[k]), k
    assert np.array_equal(a.ngidx_to_gidx[:new_n].cpu().numpy(), plan["ngidx_to_gidx"])
    m = AdamMoments.zeros(n, 3, cuda)
    for t in m.tensors():
        t.copy_(torch.from_numpy(rng.normal(0, 1, tuple(t.shape)).astype(np.float32)))
    f2g_np = np.sort(rng.choice(n, 20_000, replace=False) + 1).astype(np.int32)
    f2g = torch.from_numpy(f2g_np).to(cuda)
    counts = torch.tensor([f2g_np.size, 0, 0, 0], dtype=torch.int32, device=cuda)
    split = 1 / 1.6
    ng, nm = adc_mod.densify_apply(a, g, m, new_n, split, 99, f2g, counts)
    torch.cuda.synchronize()
    ong, onm, of2g = O.adc_apply(go, O.NpMoments.from_moments(m), plan, f2g_np,
                                 float(np.log(np.float32(split))), 99)
    for x, y in zip([t.cpu().numpy() for t in ng.tensors()], (ong.mo, ong.sf, ong.rf, ong.sh)):
        assert np.array_equal(x.view(np.uint32), y.view(np.uint32))
    for x, y in zip([t.cpu().numpy() for t in nm.tensors()], (onm.mm, onm.om, onm.sm, onm.rm, onm.shm)):
        assert np.array_equal(x, y)
    assert np.array_equal(f2g.cpu().numpy(), of2g)


def test_opacity_reset_vs_oracle(cuda):
    gv = synthetic_gaussians(SceneSpec(10_000, "uniform:1", -4.0, 1.0, 0.0, 3.0), 5)
    g = gv.to(cuda)
    m = AdamMoments.zeros(g.n, 3, cuda)
    m.opacity_features_moments.fill_(3.0)
    adc_mod.opacity_reset(g, m, 0.01)
    go = O.NpGaussians.from_vector(gv)
    om = O.NpMoments.from_moments(AdamMoments.zeros(g.n, 3, "cpu"))
    O.opacity_reset(go, om, 0.01)
    assert np.array_equal(g.means_opacity_features.cpu().numpy(), go.mo)
    assert torch.all(m.opacity_features_moments == 0)


def _cfg0_trainer(cuda, nviews=1, seed=0):
    gv = synthetic_gaussians(SceneSpec(16_384, "uniform:1", -4.0, 0.5), seed)
    cams = [look_at_camera(256, 256, 60.0, (0, 0, 3))] * nviews
    targets = [target_image(256, 256, 100 + i, cuda) for i in range(nviews)]
    opts = TrainingOptions(scene_radius=3.3)
    ro = RenderOptions.for_camera(cams[0], 3)
    t = Trainer(gv.to(cuda), cams, targets, ro, Tiling.for_camera(cams[0]), opts)
    return gv, cams, targets, ro, t


def test_training_step_matches_oracle_chain(cuda):
    gv, cams, targets, ro, t = _cfg0_trainer(cuda)
    t.iteration_nb = 2000  # past the SH-degree increases, before any densify step
    t.training_step()
    torch.cuda.synchronize()
    # oracle chain: render -> loss -> backward -> ADC stats -> Adam
    g = O.NpGaussians.from_vector(gv)
    til = Tiling.for_camera(cams[0])
    f = O.render(g, cams[0], til, ro)
    (loss, _, _), grad = O.loss(f["rgb"], targets[0].cpu().numpy(), 0.2)
    b = O.backward(g, cams[0], til, ro, f, grad)
    assert abs(float(t.last_loss[0]) - loss) <= 1e-5 * abs(loss)
    p = t.optimizer.params_c(3)
    p.update_count = 0
    bc1, bc2 = bias_corrections(t.optimizer.beta1, t.optimizer.beta2, 0)
    m = O.NpMoments.from_moments(AdamMoments.zeros(g.n, 3, "cpu"))
    O.adam(g, m, b, f["fgidx_to_gidx"], p, bc1, bc2)
    got = O.NpGaussians.from_vector(t.gaussians)
    # first Adam step moves every touched parameter by ~lr * sign(grad): compare to that scale
    for x, y, lr in ((got.mo[:, :3], g.mo[:, :3], p.lr_means), (got.mo[:, 3], g.mo[:, 3], p.lr_opacity_features),
                     (got.sf, g.sf, p.lr_scaling_features), (got.rf, g.rf, p.lr_rotation_features),
                     (got.sh[:, :, 1:], g.sh[:, :, 1:], p.lr_sh_rest)):
        d = np.abs(x - y)
        assert d.max() <= 2.01 * lr
        assert np.mean(d <= 1e-6 + 1e-3 * lr) >= 0.999


def test_host_targets_prefetched_match_device_targets(cuda):
    """Pinned host targets, uploaded one step ahead on a copy stream, give the same training
    run as device-resident targets (5 views, 12 steps: re-shuffles included): every step's
    [loss, L1, DSSIM] agree. The backward's float atomics make two runs differ in the last
    bits (and Adam with epsilon 1e-15 turns a near-zero gradient's sign flip into a full step),
    so parameters are not compared and the losses have a tolerance, far below what a wrong or
    stale target would change (the targets are independent random images)."""
    runs = []
    for on_host in (False, True):
        gv = synthetic_gaussians(SceneSpec(16_384, "uniform:1", -4.0, 0.5), 3)
        cams = [look_at_camera(256, 256, 60.0, (0.2 * i, 0, 3)) for i in range(5)]
        targets = [target_image(256, 256, 200 + i, cuda) for i in range(5)]
        if on_host:
            targets = [x.cpu().pin_memory() for x in targets]
        ro = RenderOptions.for_camera(cams[0], 3)
        t = Trainer(gv.to(cuda), cams, targets, ro, Tiling.for_camera(cams[0]),
                    TrainingOptions(scene_radius=3.3), seed=7)
        t.iteration_nb = 3000
        losses = [t.training_step().clone() for _ in range(12)]
        torch.cuda.synchronize()
        runs.append(torch.stack(losses)[:, :3].cpu())
    assert torch.allclose(runs[0], runs[1], rtol=1e-5, atol=0), (runs[0], runs[1])


def test_trainer_loss_decreases(cuda):
    _, _, _, _, t = _cfg0_trainer(cuda, nviews=1, seed=1)
    t.iteration_nb = 3000
    losses = []
    for _ in range(40):
        losses.append(float(t.training_step()[0]))
    assert losses[-1] < losses[0]
    assert t.optimizer.update_count == 40


@pytest.mark.parametrize("factored", [False, True])
def test_data_parallel_trainer_one_rank_matches_trainer(cuda, factored):
    """DataParallelTrainer without a process group (dense rows: gs3d_backward_project_dense +
    gs3d_adam_step_dense_range; factored rows: gs3d_backward_project_factored +
    gs3d_adam_step_factored_range) follows the sparse Trainer's training run (one view, 8 steps)."""
    from functools import partial

    from gs3d.dp import DataParallelTrainer
    runs = []
    for cls in (Trainer, partial(DataParallelTrainer, factored=factored)):
        gv = synthetic_gaussians(SceneSpec(16_384, "uniform:1", -4.0, 0.5), 9)
        cams = [look_at_camera(256, 256, 60.0, (0, 0, 3))]
        ro = RenderOptions.for_camera(cams[0], 3)
        t = cls(gv.to(cuda), cams, [target_image(256, 256, 300, cuda)], ro, Tiling.for_camera(cams[0]),
                TrainingOptions(scene_radius=3.3), seed=7)
        t.iteration_nb = 3000
        runs.append(torch.stack([t.training_step().clone() for _ in range(8)])[:, :3].cpu())
    assert torch.allclose(runs[0], runs[1], rtol=1e-5, atol=0), (runs[0], runs[1])


@pytest.mark.parametrize("views", [1, 2])
def test_data_parallel_sharded_sh_follows_gathered_sh(cuda, views):
    """DataParallelTrainer(shard_sh=True) on one rank: the owner adds the mean gradients'
    colour -> direction terms and computes the next step's colours, which the next render takes.
    Over 8 steps crossing a densify step (which needs every SH coefficient and takes the
    gathered path), then a jump to a densify step and two more steps, the run follows
    shard_sh=False within float rounding (the backward blend's
    float atomics make two runs differ in the last bits; with one view the split rows and the
    given colours are themselves bit-exact: test_owner_colour_direction_rows,
    test_given_colour_render_equals_render)."""
    from gs3d.dp import DataParallelTrainer
    cams = [look_at_camera(256, 256, 60.0, p)
            for p in ((0, 0, 3), (0.5, 0.2, 2.8), (-0.4, 0.3, 2.9), (0.2, -0.5, 3.1))]
    runs = []
    for shard in (False, True):
        gv = synthetic_gaussians(SceneSpec(16_384, "uniform:1", -4.0, 0.5), 9)
        ro = RenderOptions.for_camera(cams[0], 3)
        t = DataParallelTrainer(gv.to(cuda), cams, [target_image(256, 256, 300 + i, cuda) for i in range(4)],
                                ro, Tiling.for_camera(cams[0]), TrainingOptions(scene_radius=3.3), seed=7,
                                views_per_rank=views, shard_sh=shard)
        t.iteration_nb = 3096  # steps 3097 .. 3104: a densify step at 3100
        ls = [t.training_step().clone() for _ in range(8)]
        # a jump straight to a densify step (as bench.py's densify leg does), after a step that
        # prepared colours for its successor, and two more steps
        t.iteration_nb = 3199
        ls += [t.training_step().clone() for _ in range(3)]
        losses = torch.stack(ls)[:, :3].cpu()
        t.sync_parameters()
        torch.cuda.synchronize()
        runs.append((losses, [x.clone() for x in t.gaussians.tensors()], t.gaussians.n))
    (l0, p0, n0), (l1, p1, n1) = runs
    assert abs(n0 - n1) <= 2  # a borderline Gaussian may densify differently
    assert torch.allclose(l0, l1, rtol=1e-5, atol=0), (l0, l1)
    if n0 == n1:
        # Adam normalises each gradient: where a gradient is tiny, rounding differences of the
        # summed mean gradients change a step by up to the learning rate, so a few elements
        # drift; the rest agree
        for a, b in zip(p0, p1):
            close = torch.isclose(a, b, rtol=1e-4, atol=1e-5)
            assert float(close.float().mean()) >= 0.99, float(close.float().mean())


def test_data_parallel_phase_times(cuda):
    """phase_events / phase_times: every phase of a data-parallel step (two views per rank) is
    recorded once per step per view where it repeats, with non-negative times whose sum stays
    within the steps' own device time."""
    from gs3d.dp import DataParallelTrainer
    gv = synthetic_gaussians(SceneSpec(16_384, "uniform:1", -4.0, 0.5), 9)
    cams = [look_at_camera(256, 256, 60.0, p) for p in ((0, 0, 3), (0.5, 0.2, 2.8))]
    ro = RenderOptions.for_camera(cams[0], 3)
    t = DataParallelTrainer(gv.to(cuda), cams, [target_image(256, 256, 300 + i, cuda) for i in range(2)],
                            ro, Tiling.for_camera(cams[0]), TrainingOptions(scene_radius=3.3), seed=7,
                            views_per_rank=2)
    t.iteration_nb = 3000
    t.training_step()
    t.phase_events = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(4):
        t.training_step()
    t._mark("step_start")  # closes the last step
    e1.record()
    torch.cuda.synchronize()
    total = e0.elapsed_time(e1) / 4
    ph = t.phase_times()
    for k in ("render", "loss", "backward_raster", "backward_project", "wait_exchange_0", "adam_0"):
        assert k in ph, ph
    assert all(v >= 0 for v in ph.values()), ph
    assert sum(ph.values()) <= total * 1.05 + 0.05, (ph, total)
    assert t.phase_events == []


def test_checkpoint_resume_follows_the_uninterrupted_run(cuda, tmp_path):
    """gs3d.io.save_checkpoint after 5 steps, then 10 more steps (through the densify and
    opacity-reset step at iteration 3000); a fresh Trainer restored from the checkpoint takes the
    same views and reaches the same losses and (up to a borderline Gaussian) Gaussian count: the backward's
    float-atomic sums make two runs differ in the last bits."""
    from gs3d import io

    cams = [look_at_camera(192, 160, 60.0, (np.cos(a) * 3, 0.5, np.sin(a) * 3))
            for a in np.linspace(0, 2 * np.pi, 6, endpoint=False)]
    targets = [target_image(192, 160, 400 + i, cuda) for i in range(len(cams))]

    def make():
        gv = synthetic_gaussians(SceneSpec(8_192, "uniform:1", -4.0, 0.5), 11)
        t = Trainer(gv.to(cuda), cams, targets, RenderOptions.for_camera(cams[0], 3),
                    Tiling.for_camera(cams[0]), TrainingOptions(scene_radius=3.3), seed=3)
        t.iteration_nb = 2990
        return t

    t1 = make()
    for _ in range(5):
        t1.training_step()
    ck = tmp_path / "state.pt"
    io.save_checkpoint(ck, t1)
    run1, views1 = [], []
    for _ in range(10):
        run1.append(t1.training_step()[:3].cpu())
        views1.append(t1.current_camera_index())
    t2 = make()
    io.load_checkpoint(ck, t2)
    assert t2.iteration_nb == 2995 and t2.optimizer.update_count == 5
    run2, views2 = [], []
    for _ in range(10):
        run2.append(t2.training_step()[:3].cpu())
        views2.append(t2.current_camera_index())
    assert views1 == views2
    # densify decisions compare accumulated gradient norms with a threshold: a borderline
    # Gaussian may go either way between two runs
    assert abs(t1.gaussians.n - t2.gaussians.n) <= max(2, t1.gaussians.n // 1000)
    assert torch.allclose(torch.stack(run1), torch.stack(run2), rtol=1e-4, atol=0)


@pytest.mark.parametrize("factored", [False, True])
def test_multi_view_step_equals_summed_views(cuda, factored):
    """views_per_rank = 3 on one rank (a batch of three views per step): the step's gradient rows
    are the three views' dense rows summed, the update follows them, and the step returns the
    mean of the three views' losses. Dense rows: the projection backward adds the later views
    into the first view's rows (GS3D_BACKWARD_ACCUMULATE_ROWS); factored rows: the geometry rows
    add up the same way and each view keeps its colour row. The 2D gradients are float-atomic
    sums whose order differs between runs, so rows are compared within tolerances and
    the parameters after the update mostly bit for bit (Adam's first step moves a parameter by
    about its learning rate times the sign of its gradient, so a gradient that is zero up to
    rounding may move either way)."""
    import ctypes as C

    from gs3d.backward import FilteredGaussiansGradients, backward_dense
    from gs3d.dp import DataParallelTrainer, view_index
    from gs3d.optimizer import AdamOptimizer
    from gs3d.training import annealed_means_lr
    gv = synthetic_gaussians(SceneSpec(16_384, "uniform:1", -4.0, 0.5), 9)
    cams = [look_at_camera(256, 256, 60.0, p)
            for p in ((0, 0, 3), (0.5, 0.2, 2.8), (-0.4, 0.3, 2.9), (0.2, -0.5, 3.1))]
    targets = [target_image(256, 256, 300 + i, cuda) for i in range(len(cams))]
    ro = RenderOptions.for_camera(cams[0], 3)
    til = Tiling.for_camera(cams[0])
    opts = TrainingOptions(scene_radius=3.3)
    t = DataParallelTrainer(gv.to(cuda), cams, targets, ro, til, opts, seed=7, factored=factored,
                            views_per_rank=3)
    t.iteration_nb = 3000
    views = [view_index(0, 0, 1, t.perm, len(cams), 3, v) for v in range(3)]
    assert len(set(views)) == 3
    loss = t.training_step().clone()

    g = gv.to(cuda)
    n = g.n
    out = RenderOutputs.create(256, 256, cuda)
    buf = RenderBuffers.create(n, til.nb_tiles, cuda)
    lc = LossComputer(256, 256, cuda, opts.loss_dssim_vs_L1_weight)
    grad = torch.empty((256, 256, 3), dtype=torch.float32, device=cuda)
    fg = FilteredGaussiansGradients.create(n, 3, cuda)
    total, losses, live = None, [], []
    for i in views:
        gs3d.render(out, g, cams[i], til, ro, buf)
        losses.append(lc(out.rgb, targets[i], grad).clone())
        d = backward_dense(fg, grad, out, g, cams[i], til, ro, buf,
                           torch.empty((n, 60), dtype=torch.float32, device=cuda))
        live.append(d[:, 59] > 0)
        total = d.clone() if total is None else total + d
    want = (losses[0] + losses[1] + losses[2]) / 3
    assert torch.equal(loss[:3], want[:3])  # forward and loss are deterministic

    def close(a, b):
        """Within 1e-4 relative L2 overall and every entry within 1e-3 of its column's scale
        (a Gaussian whose per-pixel terms cancel carries the atomic-order noise of its 2D
        gradients into its 3D rows)."""
        rel = float((a - b).norm() / b.norm().clamp_min(1e-30))
        scale = b.abs().amax(dim=0, keepdim=True).clamp_min(1e-30)
        worst = float(((a - b).abs() / scale).max())
        assert rel <= 1e-4 and worst <= 1e-3, (rel, worst)
        return True

    if factored:
        assert close(t.geom[:n, :11], total[:, 48:59])
        assert torch.equal(t.geom[:n, 11] > 0, total[:, 59] > 0)
        for v in range(3):
            assert torch.equal(t.colour[v, :n, 3] > 0, live[v])
    else:
        assert close(t.dense[:n, :59], total[:, :59])
        assert torch.equal(t.dense[:n, 59] > 0, total[:, 59] > 0)
    adam = AdamOptimizer(g, opts.learning_rates())
    adam.lrs.means = annealed_means_lr(3001, opts)
    gc, mc, pc = g.to_c(), adam.moments.to_c(), adam.params_c(3)
    _abi.check(_abi.lib().gs3d_adam_step_dense(C.byref(gc), C.byref(mc), C.c_void_p(total.data_ptr()),
                                               C.byref(pc), None))
    torch.cuda.synchronize()
    # Adam's first step moves each parameter by its learning rate times the sign of its
    # gradient: a gradient that is zero up to the rounding noise may flip, which moves that
    # parameter by up to twice its learning rate
    lrs = opts.learning_rates()
    bounds = (max(adam.lrs.means, lrs.opacity_features), lrs.scaling_features, lrs.rotation_features,
              max(lrs.sh_coeffs_dc, lrs.sh_coeffs_rest))
    for x, y, lr in zip(t.gaussians.tensors(), g.tensors(), bounds):
        same = (x[:n] == y).float().mean().item()
        assert same >= 0.99, same
        assert float((x[:n] - y).abs().max()) <= 2.01 * lr
    assert t.optimizer.update_count == 1
