"""Oracle restatements of the optimizer and densification pinned to the reference's
test/training.jl golden data (no GPU)."""
import numpy as np

from gs3d import _abi
from gs3d.optimizer import bias_corrections
from oracle import oracle as O


def _adc_golden_state(tr):
    """test/training.jl:1-180: 8 Gaussians whose every value is its index k, SH degree 1."""
    n = 8
    k = np.arange(1, n + 1, dtype=np.float32)
    g = O.NpGaussians(np.repeat(k[:, None], 4, 1), np.repeat(k[:, None], 3, 1),
                      np.repeat(k[:, None], 4, 1), np.broadcast_to(k[:, None, None], (n, 3, 4)))
    m = O.NpMoments(*(np.broadcast_to(k.reshape((n,) + (1,) * len(s)), (n,) + s).copy()
                      for s in [(3, 2), (2,), (3, 2), (4, 2), (3, 4, 2)]))
    return g, m


def test_adc_masks_scan_and_index_map_golden(golden):
    tr = golden["training"]
    prune = np.array(tr["should_prune"], np.uint8)
    dens = np.array(tr["should_densify"], np.uint8)
    counts = (1 - prune) + dens
    assert counts.tolist() == [int(x) for x in tr["new_gaussian_counts"]]
    assert np.cumsum(counts).tolist() == [int(x) for x in tr["new_gaussian_counts_cs"]]
    # drive the oracle's plan with statistics / features that produce the golden masks
    g, _ = _adc_golden_state(tr)
    clone = np.array(tr["should_clone"], np.uint8)
    g.mo[:, 3] = np.where(prune == 1, -10.0, 5.0)           # logit opacity below / above logit(0.005)
    g.sf[:] = np.where(clone[:, None] == 1, -6.0, 0.0)      # small -> clone, large -> split
    acc = np.where(dens == 1, 1.0, 0.0).astype(np.float32)
    cnt = np.ones(8, np.int32)
    p = _abi.AdcParamsC()
    p.densification_mean2d_grad_norm_threshold_ndc = 0.0002
    p.densification_size_threshold = 0.01
    p.pruning_min_opacity = 0.005
    p.pruning_3d_max_scale = 1e6
    p.use_max_scale_pruning = 0
    plan = O.adc_plan(g, acc, cnt, p)
    assert plan["prune"].tolist() == prune.tolist()
    assert plan["densify"].tolist() == dens.tolist()
    assert plan["clone"].tolist() == clone.tolist()
    assert plan["new_n"] == 10
    assert plan["ngidx_to_gidx"].tolist() == [int(x) for x in tr["ngidx_to_gidx"]]


def test_adc_apply_golden(golden):
    tr = golden["training"]
    g, m = _adc_golden_state(tr)
    prune = np.array(tr["should_prune"], np.uint8)
    dens = np.array(tr["should_densify"], np.uint8)
    clone = np.array(tr["should_clone"], np.uint8)
    plan = dict(prune=prune, densify=dens, clone=clone,
                counts_cs=np.cumsum((1 - prune) + dens).astype(np.int32), new_n=10)
    f2g = np.array(tr["original_fgidx_to_gidx"], np.int32)
    ng, nm, f2g_new = O.adc_apply(g, m, plan, f2g, log_split=10.0, seed=7)
    ids = [int(x) - 1 for x in tr["means_after_adc_ids"]]
    assert np.array_equal(ng.mo[ids, :3], np.repeat(np.array(tr["means_after_adc"], np.float32)[:, None], 3, 1))
    assert ng.mo[:, 3].tolist() == tr["ngidx_to_gidx"]
    np.testing.assert_allclose(ng.sf, np.repeat(np.array(tr["scaling_after_adc"], np.float32)[:, None], 3, 1),
                               rtol=1e-6)
    assert np.array_equal(ng.rf, np.repeat(np.array(tr["ngidx_to_gidx"], np.float32)[:, None], 4, 1))
    assert np.array_equal(ng.sh, np.broadcast_to(np.array(tr["ngidx_to_gidx"], np.float32)[:, None, None], (10, 3, 4)))
    want = np.array(tr["moments_after_adc"], np.float32)
    for arr in (nm.mm, nm.om, nm.sm, nm.rm, nm.shm):
        assert np.array_equal(arr.reshape(10, -1), np.repeat(want[:, None], arr.reshape(10, -1).shape[1], 1))
    assert f2g_new.tolist() == [int(x) for x in tr["adjusted_fgidx_to_gidx"]]
    # split means are resampled around the original mean
    splits = [0, 1, 4, 5]
    old = np.array([2, 2, 4, 4], np.float32)[:, None]
    shift = np.linalg.norm(ng.mo[splits, :3] - old, axis=1)
    assert np.all(shift > 0) and np.all(shift < 10 * np.exp(old[:, 0]))
    assert not np.array_equal(ng.mo[0, :3], ng.mo[1, :3])


def test_adam_golden(golden):
    """test/training.jl:181-257 on the oracle's Adam."""
    tr = golden["training"]
    k = np.array(tr["ngidx_to_gidx"], np.float32)
    km = np.array(tr["moments_after_adc"], np.float32)
    n = 10
    g = O.NpGaussians(np.repeat(k[:, None], 4, 1), np.repeat(k[:, None], 3, 1), np.repeat(k[:, None], 4, 1),
                      np.broadcast_to(k[:, None, None], (n, 3, 4)))
    m = O.NpMoments(*(np.broadcast_to(km.reshape((n,) + (1,) * len(s)), (n,) + s).copy()
                      for s in [(3, 2), (2,), (3, 2), (4, 2), (3, 4, 2)]))
    F = 3
    kf = np.arange(1, F + 1, dtype=np.float32)
    grads = dict(mean2d=np.zeros((F, 2)), opacity=np.zeros(F), licov=np.zeros((F, 3)), color=np.zeros((F, 3)),
                 mean3d=np.repeat(kf[:, None], 3, 1), opacity_feature=kf, scaling=np.repeat(kf[:, None], 3, 1),
                 rotation=np.repeat(kf[:, None], 4, 1), sh=np.broadcast_to(kf[:, None, None], (F, 3, 4)).copy())
    p = _abi.AdamParamsC()
    p.lr_means = p.lr_opacity_features = p.lr_scaling_features = p.lr_rotation_features = p.lr_sh_dc = 1.0
    p.lr_sh_rest = 10.0
    p.beta1 = p.beta2 = 0.5
    p.epsilon = 0.0
    p.update_count = 0
    p.sh_degree = 1
    bc1, bc2 = bias_corrections(0.5, 0.5, 0)
    before = g.mo.copy()
    O.adam(g, m, grads, np.array(tr["adjusted_fgidx_to_gidx"], np.int32), p, bc1, bc2)
    for ngidx, gidx, fgidx in tr["adam"]["checked"]:
        i = ngidx - 1
        m1h, m2h = gidx + fgidx, gidx + fgidx ** 2
        want = gidx - m1h / np.sqrt(m2h)
        np.testing.assert_allclose(g.mo[i], want, rtol=1e-6)
        np.testing.assert_allclose(m.mm[i], [[m1h / 2, m2h / 2]] * 3, rtol=1e-6)
        np.testing.assert_allclose(g.sh[i, :, 1:], gidx - 10 * m1h / np.sqrt(m2h), rtol=1e-6)
    for i in [int(x) - 1 for x in tr["splits_second_copies_ids"]]:
        assert np.array_equal(g.mo[i], before[i])


def test_opacity_reset_golden(golden):
    """test/training.jl:307-338: opacities above the max drop to it, the others stay."""
    from gs3d.scene import create_test_scene
    gv, _ = create_test_scene(0)
    g = O.NpGaussians.from_vector(gv)
    m = O.NpMoments(np.zeros((4, 3, 2)), np.ones((4, 2)), np.zeros((4, 3, 2)), np.zeros((4, 4, 2)),
                    np.zeros((4, 3, 1, 2)))
    op = 1 / (1 + np.exp(-g.mo[:, 3].astype(np.float64)))
    O.opacity_reset(g, m, golden["training"]["opacity_reset_max"])
    op2 = 1 / (1 + np.exp(-g.mo[:, 3].astype(np.float64)))
    low = op <= 0.8
    np.testing.assert_allclose(op2[low], op[low], rtol=1e-6)
    np.testing.assert_allclose(op2[~low], 0.8, rtol=1e-5)
    assert np.all(m.om == 0)


def test_split_normals_are_standard_normal():
    z = np.concatenate([O.split_normals(11, k) for k in range(1, 20001)])
    assert abs(z.mean()) < 0.02 and abs(z.std() - 1) < 0.02
