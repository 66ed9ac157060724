"""Host-side training schedule on the CPU (training.jl:253-302, :313-330): the SH-degree
increase with its resizes of parameters, moments and gradients, and the opacity-reset and
densification predicates, checked against the reference's conditions."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from gs3d import RenderOptions
from gs3d.backward import FilteredGaussiansGradients
from gs3d.optimizer import AdamMoments
from gs3d.scene import SceneSpec, synthetic_gaussians
from gs3d.training import Trainer, TrainingOptions


def _filled(t, seed):
    rng = np.random.default_rng(seed)
    t.copy_(torch.from_numpy(rng.normal(size=t.shape).astype(np.float32)))
    return t


def test_set_sh_degree_keeps_old_coefficients_and_zeros_new_ones():
    g = synthetic_gaussians(SceneSpec(33, "uniform:1", -4.0, 0.5), 0)
    g.set_sh_degree(0)
    m = AdamMoments.zeros(g.n, 0, "cpu")
    fg = FilteredGaussiansGradients.create(g.n, 0, "cpu")
    assert g.sh_degree == 0
    _filled(g.sh_coeffs, 1)
    _filled(m.sh_coeffs_moments, 2)
    dc, mdc = g.sh_coeffs.clone(), m.sh_coeffs_moments.clone()
    for d in (1, 2, 3):
        g.set_sh_degree(d)
        m.set_sh_degree(d)
        fg.set_sh_degree(d)
        S = (d + 1) ** 2
        assert g.sh_coeffs.shape == (g.n, 3, S) and g.sh_degree == d
        assert m.sh_coeffs_moments.shape == (g.n, 3, S, 2) and m.sh_degree == d
        assert fg.sh_coeffs_grads.shape == (fg.capacity, 3, S) and fg.sh_degree == d
        # (S, 3, n) column-major in the reference = (n, 3, S) here: coefficient k of channel c
        assert torch.equal(g.sh_coeffs[:, :, :1], dc)
        assert torch.equal(m.sh_coeffs_moments[:, :, :1], mdc)
        assert not g.sh_coeffs[:, :, 1:].any() and not m.sh_coeffs_moments[:, :, 1:].any()
    # shrinking keeps the leading coefficients
    _filled(g.sh_coeffs, 3)
    keep = g.sh_coeffs[:, :, :4].clone()
    g.set_sh_degree(1)
    assert torch.equal(g.sh_coeffs, keep)


@pytest.mark.parametrize("bad", [-1, 4])
def test_set_sh_degree_rejects_invalid_degrees(bad):
    g = synthetic_gaussians(SceneSpec(4, "uniform:1", -4.0, 0.5), 0)
    with pytest.raises(ValueError):
        g.set_sh_degree(bad)
    with pytest.raises(ValueError):
        AdamMoments.zeros(4, 0, "cpu").set_sh_degree(bad)
    with pytest.raises(ValueError):
        FilteredGaussiansGradients.create(4, 0, "cpu").set_sh_degree(bad)


def _schedule_state(options, n=8):
    """The fields of a Trainer that the schedule methods read and write, on the CPU."""
    g = synthetic_gaussians(SceneSpec(n, "uniform:1", -4.0, 0.5), 0)
    g.set_sh_degree(0)
    return SimpleNamespace(
        options=options, iteration_nb=0, gaussians=g,
        render_options=RenderOptions.create(64, 48, g.sh_degree),
        fgradients=FilteredGaussiansGradients.create(n, g.sh_degree, "cpu"),
        optimizer=SimpleNamespace(moments=AdamMoments.zeros(n, g.sh_degree, "cpu")))


def test_sh_degree_increases_every_interval_up_to_three():
    o = TrainingOptions(scene_radius=1.0, sh_degree_increase_interval=1000)
    t = _schedule_state(o)
    seen = {}
    for it in range(1, 5001):
        t.iteration_nb = it
        Trainer.maybe_increase_sh_degree(t)
        seen[it] = t.gaussians.sh_degree
        assert t.render_options.sh_degree == t.fgradients.sh_degree == seen[it]
        assert t.optimizer.moments.sh_degree == seen[it]
    assert seen[999] == 0 and seen[1000] == 1 and seen[1999] == 1 and seen[2000] == 2
    assert seen[3000] == 3 and seen[4000] == 3 and seen[5000] == 3


def test_opacity_reset_and_densify_predicates(monkeypatch):
    from gs3d import training

    o = TrainingOptions(scene_radius=1.0)
    t = _schedule_state(o)
    resets = []
    monkeypatch.setattr(training.adc_mod, "opacity_reset",
                        lambda g, m, v: resets.append((t.iteration_nb, v)))
    densify = []
    for it in range(0, 16_000):
        t.iteration_nb = it
        Trainer.maybe_opacity_reset(t)
        if Trainer.densifies_this_iteration(t):
            densify.append(it)
    # training.jl:271-280: start <= it <= final and it % interval == 0
    want_resets = [it for it in range(0, 16_000) if 0 <= it <= 12_000 and it % 3_000 == 0]
    assert [r[0] for r in resets] == want_resets and all(v == o.opacity_reset_max_value for _, v in resets)
    # training.jl:313-330: adc_start <= it <= adc_final and it % adc_interval == 0
    assert densify == list(range(600, 14_901, 100))
