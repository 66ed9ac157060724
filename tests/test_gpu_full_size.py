"""Full-size checks on the bench workload (3M Gaussians, 1920x1080, 256
hemisphere cameras) and the 4K render-only config 3 (6M Gaussians, 3840x2160). The exact
comparisons with the oracle at these sizes are in test_gpu_parity_configs.py; here the CUDA path
is also held to the properties that hold at any size:

* compaction: keep_gaussians_cs is the inclusive prefix of keep_gaussians, fgidx_to_gidx lists
  the kept Gaussians in order;
* duplication + sort: the sorted codes are non-decreasing, equal codes keep ascending filtered
  indices (the stable sort), every code's depth bits are its Gaussian's depth, every (Gaussian,
  tile) pair appears once and lies in the Gaussian's tile rectangle, each Gaussian appears as
  many times as it overlaps tiles, and tiles_end is the per-tile upper bound of the codes;
* the tile-bucket pipeline and the reference-order pipeline (device radix sort) produce the
  same sorted arrays, tile ends and images bit for bit;
* images: finite colours >= 0, transmittance in (0, 1], last contributors inside their tile;
* backward + update: the rebuilt-SH update equals the update from written SH gradients, and the
  factored rows' geometry equals the dense rows', bit for bit; all gradients finite.
"""
import numpy as np
import pytest
import torch

import gs3d
from gs3d import RenderBuffers, RenderOptions, RenderOutputs, Tiling
from gs3d.backward import (FilteredGaussiansGradients, backward, backward_project_dense,
                           backward_project_factored, backward_raster)
from gs3d.optimizer import AdamOptimizer, LearningRates
from gs3d.scene import CONFIGS, synthetic_gaussians

pytestmark = pytest.mark.gpu


_SCENES = {}


def config_scene(cfg_id, device):
    """Gaussians (on the device) and cameras of a BASELINE config, built once per module."""
    if cfg_id not in _SCENES:
        _SCENES.clear()  # one full-size scene resident at a time
        cfg = CONFIGS[cfg_id]
        _SCENES[cfg_id] = (synthetic_gaussians(cfg["spec"], cfg["seed"]).to(device), cfg["cameras"]())
    return _SCENES[cfg_id]


def render_full(gv, cam, device, reference_order=False):
    opt = RenderOptions.for_camera(cam, 3)
    til = Tiling.for_camera(cam)
    out = RenderOutputs.create(cam.width, cam.height, device)
    buf = RenderBuffers.create(gv.n, til.nb_tiles, device, capacity_dup=8 * gv.n)
    gs3d.render(out, gv, cam, til, opt, buf, reference_order=reference_order)
    torch.cuda.synchronize()
    return out, buf, opt, til


@pytest.mark.parametrize("cfg_id, cam_index", [(4, 0), (4, 131), (3, 0)],
                         ids=["cfg4_cam0", "cfg4_cam131", "cfg3_4k_cam0"])
def test_full_size_forward_properties(cuda, cfg_id, cam_index):
    """Config 4 (3M, 1080p, the bench scene) and config 3 (6M, 3840x2160, 16,320 tiles, 46 key
    bits: the render-only case)."""
    gv, cams = config_scene(cfg_id, cuda)
    cam = cams[cam_index]
    out, buf, opt, til = render_full(gv, cam, cuda)
    n = gv.n
    F, D = gs3d.counts(buf)
    assert int(buf.device_counts[2]) == 0
    assert 0 < F <= n and 0 < D <= buf.capacity_dup

    # compaction
    keep = buf.keep_gaussians[:n].to(torch.int64)
    assert int(keep.max()) <= 1 and int(keep.sum()) == F
    assert torch.equal(buf.keep_gaussians_cs[:n].to(torch.int64), torch.cumsum(keep, 0))
    kept = torch.nonzero(keep).flatten() + 1
    assert torch.equal(buf.fgidx_to_gidx[:F].to(torch.int64), kept)

    # duplication + sort
    codes = buf.sdf2dgs_codes[:D]
    sfg = buf.sdfgidx_to_fgidx[:D].to(torch.int64)
    assert int(sfg.min()) >= 1 and int(sfg.max()) <= F
    assert bool((codes[1:] >= codes[:-1]).all())
    eq = codes[1:] == codes[:-1]
    assert bool((sfg[1:][eq] > sfg[:-1][eq]).all())
    tile = codes >> 32
    depth_bits = (codes & 0xFFFFFFFF).to(torch.int64)
    fg0 = sfg - 1
    want_bits = buf.depths[:F].view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    assert torch.equal(depth_bits, want_bits[fg0])
    tx = (tile - 1) % til.nb_tiles_x + 1
    ty = (tile - 1) // til.nb_tiles_x + 1
    rect = buf.intersected_tile_ranges[:F].to(torch.int64)[fg0]
    assert bool(((rect[:, 0] <= tx) & (tx <= rect[:, 2]) & (rect[:, 1] <= ty) & (ty <= rect[:, 3])).all())
    pair = fg0 * (til.nb_tiles + 1) + tile
    assert torch.unique(pair).numel() == D
    per_fg = torch.bincount(fg0, minlength=F)
    assert torch.equal(per_fg, buf.nb_overlapped_tiles[:F].to(torch.int64))
    ends = buf.tiles_end_sdfgidx[: til.nb_tiles].to(torch.int64)
    want_ends = torch.searchsorted(tile.contiguous(), torch.arange(1, til.nb_tiles + 1, device=cuda),
                                   right=True)
    assert torch.equal(ends, want_ends) and int(ends[-1]) == D

    # images
    rgb, T, last = out.rgb, out.transmittance, out.last_contributing_sdfgids.to(torch.int64)
    assert bool(torch.isfinite(rgb).all()) and float(rgb.min()) >= 0.0
    assert float(T.min()) > 0.0 and float(T.max()) <= 1.0
    w, h = cam.width, cam.height
    u = torch.arange(w, device=cuda).view(w, 1).expand(w, h)
    v = torch.arange(h, device=cuda).view(1, h).expand(w, h)
    pix_tile = (u // til.tile_width) + (v // til.tile_height) * til.nb_tiles_x  # 0-based
    t_end = ends[pix_tile]
    t_start = torch.where(pix_tile > 0, ends[(pix_tile - 1).clamp(min=0)], torch.zeros_like(t_end))
    last2 = last.view(w, h)
    assert bool(((last2 == 0) | ((last2 > t_start) & (last2 <= t_end))).all())

    # the reference-order pipeline (device radix sort) agrees bit for bit
    out_r, buf_r, _, _ = render_full(gv, cam, cuda, reference_order=True)
    assert gs3d.counts(buf_r) == (F, D)
    assert torch.equal(buf_r.sdf2dgs_codes[:D], codes)
    assert torch.equal(buf_r.sdfgidx_to_fgidx[:D], buf.sdfgidx_to_fgidx[:D])
    assert torch.equal(buf_r.tiles_end_sdfgidx[: til.nb_tiles], buf.tiles_end_sdfgidx[: til.nb_tiles])
    for a, b in ((out_r.rgb, rgb), (out_r.transmittance, T), (out_r.last_contributing_sdfgids,
                                                                out.last_contributing_sdfgids)):
        assert torch.equal(a, b)


def test_full_size_backward_and_update_paths_agree(cuda):
    gv, cams = config_scene(4, cuda)
    cam = cams[7]
    g = gv.clone()
    out, buf, opt, til = render_full(g, cam, cuda)
    n = g.n
    grad = torch.from_numpy(np.random.default_rng(5).normal(0, 1e-6, size=(cam.width, cam.height, 3))
                            .astype(np.float32)).to(cuda)
    fg = FilteredGaussiansGradients.create(n, 3, cuda)
    backward(fg, grad, out, g, cam, til, opt, buf)
    torch.cuda.synchronize()
    F, _ = gs3d.counts(buf)
    for t in (fg.mean2d_grads, fg.licov2d_grads, fg.color_grads, fg.mean3d_grads,
              fg.scaling_features_grads, fg.rotation_features_grads, fg.sh_coeffs_grads):
        assert bool(torch.isfinite(t[:F]).all())

    # update from written SH gradients == update with the SH gradients rebuilt
    g2 = g.clone()
    a1 = AdamOptimizer(g, LearningRates(means=0.001))
    a2 = AdamOptimizer(g2, LearningRates(means=0.001))
    a1.update(fg, buf.fgidx_to_gidx, buf.device_counts, 3)
    a2.update_rebuild_sh(fg, buf.fgidx_to_gidx, buf.device_counts, buf.f2d, cam.position, 3)
    torch.cuda.synchronize()
    for x, y in zip(g.tensors(), g2.tensors()):
        assert torch.equal(x, y)
    for x, y in zip(a1.moments.tensors(), a2.moments.tensors()):
        assert torch.equal(x, y)

    # factored rows carry the dense rows' geometry bit for bit (same 2D gradients)
    g3 = gv.clone()
    out3, buf3, _, _ = render_full(g3, cam, cuda)
    fg3 = FilteredGaussiansGradients.create(n, 3, cuda)
    backward_raster(fg3, grad, out3, g3, cam, til, opt, buf3)
    dense = torch.zeros((n, 60), dtype=torch.float32, device=cuda)
    geom = torch.zeros((n, 12), dtype=torch.float32, device=cuda)
    colour = torch.zeros((n, 4), dtype=torch.float32, device=cuda)
    backward_project_dense(fg3, g3, cam, til, opt, buf3, dense, 0, n)
    backward_project_factored(fg3, g3, cam, til, opt, buf3, geom, colour, 0, n)
    torch.cuda.synchronize()
    assert torch.equal(geom, dense[:, 48:60])
    assert torch.equal(colour[:, 3] > 0, dense[:, 59] > 0)
    assert int((dense[:, 59] > 0).sum()) == F
