"""Render forward on the GPU (through libgs3d.so) against the CPU oracle.

Bar: keep mask, scans, compaction, depths, tile rectangles, duplicate keys, the sorted
key/value arrays and tile ends are bit-exact; images within 1e-4 max abs (they are expected
to be bit-exact too: both sides follow the same operation order and the same exp/log).
"""
import ctypes as C

import numpy as np
import pytest
import torch

import gs3d
from gs3d import RenderBuffers, RenderOptions, RenderOutputs, Tiling
from gs3d.scene import SceneSpec, create_test_scene, look_at_camera, synthetic_gaussians
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def gpu_render(gv, cam, til, opt, device, capacity_dup=None, host_sync=True, reference_order=False):
    g = gv.to(device)
    out = RenderOutputs.create(cam.width, cam.height, device, include_depth=True)
    buf = RenderBuffers.create(g.n, til.nb_tiles, device, capacity_dup=capacity_dup)
    gs3d.render(out, g, cam, til, opt, buf, host_sync=host_sync, reference_order=reference_order)
    torch.cuda.synchronize()
    F, D = gs3d.counts(buf)
    cpu = lambda t: t.cpu().numpy()
    r = dict(F=F, D=D, keep=cpu(buf.keep_gaussians[: g.n]), keep_cs=cpu(buf.keep_gaussians_cs[: g.n]),
             fgidx_to_gidx=cpu(buf.fgidx_to_gidx[:F]), depths=cpu(buf.depths[:F]),
             f2d=cpu(buf.f2d[:F]), ranges=cpu(buf.intersected_tile_ranges[:F]),
             ntiles=cpu(buf.nb_overlapped_tiles[:F]), ntiles_cs=cpu(buf.nb_overlapped_tiles_cs[:F]),
             codes=cpu(buf.df2dgs_codes[:D]), dfg=cpu(buf.dfgidx_to_fgidx[:D]),
             scodes=cpu(buf.sdf2dgs_codes[:D]), sfg=cpu(buf.sdfgidx_to_fgidx[:D]),
             tiles_end=cpu(buf.tiles_end_sdfgidx[: til.nb_tiles]), rgb=cpu(out.rgb),
             trans=cpu(out.transmittance), depth=cpu(out.depth),
             last=cpu(out.last_contributing_sdfgids), status=int(buf.device_counts[2].item()),
             reference_order=reference_order)
    return r, buf


def compare(gpu, ref, exact_images=True):
    """The tile-bucket pipeline (default) leaves the unsorted duplicate arrays and the
    duplicate-count scan unwritten; they are compared in reference-order mode."""
    assert gpu["F"] == ref["F"] and gpu["D"] == ref["D"]
    keys = ["keep", "keep_cs", "fgidx_to_gidx", "ranges", "ntiles", "scodes", "sfg", "last"]
    if gpu["reference_order"]:
        keys += ["ntiles_cs", "codes", "dfg"]
    for k in keys:
        assert np.array_equal(gpu[k], ref[k]), k
    if ref["D"] > 0:
        assert np.array_equal(gpu["tiles_end"], ref["tiles_end"])
    assert np.array_equal(gpu["depths"].view(np.uint32), ref["depths"].view(np.uint32))
    nonempty = ref["ntiles"] > 0
    assert np.array_equal(gpu["f2d"][nonempty].view(np.uint32), ref["f2d"][nonempty].view(np.uint32))
    for k in ("rgb", "trans", "depth"):
        with np.errstate(invalid="ignore"):       # inf - inf where both are the same infinity
            diff = np.abs(gpu[k].astype(np.float64) - ref[k])
        diff[gpu[k] == ref[k]] = 0.0
        assert diff.max() <= 1e-4, (k, diff.max())
        if exact_images:
            assert np.array_equal(gpu[k], ref[k]), (k, np.count_nonzero(gpu[k] != ref[k]))


@pytest.mark.parametrize("reference_order", [False, True])
@pytest.mark.parametrize("deg", [0, 1, 2, 3])
def test_test_scene(cuda, deg, reference_order):
    gv, cams = create_test_scene(deg)
    cam = cams[0]
    opt = RenderOptions.for_camera(cam, deg)
    til = Tiling.for_camera(cam, 16, 16)
    gpu, _ = gpu_render(gv, cam, til, opt, cuda, reference_order=reference_order)
    ref = O.render(O.NpGaussians.from_vector(gv), cam, til, opt)
    compare(gpu, ref)


CASES = [
    # name, spec, seed, (w, h, fov, pos), tile, options kwargs, render degree
    ("cfg0", SceneSpec(16_384, "uniform:1", -4.0, 0.5), 0, (256, 256, 60.0, (0, 0, 3)), None, {}, 3),
    ("cfg0_filter", SceneSpec(16_384, "uniform:1", -4.0, 0.5), 0, (256, 256, 60.0, (0, 0, 3)), None,
     dict(clipping_mode=gs3d.FILTER), 3),
    ("cfg0_aa_bg", SceneSpec(16_384, "uniform:1", -4.0, 0.5), 5, (256, 256, 60.0, (0.3, 0.2, 2.5)),
     None, dict(use_antialiasing=True, background=(0.2, 0.5, 0.9)), 3),
    ("deg1_of3", SceneSpec(20_000, "uniform:1.5", -4.5, 0.5), 6, (320, 200, 70.0, (0, 1, 3)), None, {}, 1),
    ("ragged_720p", SceneSpec(60_000, "uniform:3", -4.0, 0.6), 7, (1280, 720, 50.0, (0, 1.5, 6)),
     (16, 16), {}, 3),
    ("big_tiles_1080", SceneSpec(40_000, "normal:1.5", -4.0, 0.5), 8, (1920, 1080, 50.0, (1, 2, 5)),
     (16, 32), {}, 2),
    ("odd_size", SceneSpec(5_000, "uniform:1", -3.5, 0.5), 9, (333, 171, 80.0, (0, 0, 2.2)), (32, 8), {}, 0),
]


@pytest.mark.parametrize("reference_order", [False, True])
@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_random_scenes(cuda, case, reference_order):
    _, spec, seed, (w, h, fov, pos), tile, kw, deg = case
    gv = synthetic_gaussians(spec, seed)
    cam = look_at_camera(w, h, fov, pos)
    opt = RenderOptions.for_camera(cam, deg, **kw)
    til = Tiling.for_camera(cam, *(tile or (None, None)))
    gpu, _ = gpu_render(gv, cam, til, opt, cuda, reference_order=reference_order)
    ref = O.render(O.NpGaussians.from_vector(gv), cam, til, opt)
    assert ref["F"] > 0 and ref["D"] > 0
    compare(gpu, ref)


def test_empty_and_void(cuda):
    cam = look_at_camera(64, 48, 60.0, (0, 0, 3))
    til = Tiling.for_camera(cam)
    opt = RenderOptions.for_camera(cam, 0, background=(0.1, 0.2, 0.3))
    # n = 0
    empty = synthetic_gaussians(SceneSpec(0, "uniform:1", -4, 0.5, sh_degree=0), 0)
    gpu, _ = gpu_render(empty, cam, til, opt, cuda, reference_order=True)
    assert gpu["F"] == 0 and np.all(gpu["trans"] == 1) and np.all(np.isinf(gpu["depth"]))
    assert np.allclose(gpu["rgb"], [0.1, 0.2, 0.3]) and np.all(gpu["last"] == 0)
    # everything behind the camera: F = 0
    gv = synthetic_gaussians(SceneSpec(100, "uniform:0.5", -4, 0.5, sh_degree=0), 1)
    gv.means_opacity_features[:, 2] += 10.0  # z in [9.5, 10.5], camera at z=3 looking at -z
    gpu, _ = gpu_render(gv, cam, til, opt, cuda)
    ref = O.render(O.NpGaussians.from_vector(gv), cam, til, opt)
    assert gpu["F"] == ref["F"] == 0
    compare(gpu, ref)
    # in front but far off-screen: F > 0, D = 0
    gv = synthetic_gaussians(SceneSpec(100, "uniform:0.5", -6, 0.1, sh_degree=0), 2)
    gv.means_opacity_features[:, 0] += 50.0
    gpu, _ = gpu_render(gv, cam, til, opt, cuda)
    ref = O.render(O.NpGaussians.from_vector(gv), cam, til, opt)
    assert ref["F"] > 0 and ref["D"] == 0
    compare(gpu, ref)


@pytest.mark.parametrize("reference_order", [False, True])
def test_dup_capacity_growth_and_overflow_flag(cuda, reference_order):
    gv = synthetic_gaussians(SceneSpec(16_384, "uniform:1", -4.0, 0.5), 0)
    cam = look_at_camera(256, 256, 60.0, (0, 0, 3))
    opt = RenderOptions.for_camera(cam, 3)
    til = Tiling.for_camera(cam)
    ref = O.render(O.NpGaussians.from_vector(gv), cam, til, opt)
    gpu, buf = gpu_render(gv, cam, til, opt, cuda, capacity_dup=1000,
                          reference_order=reference_order)  # grows and retries
    assert buf.capacity_dup >= ref["D"]
    compare(gpu, ref)
    gpu, _ = gpu_render(gv, cam, til, opt, cuda, capacity_dup=1000, host_sync=False,
                        reference_order=reference_order)
    assert gpu["status"] & 1  # GS3D_STATUS_DUP_OVERFLOW, outputs undefined but in bounds


@pytest.mark.parametrize("n", [20_000, 120_000])
def test_large_tile_segments(cuda, n):
    """Tiles with more entries than the shared-memory segment sort holds (4096): 64 x 64 pixels
    in 16 tiles, segments of several thousand (n = 20K) and above 8192 (n = 120K), sorted in
    global memory; sorted arrays, tile ends and images as the oracle's."""
    gv = synthetic_gaussians(SceneSpec(n, "uniform:0.6", -5.0, 0.4), 12)
    cam = look_at_camera(64, 64, 60.0, (0, 0, 3))
    opt = RenderOptions.for_camera(cam, 3)
    til = Tiling.for_camera(cam, 16, 16)
    gpu, _ = gpu_render(gv, cam, til, opt, cuda)
    ref = O.render(O.NpGaussians.from_vector(gv), cam, til, opt)
    seg = np.diff(np.concatenate([[0], ref["tiles_end"]]))
    assert seg.max() > (8192 if n > 100_000 else 4096)
    compare(gpu, ref)


def _sort_gpu(keys, vals, bits, device):
    lib = gs3d.lib()
    n = keys.size
    k_in = torch.from_numpy(keys).to(device)
    v_in = torch.from_numpy(vals).to(device)
    k_out = torch.empty_like(k_in)
    v_out = torch.empty_like(v_in)
    nbytes = lib.determine_sort_pairs_temp_storage(None, None, None, None, n, bits)
    tmp = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
    torch.cuda.synchronize()
    lib.sort_pairs(C.c_void_p(tmp.data_ptr()), nbytes, C.c_void_p(k_in.data_ptr()),
                   C.c_void_p(k_out.data_ptr()), C.c_void_p(v_in.data_ptr()),
                   C.c_void_p(v_out.data_ptr()), n, bits)
    torch.cuda.synchronize()
    assert np.array_equal(k_in.cpu().numpy(), keys)  # input untouched
    return k_out.cpu().numpy(), v_out.cpu().numpy()


@pytest.mark.parametrize("n,bits", [(1, 35), (7, 35), (4096, 41), (4097, 44), (100_003, 46),
                                    (250_000, 64), (10_000, 8), (10_000, 1)])
def test_sort_pairs_dropin(cuda, n, bits):
    rng = np.random.default_rng(n + bits)
    keys = rng.integers(0, 1 << 62, n, dtype=np.int64)
    keys[: n // 3] = keys[0]  # many exact duplicates: stability matters
    vals = rng.permutation(n).astype(np.int32)
    ko, vo = _sort_gpu(keys, vals, bits, cuda)
    rk, rv = O.sort_pairs(keys, vals, bits)
    assert np.array_equal(ko, rk) and np.array_equal(vo, rv)


@pytest.mark.parametrize("dist,n,bits", [("tiles", 2_000_000, 44), ("tiles", 700_001, 46),
                                          ("one_bucket", 300_000, 40), ("low_ties", 500_000, 36),
                                          ("random", 123_457, 33), ("random", 1_000_000, 46)])
def test_sort_pairs_bucket_path(cuda, dist, n, bits):
    """Key widths 33..46 take the bucket path (bits above 32 pick a bucket, each bucket sorted in
    shared memory): render-like keys tile << 32 | depth bits, every key in one bucket (the
    global-memory network), many equal low words (stability), random keys with bits above
    highest_key_bit set (ignored by the order, kept in the output)."""
    rng = np.random.default_rng(n + bits)
    nb = 1 << (bits - 32)
    if dist == "tiles":
        tiles = rng.integers(1, nb, n)
        depth = rng.uniform(0.2, 50.0, n).astype(np.float32).view(np.int32).astype(np.int64)
        keys = (tiles.astype(np.int64) << 32) | depth
    elif dist == "one_bucket":
        keys = (np.int64(5) << 32) | rng.integers(0, 1 << 32, n, dtype=np.int64)
    elif dist == "low_ties":
        keys = (rng.integers(0, nb, n).astype(np.int64) << 32) | rng.integers(0, 50, n)
    else:
        keys = rng.integers(0, 1 << 62, n, dtype=np.int64)
    vals = rng.permutation(n).astype(np.int32)
    ko, vo = _sort_gpu(keys, vals, bits, cuda)
    rk, rv = O.sort_pairs(keys, vals, bits)
    assert np.array_equal(ko, rk) and np.array_equal(vo, rv)


def _reference_sort_lib():
    """The reference's own CUB wrapper (deps/cub_sort_pairs/cub_sort_pairs_wrapper.cu),
    compiled from the reference checkout by oracle/build.py into oracle/_ref/."""
    from oracle.build import REF_LIB
    if not REF_LIB.exists():
        pytest.skip("reference CUB sort wrapper was not built (no reference checkout at build time)")
    lib = C.CDLL(str(REF_LIB))
    lib.determine_sort_pairs_temp_storage.restype = C.c_size_t
    lib.determine_sort_pairs_temp_storage.argtypes = [C.c_void_p] * 4 + [C.c_int, C.c_int]
    lib.sort_pairs.restype = None
    lib.sort_pairs.argtypes = [C.c_void_p, C.c_size_t] + [C.c_void_p] * 4 + [C.c_int, C.c_int]
    return lib


@pytest.mark.parametrize("n,bits", [(5, 35), (4097, 44), (300_001, 46), (1_000_000, 64)])
def test_sort_pairs_matches_reference_cub_wrapper(cuda, n, bits):
    """Same inputs through the reference's CUB DeviceRadixSort wrapper and through libgs3d's
    drop-in: identical keys and values (CUB's sort is stable, so the result is unique)."""
    ref = _reference_sort_lib()
    rng = np.random.default_rng(7 * n + bits)
    keys = rng.integers(0, 1 << 62, n, dtype=np.int64)
    keys[: n // 4] = keys[n // 2]
    vals = rng.permutation(n).astype(np.int32)
    ko, vo = _sort_gpu(keys, vals, bits, cuda)
    k_in = torch.from_numpy(keys).to(cuda)
    v_in = torch.from_numpy(vals).to(cuda)
    k_out, v_out = torch.empty_like(k_in), torch.empty_like(v_in)
    nbytes = ref.determine_sort_pairs_temp_storage(None, None, None, None, n, bits)
    tmp = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=cuda)
    torch.cuda.synchronize()
    ref.sort_pairs(tmp.data_ptr(), nbytes, k_in.data_ptr(), k_out.data_ptr(), v_in.data_ptr(),
                   v_out.data_ptr(), n, bits)
    torch.cuda.synchronize()
    assert np.array_equal(ko, k_out.cpu().numpy()) and np.array_equal(vo, v_out.cpu().numpy())


@pytest.mark.parametrize("levels", [1, 40])
def test_equal_depths_sort_by_filtered_index(cuda, levels):
    """Gaussians on planes facing the camera share their depth bits exactly: within a tile they
    must come in filtered-index order (the reference's stable sort). One plane gives runs
    longer than the per-run fix-up handles (whole-segment bitonic instead); 40 planes give
    short runs."""
    gv = synthetic_gaussians(SceneSpec(6_000, "uniform:1", -4.0, 0.5), 13)
    z = np.floor(np.random.default_rng(1).uniform(0, levels, gv.n)) * 0.01
    gv.means_opacity_features[:, 2] = torch.from_numpy(z.astype(np.float32))
    cam = look_at_camera(128, 128, 60.0, (0, 0, 3))
    opt = RenderOptions.for_camera(cam, 3)
    til = Tiling.for_camera(cam, 16, 16)
    ref = O.render(O.NpGaussians.from_vector(gv), cam, til, opt)
    d = ref["depths"]
    assert len(np.unique(d)) <= levels and ref["D"] > 0
    gpu, _ = gpu_render(gv, cam, til, opt, cuda)
    compare(gpu, ref)


RO_CASES = [c for c in CASES if c[0] in ("cfg0", "cfg0_filter", "cfg0_aa_bg", "ragged_720p", "odd_size")]


@pytest.mark.parametrize("case", RO_CASES, ids=[c[0] for c in RO_CASES])
def test_render_only_input_matches_oracle(cuda, case):
    """RenderOnlyGaussiansVector (stored opacities and 3D covariances, gaussians.jl:342-392):
    gs3d_render_forward_render_only against the oracle's render-only path, bit for bit; and the
    same Gaussians rendered from their features agree to float rounding (the 2D covariance is
    J V J^T instead of (J R S)(J R S)^T, so rare pixels flip at the alpha thresholds)."""
    from gs3d import RenderOnlyGaussiansVector
    _, spec, seed, (w, h, fov, pos), tile, kw, deg = case
    gv = synthetic_gaussians(spec, seed)
    cam = look_at_camera(w, h, fov, pos)
    opt = RenderOptions.for_camera(cam, deg, **kw)
    til = Tiling.for_camera(cam, *(tile or (None, None)))
    ro = RenderOnlyGaussiansVector.from_trainable(gv)
    gpu, _ = gpu_render(ro, cam, til, opt, cuda)
    ref = O.render(O.NpRenderOnlyGaussians(*(t.numpy() for t in ro.tensors())), cam, til, opt)
    compare(gpu, ref)
    tr, _ = gpu_render(gv, cam, til, opt, cuda)
    d = np.abs(gpu["rgb"].astype(np.float64) - tr["rgb"])
    assert np.mean(d <= 1e-4) >= 0.999 and d.mean() <= 1e-5, (d.max(), d.mean())


@pytest.mark.parametrize("case", [c for c in CASES if c[0] in ("cfg0", "cfg0_aa_bg", "ragged_720p",
                                                                "big_tiles_1080", "odd_size")],
                         ids=lambda c: c[0])
def test_work_counts_vs_oracle(cuda, case):
    """gs3d_render_work_counts (blends and contributions of the reference's blend loop) equal
    the oracle's counts over the same render."""
    from gs3d.render import work_counts
    _, spec, seed, (w, h, fov, pos), tile, kw, deg = case
    gv = synthetic_gaussians(spec, seed)
    cam = look_at_camera(w, h, fov, pos)
    opt = RenderOptions.for_camera(cam, deg, **kw)
    til = Tiling.for_camera(cam, *(tile or (None, None)))
    _, buf = gpu_render(gv, cam, til, opt, cuda)
    blends, contrib = work_counts(cam, til, opt, buf)
    ref = O.render(O.NpGaussians.from_vector(gv), cam, til, opt)
    want = O.work_counts(ref, cam, til, opt)
    assert (blends, contrib) == want
    assert 0 < contrib <= blends


@pytest.mark.parametrize("case", [c for c in CASES if c[0] in ("cfg0", "ragged_720p", "big_tiles_1080")],
                         ids=lambda c: c[0])
def test_tile_order(cuda, case):
    """RenderBuffers.tile_order: a permutation of the tiles by non-increasing bucket of their
    duplicate counts (8 per octave); the render with it equals the row-major render bit for bit
    (outputs and contribution masks)."""
    _, spec, seed, (w, h, fov, pos), tile, kw, deg = case
    gv = synthetic_gaussians(spec, seed)
    cam = look_at_camera(w, h, fov, pos)
    opt = RenderOptions.for_camera(cam, deg, **kw)
    til = Tiling.for_camera(cam, *(tile or (None, None)))
    g = gv.to(cuda)
    res = []
    for order in (True, False):
        out = RenderOutputs.create(cam.width, cam.height, cuda, include_depth=True)
        buf = RenderBuffers.create(g.n, til.nb_tiles, cuda, tile_order=order, mask_dup=16 * g.n)
        buf.contrib_masks.zero_()
        gs3d.render(out, g, cam, til, opt, buf)
        torch.cuda.synchronize()
        res.append((out, buf))
    (o1, b1), (o2, b2) = res
    T = til.nb_tiles
    order = b1.tile_order[:T].cpu().numpy()
    assert np.array_equal(np.sort(order), np.arange(T))
    ends = b1.tiles_end_sdfgidx[:T].cpu().numpy().astype(np.int64)
    n = np.diff(np.concatenate([[0], ends]))
    assert n.sum() > 0
    e = np.floor(np.log2(np.maximum(n, 1))).astype(np.int64)
    m = np.where(e >= 3, n >> np.maximum(e - 3, 0), n << np.maximum(3 - e, 0)) & 7
    bucket = np.where(n > 0, 1 + 8 * e + m, 0)
    assert np.all(np.diff(bucket[order]) <= 0)
    for a, b in ((o1.rgb, o2.rgb), (o1.transmittance, o2.transmittance), (o1.depth, o2.depth),
                 (o1.last_contributing_sdfgids, o2.last_contributing_sdfgids),
                 (b1.contrib_masks, b2.contrib_masks)):
        assert torch.equal(a, b)
    assert int(b1.device_counts[3]) == 1


@pytest.mark.parametrize("case", [c for c in CASES if c[0] in ("cfg0", "ragged_720p", "deg1_of3")],
                         ids=lambda c: c[0])
def test_deferred_colour_render_equals_render(cuda, case):
    """render(defer_colour=True) (filter, projection without colours, duplication, sort) followed
    by render_colour (colours, blend) gives the render's outputs and buffers bit for bit."""
    from gs3d.render import render_colour
    _, spec, seed, (w, h, fov, pos), tile, kw, deg = case
    gv = synthetic_gaussians(spec, seed)
    cam = look_at_camera(w, h, fov, pos)
    opt = RenderOptions.for_camera(cam, deg, **kw)
    til = Tiling.for_camera(cam, *(tile or (None, None)))
    one, buf1 = gpu_render(gv, cam, til, opt, cuda)
    g = gv.to(cuda)
    out = RenderOutputs.create(cam.width, cam.height, cuda, include_depth=True)
    buf = RenderBuffers.create(g.n, til.nb_tiles, cuda)
    gs3d.render(out, g, cam, til, opt, buf, defer_colour=True)
    render_colour(out, g, cam, til, opt, buf)
    torch.cuda.synchronize()
    F, D = one["F"], one["D"]
    assert gs3d.counts(buf) == (F, D)
    for a, b in ((out.rgb, one["rgb"]), (out.transmittance, one["trans"]), (out.depth, one["depth"]),
                 (out.last_contributing_sdfgids, one["last"]), (buf.f2d[:F], one["f2d"]),
                 (buf.sdfgidx_to_fgidx[:D], one["sfg"])):
        assert np.array_equal(a.cpu().numpy().view(np.uint32) if a.dtype == torch.float32 else a.cpu().numpy(),
                              b.view(np.uint32) if b.dtype == np.float32 else b)


@pytest.mark.parametrize("case", [c for c in CASES if c[0] in ("cfg0", "ragged_720p", "deg1_of3")],
                         ids=lambda c: c[0])
def test_given_colour_render_equals_render(cuda, case):
    """shard_sh's render: colours computed per owner sub-range (gs3d_shard_colours, here for 3
    ranks x 2 views x 2 chunks, the camera under test as view 1 of rank 0), laid out as rank 0
    receives them, then render(defer_colour=True) + gs3d_render_forward_given_colour: the
    render's outputs and buffers bit for bit."""
    from gs3d.dp import chunk_layout, given_colour_row
    from gs3d.render import render_given_colour, shard_colours
    _, spec, seed, (w, h, fov, pos), tile, kw, deg = case
    gv = synthetic_gaussians(spec, seed)
    cam = look_at_camera(w, h, fov, pos)
    opt = RenderOptions.for_camera(cam, deg, **kw)
    til = Tiling.for_camera(cam, *(tile or (None, None)))
    one, _ = gpu_render(gv, cam, til, opt, cuda)
    g = gv.to(cuda)
    n = g.n
    world, views, chunks = 3, 2, 2
    S, C_ = chunk_layout(n, world, chunks)
    # slot r * V + v: view v of rank r; rank 0's view 1 is the camera under test
    slots = [look_at_camera(w, h, fov, (0.3 * s_, 1.0, 4.0)).position for s_ in range(world * views)]
    slots[0 * views + 1] = cam.position
    slots = np.array(slots, dtype=np.float32)
    recv = torch.full((chunks, world * views * S, 4), float("nan"), device=cuda)
    tmp = torch.empty((world * views * S, 4), device=cuda)
    for c in range(chunks):
        for q in range(world):  # owner q's block for rank 0: its slots 0 * V + v
            lo, hi = c * C_ + q * S, min(c * C_ + (q + 1) * S, n)
            if lo >= hi:
                continue
            shard_colours(g, deg, slots, lo, hi, tmp, S)
            for v in range(views):
                recv[c, (q * views + v) * S:(q * views + v) * S + (hi - lo)] = \
                    tmp[(0 * views + v) * S:(0 * views + v) * S + (hi - lo)]
    flat = recv.reshape(-1, 4)
    gi = 12345 % n
    assert given_colour_row(gi, S, world, views, 1) < flat.shape[0]
    out = RenderOutputs.create(cam.width, cam.height, cuda, include_depth=True)
    buf = RenderBuffers.create(g.n, til.nb_tiles, cuda)
    gs3d.render(out, g, cam, til, opt, buf, defer_colour=True)
    render_given_colour(out, g, cam, til, opt, buf, recv, S, world, views, 1)
    torch.cuda.synchronize()
    F, D = one["F"], one["D"]
    assert gs3d.counts(buf) == (F, D)
    for a, b in ((out.rgb, one["rgb"]), (out.transmittance, one["trans"]), (out.depth, one["depth"]),
                 (out.last_contributing_sdfgids, one["last"]), (buf.f2d[:F], one["f2d"])):
        assert np.array_equal(a.cpu().numpy().view(np.uint32) if a.dtype == torch.float32 else a.cpu().numpy(),
                              b.view(np.uint32) if b.dtype == np.float32 else b)
