"""ctypes front end of the CPU oracle — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs may import
this module, and only as the checker or the timed CPU baseline, never as a product path.
The C++ it loads restates ThreeDGaussianSplatting.jl (see the .cpp headers for file:line).

Parity pinning: the oracle is checked against every golden vector of the reference's own
tests (tests/test_oracle_golden.py, fixtures in tests/golden/); the SSIM term of the loss is
the exception (FastCUDASSIM is not vendored: parity unpinned).
"""
from __future__ import annotations

import ctypes as C
import sys
from pathlib import Path

import numpy as np

_REPO = Path(__file__).resolve().parent.parent
_PKG = _REPO / "threedgaussiansplatting.jl_b200"
if str(_PKG) not in sys.path:
    sys.path.insert(0, str(_PKG))

from gs3d import _abi  # noqa: E402  (ctypes mirrors of include/gs3d.h)

from . import build as _build  # noqa: E402

_LIB = None


def lib():
    global _LIB
    if _LIB is None:
        path = _build.build_oracle()
        _LIB = C.CDLL(str(path))
        vp = C.c_void_p
        P = C.POINTER
        _LIB.oracle_render.restype = C.c_int
        _LIB.oracle_render.argtypes = [P(_abi.GaussiansC), P(_abi.Camera), P(_abi.TilingC),
                                       P(_abi.RenderOptionsC)] + [vp] * 8 + [C.c_int64] + [vp] * 10
        _LIB.oracle_render_ro.restype = C.c_int
        _LIB.oracle_render_ro.argtypes = [P(_abi.GaussiansC), vp, P(_abi.Camera), P(_abi.TilingC),
                                          P(_abi.RenderOptionsC)] + [vp] * 8 + [C.c_int64] + [vp] * 10
        _LIB.oracle_backward.restype = C.c_int
        _LIB.oracle_backward.argtypes = [P(_abi.GaussiansC), P(_abi.Camera), P(_abi.TilingC),
                                         P(_abi.RenderOptionsC), C.c_int32] + [vp] * 7 + \
            [C.c_uint32] + [vp] * 9 + [C.c_int32]
        _LIB.oracle_backward_ex.restype = C.c_int
        _LIB.oracle_backward_ex.argtypes = _LIB.oracle_backward.argtypes + [C.c_int32, vp]
        _LIB.oracle_sort_pairs.restype = C.c_int
        _LIB.oracle_sort_pairs.argtypes = [vp, vp, vp, vp, C.c_int64, C.c_int]
        _LIB.oracle_cpu_render.restype = C.c_int32
        _LIB.oracle_cpu_render.argtypes = [P(_abi.GaussiansC), P(_abi.Camera),
                                           P(_abi.RenderOptionsC), vp, vp, vp, C.c_int32]
        _LIB.oracle_adam.restype = C.c_int
        _LIB.oracle_adam.argtypes = [P(_abi.GaussiansC), P(_abi.AdamMomentsC), P(_abi.FGradientsC),
                                     vp, C.c_int32, P(_abi.AdamParamsC), C.c_float, C.c_float]
        _LIB.oracle_loss.restype = C.c_int
        _LIB.oracle_loss.argtypes = [vp, vp, C.c_int32, C.c_int32, C.c_float, vp, vp]
        _LIB.oracle_adc_stats.restype = C.c_int
        _LIB.oracle_adc_stats.argtypes = [vp, vp, vp, vp, C.c_int32, C.c_int32, C.c_int32]
        _LIB.oracle_adc_plan.restype = C.c_int32
        _LIB.oracle_adc_plan.argtypes = [P(_abi.GaussiansC), vp, vp, P(_abi.AdcParamsC)] + [vp] * 7
        _LIB.oracle_adc_apply.restype = C.c_int
        _LIB.oracle_adc_apply.argtypes = [P(_abi.GaussiansC), P(_abi.AdamMomentsC),
                                          P(_abi.GaussiansC), P(_abi.AdamMomentsC)] + [vp] * 5 + \
            [C.c_int32, C.c_float, C.c_uint64]
        _LIB.oracle_opacity_reset.restype = C.c_int
        _LIB.oracle_opacity_reset.argtypes = [P(_abi.GaussiansC), P(_abi.AdamMomentsC), C.c_float]
        _LIB.oracle_expf.restype = C.c_float
        _LIB.oracle_expf.argtypes = [C.c_float]
        _LIB.oracle_logf.restype = C.c_float
        _LIB.oracle_logf.argtypes = [C.c_float]
        _LIB.oracle_split_normals.restype = None
        _LIB.oracle_split_normals.argtypes = [C.c_uint64, C.c_uint64, vp]
        _LIB.oracle_work_counts.restype = None
        _LIB.oracle_work_counts.argtypes = [vp, vp, vp, P(_abi.Camera), P(_abi.TilingC),
                                            P(_abi.RenderOptionsC), vp]
        _LIB.oracle_set_threads.restype = None
        _LIB.oracle_set_threads.argtypes = [C.c_int32]
        _LIB.oracle_compact.restype = C.c_int32
        _LIB.oracle_compact.argtypes = [vp, C.c_int64, vp, vp]
        _LIB.oracle_dup_keys.restype = C.c_int64
        _LIB.oracle_dup_keys.argtypes = [C.c_int32, vp, vp, vp, C.c_int32, vp, vp]
        _LIB.oracle_tiles_end.restype = None
        _LIB.oracle_tiles_end.argtypes = [vp, C.c_int64, C.c_int32, vp]
    return _LIB


def compact(keep: np.ndarray):
    keep = np.ascontiguousarray(keep, np.uint8)
    cs = np.zeros(keep.size, np.int32)
    f2g = np.zeros(keep.size, np.int32)
    F = lib().oracle_compact(_p(keep), keep.size, _p(cs), _p(f2g))
    return cs, f2g[:F]


def dup_keys(ntiles: np.ndarray, ranges: np.ndarray, depths: np.ndarray, tiles_x: int):
    ntiles = np.ascontiguousarray(ntiles, np.int32)
    ranges = np.ascontiguousarray(ranges, np.int32).reshape(-1, 4)
    depths = np.ascontiguousarray(depths, np.float32)
    D = int(ntiles.sum())
    codes = np.zeros(max(D, 1), np.int64)
    dfg = np.zeros(max(D, 1), np.int32)
    lib().oracle_dup_keys(ntiles.size, _p(ntiles), _p(ranges), _p(depths), tiles_x, _p(codes), _p(dfg))
    return codes[:D], dfg[:D]


def tiles_end(scodes: np.ndarray, nb_tiles: int):
    scodes = np.ascontiguousarray(scodes, np.int64)
    out = np.zeros(nb_tiles, np.int32)
    lib().oracle_tiles_end(_p(scodes), scodes.size, nb_tiles, _p(out))
    return out


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class NpGaussians:
    """Gaussians as C-contiguous float32 numpy arrays in the reference layouts."""

    def __init__(self, means_opacity_features, scaling_features, rotation_features, sh_coeffs):
        f = lambda a: np.ascontiguousarray(np.asarray(a, dtype=np.float32))
        self.mo, self.sf, self.rf, self.sh = map(f, (means_opacity_features, scaling_features,
                                                     rotation_features, sh_coeffs))

    @classmethod
    def from_vector(cls, gv) -> "NpGaussians":
        return cls(*(t.detach().cpu().numpy() for t in gv.tensors()))

    @property
    def n(self):
        return self.mo.shape[0]

    @property
    def sh_degree(self):
        return int(round(np.sqrt(self.sh.shape[2]))) - 1

    def to_c(self):
        g = _abi.GaussiansC()
        g.n, g.sh_degree = self.n, self.sh_degree
        g.means_opacity_features = _p(self.mo)
        g.scaling_features = _p(self.sf)
        g.rotation_features = _p(self.rf)
        g.sh_coeffs = _p(self.sh)
        return g

    def copy(self):
        return NpGaussians(self.mo.copy(), self.sf.copy(), self.rf.copy(), self.sh.copy())


class NpRenderOnlyGaussians:
    """RenderOnlyGaussiansVector (gaussians.jl:342-392) as numpy arrays: (n, 4) x y z opacity,
    (n, 6) lower covariances (11 21 31 22 32 33), (n, 3, (d+1)^2) SH coefficients."""

    def __init__(self, means_opacities, covariances, sh_coeffs):
        f = lambda a: np.ascontiguousarray(np.asarray(a, dtype=np.float32))
        self.mo, self.cov, self.sh = map(f, (means_opacities, covariances, sh_coeffs))

    @property
    def n(self):
        return self.mo.shape[0]

    @property
    def sh_degree(self):
        return int(round(np.sqrt(self.sh.shape[2]))) - 1

    def to_c(self):
        g = _abi.GaussiansC()
        g.n, g.sh_degree = self.n, self.sh_degree
        g.means_opacity_features = _p(self.mo)
        g.sh_coeffs = _p(self.sh)
        return g


def render(g, camera, tiling, options, dup_capacity: int | None = None) -> dict:
    """GPU-path render restatement; returns every intermediate in reference layouts. `g` is an
    NpGaussians or an NpRenderOnlyGaussians."""
    n, W, H = g.n, camera.width, camera.height
    cap = max(n, 1)
    out = dict(
        keep=np.zeros(cap, np.uint8), keep_cs=np.zeros(cap, np.int32),
        fgidx_to_gidx=np.zeros(cap, np.int32), depths=np.zeros(cap, np.float32),
        f2d=np.zeros((cap, 9), np.float32), ranges=np.zeros((cap, 4), np.int32),
        ntiles=np.zeros(cap, np.int32), ntiles_cs=np.zeros(cap, np.int32),
        tiles_end=np.zeros(tiling.nb_tiles, np.int32), rgb=np.zeros((W, H, 3), np.float32),
        trans=np.zeros((W, H), np.float32), depth=np.zeros((W, H), np.float32),
        last=np.zeros((W, H), np.int32))
    counts = np.zeros(2, np.int64)
    dc = dup_capacity or max(4 * n, 1024)
    gc, cc, tc, oc = g.to_c(), camera.to_c(), tiling.to_c(), options.to_c()
    while True:
        dup = dict(codes=np.zeros(dc, np.int64), dfg=np.zeros(dc, np.int32),
                   scodes=np.zeros(dc, np.int64), sfg=np.zeros(dc, np.int32))
        ro = isinstance(g, NpRenderOnlyGaussians)
        head = ((lib().oracle_render_ro, C.byref(gc), _p(g.cov)) if ro
                else (lib().oracle_render, C.byref(gc)))
        st = head[0](*head[1:], C.byref(cc), C.byref(tc), C.byref(oc),
                                 _p(out["keep"]), _p(out["keep_cs"]), _p(out["fgidx_to_gidx"]),
                                 _p(out["depths"]), _p(out["f2d"]), _p(out["ranges"]),
                                 _p(out["ntiles"]), _p(out["ntiles_cs"]), dc, _p(dup["codes"]),
                                 _p(dup["dfg"]), _p(dup["scodes"]), _p(dup["sfg"]),
                                 _p(out["tiles_end"]), _p(out["rgb"]), _p(out["trans"]),
                                 _p(out["depth"]), _p(out["last"]), _p(counts))
        if st == _abi.GS3D_ERR_CAPACITY:
            dc = int(counts[1]) + 16
            continue
        assert st == 0
        break
    F, D = int(counts[0]), int(counts[1])
    out.update(dup)
    out["F"], out["D"] = F, D
    for k in ("keep", "keep_cs"):
        out[k] = out[k][:n]
    for k in ("fgidx_to_gidx", "depths", "f2d", "ranges", "ntiles", "ntiles_cs"):
        out[k] = out[k][:F]
    for k in ("codes", "dfg", "scodes", "sfg"):
        out[k] = out[k][:D]
    return out


def work_counts(fwd: dict, camera, tiling, options) -> tuple[int, int]:
    """(blends, contributions) of the blend loop over a render() result: (pixel, Gaussian)
    evaluations until each pixel stops, and the evaluations blended into a pixel."""
    out = np.zeros(2, np.int64)
    if fwd["D"] == 0:
        return 0, 0
    cc, tc, oc = camera.to_c(), tiling.to_c(), options.to_c()
    lib().oracle_work_counts(_p(np.ascontiguousarray(fwd["f2d"])), _p(np.ascontiguousarray(fwd["sfg"])),
                             _p(fwd["tiles_end"]), C.byref(cc), C.byref(tc), C.byref(oc), _p(out))
    return int(out[0]), int(out[1])


def backward(g: NpGaussians, camera, tiling, options, fwd: dict, rgb_grad: np.ndarray,
             flags: int = 0, sh_grad_degree: int | None = None, grads_2d: dict | None = None,
             with_magnitudes: bool = False) -> dict:
    """backward! restated. `grads_2d` (mean2d, opacity, licov, color arrays of F rows): run only
    the projection backward on these 2D gradients. `with_magnitudes`: also return "mag", per
    filtered Gaussian the sums of the absolute per-pixel terms of the 9 2D gradient components
    (mean2d 2, opacity 1, licov 3, colour 3), each term evaluated on absolute values (its
    colour differences taken as sums of magnitudes): the scale of float rounding errors."""
    F = fwd["F"]
    d = g.sh_degree if sh_grad_degree is None else sh_grad_degree
    S = (d + 1) ** 2
    cap = max(F, 1)
    o = dict(mean2d=np.zeros((cap, 2), np.float32), opacity=np.zeros(cap, np.float32),
             licov=np.zeros((cap, 3), np.float32), color=np.zeros((cap, 3), np.float32),
             mean3d=np.zeros((cap, 3), np.float32), opacity_feature=np.zeros(cap, np.float32),
             scaling=np.zeros((cap, 3), np.float32), rotation=np.zeros((cap, 4), np.float32),
             sh=np.zeros((cap, 3, S), np.float32))
    if grads_2d is not None:
        for k, shape in (("mean2d", (F, 2)), ("opacity", (F,)), ("licov", (F, 3)), ("color", (F, 3))):
            o[k][:F] = np.asarray(grads_2d[k], np.float32).reshape(shape)
    mag = np.zeros((cap, 9), np.float32) if with_magnitudes else None
    rg = np.ascontiguousarray(rgb_grad, dtype=np.float32)
    sfg = fwd["sfg"] if fwd["D"] > 0 else np.zeros(1, np.int32)
    gc, cc, tc, oc = g.to_c(), camera.to_c(), tiling.to_c(), options.to_c()
    st = lib().oracle_backward_ex(C.byref(gc), C.byref(cc), C.byref(tc), C.byref(oc), F,
                               _p(np.ascontiguousarray(fwd["fgidx_to_gidx"])), _p(np.ascontiguousarray(fwd["f2d"])),
                               _p(np.ascontiguousarray(sfg)), _p(fwd["tiles_end"]), _p(fwd["trans"]),
                               _p(fwd["last"]), _p(rg), flags, _p(o["mean2d"]), _p(o["opacity"]),
                               _p(o["licov"]), _p(o["color"]), _p(o["mean3d"]),
                               _p(o["opacity_feature"]), _p(o["scaling"]), _p(o["rotation"]),
                               _p(o["sh"]), d, 1 if grads_2d is not None else 0, _p(mag))
    assert st == 0
    out = {k: v[:F] for k, v in o.items()}
    if mag is not None:
        out["mag"] = mag[:F]
    return out


class NpMoments:
    """Adam moments as numpy arrays: (n,3,2) (n,2) (n,3,2) (n,4,2) (n,3,S,2)."""

    def __init__(self, mm, om, sm, rm, shm):
        f = lambda a: np.ascontiguousarray(np.asarray(a, dtype=np.float32))
        self.mm, self.om, self.sm, self.rm, self.shm = map(f, (mm, om, sm, rm, shm))

    @classmethod
    def from_moments(cls, m) -> "NpMoments":
        return cls(*(t.detach().cpu().numpy() for t in m.tensors()))

    @property
    def sh_degree(self):
        return int(round(np.sqrt(self.shm.shape[2]))) - 1

    def to_c(self):
        m = _abi.AdamMomentsC()
        m.sh_degree = self.sh_degree
        m.means_moments, m.opacity_features_moments = _p(self.mm), _p(self.om)
        m.scaling_features_moments, m.rotation_features_moments = _p(self.sm), _p(self.rm)
        m.sh_coeffs_moments = _p(self.shm)
        return m

    def copy(self):
        return NpMoments(self.mm.copy(), self.om.copy(), self.sm.copy(), self.rm.copy(), self.shm.copy())


def fgradients_c(grads: dict):
    """FGradientsC over the numpy dict returned by backward() (3D parts only are read)."""
    f = _abi.FGradientsC()
    keep = {k: np.ascontiguousarray(v, np.float32) for k, v in grads.items()}
    f.sh_degree = int(round(np.sqrt(keep["sh"].shape[2]))) - 1
    f.mean2d_grads, f.opacity_grads = _p(keep["mean2d"]), _p(keep["opacity"])
    f.licov2d_grads, f.color_grads = _p(keep["licov"]), _p(keep["color"])
    f.mean3d_grads, f.opacity_feature_grads = _p(keep["mean3d"]), _p(keep["opacity_feature"])
    f.scaling_features_grads, f.rotation_features_grads = _p(keep["scaling"]), _p(keep["rotation"])
    f.sh_coeffs_grads = _p(keep["sh"])
    return f, keep


def adam(g: NpGaussians, m: NpMoments, grads: dict, fgidx_to_gidx: np.ndarray, params, bc1: float,
         bc2: float) -> None:
    """In-place sparse Adam step on (g, m); params is an _abi.AdamParamsC."""
    f2g = np.ascontiguousarray(fgidx_to_gidx, np.int32)
    fc, _keep = fgradients_c(grads)
    gc, mc = g.to_c(), m.to_c()
    assert lib().oracle_adam(C.byref(gc), C.byref(mc), C.byref(fc), _p(f2g), f2g.size,
                             C.byref(params), bc1, bc2) == 0


def adc_stats(acc: np.ndarray, cnt: np.ndarray, mean2d_g: np.ndarray, fgidx_to_gidx: np.ndarray,
              width: int, height: int) -> None:
    m2 = np.ascontiguousarray(mean2d_g, np.float32)
    f2g = np.ascontiguousarray(fgidx_to_gidx, np.int32)
    assert acc.dtype == np.float32 and cnt.dtype == np.int32
    lib().oracle_adc_stats(_p(acc), _p(cnt), _p(m2), _p(f2g), f2g.size, width, height)


def adc_plan(g: NpGaussians, acc, cnt, params) -> dict:
    n = g.n
    out = dict(max_sf=np.zeros(n, np.float32), prune=np.zeros(n, np.uint8),
               densify=np.zeros(n, np.uint8), clone=np.zeros(n, np.uint8),
               counts=np.zeros(n, np.uint8), counts_cs=np.zeros(n, np.int32),
               ngidx_to_gidx=np.zeros(2 * max(n, 1), np.int32))
    gc = g.to_c()
    acc = np.ascontiguousarray(acc, np.float32)
    cnt = np.ascontiguousarray(cnt, np.int32)
    new_n = lib().oracle_adc_plan(C.byref(gc), _p(acc), _p(cnt), C.byref(params), _p(out["max_sf"]),
                                  _p(out["prune"]), _p(out["densify"]), _p(out["clone"]),
                                  _p(out["counts"]), _p(out["counts_cs"]), _p(out["ngidx_to_gidx"]))
    out["new_n"] = int(new_n)
    out["ngidx_to_gidx"] = out["ngidx_to_gidx"][:new_n]
    return out


def adc_apply(g: NpGaussians, m: NpMoments, plan: dict, fgidx_to_gidx: np.ndarray | None,
              log_split: float, seed: int):
    """Returns (new NpGaussians, new NpMoments, retargeted fgidx_to_gidx)."""
    nn = plan["new_n"]
    S = g.sh.shape[2]
    Sm = m.shm.shape[2]
    ng = NpGaussians(np.zeros((nn, 4)), np.zeros((nn, 3)), np.zeros((nn, 4)), np.zeros((nn, 3, S)))
    nm = NpMoments(np.zeros((nn, 3, 2)), np.zeros((nn, 2)), np.zeros((nn, 3, 2)), np.zeros((nn, 4, 2)),
                   np.zeros((nn, 3, Sm, 2)))
    f2g = np.ascontiguousarray(fgidx_to_gidx if fgidx_to_gidx is not None else np.zeros(0), np.int32).copy()
    gc, mc, ngc, nmc = g.to_c(), m.to_c(), ng.to_c(), nm.to_c()
    assert lib().oracle_adc_apply(C.byref(gc), C.byref(mc), C.byref(ngc), C.byref(nmc),
                                  _p(plan["prune"]), _p(plan["densify"]), _p(plan["clone"]),
                                  _p(plan["counts_cs"]), _p(f2g), f2g.size, log_split,
                                  seed & 0xFFFFFFFFFFFFFFFF) == 0
    return ng, nm, f2g


def opacity_reset(g: NpGaussians, m: NpMoments, max_opacity: float) -> None:
    gc, mc = g.to_c(), m.to_c()
    lib().oracle_opacity_reset(C.byref(gc), C.byref(mc), max_opacity)


def split_normals(seed: int, key: int) -> np.ndarray:
    out = np.zeros(6, np.float32)
    lib().oracle_split_normals(seed & 0xFFFFFFFFFFFFFFFF, key, _p(out))
    return out


def sort_pairs(keys: np.ndarray, vals: np.ndarray, highest_key_bit: int):
    keys = np.ascontiguousarray(keys, np.int64)
    vals = np.ascontiguousarray(vals, np.int32)
    ko, vo = np.empty_like(keys), np.empty_like(vals)
    lib().oracle_sort_pairs(_p(keys), _p(ko), _p(vals), _p(vo), keys.size, highest_key_bit)
    return ko, vo


def cpu_render(g: NpGaussians, camera, options, nthreads: int = 1):
    W, H = camera.width, camera.height
    rgb = np.zeros((W, H, 3), np.float32)
    trans = np.zeros((W, H), np.float32)
    depth = np.zeros((W, H), np.float32)
    gc, cc, oc = g.to_c(), camera.to_c(), options.to_c()
    F = lib().oracle_cpu_render(C.byref(gc), C.byref(cc), C.byref(oc), _p(rgb), _p(trans),
                                _p(depth), nthreads)
    return dict(rgb=rgb, trans=trans, depth=depth, F=F)


def loss(rendered: np.ndarray, target: np.ndarray, weight: float = 0.2):
    """(loss, l1, dssim), gradient (w, h, 3)."""
    K = np.ascontiguousarray(rendered, np.float32)
    I = np.ascontiguousarray(target, np.float32)
    W, H = K.shape[0], K.shape[1]
    out = np.zeros(3, np.float64)
    grad = np.zeros_like(K)
    lib().oracle_loss(_p(K), _p(I), W, H, weight, _p(out), _p(grad))
    return out, grad


def expf(x: float) -> float:
    return lib().oracle_expf(x)


def logf(x: float) -> float:
    return lib().oracle_logf(x)
