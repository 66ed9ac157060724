"""render! (forward_core.jl:196-314) through libgs3d.so."""
from __future__ import annotations

import ctypes as C

import torch

from . import _abi
from .structs import (GaussiansVector, PinholeCamera, RenderBuffers, RenderOnlyGaussiansVector,
                      RenderOptions,
                      RenderOutputs, Tiling)


def _stream_handle(stream: torch.cuda.Stream | None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def render(outputs: RenderOutputs, gaussians: GaussiansVector, camera: PinholeCamera,
           tiling: Tiling, options: RenderOptions, buffers: RenderBuffers,
           stream: torch.cuda.Stream | None = None, host_sync: bool = True,
           reference_order: bool = False, contrib_masks: bool = True,
           defer_colour: bool = False) -> RenderOutputs:
    """Render `gaussians` for `camera` into `outputs` (in place), like the reference's
    GPU `render!`. With `host_sync` the call waits once for the duplicate count and grows the
    duplicate buffers when they are too small (the reference's set_nb_dfgaussians!);
    without it nothing blocks and an overflow shows up in buffers.device_counts[2].
    `reference_order` also fills the unsorted duplicate arrays and the duplicate-count scan
    as the reference does (GS3D_RENDER_REFERENCE_ORDER); the sorted arrays, tile ends and
    images are the same either way. `gaussians` may also be a RenderOnlyGaussiansVector
    (stored opacities and 3D covariances; gs3d_render_forward_render_only).
    `contrib_masks=False` leaves the buffers' contribution masks unwritten (for renders that no
    backward follows; GS3D_RENDER_NO_CONTRIB_MASKS). `defer_colour=True` stops before the colours
    and the blend (the SH coefficients are not read); `render_colour` completes the render."""
    if gaussians.n > buffers.capacity_n:
        raise ValueError(f"{gaussians.n} Gaussians exceed the buffers' capacity {buffers.capacity_n}")
    lib = _abi.lib()
    flags = 0 if host_sync else _abi.GS3D_RENDER_NO_HOST_SYNC
    if reference_order:
        flags |= _abi.GS3D_RENDER_REFERENCE_ORDER
    if not contrib_masks:
        flags |= _abi.GS3D_RENDER_NO_CONTRIB_MASKS
    if defer_colour:
        flags |= _abi.GS3D_RENDER_DEFER_COLOUR
    host = buffers.host_counts
    hptr = C.c_void_p(host.data_ptr()) if host is not None else None
    args = (outputs.to_c(), gaussians.to_c(), camera.to_c(), tiling.to_c(), options.to_c())
    entry = (lib.gs3d_render_forward_render_only if isinstance(gaussians, RenderOnlyGaussiansVector)
             else lib.gs3d_render_forward)
    for _ in range(4):
        b = buffers.to_c()
        st = entry(C.byref(args[0]), C.byref(args[1]), C.byref(args[2]),
                                     C.byref(args[3]), C.byref(args[4]), C.byref(b), hptr,
                                     flags, C.c_void_p(_stream_handle(stream)))
        if st == _abi.GS3D_ERR_CAPACITY:
            buffers.grow_dup(int(host[1]) if host is not None else 2 * buffers.capacity_dup)
            continue
        _abi.check(st)
        return outputs
    raise RuntimeError("duplicate-key capacity did not converge")


def render_colour(outputs: RenderOutputs, gaussians: GaussiansVector, camera: PinholeCamera,
                  tiling: Tiling, options: RenderOptions, buffers: RenderBuffers,
                  stream: torch.cuda.Stream | None = None, contrib_masks: bool = True) -> RenderOutputs:
    """Second half of render(..., defer_colour=True) with the same arguments: the filtered
    Gaussians' colours and the blend (gs3d_render_forward_colour). The two halves equal one
    render bit for bit."""
    flags = 0 if contrib_masks else _abi.GS3D_RENDER_NO_CONTRIB_MASKS
    args = (outputs.to_c(), gaussians.to_c(), camera.to_c(), tiling.to_c(), options.to_c(),
            buffers.to_c())
    _abi.check(_abi.lib().gs3d_render_forward_colour(*(C.byref(x) for x in args), flags,
                                                     C.c_void_p(_stream_handle(stream))))
    return outputs


def render_given_colour(outputs: RenderOutputs, gaussians: GaussiansVector, camera: PinholeCamera,
                        tiling: Tiling, options: RenderOptions, buffers: RenderBuffers,
                        colours: torch.Tensor, shard_rows: int, n_ranks: int = 1,
                        n_views: int = 1, view: int = 0, stream: torch.cuda.Stream | None = None,
                        contrib_masks: bool = True) -> RenderOutputs:
    """Second half of render(..., defer_colour=True) with the colours given (float4 rows of
    `colours` in the layout of gs3d_render_forward_given_colour: Gaussian g = c N S + q S + i takes
    row ((c N + q) V + view) S + i) instead of computed from the SH coefficients."""
    assert colours.is_contiguous() and colours.dtype == torch.float32
    flags = 0 if contrib_masks else _abi.GS3D_RENDER_NO_CONTRIB_MASKS
    args = (outputs.to_c(), gaussians.to_c(), camera.to_c(), tiling.to_c(), options.to_c(),
            buffers.to_c())
    _abi.check(_abi.lib().gs3d_render_forward_given_colour(
        *(C.byref(x) for x in args), C.c_void_p(colours.data_ptr()), int(shard_rows), int(n_ranks),
        int(n_views), int(view), flags, C.c_void_p(_stream_handle(stream))))
    return outputs


def shard_colours(gaussians: GaussiansVector, sh_degree: int, positions, g_begin: int, g_end: int,
                  out: torch.Tensor, view_stride: int, stream: torch.cuda.Stream | None = None) -> None:
    """Colours of Gaussians [g_begin, g_end) from the cameras at `positions` ((n, 3) float32,
    host) into float4 rows v * view_stride + g - g_begin of `out` (gs3d_shard_colours)."""
    import numpy as np
    pos = np.ascontiguousarray(positions, dtype=np.float32)
    assert out.is_contiguous() and out.dtype == torch.float32
    _abi.check(_abi.lib().gs3d_shard_colours(
        C.byref(gaussians.to_c()), int(sh_degree), pos.ctypes.data_as(C.POINTER(C.c_float)),
        int(pos.shape[0]), int(g_begin), int(g_end), C.c_void_p(out.data_ptr()), int(view_stride),
        C.c_void_p(_stream_handle(stream))))


def counts(buffers: RenderBuffers) -> tuple[int, int]:
    """(F, D) of the last render (reads device memory; synchronises)."""
    c = buffers.device_counts.cpu()
    return int(c[0]), int(c[1])


def work_counts(camera: PinholeCamera, tiling: Tiling, options: RenderOptions,
                buffers: RenderBuffers, stream: torch.cuda.Stream | None = None) -> tuple[int, int]:
    """(blends, contributions) of the last render with `buffers`, as the reference's blend loop
    performs the work (gs3d_render_work_counts): (pixel, Gaussian) evaluations until each pixel
    stops, and the evaluations blended into a pixel (the pairs the backward blend
    differentiates). Synchronises; for rooflines and tests."""
    out = torch.zeros(2, dtype=torch.int64, device=buffers.device_counts.device)
    _abi.check(_abi.lib().gs3d_render_work_counts(
        C.byref(camera.to_c()), C.byref(tiling.to_c()), C.byref(options.to_c()),
        C.byref(buffers.to_c()), C.c_void_p(out.data_ptr()), C.c_void_p(_stream_handle(stream))))
    c = out.cpu()
    return int(c[0]), int(c[1])
