"""Multi-view data-parallel training: one process per GPU.

Each rank renders and back-propagates its own view of the step with the 3D gradients written
straight into dense rows indexed by Gaussian (no scatter pass). The optimizer step is sharded
over the ranks and pipelined over `chunks` ranges of Gaussians: chunk c holds rows
[c C, (c + 1) C), C = world * S, and rank r owns the sub-range [c C + r S, c C + (r + 1) S) of
every chunk. For each chunk in turn the projection backward writes its rows
(gs3d_backward_project_dense) and an in-place NCCL reduce-scatter sums them into the owners'
sub-ranges while the next chunk's rows are computed; then, chunk by chunk, each rank applies
the Adam update to the touched Gaussians of its sub-range (gs3d_adam_step_dense_range) and
in-place all-gathers of the parameter arrays replicate the result while the next chunk is
updated. Parameters are identical on every rank after each step (with sharded SH coefficients,
the default with several ranks, the SH coefficients after sync_parameters(): between steps each
rank holds current coefficients only for its own sub-ranges and receives the colours of its
next views instead); each rank keeps its own sub-ranges' moments current. Parameters, moments and rows live in storage padded to
chunks * C rows so that every collective runs in place. A densify step all-gathers the
moments, all-reduces the rows and the statistics, and every rank then makes the same
decisions and the full update, as the reference retargets fgidx_to_gidx. With one rank this
is the reference's sparse update. `optimizer_step="replicated"` instead all-reduces each chunk's
rows and lets every rank apply the full update (no parameter exchange; measured slower).
Views: a permutation of the cameras drawn from a seed shared by all ranks; at step k rank r
takes entries ((k * world + r) * V + v) mod #cameras, v < V, for V views per rank
(`views_per_rank`; a global batch of world * V views). Every view is rendered and
back-propagated in turn; the rows of a step carry the sum over its views (the first view
writes them, later views add: GS3D_BACKWARD_ACCUMULATE_ROWS; factored rows keep one colour row
per view), the last view's projection backward is the one pipelined with the exchange, and the
update is applied once per step.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist
from torch.distributed.distributed_c10d import _coalescing_manager

from . import _abi
from . import adc as adc_mod
from .backward import (backward_project_dense, backward_project_factored, backward_raster,
                       colour_direction_rows)
from .render import _stream_handle, render, render_colour, render_given_colour, shard_colours
from .training import Trainer

DENSE_ROW = _abi.GS3D_DENSE_ROW
GEOM_ROW = _abi.GS3D_GEOM_ROW
COLOUR_ROW = _abi.GS3D_COLOUR_ROW
CHUNKS = 2


def view_index(step: int, rank: int, world: int, perm, ncams: int, views: int = 1, v: int = 0) -> int:
    """Camera of view v of rank `rank` at (0-based) step `step`: entry
    ((step * world + rank) * views + v) of the shared permutation, taken modulo #cameras."""
    k = (step * world + rank) * views + v
    return int(perm[k % ncams])


def shard_range(n: int, world: int, rank: int) -> tuple[int, int, int]:
    """(S, begin, end) of an unchunked split: shard size and this rank's Gaussian range."""
    S = max(1, -(-n // world))
    return S, min(n, rank * S), min(n, (rank + 1) * S)


def chunk_layout(n: int, world: int, chunks: int) -> tuple[int, int]:
    """(S, C): per-rank sub-range size and chunk size (C = world * S, chunks * C >= n)."""
    S = max(1, -(-n // (chunks * world)))
    return S, S * world


def exchange_factored_chunk(geom: torch.Tensor, colour: torch.Tensor, colour_recv: torch.Tensor,
                            c: int, S: int, C_: int, rank: int, group=None, in_place: bool = True):
    """Chunk c of the factored rows: reduce-scatter of its geometry rows into the owners'
    sub-ranges (in place) and, per view v, all-to-all of its colour rows: rank p receives, in
    slot (v, q) of `colour_recv` ((V, world, S, COLOUR_ROW)), rank q's colour rows of view v for
    p's sub-range. `colour` is (V, rows, COLOUR_ROW) (or (rows, COLOUR_ROW) for one view).
    Returns the async works. `in_place=False` reduces from a copy (for backends without
    in-place reduce-scatter)."""
    gflat = geom[c * C_:(c + 1) * C_].reshape(-1)
    per = S * GEOM_ROW
    works = [dist.reduce_scatter_tensor(gflat[rank * per:(rank + 1) * per],
                                        gflat if in_place else gflat.clone(),
                                        op=dist.ReduceOp.SUM, group=group, async_op=True)]
    col = colour if colour.dim() == 3 else colour.unsqueeze(0)
    recv = colour_recv if colour_recv.dim() == 4 else colour_recv.unsqueeze(0)
    for v in range(col.shape[0]):
        works.append(dist.all_to_all_single(recv[v].reshape(-1),
                                            col[v, c * C_:(c + 1) * C_].reshape(-1),
                                            group=group, async_op=True))
    return tuple(works)


def exchange_next_colours_chunk(send: torch.Tensor, recv: torch.Tensor, group=None):
    """One all-to-all of chunk c's next-step colours (shard_sh): `send` is this rank's
    (world * V * S, 4) block, slot r * V + v holding its sub-range's colours for view v of rank r;
    rank r receives in `recv` ((world * V * S, 4)) slot q * V + v from owner q. Over all chunks
    the received rows are laid out as gs3d_render_forward_given_colour reads them
    (given_colour_row). Returns the async work."""
    return dist.all_to_all_single(recv.reshape(-1), send.reshape(-1), group=group, async_op=True)


def given_colour_row(gi: int, S: int, world: int, views: int, v: int) -> int:
    """Row of Gaussian gi's colour for view v in the chunks' received colours (the index
    k_fill_colours uses): gi = c N S + q S + i -> ((c N + q) V + v) S + i."""
    C_ = world * S
    c, rem = divmod(gi, C_)
    q, i = divmod(rem, S)
    return ((c * world + q) * views + v) * S + i


class DataParallelTrainer(Trainer):
    """`optimizer_step`: "sharded" (reduce-scatter rows, Adam on the rank's sub-ranges,
    all-gather parameters) or "replicated" (all-reduce rows chunk by chunk, the full Adam update
    on every rank, no parameter exchange). `factored` (sharded step, SH storage degree 3, outside
    densify steps): exchange factored rows instead of dense rows, i.e. reduce-scatter the 12
    geometry floats per Gaussian and send each owner the 3 colour gradients of every view
    (all-to-all), from which it rebuilds the 48 SH gradients (gs3d_adam_step_factored_range):
    16 floats per Gaussian cross the links instead of 60. `shard_sh` (factored steps): the SH
    coefficients stay with their owners; the projection backward leaves the colour -> direction
    term of the mean gradient to the owner (gs3d_factored_colour_direction_range), and after its
    update the owner computes the colours of its Gaussians for every view of the next step
    (gs3d_shard_colours) and sends them (one all-to-all per chunk, 16 B per Gaussian and view)
    instead of all-gathering 192 B of SH coefficients per Gaussian; the next render takes them
    (gs3d_render_forward_given_colour). Steps that need every SH coefficient everywhere (a
    densify step, sync_parameters) all-gather them first."""

    def __init__(self, *args, group=None, optimizer_step: str = "sharded", chunks: int | None = None,
                 factored: bool = True, views_per_rank: int = 1, shard_sh: bool | None = None,
                 **kw):
        super().__init__(*args, **kw)
        if views_per_rank < 1:
            raise ValueError(f"views_per_rank {views_per_rank} < 1")
        self.views = int(views_per_rank)
        self._vi = 0  # view of the current step being processed
        if optimizer_step not in ("sharded", "replicated"):
            raise ValueError(f"optimizer_step {optimizer_step!r}")
        self.optimizer_step = optimizer_step
        self.factored = bool(factored)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        # pipeline depth (measured at 3M Gaussians on 2 B200s with factored rows: 2 chunks
        # 4.61 ms/step, 4: 4.74, 6: 4.90, 8: 5.03; the exchange is small enough that each
        # chunk's launches and collective calls cost more than the extra overlap gains)
        self.chunks = int(chunks) if chunks else CHUNKS
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.step_index = 0
        self.perm = self.rng.permutation(len(self.cameras))
        self._bases = {}
        self.dense = None
        self.geom = None
        self.colour = None
        self.colour_recv = None
        self._side = None
        # all-gathers of the last update still in flight: geometry arrays, SH coefficients
        self._pending_geom = []
        self._pending_sh = []
        self.defer_colour = True  # False: every render waits for all of the last update's gathers
        # default: on with several ranks (one rank saves no traffic and would only add the
        # owner's work)
        self.shard_sh = self.world > 1 if shard_sh is None else bool(shard_sh)
        self._sh_stale = False  # other ranks' SH sub-ranges out of date here (shard_sh)
        self._given = None  # colours of this step's views from their owners (shard_sh)
        self._pending_colours = []  # their all-to-alls still in flight
        self.colour_send = None
        self.colour_next = None
        # a list: each training step appends (phase name, CUDA event recorded on the compute
        # stream at the end of that phase); see phase_times
        self.phase_events = None
        self._ensure_padded()

    # -- padded storage -------------------------------------------------------------------
    def _padded_rows(self) -> int:
        _, C_ = chunk_layout(self.gaussians.n, self.world, self.chunks)
        return self.chunks * C_

    def _pad(self, key: str, t: torch.Tensor, rows: int) -> torch.Tensor:
        """t as the leading n rows of a (rows, ...) base tensor (reused when t already is)."""
        base = self._bases.get(key)
        if (base is not None and base.shape[0] == rows and base.shape[1:] == t.shape[1:]
                and base.data_ptr() == t.data_ptr()):
            return t
        base = torch.zeros((rows,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        base[: t.shape[0]].copy_(t)
        self._bases[key] = base
        return base[: t.shape[0]]

    def _ensure_padded(self) -> None:
        rows = self._padded_rows()
        g, m = self.gaussians, self.optimizer.moments
        g.means_opacity_features = self._pad("mo", g.means_opacity_features, rows)
        g.scaling_features = self._pad("sf", g.scaling_features, rows)
        g.rotation_features = self._pad("rf", g.rotation_features, rows)
        g.sh_coeffs = self._pad("sh", g.sh_coeffs, rows)
        m.means_moments = self._pad("mm", m.means_moments, rows)
        m.opacity_features_moments = self._pad("om", m.opacity_features_moments, rows)
        m.scaling_features_moments = self._pad("sm", m.scaling_features_moments, rows)
        m.rotation_features_moments = self._pad("rm", m.rotation_features_moments, rows)
        m.sh_coeffs_moments = self._pad("shm", m.sh_coeffs_moments, rows)
        if self.dense is None or self.dense.shape[0] != rows:
            self.dense = torch.zeros((rows, DENSE_ROW), dtype=torch.float32, device=self.device)
        if self.factored and self.optimizer_step == "sharded":
            S, _ = chunk_layout(self.gaussians.n, self.world, self.chunks)
            f = dict(dtype=torch.float32, device=self.device)
            if self.geom is None or self.geom.shape[0] != rows:
                self.geom = torch.zeros((rows, GEOM_ROW), **f)
                self.colour = torch.zeros((self.views, rows, COLOUR_ROW), **f)
            if self.world > 1 and (self.colour_recv is None or self.colour_recv.shape[3] != S):
                self.colour_recv = torch.empty((self.chunks, self.views, self.world, S, COLOUR_ROW), **f)
            if self.shard_sh:
                shape = (self.chunks, self.world * self.views * S, 4)
                if self.colour_send is None or self.colour_send.shape != shape:
                    self.colour_send = torch.zeros(shape, **f)
                    self.colour_next = torch.zeros(shape, **f) if self.world > 1 else None
                    self._given = None

    def _use_factored(self, in_adc: bool) -> bool:
        return (self.factored and self.optimizer_step == "sharded" and not in_adc and
                self.gaussians.sh_degree == 3 and
                self.world * self.views <= _abi.GS3D_MAX_FACTORED_VIEWS)

    def _view_positions(self):
        """Camera positions (float32) of this step's views in the order of the colour-row slots
        the update reads: view v of rank p at slot v * world + p."""
        import numpy as np
        pos = np.stack([self.cameras[view_index(self.step_index, p, self.world, self.perm,
                                                len(self.cameras), self.views, v)].position
                        for v in range(self.views) for p in range(self.world)]).astype(np.float32)
        return np.ascontiguousarray(pos)

    def _next_positions(self):
        """Camera positions (float32) of the next step's views in the order of the colour slots
        the owners fill: view v of rank r at slot r * views + v."""
        import numpy as np
        pos = np.stack([self.cameras[view_index(self.step_index + 1, r, self.world, self.perm,
                                                len(self.cameras), self.views, v)].position
                        for r in range(self.world) for v in range(self.views)]).astype(np.float32)
        return np.ascontiguousarray(pos)

    def _densifies_at(self, it: int) -> bool:
        o = self.options
        return o.adc_start_iteration_nb <= it <= o.adc_final_iteration_nb and it % o.adc_interval == 0

    def _exchange_factored(self, c: int, S: int, C_: int):
        return exchange_factored_chunk(self.geom, self.colour, self.colour_recv[c], c, S, C_,
                                       self.rank, self.group)

    def _gather_chunk(self, keys, c: int, async_op: bool):
        """In-place all-gather of chunk c of each padded array (rank r's sub-range to all), as
        one NCCL group."""
        if self.world <= 1:
            return []
        S, C_ = chunk_layout(self.gaussians.n, self.world, self.chunks)
        with _coalescing_manager(group=self.group, device=self.device, async_ops=async_op) as cm:
            for key in keys:
                base = self._bases[key]
                flat = base[c * C_:(c + 1) * C_].reshape(-1)
                per = flat.numel() // self.world
                dist.all_gather_into_tensor(flat, flat[self.rank * per:(self.rank + 1) * per],
                                            group=self.group)
        return [cm] if async_op else []

    def _allreduce(self, t: torch.Tensor) -> None:
        if self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def current_camera_index(self) -> int:
        return view_index(self.step_index, self.rank, self.world, self.perm, len(self.cameras),
                          self.views, self._vi)

    def peek_camera_index(self, ahead: int) -> int:
        """Camera of the view `ahead` views after the current one (of this rank)."""
        k = self._vi + ahead
        return view_index(self.step_index + k // self.views, self.rank, self.world, self.perm,
                          len(self.cameras), self.views, k % self.views)

    # -- one step ---------------------------------------------------------------------------
    def maybe_increase_sh_degree(self) -> None:
        if (self.iteration_nb % self.options.sh_degree_increase_interval == 0 and
                self.gaussians.sh_degree < 3):
            self.sync_parameters()  # the SH arrays are replaced
        super().maybe_increase_sh_degree()

    def maybe_opacity_reset(self) -> None:
        o = self.options
        if (o.opacity_reset_start_iteration_nb <= self.iteration_nb <= o.opacity_reset_final_iteration_nb
                and self.iteration_nb % o.opacity_reset_interval == 0):
            self.sync_parameters()  # the reset writes every opacity, the all-gathers some
        super().maybe_opacity_reset()

    def _mark(self, name: str) -> None:
        if self.phase_events is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.phase_events.append((name, ev))

    def phase_times(self) -> dict:
        """Average milliseconds per step of each phase recorded in phase_events (the compute
        stream's time from the previous marker to this one: a wait for a collective falls in
        the phase that ends with it). Synchronizes the device and clears the record."""
        torch.cuda.synchronize()
        ev = self.phase_events or []
        tot, cnt = {}, {}
        for (_, a), (name, b) in zip(ev, ev[1:]):
            if name == "step_start":
                continue
            tot[name] = tot.get(name, 0.0) + a.elapsed_time(b)
            cnt[name] = cnt.get(name, 0) + 1
        self.phase_events = [] if self.phase_events is not None else None
        # steps recorded: step_start markers followed by a phase (a trailing one only closes)
        steps = max(1, sum(1 for (n, _), (m, _) in zip(ev, ev[1:] + [("", None)])
                           if n == "step_start" and m not in ("", "step_start")))
        return {k: round(v / steps, 4) for k, v in tot.items()}

    def sync_parameters(self) -> None:
        """Make the current stream wait for the parameter all-gathers of the last update (a
        training step starts its first render before the SH coefficients have arrived) and,
        with sharded SH coefficients, all-gather them; call it before reading the parameters
        outside training_step. With shard_sh it is a collective: every rank calls it at the same
        point."""
        for w in self._pending_geom + self._pending_sh + self._pending_colours:
            w.wait()
        self._pending_geom, self._pending_sh, self._pending_colours = [], [], []
        if self._sh_stale:
            for c in range(self.chunks):
                self._gather_chunk(("sh",), c, async_op=False)
            self._sh_stale = False

    def _render_view(self, compute):
        """Render the current view, its loss and its 2D gradients (backward_raster); returns
        (camera, loss tensor). While the last update's SH all-gathers are in flight, the render
        runs without colours (filter, projection, duplication, sort) once the geometry arrays
        have arrived, then waits for the SH coefficients and completes (render_colour)."""
        idx = self.current_camera_index()
        cam = self.cameras[idx]
        rb = self.render_buffers
        if self._given is not None:
            # the colours of this view come from their owners (shard_sh)
            for w in self._pending_geom:
                w.wait()
            self._pending_geom = []
            self._mark("wait_geometry_gather")
            render(self.render_outputs, self.gaussians, cam, self.tiling, self.render_options, rb,
                   host_sync=self.render_host_sync, defer_colour=True)
            self._mark("render_geometry")
            for w in self._pending_colours:
                w.wait()
            self._pending_colours = []
            self._mark("wait_colours")
            S, _ = chunk_layout(self.gaussians.n, self.world, self.chunks)
            render_given_colour(self.render_outputs, self.gaussians, cam, self.tiling,
                                self.render_options, rb, self._given, S, self.world, self.views,
                                self._vi)
        elif self._pending_sh and self.defer_colour:
            for w in self._pending_geom:
                w.wait()
            self._mark("wait_geometry_gather")
            render(self.render_outputs, self.gaussians, cam, self.tiling, self.render_options, rb,
                   host_sync=self.render_host_sync, defer_colour=True)
            self._mark("render_geometry")
            for w in self._pending_sh:
                w.wait()
            self._pending_geom, self._pending_sh = [], []
            self._mark("wait_sh_gather")
            render_colour(self.render_outputs, self.gaussians, cam, self.tiling, self.render_options, rb)
        else:
            self.sync_parameters()
            self._mark("wait_gathers")
            render(self.render_outputs, self.gaussians, cam, self.tiling, self.render_options, rb,
                   host_sync=self.render_host_sync)
        self._mark("render")
        gt = self.target_for(idx)
        loss = self.loss(self.render_outputs.rgb, gt, self.rgb_image_grad)
        if gt is self._gt_buffers[self._gt_slot]:
            self._gt_free[self._gt_slot].record(compute)
        self.prefetch_target()
        self._mark("loss")
        backward_raster(self.fgradients, self.rgb_image_grad, self.render_outputs, self.gaussians,
                        cam, self.tiling, self.render_options, rb)
        self._mark("backward_raster")
        return cam, loss

    def training_step(self) -> torch.Tensor:
        lib = _abi.lib()
        self.iteration_nb += 1
        self.maybe_increase_sh_degree()
        self._ensure_padded()
        compute = torch.cuda.current_stream(self.device)
        o = self.options
        in_adc = self.densifies_this_iteration()
        factored = self._use_factored(in_adc)
        V = self.views
        if self._sh_stale and not factored:
            self.sync_parameters()  # this step reads every SH coefficient on every rank
        self._mark("step_start")
        # zero the rows on a side stream while the first forward runs
        if self._side is None:
            self._side = torch.cuda.Stream(self.device)
        self._side.wait_stream(compute)
        with torch.cuda.stream(self._side):
            if factored:
                self.geom.zero_()
                self.colour.zero_()
            else:
                self.dense.zero_()
        zeroed = torch.cuda.Event()
        zeroed.record(self._side)

        stream = C.c_void_p(_stream_handle(None))
        n = self.gaussians.n
        S, C_ = chunk_layout(n, self.world, self.chunks)
        rb = self.render_buffers
        track_adc = self.iteration_nb <= o.adc_final_iteration_nb
        loss_sum = None
        # views 0 .. V-2: rows of every Gaussian at once, added up (no exchange yet)
        for v in range(V - 1):
            self._vi = v
            cam, loss = self._render_view(compute)
            loss_sum = loss.clone() if loss_sum is None else loss_sum.add_(loss)
            if v == 0:
                compute.wait_event(zeroed)
            if factored:
                backward_project_factored(self.fgradients, self.gaussians, cam, self.tiling,
                                          self.render_options, rb, self.geom, self.colour[v], 0, n,
                                          accumulate=v > 0, colour_direction=not self.shard_sh)
            else:
                backward_project_dense(self.fgradients, self.gaussians, cam, self.tiling,
                                       self.render_options, rb, self.dense, 0, n, accumulate=v > 0)
            if track_adc or in_adc:
                adc_mod.adc_stats(self.adc_buffers, self.fgradients, rb.fgidx_to_gidx, rb.device_counts,
                                  self.width, self.height)
            self._mark("backward_project")
        # the last view: its projection backward pipelined with the exchange, chunk by chunk
        self._vi = V - 1
        acc = V > 1
        cam, loss = self._render_view(compute)
        self._given = None  # every view of this step has been rendered
        loss_sum = loss if loss_sum is None else loss_sum.add_(loss)
        if V == 1:
            compute.wait_event(zeroed)
        if in_adc:
            backward_project_dense(self.fgradients, self.gaussians, cam, self.tiling,
                                   self.render_options, rb, self.dense, 0, n, accumulate=acc)
            adc_mod.adc_stats(self.adc_buffers, self.fgradients, rb.fgidx_to_gidx, rb.device_counts,
                              self.width, self.height)
            self.update_learning_rates()
            params = self.optimizer.params_c(self.render_options.sh_degree)
            # every rank needs every moment and the summed rows: the update is not sharded
            if self.optimizer_step == "sharded":
                for c in range(self.chunks):
                    self._gather_chunk(("mm", "om", "sm", "rm", "shm"), c, async_op=False)
            self._allreduce(self.dense)
            self._densify()
            g, m = self.gaussians.to_c(), self.optimizer.moments.to_c()
            _abi.check(lib.gs3d_adam_step_dense(C.byref(g), C.byref(m), C.c_void_p(self.dense.data_ptr()),
                                                C.byref(params), stream))
        elif self.optimizer_step == "replicated" or (self.world == 1 and not factored):
            # chunk c: its rows, then their all-reduce while chunk c + 1 is computed; then the
            # full update of chunk c on every rank while the later chunks are still exchanged
            ar = []
            for c in range(self.chunks):
                lo, hi = c * C_, min((c + 1) * C_, n)
                if lo < hi:
                    backward_project_dense(self.fgradients, self.gaussians, cam, self.tiling,
                                           self.render_options, rb, self.dense[lo:], lo, hi,
                                           accumulate=acc)
                if self.world > 1:
                    ar.append(dist.all_reduce(self.dense[c * C_:(c + 1) * C_], op=dist.ReduceOp.SUM,
                                              group=self.group, async_op=True))
            if track_adc:
                adc_mod.adc_stats(self.adc_buffers, self.fgradients, rb.fgidx_to_gidx, rb.device_counts,
                                  self.width, self.height)
            self.update_learning_rates()
            params = self.optimizer.params_c(self.render_options.sh_degree)
            g, m = self.gaussians.to_c(), self.optimizer.moments.to_c()
            for c in range(self.chunks):
                if ar:
                    ar[c].wait()
                lo, hi = c * C_, min((c + 1) * C_, n)
                if lo < hi:
                    _abi.check(lib.gs3d_adam_step_dense_range(C.byref(g), C.byref(m),
                                                              C.c_void_p(self.dense[lo:].data_ptr()), lo, hi,
                                                              C.byref(params), stream))
        else:
            # chunk c: its rows, then the reduce-scatter of those rows while chunk c + 1 is computed
            rs = []
            for c in range(self.chunks):
                lo, hi = c * C_, min((c + 1) * C_, n)
                if factored:
                    if lo < hi:
                        backward_project_factored(self.fgradients, self.gaussians, cam, self.tiling,
                                                  self.render_options, rb, self.geom[lo:],
                                                  self.colour[V - 1, lo:], lo, hi, accumulate=acc,
                                                  colour_direction=not self.shard_sh)
                    if self.world > 1:
                        rs.append(self._exchange_factored(c, S, C_))
                    continue
                if lo < hi:
                    backward_project_dense(self.fgradients, self.gaussians, cam, self.tiling,
                                           self.render_options, rb, self.dense[lo:], lo, hi,
                                           accumulate=acc)
                if self.world > 1:
                    flat = self.dense[c * C_:(c + 1) * C_].reshape(-1)
                    per = S * DENSE_ROW
                    rs.append(dist.reduce_scatter_tensor(flat[self.rank * per:(self.rank + 1) * per], flat,
                                                         op=dist.ReduceOp.SUM, group=self.group,
                                                         async_op=True))
            if track_adc:
                adc_mod.adc_stats(self.adc_buffers, self.fgradients, rb.fgidx_to_gidx, rb.device_counts,
                                  self.width, self.height)
            self._mark("backward_project")
            self.update_learning_rates()
            params = self.optimizer.params_c(self.render_options.sh_degree)
            g, m = self.gaussians.to_c(), self.optimizer.moments.to_c()
            ag = []
            cw = []
            # shard_sh: the owners send the next step's colours instead of all-gathering the SH
            # coefficients, unless the next step densifies (it needs them everywhere)
            give = factored and self.shard_sh and not self._densifies_at(self.iteration_nb + 1)
            if factored:
                pos = self._view_positions()
                pos_p = pos.ctypes.data_as(C.POINTER(C.c_float))
                if give:
                    next_pos = self._next_positions()
            for c in range(self.chunks):
                if rs:
                    for w in (rs[c] if factored else (rs[c],)):
                        w.wait()
                self._mark(f"wait_exchange_{c}")
                lo = c * C_ + self.rank * S
                hi = min(lo + S, n)
                if factored:
                    if lo < hi:
                        if self.world > 1:
                            views, stride = self.colour_recv[c], S
                        else:
                            views, stride = self.colour[0, lo:], self.colour.shape[1]
                        if self.shard_sh:
                            # the mean gradients' colour -> direction terms, from the SH
                            # coefficients and means before their update
                            colour_direction_rows(self.gaussians, self.geom[lo:], views,
                                                  self.world * V, stride, pos, lo, hi,
                                                  self.render_options.sh_degree)
                        _abi.check(lib.gs3d_adam_step_factored_range(
                            C.byref(g), C.byref(m), C.c_void_p(self.geom[lo:].data_ptr()),
                            C.c_void_p(views.data_ptr()), self.world * V, stride, pos_p, lo, hi,
                            C.byref(params), stream))
                        if give:
                            shard_colours(self.gaussians, self.render_options.sh_degree, next_pos,
                                          lo, hi, self.colour_send[c], S)
                elif lo < hi:
                    rows = self.dense[lo:]
                    _abi.check(lib.gs3d_adam_step_dense_range(C.byref(g), C.byref(m),
                                                              C.c_void_p(rows.data_ptr()), lo, hi,
                                                              C.byref(params), stream))
                self._mark(f"adam_{c}")
                ag.extend(self._gather_chunk(("mo", "sf", "rf"), c, async_op=True))
                if give and self.world > 1:
                    cw.append(exchange_next_colours_chunk(self.colour_send[c], self.colour_next[c],
                                                          self.group))
            # the SH coefficients (192 of the 236 bytes per Gaussian) go last; the next step's
            # first render waits for the geometry arrays, filters, projects, duplicates and sorts,
            # and only then for the SH coefficients or the colours (_render_view)
            sh = []
            if give:
                self._given = self.colour_next if self.world > 1 else self.colour_send
                self._sh_stale = self.world > 1
            else:
                for c in range(self.chunks):
                    sh.extend(self._gather_chunk(("sh",), c, async_op=True))
                self._sh_stale = False
            self._pending_geom, self._pending_sh, self._pending_colours = ag, sh, cw
        self.optimizer.update_count += 1
        if in_adc:
            self.complete_adc_step()
            self._ensure_padded()
        self.maybe_opacity_reset()
        self.step_index += 1
        self._vi = 0
        if V > 1:
            loss_sum.div_(V)
        self.last_loss = loss_sum
        return loss_sum

    def _densify(self) -> None:
        self.sync_parameters()
        o = self.options
        a = self.adc_buffers
        self._allreduce(a.accumulated_mean2d_grad_norms_ndc)
        self._allreduce(a.rendering_contribution_counts)
        old_n = self.gaussians.n
        new_n = adc_mod.densify_prune_plan(a, self.gaussians, o.densification_mean2d_grad_norm_threshold_ndc,
                                           o.densification_size_threshold, o.pruning_min_opacity,
                                           o.pruning_3d_max_scale, self.iteration_nb > o.opacity_reset_interval)
        ng, nm = adc_mod.densify_apply(a, self.gaussians, self.optimizer.moments, new_n,
                                       o.splitting_scale_factor, self.adc_seed + self.iteration_nb)
        dense_new = torch.empty((max(new_n, 1), DENSE_ROW), dtype=torch.float32, device=self.device)
        ac = a.to_c()
        _abi.check(_abi.lib().gs3d_densify_remap_dense(C.byref(ac), old_n, C.c_void_p(self.dense.data_ptr()),
                                                       C.c_void_p(dense_new.data_ptr()),
                                                       C.c_void_p(_stream_handle(None))))
        self.dense = dense_new
        self.gaussians.replace(ng)
        self.optimizer.moments = nm
        a.set_nb_gaussians(new_n)
