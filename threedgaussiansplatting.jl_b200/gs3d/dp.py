"""Multi-view data-parallel training: one process per GPU.

Each rank renders and back-propagates its own view of the step with the 3D gradients written
straight into dense rows indexed by Gaussian (gs3d_backward_dense). The optimizer step is
sharded over the ranks: the rows are summed with one NCCL reduce-scatter, rank r applies the
Adam update to the touched Gaussians of its range [r S, (r + 1) S) (S = ceil(n / world)) with
gs3d_adam_step_dense_range, and the updated parameters are all-gathered, so the parameters are
identical on every rank after each step while each rank keeps its own range's moments current.
Parameters, moments and rows live in storage padded to world * S rows so that both
collectives run in place. A densify step all-gathers the moments, all-reduces the rows and
the statistics, and every rank then makes the same decisions and the full dense update, as
the reference retargets fgidx_to_gidx. With one rank this is the reference's sparse update.
Views: a permutation of the cameras drawn from a seed shared by all ranks; at step k rank r
takes entry (k * world + r) mod #cameras.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from . import _abi
from . import adc as adc_mod
from .backward import backward_dense
from .render import _stream_handle, render
from .training import Trainer

DENSE_ROW = 60


def view_index(step: int, rank: int, world: int, perm, ncams: int) -> int:
    """Camera of rank `rank` at (0-based) step `step`: entry (step * world + rank) of the
    shared permutation, re-drawn every #cameras views."""
    k = step * world + rank
    return int(perm[k % ncams])


def shard_range(n: int, world: int, rank: int) -> tuple[int, int, int]:
    """(S, begin, end): shard size and this rank's Gaussian range."""
    S = max(1, -(-n // world))
    return S, min(n, rank * S), min(n, (rank + 1) * S)


class DataParallelTrainer(Trainer):
    def __init__(self, *args, group=None, **kw):
        super().__init__(*args, **kw)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.step_index = 0
        self.perm = self.rng.permutation(len(self.cameras))
        self._bases = {}
        self.dense = None
        self._ensure_padded()

    # -- padded storage -------------------------------------------------------------------
    def _padded_rows(self) -> int:
        S, _, _ = shard_range(self.gaussians.n, self.world, self.rank)
        return S * self.world

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

    def _all_gather_rows(self, keys) -> None:
        """In-place all-gather of each padded array's shards."""
        if self.world <= 1:
            return
        for key in keys:
            flat = self._bases[key].view(-1)
            per = flat.numel() // self.world
            dist.all_gather_into_tensor(flat, flat[self.rank * per:(self.rank + 1) * per],
                                        group=self.group)

    def _allreduce(self, t: torch.Tensor) -> None:
        if self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def current_camera_index(self) -> int:
        return view_index(self.step_index, self.rank, self.world, self.perm, len(self.cameras))

    def peek_camera_index(self, ahead: int) -> int:
        return view_index(self.step_index + ahead, self.rank, self.world, self.perm, len(self.cameras))

    # -- one step ---------------------------------------------------------------------------
    def training_step(self) -> torch.Tensor:
        lib = _abi.lib()
        self.iteration_nb += 1
        self.maybe_increase_sh_degree()
        self._ensure_padded()
        idx = self.current_camera_index()
        cam = self.cameras[idx]
        rb = self.render_buffers
        render(self.render_outputs, self.gaussians, cam, self.tiling, self.render_options, rb,
               host_sync=self.render_host_sync)
        gt = self.target_for(idx)
        loss = self.loss(self.render_outputs.rgb, gt, self.rgb_image_grad)
        if gt is self._gt_buffers[self._gt_slot]:
            self._gt_free[self._gt_slot].record(torch.cuda.current_stream(self.device))
        self.prefetch_target()
        backward_dense(self.fgradients, self.rgb_image_grad, self.render_outputs, self.gaussians,
                       cam, self.tiling, self.render_options, rb, self.dense)
        o = self.options
        stream = C.c_void_p(_stream_handle(None))
        in_adc = False
        if self.iteration_nb <= o.adc_final_iteration_nb:
            adc_mod.adc_stats(self.adc_buffers, self.fgradients, rb.fgidx_to_gidx, rb.device_counts,
                              self.width, self.height)
            in_adc = self.iteration_nb >= o.adc_start_iteration_nb and self.iteration_nb % o.adc_interval == 0
        self.update_learning_rates()
        params = self.optimizer.params_c(self.render_options.sh_degree)
        if in_adc:
            # every rank needs every moment and the summed rows: the update is not sharded
            self._all_gather_rows(("mm", "om", "sm", "rm", "shm"))
            self._allreduce(self.dense)
            self._densify()
            g, m = self.gaussians.to_c(), self.optimizer.moments.to_c()
            _abi.check(lib.gs3d_adam_step_dense(C.byref(g), C.byref(m), C.c_void_p(self.dense.data_ptr()),
                                                C.byref(params), stream))
        else:
            n = self.gaussians.n
            S, lo, hi = shard_range(n, self.world, self.rank)
            if self.world > 1:
                flat = self.dense.view(-1)
                per = S * DENSE_ROW
                dist.reduce_scatter_tensor(flat[self.rank * per:(self.rank + 1) * per], flat,
                                           op=dist.ReduceOp.SUM, group=self.group)
            g, m = self.gaussians.to_c(), self.optimizer.moments.to_c()
            rows = self.dense[lo:]
            _abi.check(lib.gs3d_adam_step_dense_range(C.byref(g), C.byref(m), C.c_void_p(rows.data_ptr()),
                                                      lo, hi, C.byref(params), stream))
            self._all_gather_rows(("mo", "sf", "rf", "sh"))
        self.optimizer.update_count += 1
        if in_adc:
            self.complete_adc_step()
            self._ensure_padded()
        self.maybe_opacity_reset()
        self.step_index += 1
        self.last_loss = loss
        return loss

    def _densify(self) -> None:
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
