"""Multi-view data-parallel training: one process per GPU, model replicated.

Each rank renders and back-propagates its own view of the step with the 3D gradients written
straight into dense rows indexed by Gaussian (gs3d_backward_dense), the rows are summed across
ranks with one all-reduce over NCCL (torch.distributed), and every rank applies the identical
Adam update to the union of touched Gaussians (gs3d_adam_step_dense). With one rank this is exactly the
reference's sparse update. Densify steps all-reduce the statistics first, so every rank makes
the same decisions, and remap the dense rows like the reference retargets fgidx_to_gidx.
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


class DataParallelTrainer(Trainer):
    def __init__(self, *args, group=None, **kw):
        super().__init__(*args, **kw)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.dense = torch.empty((max(self.gaussians.n, 1), DENSE_ROW), dtype=torch.float32,
                                 device=self.device)
        self.step_index = 0
        self.perm = self.rng.permutation(len(self.cameras))

    def _allreduce(self, t: torch.Tensor) -> None:
        if self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def current_camera_index(self) -> int:
        return view_index(self.step_index, self.rank, self.world, self.perm, len(self.cameras))

    def peek_camera_index(self, ahead: int) -> int:
        return view_index(self.step_index + ahead, self.rank, self.world, self.perm, len(self.cameras))

    def training_step(self) -> torch.Tensor:
        lib = _abi.lib()
        self.iteration_nb += 1
        self.maybe_increase_sh_degree()
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
        self._allreduce(self.dense)
        in_adc = False
        if self.iteration_nb <= o.adc_final_iteration_nb:
            adc_mod.adc_stats(self.adc_buffers, self.fgradients, rb.fgidx_to_gidx, rb.device_counts,
                              self.width, self.height)
            if self.iteration_nb >= o.adc_start_iteration_nb and self.iteration_nb % o.adc_interval == 0:
                in_adc = True
                self._densify()
        self.update_learning_rates()
        params = self.optimizer.params_c(self.render_options.sh_degree)
        g, m = self.gaussians.to_c(), self.optimizer.moments.to_c()
        _abi.check(lib.gs3d_adam_step_dense(C.byref(g), C.byref(m), C.c_void_p(self.dense.data_ptr()),
                                            C.byref(params), stream))
        self.optimizer.update_count += 1
        if in_adc:
            self.complete_adc_step()
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
