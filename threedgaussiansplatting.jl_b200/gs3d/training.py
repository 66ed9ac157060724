"""Training orchestration of ThreeDGaussianSplatting.jl: TrainingOptions
(training_structs.jl:43-228), Trainer and training_step! (training.jl:40-244) with the
SH-degree increase, learning-rate annealing, densify/prune and opacity reset schedule
(training.jl:253-459). Every compute step is a libgs3d.so call on one CUDA stream; the host
only orders the calls (and, like the reference, reads n' back at a densify step)."""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from . import adc as adc_mod
from .backward import FilteredGaussiansGradients, backward
from .loss import LossComputer
from .optimizer import AdamOptimizer, LearningRates
from .render import render
from .structs import GaussiansVector, PinholeCamera, RenderBuffers, RenderOptions, RenderOutputs, Tiling

F32 = np.float32


@dataclass
class TrainingOptions:
    """TrainingOptions with the reference defaults; radius-scaled values already scaled."""

    scene_radius: float
    nb_iterations: int = 30_000
    loss_dssim_vs_L1_weight: float = 0.2
    base_initial_means_lr: float = 0.00016
    base_final_means_lr_rel_factor: float = 1 / 100
    opacity_features_lr: float = 0.05
    scaling_features_lr: float = 0.005
    rotation_features_lr: float = 0.001
    sh_coeffs_dc_lr: float = 0.0025
    sh_coeffs_rest_lr_rel_factor: float = 1 / 20
    nb_lr_annealing_steps: int | None = None
    sh_degree_increase_interval: int = 1_000
    opacity_reset_interval: int = 3_000
    opacity_reset_start_iteration_nb: int = 0
    opacity_reset_final_iteration_nb: int = 12_000
    opacity_reset_max_value: float = 0.01
    adc_interval: int = 100
    adc_start_iteration_nb: int = 600
    adc_final_iteration_nb: int = 14_900
    densification_mean2d_grad_norm_threshold_ndc: float = 0.0002
    base_densification_size_threshold: float = 0.01
    splitting_scale_factor: float = 1 / (0.8 * 2)
    pruning_min_opacity: float = 0.005
    base_pruning_3d_max_scale: float = 0.1

    def __post_init__(self):
        if self.nb_lr_annealing_steps is None:
            self.nb_lr_annealing_steps = self.nb_iterations
        if not (self.scene_radius > 0):
            raise ValueError("scene radius must be positive (the reference's _check_positive "
                             "rejects a zero means learning rate)")

    @property
    def initial_means_lr(self) -> float:
        return float(F32(self.base_initial_means_lr * self.scene_radius))

    @property
    def final_means_lr(self) -> float:
        return float(F32(self.base_initial_means_lr * self.base_final_means_lr_rel_factor * self.scene_radius))

    @property
    def sh_coeffs_rest_lr(self) -> float:
        return float(F32(self.sh_coeffs_dc_lr * self.sh_coeffs_rest_lr_rel_factor))

    @property
    def densification_size_threshold(self) -> float:
        return float(F32(self.base_densification_size_threshold * self.scene_radius))

    @property
    def pruning_3d_max_scale(self) -> float:
        return float(F32(self.base_pruning_3d_max_scale * self.scene_radius))

    def learning_rates(self) -> LearningRates:
        return LearningRates(self.initial_means_lr, self.opacity_features_lr, self.scaling_features_lr,
                             self.rotation_features_lr, self.sh_coeffs_dc_lr, self.sh_coeffs_rest_lr)


def annealed_means_lr(iteration_nb: int, o: TrainingOptions) -> float:
    """Means learning rate of update_learning_rates! (training.jl:287-302) in Float32
    arithmetic: x = clamp((it - 1) / Float32(steps - 1), 0, 1) and
    exp((1 - x) log(initial) + x log(final)), each log and exp rounded once to Float32 (Julia's
    Float32 log and exp evaluate in Float64 and round), products and sum rounded as Float32."""
    den = F32(o.nb_lr_annealing_steps - 1)
    if den == 0:
        # one annealing step: the reference divides by zero, Inf clamps to 1 and 0 / 0 = NaN
        # fails its positivity check on the learning rate
        if iteration_nb == 1:
            raise ValueError("nb_lr_annealing_steps == 1 gives a NaN means learning rate at "
                             "iteration 1")
        x = F32(1)
    else:
        x = F32(iteration_nb - 1) / den
    x = F32(min(max(x, F32(0)), F32(1)))
    la = F32(math.log(o.initial_means_lr))
    lb = F32(math.log(o.final_means_lr))
    t = F32(F32(F32(1) - x) * la) + F32(x * lb)
    return float(F32(math.exp(float(t))))


class Trainer:
    """Trainer (training.jl:40-151). `targets[i]` is the ground-truth image of camera i as a
    (w, h, 3) float32 tensor, on the device or in (pinned) host memory; host images are
    copied to a device buffer at each step."""

    def __init__(self, gaussians: GaussiansVector, cameras: list[PinholeCamera], targets,
                 render_options: RenderOptions, tiling: Tiling, options: TrainingOptions,
                 seed: int = 0, capacity_dup: int | None = None, adc_seed: int = 1234,
                 rebuild_sh_grads: bool = True):
        # outside densify steps the Adam kernel recomputes the SH gradients from the colour
        # gradients instead of reading them back (the same update, without the 192 bytes per
        # filtered Gaussian written by the backward and read by the update)
        self.rebuild_sh_grads = rebuild_sh_grads
        self.gaussians = gaussians
        self.cameras = cameras
        self.targets = targets
        self.render_options = render_options
        self.tiling = tiling
        self.options = options
        dev = gaussians.device
        self.device = dev
        cam0 = cameras[0]
        self.width, self.height = cam0.width, cam0.height
        self.render_buffers = RenderBuffers.create(gaussians.n, tiling.nb_tiles, dev, capacity_dup=capacity_dup)
        self.render_outputs = RenderOutputs.create(self.width, self.height, dev)
        self.rgb_image_grad = torch.empty((self.width, self.height, 3), dtype=torch.float32, device=dev)
        # host targets: two device buffers, filled on a copy stream one step ahead
        self._gt_buffers = [torch.empty((self.width, self.height, 3), dtype=torch.float32, device=dev)
                            for _ in range(2)]
        self._gt_ready = [torch.cuda.Event() for _ in range(2)] if dev.type == "cuda" else None
        self._gt_free = [torch.cuda.Event() for _ in range(2)] if dev.type == "cuda" else None
        self._gt_slot = 0
        self._prefetched = None
        self._copy_stream = None
        self._next_orders = []
        self.loss = LossComputer(self.width, self.height, dev, options.loss_dssim_vs_L1_weight)
        self.fgradients = FilteredGaussiansGradients.create(gaussians.n, gaussians.sh_degree, dev)
        self.optimizer = AdamOptimizer(gaussians, options.learning_rates())
        self.adc_buffers = adc_mod.AdcBuffers.create(gaussians.n, dev)
        self.iteration_nb = 0
        self.rng = np.random.default_rng(seed)
        self.cameras_order = self.rng.permutation(len(cameras))
        self.cameras_order_idx = -1
        self.adc_seed = adc_seed
        self.last_loss = None
        # False: renders never block; a duplicate-key overflow is flagged in
        # render_buffers.device_counts[2] instead of growing the buffers
        self.render_host_sync = True

    # -- schedule pieces (training.jl:253-302) ---------------------------------------------
    def current_camera_index(self) -> int:
        return int(self.cameras_order[self.cameras_order_idx])

    def maybe_increase_sh_degree(self) -> None:
        if self.iteration_nb % self.options.sh_degree_increase_interval != 0:
            return
        d = self.gaussians.sh_degree
        if d >= 3:
            return
        d += 1
        self.render_options = self.render_options.with_sh_degree(d)
        self.gaussians.set_sh_degree(d)
        self.fgradients.set_sh_degree(d)
        self.optimizer.moments.set_sh_degree(d)

    def maybe_opacity_reset(self) -> None:
        o = self.options
        if (o.opacity_reset_start_iteration_nb <= self.iteration_nb <= o.opacity_reset_final_iteration_nb
                and self.iteration_nb % o.opacity_reset_interval == 0):
            adc_mod.opacity_reset(self.gaussians, self.optimizer.moments, o.opacity_reset_max_value)

    def update_learning_rates(self) -> None:
        self.optimizer.lrs.means = annealed_means_lr(self.iteration_nb, self.options)

    def densifies_this_iteration(self) -> bool:
        """Whether maybe_densify_and_prune densifies at the current iteration_nb."""
        o = self.options
        return (self.iteration_nb <= o.adc_final_iteration_nb and
                self.iteration_nb >= o.adc_start_iteration_nb and
                self.iteration_nb % o.adc_interval == 0)

    def maybe_densify_and_prune(self) -> bool:
        o = self.options
        if self.iteration_nb > o.adc_final_iteration_nb:
            return False
        rb = self.render_buffers
        adc_mod.adc_stats(self.adc_buffers, self.fgradients, rb.fgidx_to_gidx, rb.device_counts,
                          self.width, self.height)
        if not (self.iteration_nb >= o.adc_start_iteration_nb and self.iteration_nb % o.adc_interval == 0):
            return False
        new_n = adc_mod.densify_prune_plan(
            self.adc_buffers, self.gaussians, o.densification_mean2d_grad_norm_threshold_ndc,
            o.densification_size_threshold, o.pruning_min_opacity, o.pruning_3d_max_scale,
            self.iteration_nb > o.opacity_reset_interval)
        ng, nm = adc_mod.densify_apply(self.adc_buffers, self.gaussians, self.optimizer.moments, new_n,
                                       o.splitting_scale_factor, self.adc_seed + self.iteration_nb,
                                       rb.fgidx_to_gidx, rb.device_counts)
        self.gaussians.replace(ng)
        self.optimizer.moments = nm
        self.adc_buffers.set_nb_gaussians(new_n)
        return True

    def complete_adc_step(self) -> None:
        """complete_adc_step! (training.jl:455-459): buffers for the new Gaussian count. The
        gradient and render buffers are kept while they hold n Gaussians, else replaced with
        25% headroom (the reference reallocates them at every densify step)."""
        n = self.gaussians.n
        if n > self.fgradients.capacity:
            self.fgradients.resize(n + n // 4)
        rb = self.render_buffers
        if n > rb.capacity_n:
            cap = n + n // 4
            self.render_buffers = RenderBuffers.create(cap, self.tiling.nb_tiles, self.device,
                                                       capacity_dup=max(rb.capacity_dup, 4 * cap))

    # -- one iteration (training.jl:173-244) -----------------------------------------------
    def target_for(self, idx: int) -> torch.Tensor:
        """Device copy of camera idx's target. Host targets are uploaded on a side stream one
        step ahead (prefetch_target), into one of two device buffers, so the copy overlaps the
        previous step's kernels; a target that was not prefetched is copied here."""
        t = self.targets[idx]
        if t.device == self.device:
            return t
        stream = torch.cuda.current_stream(self.device)
        pf = self._prefetched
        if pf is not None and pf[0] == idx and pf[1] is t:
            _, _, slot = pf
            stream.wait_event(self._gt_ready[slot])
        else:
            slot = self._gt_slot ^ 1
            stream.wait_event(self._gt_free[slot])
            self._gt_buffers[slot].copy_(t, non_blocking=True)
        self._prefetched = None
        self._gt_slot = slot
        return self._gt_buffers[slot]

    def advance_camera(self) -> None:
        """Next camera of the shuffled order, re-shuffled after every pass over the cameras
        (training.jl:174-178)."""
        self.cameras_order_idx += 1
        if self.cameras_order_idx >= len(self.cameras_order):
            self.cameras_order = (self._next_orders.pop(0) if self._next_orders
                                  else self.rng.permutation(len(self.cameras)))
            self.cameras_order_idx = 0

    def peek_camera_index(self, ahead: int) -> int:
        """Camera of the step `ahead` steps after the current one (drawing the coming
        permutations from the same generator, in the same order, as training_step would)."""
        pos = self.cameras_order_idx + ahead
        order = self.cameras_order
        k = 0
        while pos >= len(order):
            pos -= len(order)
            if k == len(self._next_orders):
                self._next_orders.append(self.rng.permutation(len(self.cameras)))
            order = self._next_orders[k]
            k += 1
        return int(order[pos])

    def prefetch_target(self) -> None:
        """Start the upload of the next step's host target on the copy stream."""
        idx = self.peek_camera_index(1)
        t = self.targets[idx]
        if t.device == self.device:
            return
        slot = self._gt_slot ^ 1
        if self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(self.device)
        cs = self._copy_stream
        cs.wait_event(self._gt_free[slot])
        with torch.cuda.stream(cs):
            self._gt_buffers[slot].copy_(t, non_blocking=True)
            self._gt_ready[slot].record(cs)
        self._prefetched = (idx, t, slot)

    def training_step(self) -> torch.Tensor:
        """One iteration; returns the device tensor [loss, L1, DSSIM, -] (no host sync)."""
        self.iteration_nb += 1
        self.advance_camera()
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
        rebuild = (self.rebuild_sh_grads and not self.densifies_this_iteration() and
                   self.gaussians.sh_degree == 3)
        backward(self.fgradients, self.rgb_image_grad, self.render_outputs, self.gaussians, cam,
                 self.tiling, self.render_options, rb, skip_sh_grads=rebuild)
        in_adc = self.maybe_densify_and_prune()
        self.update_learning_rates()
        if rebuild:
            self.optimizer.update_rebuild_sh(self.fgradients, rb.fgidx_to_gidx, rb.device_counts,
                                             rb.f2d, cam.position, self.render_options.sh_degree)
        else:
            self.optimizer.update(self.fgradients, rb.fgidx_to_gidx, rb.device_counts,
                                  self.render_options.sh_degree)
        if in_adc:
            self.complete_adc_step()
        self.maybe_opacity_reset()
        self.last_loss = loss
        return loss
