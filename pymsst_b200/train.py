"""Training step, benchmark configurations and the seeded loss-curve runner.

``Trainer.step`` is one training step of the reference's manual loop
(src/pymsst/validation/direct_compare.py:350-384): forward with the loss under
autocast (bf16 / fp16 or off), backward of the (fp16: scaled) loss, optional
gradient clipping, Adam step through the gradient scaler.  Data parallelism
follows the reference's Lightning ``strategy="ddp"`` (src/pymsst/cli.py:
357-372): one process per GPU, gradients averaged over ranks by NCCL -- one
all-reduce of the flat gradient buffer (optionally in buckets that overlap
the backward) in the flat / captured step, torch DDP otherwise.
``run_loss_curve`` is the ``compare-direct`` analogue: a seeded run that
records the loss of every step.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from . import config as cfg
from . import synthetic

BSR_BASE = dict(dim=192, depth=6, stereo=True, num_stems=1, time_transformer_depth=1, freq_transformer_depth=1,
                dim_head=64, heads=8, mask_estimator_depth=2, mlp_expansion_factor=4)


@dataclass(frozen=True)
class BenchConfig:
    """A benchmark workload: model, per-GPU batch, chunk length and precision."""

    name: str
    model_type: str
    model: dict
    batch: int
    chunk: int
    amp: torch.dtype | None
    stems: int = 1
    lr: float = 1e-4
    notes: str = ""
    extra: dict = field(default_factory=dict)

    @property
    def audio_seconds_per_step(self) -> float:
        return self.batch * self.chunk / synthetic.SAMPLE_RATE

    @property
    def frames(self) -> int:
        return self.chunk // self.model.get("stft_hop_length", 512) + 1


CONFIGS = {
    "config0": BenchConfig("config0", "bs_roformer", BSR_BASE, batch=2, chunk=32768, amp=None,
                           notes="BS-RoFormer fp32, batch 2 x 32768"),
    "config1": BenchConfig("config1", "mel_band_roformer",
                           dict(BSR_BASE, num_bands=60, sample_rate=44100), batch=2, chunk=32768,
                           amp=torch.bfloat16, notes="Mel-band RoFormer, 60 bands, batch 2 x 32768"),
    "config3": BenchConfig("config3", "bs_roformer", BSR_BASE, batch=4, chunk=131584, amp=torch.bfloat16,
                           notes="BS-RoFormer bf16 AMP, chunk 131584 (258 frames), batch 4 per GPU"),
    "config4": BenchConfig("config4", "bs_roformer", dict(BSR_BASE, dim=384, depth=12, num_stems=4), batch=2,
                           chunk=352800, amp=torch.bfloat16, stems=4,
                           notes="BS-RoFormer dim 384 depth 12, 4 stems, chunk 352800, batch 2 per GPU"),
}


def build_model(bench: BenchConfig, seed: int = 0) -> torch.nn.Module:
    torch.manual_seed(seed)
    return cfg.build_model(bench.model_type, **bench.model)


class Trainer:
    """Owns the model (optionally data-parallel), its Adam optimizer and, for fp16, its gradient scaler.

    One ``step`` is one iteration of the reference's manual loop
    (src/pymsst/validation/direct_compare.py:350-384): forward and loss under
    autocast, ``scaler.scale(loss).backward()``, ``scaler.unscale_`` before
    gradient clipping, ``scaler.step`` / ``scaler.update``.  As there, the
    ``torch.amp.GradScaler`` is enabled for fp16 autocast (``grad_scaler``
    None) and off otherwise; bf16 and fp32 steps are plain Adam steps.

    ``flat_params`` (default: on with ``cuda_graph``) makes every parameter a
    view of one flat fp32 buffer and every gradient a slot of one flat
    gradient buffer: Adam updates one tensor, and with more than one rank the
    flat gradients are all-reduced directly (mean over ranks) instead of
    through DDP, after rank 0's parameters are broadcast to every rank.
    ``overlap_allreduce`` splits that all-reduce into buckets of about
    ``bucket_cap_mb`` that start, asynchronously, as soon as the backward has
    finished every gradient of a bucket; the flat layout is rebuilt after the
    first backward so each bucket is a contiguous range in the order the
    gradients become final.

    ``cuda_graph=True`` captures the whole training step (forward, backward,
    gradient all-reduce, scaler and Adam) once into a CUDA graph and replays
    it; the step is then free of per-kernel host launch cost, which otherwise
    bounds a training step of this size.  The first call runs three untimed
    forward/backward passes on its batch (no parameter update) so every
    library plan and cached table exists before the capture, initialises the
    Adam state with an update of zero, and then captures; every call,
    including the first, applies exactly one update.  Input shapes must stay
    fixed; the returned loss tensor is overwritten by the next step."""

    def __init__(self, model: torch.nn.Module, *, lr: float = 1e-4, amp_dtype: torch.dtype | None = None,
                 grad_clip: float = 0.0, distributed: bool = False, device: torch.device | None = None,
                 fused_adam: bool = True, bucket_cap_mb: float = 64.0, cuda_graph: bool = False,
                 grad_scaler: bool | None = None, flat_params: bool | None = None, overlap_allreduce: bool = False):
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.model = model.to(self.device)
        self.amp_dtype = amp_dtype
        self.grad_clip = float(grad_clip)
        self.module = self.model
        self.distributed = distributed
        self.cuda_graph = bool(cuda_graph) and self.device.type == "cuda"
        on_cuda = self.device.type == "cuda"
        params = [p for p in self.model.parameters() if p.requires_grad]
        self.params = params
        flat = self.cuda_graph if flat_params is None else bool(flat_params)
        self.flat = flat and bool(params) and all(p.dtype == torch.float32 for p in params)
        if self.cuda_graph and not self.flat and distributed:
            raise ValueError("a captured multi-rank step needs fp32 parameters in the flat layout")
        use_scaler = (amp_dtype == torch.float16) if grad_scaler is None else bool(grad_scaler)
        self.scaler = torch.amp.GradScaler(self.device.type, enabled=use_scaler)
        if distributed and not self.flat:
            from torch.nn.parallel import DistributedDataParallel

            self.module = DistributedDataParallel(
                self.model, device_ids=[self.device.index] if on_cuda else None,
                bucket_cap_mb=bucket_cap_mb, gradient_as_bucket_view=True, broadcast_buffers=False,
            )
        self.flat_param = self.flat_grad = self.flat_half = None
        self._half_live = [False]  # True only inside _forward_backward, after the mirror's refresh
        self.bucket_bytes = int(bucket_cap_mb * 2**20)
        self.overlap = bool(overlap_allreduce) and distributed and self.flat
        self._buckets: list[tuple[int, int, list[int]]] = []
        self._bucket_of: list[int] = []
        self._pending: list[int] = []
        self._works: list = []
        self._launched: list[bool] = []
        self._relayout_done = not self.overlap
        self._ready_order: list[int] | None = None
        self.bucket_launches = 0  # bucketed all-reduces issued so far (host-side count)
        self._profiling = False
        self._hook_handles: list = []
        opt_params = params
        if self.flat:
            self._build_flat(list(range(len(params))))
            if distributed:
                # every rank starts from rank 0's parameters (DDP does the same broadcast at construction)
                dist.broadcast(self.flat_param.data, 0)
            opt_params = [self.flat_param]
            if self.overlap:
                self._hook_handles = [p.register_post_accumulate_grad_hook(self._grad_ready_hook(i))
                                      for i, p in enumerate(params)]
        self.optimizer = torch.optim.Adam(opt_params, lr=lr, fused=fused_adam and on_cuda,
                                          capturable=self.cuda_graph)
        self._graph = None
        self._static = None
        self.launches_per_step = None  # this package's kernels in one captured step

    def close(self) -> None:
        """Release the captured step (which holds this trainer's NCCL calls when distributed) and the gradient
        hooks.  Call it before destroy_process_group: a live graph with captured collectives keeps the process
        group's teardown waiting, and the hooks (closures over the trainer) keep the trainer, and so its graph,
        alive until a garbage collection."""
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        for h in self._hook_handles:
            h.remove()
        self._hook_handles = []
        self._works = []
        self._graph = None
        self._static = None

    # ------------------------------------------------------------- flat layout
    def _build_flat(self, order: list[int]):
        """(Re)build the flat fp32 parameter and gradient buffers with the parameters in ``order``.

        Every parameter starts on a 128-element boundary (512 bytes fp32, 256 bytes in the 16-bit mirror), as
        a fresh allocation would: libraries pick their kernels by operand alignment, and a view at an odd
        offset would get a different (differently rounded) GEMM than the per-step cast it replaces.  The
        padding holds zeros, which Adam leaves at zero and the all-reduce averages as zeros."""
        params = self.params
        offsets = [0] * len(params)
        total = 0
        for i in order:
            offsets[i] = total
            total += (params[i].numel() + 127) // 128 * 128
        flat_param = torch.zeros(total, dtype=torch.float32, device=self.device)
        flat_grad = torch.zeros(total, dtype=torch.float32, device=self.device)
        with torch.no_grad():
            for p, off in zip(params, offsets):
                flat_param[off:off + p.numel()].copy_(p.reshape(-1))
        if self.flat_param is None:
            self.flat_param = torch.nn.Parameter(flat_param)
        else:
            self.flat_param.data = flat_param
        self.flat_grad = flat_grad
        self.flat_param.grad = flat_grad
        self._offsets = offsets
        self._grad_views = []
        for p, off in zip(params, offsets):
            n = p.numel()
            p.data = self.flat_param.data[off:off + n].view_as(p)
            self._grad_views.append(flat_grad[off:off + n].view_as(p))
        if self.amp_dtype in (torch.bfloat16, torch.float16) and self.device.type == "cuda":
            # the parameters in the activation type, refreshed by one copy kernel per step (the fused ops read
            # them through fused.lowp_weight instead of casting each weight with its own kernel)
            self.flat_half = torch.zeros(total, dtype=self.amp_dtype, device=self.device)
            for p, off in zip(params, offsets):
                p._pmb_half = self.flat_half[off:off + p.numel()].view_as(p)
                p._pmb_half_live = self._half_live
        # all-reduce buckets: contiguous ranges of the flat buffer, in layout order
        self._buckets = []
        cur: list[int] = []
        start = 0
        size = 0
        for i in order:
            cur.append(i)
            size += ((params[i].numel() + 127) // 128 * 128) * 4
            if size >= self.bucket_bytes:
                end = offsets[i] + (params[i].numel() + 127) // 128 * 128
                self._buckets.append((start, end, cur))
                start, cur, size = end, [], 0
        if cur:
            self._buckets.append((start, total, cur))
        self._bucket_of = [0] * len(params)
        for b, (_, _, idx) in enumerate(self._buckets):
            for i in idx:
                self._bucket_of[i] = b

    def _grad_ready_hook(self, index: int):
        def hook(p):
            if self._ready_order is not None:
                self._ready_order.append(index)
            if self._relayout_done and self._pending:
                b = self._bucket_of[index]
                self._pending[b] -= 1
                if self._pending[b] == 0:
                    self._launch_bucket(b)
        return hook

    def _launch_bucket(self, b: int):
        start, end, idx = self._buckets[b]
        pairs = [(self._grad_views[i], self.params[i].grad) for i in idx if self.params[i].grad is not None]
        if pairs:
            torch._foreach_copy_([v for v, _ in pairs], [g for _, g in pairs])
        self._works.append(dist.all_reduce(self.flat_grad[start:end], async_op=True))
        self._launched[b] = True
        self.bucket_launches += 1

    def _begin_backward(self):
        if self.overlap and self._relayout_done and not self._profiling:
            self._pending = [len(idx) for _, _, idx in self._buckets]
            self._launched = [False] * len(self._buckets)
            self._works = []

    def _finish_grads(self):
        """After the backward: the gradients in the flat buffer, all-reduced (mean) when distributed."""
        if self.overlap and self._relayout_done and self._pending:
            for b in range(len(self._buckets)):
                if not self._launched[b]:  # a bucket with parameters that got no gradient this step
                    self._launch_bucket(b)
            for w in self._works:
                w.wait()
            self._works = []
            self._pending = []
            self.flat_grad.div_(dist.get_world_size())
            return
        if self.flat:
            self._gather_flat_grads()
        if self.distributed:
            self._allreduce_grads()

    def _maybe_relayout(self):
        """First backward with overlap on: lay the flat buffers out in the order the gradients became final."""
        if self._relayout_done or self._ready_order is None:
            return
        seen = []
        for i in self._ready_order:
            if i not in seen:
                seen.append(i)
        seen += [i for i in range(len(self.params)) if i not in seen]
        # every rank must use the same layout: take rank 0's order
        order = torch.tensor(seen, dtype=torch.int64, device=self.device)
        dist.broadcast(order, 0)
        self._build_flat([int(i) for i in order.tolist()])
        self._ready_order = None
        self._relayout_done = True

    # ------------------------------------------------------------- eager
    def _forward_backward(self, mixture, target):
        if self.flat_half is not None:
            # this step's low-precision mirror of the parameters (one kernel), served by fused.lowp_weight
            # only within this forward / backward
            with torch.no_grad():
                self.flat_half.copy_(self.flat_param)
            self._half_live[0] = True
        try:
            with torch.autocast(self.device.type, dtype=self.amp_dtype or torch.bfloat16,
                                enabled=self.amp_dtype is not None, cache_enabled=not self.cuda_graph):
                loss = self.module(mixture, target)
            self._begin_backward()
            self.scaler.scale(loss).backward()
        finally:
            self._half_live[0] = False
        return loss

    def _gather_flat_grads(self):
        """Per-parameter gradients into the flat gradient buffer (multi-tensor copies); parameters that got
        no gradient keep zeros there."""
        pairs = [(v, p.grad) for v, p in zip(self._grad_views, self.params) if p.grad is not None]
        torch._foreach_copy_([v for v, _ in pairs], [g for _, g in pairs])

    def _allreduce_grads(self):
        if self.flat_grad is not None:
            dist.all_reduce(self.flat_grad)
            self.flat_grad.div_(dist.get_world_size())
            return
        grads = [p.grad for p in self.params if p.grad is not None]
        flat = torch.cat([g.reshape(-1) for g in grads])
        dist.all_reduce(flat)
        flat.div_(dist.get_world_size())
        # back into the gradients with multi-tensor copies (a handful of launches, not one per parameter)
        parts = flat.split([g.numel() for g in grads])
        torch._foreach_copy_(grads, [v.view_as(g) for v, g in zip(parts, grads)])

    def _update(self):
        if self.grad_clip:
            self.scaler.unscale_(self.optimizer)
            torch.nn.utils.clip_grad_norm_([self.flat_param] if self.flat else self.model.parameters(),
                                           self.grad_clip)
        self.scaler.step(self.optimizer)
        self.scaler.update()

    def _warm_relayout(self, mixture, target):
        """One untimed forward/backward that records the order in which gradients become final, then the
        flat layout in that order (overlap_allreduce only)."""
        if self._relayout_done:
            return
        self._zero_grads()
        self._ready_order = []
        self._forward_backward(mixture, target)
        self._maybe_relayout()
        self._zero_grads()

    def step(self, mixture: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
        """One training step on device tensors; returns the detached loss (device)."""
        if self.cuda_graph:
            return self._graph_step(mixture, target)
        self._warm_relayout(mixture, target)
        self._zero_grads()
        if not self.flat:
            self.optimizer.zero_grad(set_to_none=True)
        loss = self._forward_backward(mixture, target)
        self._finish_grads()
        self._update()
        return loss.detach()

    def check_kernels(self) -> None:
        """Raise if a tensor-core kernel of this package gave up waiting (its outputs would be incomplete).

        Every tcgen05 / TMA wait in the library is bounded; a wait that runs out sets a device flag and the
        kernel winds down instead of hanging.  Reading the flag synchronises with the device."""
        from . import _native as nat

        if self.device.type != "cuda":
            return
        torch.cuda.synchronize(self.device)
        code = int(nat.library().pmb_umma_timeout(0))
        if code:
            raise nat.KernelError(f"a tensor-core kernel timed out waiting (site code {code:#x}); "
                                  "the last steps' results are not valid")

    # ------------------------------------------------------------- graph
    def _capture(self, mixture, target):
        from . import _native as nat

        static_mix, static_tgt = mixture.clone(), target.clone()
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self._warm_relayout(static_mix, static_tgt)
            for _ in range(3):
                self._zero_grads()
                self._forward_backward(static_mix, static_tgt)
                self._finish_grads()
            # Adam state (moments, device step counters) created by an update of zero
            if self.flat_grad is not None:
                self.flat_grad.zero_()
            else:
                for p in self.params:
                    p.grad = torch.zeros_like(p)
            self.optimizer.step()
            for group in self.optimizer.param_groups:
                for p in group["params"]:
                    st = self.optimizer.state[p]
                    if "step" in st:
                        st["step"].zero_()
        torch.cuda.current_stream(self.device).wait_stream(side)
        self._zero_grads()
        self.check_kernels()
        graph = torch.cuda.CUDAGraph()
        before = nat.library().pmb_launch_count()
        with torch.cuda.graph(graph):
            loss = self._forward_backward(static_mix, static_tgt)
            self._finish_grads()
            self._update()
        self.launches_per_step = int(nat.library().pmb_launch_count() - before)
        self._graph = graph
        self._static = (static_mix, static_tgt, loss.detach())

    def profile_graph(self) -> torch.cuda.CUDAGraph:
        """A second captured graph of this step's forward and backward alone (no collective, no update) on the
        captured step's static inputs, for per-kernel device timing: entry points called under
        ``_native.time_entries(..., external=True)`` while it is captured get timing events in the graph."""
        if self._static is None:
            raise RuntimeError("profile_graph needs the captured step: run one step first")
        static_mix, static_tgt, _ = self._static
        self._zero_grads()
        graph = torch.cuda.CUDAGraph()
        self._profiling = True
        try:
            with torch.cuda.graph(graph):
                self._forward_backward(static_mix, static_tgt)
        finally:
            self._profiling = False
        return graph

    def _zero_grads(self):
        """Drop the per-parameter gradients (the backward allocates fresh ones); the flat buffer, when there
        is one, stays attached to the optimizer's single tensor."""
        for p in self.params:
            p.grad = None

    def _graph_step(self, mixture, target):
        if self._graph is None:
            self._capture(mixture, target)
        static_mix, static_tgt, loss = self._static
        if mixture.data_ptr() != static_mix.data_ptr():
            static_mix.copy_(mixture, non_blocking=True)
        if target.data_ptr() != static_tgt.data_ptr():
            static_tgt.copy_(target, non_blocking=True)
        self._graph.replay()
        return loss

    def step_host(self, mixture: torch.Tensor, target: torch.Tensor, loss_out: torch.Tensor | None = None):
        """Step from host tensors (pinned for async copies); the loss is copied back to ``loss_out``, or
        returned as a float (after checking the kernels' timeout flag) when no ``loss_out`` is given."""
        if self.cuda_graph and self._static is not None:
            static_mix, static_tgt, _ = self._static
            static_mix.copy_(mixture, non_blocking=True)
            static_tgt.copy_(target, non_blocking=True)
            loss = self._graph_step(static_mix, static_tgt)
        else:
            mix = mixture.to(self.device, non_blocking=True)
            tgt = target.to(self.device, non_blocking=True)
            loss = self.step(mix, tgt)
        if loss_out is None:
            value = float(loss)
            self.check_kernels()
            return value
        loss_out.copy_(loss, non_blocking=True)
        return loss_out


def run_loss_curve(model: torch.nn.Module, batches, *, lr: float = 1e-4, amp_dtype=None,
                   device: torch.device | None = None, grad_clip: float = 0.0, cuda_graph: bool = False,
                   grad_scaler: bool | None = None) -> list[float]:
    """Seeded training run; returns the loss of every step (the compare-direct curve)."""
    trainer = Trainer(model, lr=lr, amp_dtype=amp_dtype, device=device, grad_clip=grad_clip, cuda_graph=cuda_graph,
                      grad_scaler=grad_scaler)
    losses = []
    for mix, tgt in batches:
        losses.append(float(trainer.step(mix.to(trainer.device), tgt.to(trainer.device))))
    trainer.check_kernels()
    return losses


def compare_loss_curves(a: list[float], b: list[float]) -> dict:
    """Mean / max absolute difference over the overlapping steps (comparison.py:223-241)."""
    n = min(len(a), len(b))
    if n == 0:
        raise ValueError("no overlapping loss points to compare")
    diffs = [abs(x - y) for x, y in zip(a[:n], b[:n])]
    return {"compared_points": n, "mean_abs_diff": sum(diffs) / n, "max_abs_diff": max(diffs)}


def max_over_ranks(values: list[float], device: torch.device) -> list[float]:
    """Element-wise max of per-rank timings (the job's time is its slowest rank's)."""
    t = torch.tensor(values, dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.cpu()]


def init_distributed(timeout_s: float = 120.0) -> tuple[int, int, int]:
    """(rank, world, local_rank) from torchrun's environment; NCCL on CUDA, gloo otherwise."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        import datetime

        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return rank, world, local
