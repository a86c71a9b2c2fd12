"""Training engine: one optimizer step over gradient-accumulated micro-batches.

Reference loop: ``scripts/train.py:363-462`` (micro-batch forward, loss / grad_accum backward,
NaN/Inf skip, clip 1.0, AdamW step, scheduler step).  Here:

* the model runs in the bf16 compute layout with fp32 masters in ``MixedPrecisionAdamW``;
* ``return_logits=False`` so the main and MTP losses use the fused linear-cross-entropy path;
* the step never synchronises with the host unless asked (``sync_loss=True``): the loss is
  accumulated on the device and the clip factor is computed on the device;
* with ``sync_loss=True`` the step reads the loss back and, like the reference, skips the
  update when it is not finite.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from mamformer_b200.models.model import MamformerForCausalLM
from mamformer_b200.optim import MixedPrecisionAdamW, create_lr_scheduler, param_groups
from mamformer_b200.utils.precision import to_compute_dtype


@dataclass
class TrainConfig:
    learning_rate: float = 3e-4
    weight_decay: float = 0.1
    adam_beta1: float = 0.9
    adam_beta2: float = 0.95
    adam_epsilon: float = 1e-8
    warmup_steps: int = 2000
    max_steps: int = 100000
    min_lr_ratio: float = 0.1
    max_grad_norm: float = 1.0
    micro_batch: int = 1
    grad_accum: int = 1
    compute_dtype: torch.dtype = torch.bfloat16
    gradient_checkpointing: bool = False


class Trainer:
    """Owns model + optimizer + schedule; ``train_step`` is the public per-step API."""

    def __init__(self, model: MamformerForCausalLM, cfg: TrainConfig,
                 dp_group: Optional[dist.ProcessGroup] = None, expert_params=None,
                 expert_dp_group: Optional[dist.ProcessGroup] = None,
                 ep_group: Optional[dist.ProcessGroup] = None, bucket_mb: float = 64.0,
                 zero_stage: int = 0, dp_transport: str = "nccl"):
        self.cfg = cfg
        self.model = model
        if cfg.compute_dtype != torch.float32:
            to_compute_dtype(model, cfg.compute_dtype)
            if next(model.parameters()).is_cuda:
                from mamformer_b200.ops.linear import use_native_linear
                use_native_linear(model)
        model.return_logits = False
        model.train()
        if cfg.gradient_checkpointing:
            model.model.enable_gradient_checkpointing()
        if expert_params is None:
            expert_params = [p for p in model.parameters() if getattr(p, "_mamf_expert", False)] or None
        self.dp_group = dp_group
        self.optimizer = MixedPrecisionAdamW(
            param_groups(model, cfg.weight_decay), lr=cfg.learning_rate,
            betas=(cfg.adam_beta1, cfg.adam_beta2), eps=cfg.adam_epsilon,
            weight_decay=cfg.weight_decay, max_grad_norm=cfg.max_grad_norm, dp_group=dp_group,
            no_dp_reduce=expert_params, expert_dp_group=expert_dp_group, ep_group=ep_group,
            bucket_mb=bucket_mb, param_order={id(p): i for i, p in enumerate(model.parameters())},
            zero_stage=zero_stage, dp_transport=dp_transport)
        self.scheduler = create_lr_scheduler(self.optimizer, cfg.warmup_steps, cfg.max_steps,
                                             cfg.learning_rate, cfg.min_lr_ratio)
        dev = next(model.parameters()).device
        self.device = dev
        self._loss_acc = torch.zeros((), device=dev)
        self.step_count = 0
        self.skipped_steps = 0
        from mamformer_b200.utils.nvtx import PhaseTimer
        # CUDA-event breakdown of a step (forward / backward / exposed gradient reduction /
        # optimizer); off unless enabled, e.g. by bench.py --breakdown
        self.timer = PhaseTimer(False)

    def train_step(self, input_ids: torch.Tensor, labels: Optional[torch.Tensor] = None,
                   sync_loss: bool = False, check_grads: bool = False):
        """One optimizer step.  ``input_ids`` (micro_batch*grad_accum, S) on the device or in
        (pinned) host memory.  Returns the mean loss (device tensor, or float if sync_loss)."""
        cfg = self.cfg
        if not input_ids.is_cuda and self.device.type == "cuda":
            input_ids = input_ids.to(self.device, non_blocking=True)
            if labels is not None:
                labels = labels.to(self.device, non_blocking=True)
        labels = input_ids if labels is None else labels
        n_micro = max(1, input_ids.shape[0] // cfg.micro_batch)
        eng = getattr(self.model, "_mamf_ep_engine", None)
        self.optimizer.zero_grad()
        self._loss_acc.zero_()
        if eng is not None:
            eng.begin_step(self.model)
        tm = self.timer
        tm.mark("begin")
        for i in range(n_micro):
            sl = slice(i * cfg.micro_batch, (i + 1) * cfg.micro_batch)
            out = self.model(input_ids[sl], labels=labels[sl])
            loss = out["loss"]
            tm.mark("forward")
            if i == n_micro - 1:
                if eng is not None:
                    eng.record_status()           # expert-parallel capacity check of this step
                self.optimizer.reducer.arm()      # overlap the gradient all-reduce with this backward
            (loss / n_micro).backward()
            self._loss_acc += loss.detach().float() / n_micro
            tm.mark("backward")
        if eng is not None and eng.step_overflowed():
            # some expert owner needed more rows than its fixed capacity: discard and rerun the
            # step with the larger capacity the engine has just set (identically on every rank)
            self.optimizer.reduce_gradients()
            self.optimizer.zero_grad()
            return self.train_step(input_ids, labels, sync_loss=sync_loss, check_grads=check_grads)
        loss_val = None
        if sync_loss:
            self.optimizer.reduce_gradients()
            if self.dp_group is not None and dist.is_initialized() and dist.get_world_size(self.dp_group) > 1:
                dist.all_reduce(self._loss_acc, group=self.dp_group)   # same skip decision on all ranks
                self._loss_acc /= dist.get_world_size(self.dp_group)
            eng = getattr(self.model, "_mamf_ep_engine", None)
            if eng is not None:
                eng.check_error()
            loss_val = float(self._loss_acc)
            if loss_val != loss_val or loss_val in (float("inf"), float("-inf")):
                # non-finite loss: skip the update (reference train.py:406-432)
                self.skipped_steps += 1
                self.optimizer.zero_grad()
                return loss_val
        if check_grads:
            # non-finite gradient: zero and skip (reference train.py:436-447); the flag is
            # reduced over the data-parallel group so every rank takes the same decision
            from mamformer_b200.fault import grads_finite
            self.optimizer.reduce_gradients()
            ok = torch.tensor([1.0 if grads_finite(self.optimizer) else 0.0], device=self.device)
            if self.dp_group is not None and dist.is_initialized() and dist.get_world_size(self.dp_group) > 1:
                dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.dp_group)
            if float(ok) < 1.0:
                self.skipped_steps += 1
                self.optimizer.zero_grad()
                return loss_val if sync_loss else self._loss_acc
        if tm.enabled:
            self.optimizer.reduce_gradients()
            tm.mark("dp_reduce_exposed")
        self.optimizer.step()
        tm.mark("optimizer")
        self.scheduler.step()
        self.step_count += 1
        return loss_val if sync_loss else self._loss_acc


def build_trainer(config, train_cfg: TrainConfig, device="cuda", seed: int = 0, dp_group=None):
    torch.manual_seed(seed)
    model = MamformerForCausalLM(config).to(device)
    return Trainer(model, train_cfg, dp_group=dp_group)
