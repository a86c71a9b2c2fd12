"""Pipeline parallelism: contiguous layer slices per stage, 1F1B schedule over NCCL p2p.

Reference: ``mamformer/parallelism/pipeline_parallel.py`` (``_SendForward``/``_RecvForward``
39-96, ``PipelineStage`` 105-240, ``PipelineScheduler1F1B`` 243-438, ``shard_model_pp``
440-480).  Differences:

* the cross-layer SSM state (``pending`` per-step state of the last SSM-only layer, consumed by
  the next attention-only layer) crosses stage boundaries with the activations; whether a
  boundary carries one is fixed by the layer layout and computed once, so both sides agree on
  the messages without a handshake (the reference drops it at stage boundaries);
* activations travel in the compute dtype (the reference receives into fp32 regardless);
* sends and receives that can cross in flight are posted together with ``batch_isend_irecv``
  (send-forward with receive-backward, send-backward with receive-forward), so neighbouring
  stages never wait on each other's unposted operation; the reference's blocking send/recv and
  its 1-element "gradient done" messages are dropped - real gradient tensors flow instead;
* the tied embedding lives on the first stage (lookup) and on the last stage (LM head / MTP
  logits); the two copies start equal and their gradients are summed over the embedding group
  ({first, last}) before the optimizer step.
"""

from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn


class _Absent(nn.Module):
    """Placeholder for a layer owned by another stage (keeps global layer indices)."""

    has_attention = False
    has_ssm = False

    def forward(self, *a, **k):
        raise RuntimeError("layer lives on another pipeline stage")


def split_layers(n_layers: int, pp_size: int) -> List[Tuple[int, int]]:
    """Contiguous, as-even-as-possible layer ranges (earlier stages take the remainder)."""
    base, rem = divmod(n_layers, pp_size)
    out, s = [], 0
    for r in range(pp_size):
        n = base + (1 if r < rem else 0)
        out.append((s, s + n))
        s += n
    return out


def _pending_after(layers, end: int) -> bool:
    """Static: does an SSM state wait for an attention-only layer after layer ``end - 1``?"""
    pending = False
    for i in range(end):
        lt = layers[i]
        if not lt.has_attention and lt.has_ssm and getattr(lt, "h_states_needed", False):
            pending = True
        elif lt.has_attention and not lt.has_ssm and pending:
            pending = False
    return pending


class PipelineStage(nn.Module):
    """One pipeline stage of a ``MamformerForCausalLM``."""

    def __init__(self, model: nn.Module, pp_size: int, pp_rank: int, group=None,
                 ranges: Optional[List[Tuple[int, int]]] = None):
        super().__init__()
        self.pp_size, self.pp_rank, self.group = pp_size, pp_rank, group
        trunk = model.model
        n = len(trunk.layers)
        self.ranges = ranges or split_layers(n, pp_size)
        self.start, self.end = self.ranges[pp_rank]
        self.is_first = pp_rank == 0
        self.is_last = pp_rank == pp_size - 1
        self.recv_state = self.start > 0 and _pending_after(trunk.layers, self.start)
        self.send_state = self.end < n and _pending_after(trunk.layers, self.end)
        for i in range(n):
            if not (self.start <= i < self.end):
                trunk.layers[i] = _Absent()
        if not self.is_last:
            model.mtp = None
            trunk.norm = None
            model.lm_head = None
        if not (self.is_first or self.is_last):
            trunk.embed_tokens = None
        self.model = model
        self.config = model.config
        self.gradient_checkpointing = False

    # -- ranks -------------------------------------------------------------------------------
    def _peer(self, delta: int) -> int:
        r = self.pp_rank + delta
        return dist.get_global_rank(self.group, r) if self.group is not None else r

    def embedding_group_members(self) -> List[int]:
        return [self._peer(-self.pp_rank), self._peer(self.pp_size - 1 - self.pp_rank)]

    # -- compute -----------------------------------------------------------------------------
    def forward(self, x: torch.Tensor, pending: Optional[torch.Tensor] = None,
                input_ids: Optional[torch.Tensor] = None, labels: Optional[torch.Tensor] = None):
        trunk = self.model.model
        h = trunk.embed_tokens(x) if self.is_first else x
        h, pending, _, aux = trunk.run_layers(h, None, self.start, self.end, pending)
        if not self.is_last:
            return h, pending
        h = trunk.norm(h)
        res = self.model.compute_head(h, input_ids, labels, None, False, {})
        return res["loss"], res

    def compute_loss(self, hidden: torch.Tensor, input_ids: torch.Tensor, labels: torch.Tensor):
        """Loss on the last stage from its final hidden state (before the norm)."""
        h = self.model.model.norm(hidden)
        return self.model.compute_head(h, input_ids, labels, None, False, {})["loss"]

    def enable_gradient_checkpointing(self) -> None:
        self.model.model.gradient_checkpointing = True

    def disable_gradient_checkpointing(self) -> None:
        self.model.model.gradient_checkpointing = False


class PipelineScheduler1F1B:
    """One-forward-one-backward schedule over ``num_microbatches`` micro-batches."""

    def __init__(self, stage: PipelineStage, num_microbatches: int, d_model: int,
                 dtype: torch.dtype = torch.bfloat16, d_state: Optional[int] = None):
        self.stage = stage
        self.m = int(num_microbatches)
        self.d_model = d_model
        self.dtype = dtype
        self.d_state = d_state if d_state is not None else stage.config.mamba.d_state
        self._pending_sends = []

    # -- p2p ---------------------------------------------------------------------------------
    def _shapes(self, mb: int, S: int, with_state: bool):
        sh = [(mb, S, self.d_model)]
        if with_state:
            sh.append((mb, S, self.d_state))
        return sh

    def _exchange(self, send: Optional[List[torch.Tensor]], send_to: Optional[int],
                  recv_shapes: Optional[list], recv_from: Optional[int], device) -> Optional[List[torch.Tensor]]:
        ops, recv = [], None
        if send is not None and send_to is not None:
            for t in send:
                ops.append(dist.P2POp(dist.isend, t.contiguous(), send_to, group=self.stage.group))
        if recv_shapes is not None and recv_from is not None:
            recv = [torch.empty(s, device=device, dtype=self.dtype) for s in recv_shapes]
            for t in recv:
                ops.append(dist.P2POp(dist.irecv, t, recv_from, group=self.stage.group))
        if ops:
            reqs = dist.batch_isend_irecv(ops)
            for r in reqs:
                r.wait()
            if send is not None:
                self._pending_sends.append(send)     # keep alive until the step ends
        return recv

    # -- schedule ----------------------------------------------------------------------------
    def run_forward_backward(self, input_ids: torch.Tensor, labels: Optional[torch.Tensor] = None):
        """``input_ids`` (m*mb, S) on every stage (the last stage needs the labels and the
        MTP targets).  Returns the mean loss on the last stage, None elsewhere."""
        st = self.stage
        labels = input_ids if labels is None else labels
        mb = input_ids.shape[0] // self.m
        S = input_ids.shape[1]
        dev = input_ids.device
        prev = st._peer(-1) if not st.is_first else None
        nxt = st._peer(1) if not st.is_last else None
        in_shapes = self._shapes(mb, S, st.recv_state) if not st.is_first else None
        out_shapes = self._shapes(mb, S, st.send_state) if not st.is_last else None
        n_warm = min(st.pp_size - st.pp_rank - 1, self.m)
        n_steady = self.m - n_warm
        inputs, outputs, losses = [], [], []

        def fwd(i, recv):
            ids = input_ids[i * mb:(i + 1) * mb]
            lab = labels[i * mb:(i + 1) * mb]
            if st.is_first:
                x, pend, ins = ids, None, []
            else:
                x = recv[0].requires_grad_()
                pend = recv[1].requires_grad_() if st.recv_state else None
                ins = [x] + ([pend] if pend is not None else [])
            if st.is_last:
                loss, _ = st(x, pend, ids, lab)
                losses.append(loss.detach())
                inputs.append(ins)
                outputs.append([loss / self.m])
                return None
            h, pend_out = st(x, pend)
            outs = [h] + ([pend_out.to(self.dtype)] if st.send_state else [])
            inputs.append(ins)
            outputs.append(outs)
            return [o.detach() for o in outs]

        def bwd(i, grads):
            outs = outputs[i]
            if st.is_last:
                torch.autograd.backward(outs[0])
            else:
                torch.autograd.backward(outs, grads)
            ins = inputs[i]
            outputs[i] = inputs[i] = None
            if st.is_first:
                return None
            return [t.grad if t.grad is not None else torch.zeros_like(t) for t in ins]

        for i in range(n_warm):
            recv = self._exchange(None, None, in_shapes, prev, dev)
            y = fwd(i, recv)
            self._exchange(y, nxt, None, None, dev)
        recv = self._exchange(None, None, in_shapes, prev, dev) if n_steady > 0 else None
        for j in range(n_steady):
            y = fwd(n_warm + j, recv)
            g = self._exchange(y, nxt, out_shapes, nxt, dev)
            dx = bwd(j, g)
            if j == n_steady - 1:
                self._exchange(dx, prev, None, None, dev)
                recv = None
            else:
                recv = self._exchange(dx, prev, in_shapes, prev, dev)
        for j in range(n_steady, self.m):
            g = self._exchange(None, None, out_shapes, nxt, dev)
            dx = bwd(j, g)
            self._exchange(dx, prev, None, None, dev)
        self._pending_sends.clear()
        if st.is_last:
            return torch.stack(losses).mean()
        return None

    def sync_tied_embedding_grads(self, embedding_group=None) -> None:
        """Sum the tied-embedding gradient over the first and last stage."""
        st = self.stage
        if st.pp_size == 1 or embedding_group is None or not (st.is_first or st.is_last):
            return
        w = st.model.model.embed_tokens.weight
        g = getattr(w, "main_grad", None)
        if g is None:
            g = w.grad
        if g is not None:
            dist.all_reduce(g, group=embedding_group)


def shard_model_pp(model: nn.Module, pp_size: int, pp_rank: int, group=None) -> nn.Module:
    """Keep this stage's layers (plus embedding / head where they belong); returns a
    :class:`PipelineStage`.  Must run before the optimizer is built."""
    if pp_size <= 1:
        return model
    return PipelineStage(model, pp_size, pp_rank, group)


def bubble_fraction(pp_size: int, num_microbatches: int) -> float:
    """Idle fraction of the 1F1B schedule: (p - 1) / (p - 1 + m)."""
    return (pp_size - 1) / (pp_size - 1 + num_microbatches)
