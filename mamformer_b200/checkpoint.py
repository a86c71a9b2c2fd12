"""Checkpoints: the reference's single-file format, per-rank shards, consolidation, resume.

Reference format (``scripts/train.py:535-576``, ``train_distributed.py:356-377``,
``train_grpo.py:774-810``): ``torch.save({"model": state_dict, "optimizer": ..., "scheduler": ...,
"step": N})`` to ``checkpoint_step_{N}.pt`` / ``checkpoint_final.pt``, fp32 weights, and the
state-dict key layout of the reference model (kept by the model code: the same module names;
the stacked routed experts are written and read as per-expert keys).  Inference loads
``ckpt["model"]`` or a raw state dict with ``strict=False``.

B200 layout:

* the model's bf16 parameters are views into the optimizer's flat buffers; checkpoints store
  the fp32 master weights (the parameters are pointed at their masters while the state dict is
  taken), so a saved model equals the reference's fp32 checkpoint of the same weights;
* a parallel job (TP / EP / PP / DP) writes one shard per rank plus the slicing metadata
  (``checkpoint_step_{N}/rank{r:05d}.pt``); :func:`consolidate` rebuilds the single-file layout
  (TP slices placed by their recorded indices, EP experts by their global indices, PP stages by
  their global layer indices, DP replicas deduplicated) and :func:`load_model_state` loads a
  consolidated state into any (re)sharded model.  The optimizer state of a sharded job is
  resumable only with the same layout; a new layout restarts the moments from the weights.
"""

from __future__ import annotations

import contextlib
import glob
import os
import re
from typing import Dict, Optional

import torch
import torch.distributed as dist


def _masters(optimizer):
    """param id -> fp32 weight (a temporary full copy for ZeRO-sharded segments, gathered
    collectively); empty without a mixed-precision optimizer."""
    if optimizer is None or not hasattr(optimizer, "master_views"):
        return {}
    return optimizer.master_views()


@contextlib.contextmanager
def fp32_parameters(model, optimizer, ms=None):
    """Temporarily point every parameter at its fp32 master weight."""
    ms = _masters(optimizer) if ms is None else ms
    saved = []
    for p in model.parameters():
        m = ms.get(id(p))
        if m is not None:
            saved.append((p, p.data))
            p.data = m
    try:
        yield
    finally:
        for p, d in saved:
            p.data = d


def model_state_dict(model, optimizer=None, cpu: bool = True) -> Dict[str, torch.Tensor]:
    with fp32_parameters(model, optimizer):
        sd = model.state_dict()
        sd = {k: (v.detach().float() if v.is_floating_point() else v.detach()) for k, v in sd.items()}
    if cpu:
        sd = {k: v.cpu() for k, v in sd.items()}
    return sd


def load_model_state(model, state: Dict[str, torch.Tensor], optimizer=None, strict: bool = False):
    """Load a consolidated state dict into a (possibly sharded) model.  Tensor-parallel slices are
    cut out of the full tensors; expert-parallel experts are picked by the MoE load hook; keys of
    other pipeline stages are ignored.  With a mixed-precision optimizer the fp32 values land in
    the masters and the bf16 copies are refreshed."""
    local = {}
    named = dict(model.named_parameters())
    for k, v in state.items():
        p = named.get(k)
        sl = getattr(p, "_mamf_tp_slice", None) if p is not None else None
        local[k] = v.index_select(sl[0], sl[1].to(v.device)) if (sl is not None and v.shape != p.shape) else v
    ms = _masters(optimizer)
    with fp32_parameters(model, optimizer, ms):
        res = model.load_state_dict(local, strict=strict)
    if optimizer is not None and hasattr(optimizer, "segments"):
        with torch.no_grad():
            for _, seg in optimizer.segments:
                if not seg.low:
                    continue
                if seg.sharded:          # the loaded values sit in the gathered temporary
                    p0, o0 = seg.params[0], seg.offsets[0]
                    full = ms[id(p0)].reshape(-1).view(-1)
                    flat = torch.empty(0, device=full.device, dtype=torch.float32).set_(
                        full.untyped_storage(), full.storage_offset() - o0, (seg.numel,))
                    seg.master.copy_(flat[seg.lo:seg.hi])
                    seg.low_flat.copy_(flat)
                else:
                    seg.low_flat.copy_(seg.master)
    return res


def save_checkpoint(path: str, model, optimizer=None, scheduler=None, step: int = 0, extra: Optional[dict] = None,
                    write: bool = True):
    """Checkpoint in the reference format.  With a ZeRO-sharded optimizer every rank must call
    this (the fp32 weights are gathered); only ranks with ``write`` touch the file."""
    state = model_state_dict(model, optimizer)
    if not write:
        return path
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    # a ZeRO-sharded optimizer state belongs in per-rank shards (save_sharded), not in one file
    keep_opt = optimizer is not None and not getattr(optimizer, "sharded", False)
    ck = {"model": state, "step": int(step),
          "optimizer": optimizer.state_dict() if keep_opt else None,
          "scheduler": scheduler.state_dict() if scheduler is not None else None}
    if extra:
        ck.update(extra)
    tmp = path + ".tmp"
    torch.save(ck, tmp)
    os.replace(tmp, path)
    return path


def load_checkpoint(path: str, model, optimizer=None, scheduler=None, strict: bool = False,
                    map_location="cpu") -> int:
    """Resume: model (+ optimizer, scheduler); returns the saved step."""
    ck = torch.load(path, map_location=map_location, weights_only=False)
    state = ck["model"] if isinstance(ck, dict) and "model" in ck else ck
    load_model_state(model, state, optimizer, strict=strict)
    if optimizer is not None and isinstance(ck, dict) and ck.get("optimizer") is not None:
        try:
            optimizer.load_state_dict(ck["optimizer"])
        except (KeyError, ValueError, RuntimeError) as e:   # another layout: moments restart
            import logging
            logging.getLogger(__name__).warning("optimizer state not restored: %s", e)
    if scheduler is not None and isinstance(ck, dict) and ck.get("scheduler") is not None:
        scheduler.load_state_dict(ck["scheduler"])
    return int(ck.get("step", 0)) if isinstance(ck, dict) else 0


# ---- sharded --------------------------------------------------------------------------------------
def _slice_meta(model) -> dict:
    meta = {}
    for n, p in model.named_parameters():
        sl = getattr(p, "_mamf_tp_slice", None)
        if sl is not None:
            meta[n] = {"dim": int(sl[0]), "index": sl[1].cpu(), "full": None}
    return meta


def save_sharded(directory: str, model, optimizer=None, scheduler=None, step: int = 0, rank: Optional[int] = None,
                 full_shapes: Optional[Dict[str, tuple]] = None) -> str:
    """Every rank writes its shard (model fp32 weights + optimizer + slicing metadata)."""
    r = rank if rank is not None else (dist.get_rank() if dist.is_available() and dist.is_initialized() else 0)
    os.makedirs(directory, exist_ok=True)
    meta = _slice_meta(model)
    for n, m in meta.items():
        if full_shapes and n in full_shapes:
            m["full"] = tuple(full_shapes[n])
    shard = {"model": model_state_dict(model, optimizer), "step": int(step), "tp_slices": meta,
             "optimizer": optimizer.state_dict() if optimizer is not None else None,
             "scheduler": scheduler.state_dict() if scheduler is not None else None}
    path = os.path.join(directory, f"rank{r:05d}.pt")
    torch.save(shard, path + ".tmp")
    os.replace(path + ".tmp", path)
    return path


def consolidate(directory: str, out_path: Optional[str] = None) -> Dict[str, torch.Tensor]:
    """Merge the rank shards of ``directory`` into one state dict in the reference layout."""
    files = sorted(glob.glob(os.path.join(directory, "rank*.pt")))
    if not files:
        raise FileNotFoundError(f"no rank*.pt shards in {directory}")
    full: Dict[str, torch.Tensor] = {}
    pieces: Dict[str, list] = {}
    step = 0
    for f in files:
        sh = torch.load(f, map_location="cpu", weights_only=False)
        step = max(step, int(sh.get("step", 0)))
        meta = sh.get("tp_slices", {})
        for k, v in sh["model"].items():
            if k in meta:
                pieces.setdefault(k, []).append((meta[k], v))
            elif k not in full:
                full[k] = v
    for k, parts in pieces.items():
        m0 = parts[0][0]
        dim = m0["dim"]
        n_total = sum(int(m["index"].numel()) for m, _ in parts)
        if m0.get("full") is not None:
            shape = list(m0["full"])
        else:
            shape = list(parts[0][1].shape)
            shape[dim] = max(int(m["index"].max()) + 1 for m, _ in parts)
        t = torch.zeros(shape, dtype=parts[0][1].dtype)
        seen = set()
        for m, v in parts:
            key = tuple(m["index"].tolist())
            if key in seen:          # a replica of the same slice (DP)
                continue
            seen.add(key)
            t.index_copy_(dim, m["index"], v)
        full[k] = t
    if out_path:
        torch.save({"model": full, "step": step, "optimizer": None, "scheduler": None}, out_path)
    return full


def latest_checkpoint(directory: str) -> Optional[str]:
    """Highest ``checkpoint_step_{N}.pt`` (or sharded directory) in ``directory``."""
    best, best_n = None, -1
    for p in glob.glob(os.path.join(directory, "checkpoint_*step_*")):
        m = re.search(r"step_(\d+)", os.path.basename(p))
        if m and int(m.group(1)) > best_n:
            best, best_n = p, int(m.group(1))
    return best
