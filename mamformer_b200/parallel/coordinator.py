"""4-D process topology: data x tensor x pipeline x expert parallelism.

Reference: ``mamformer/parallelism/coordinator.py`` (``ParallelConfig`` 41-122,
``DistributedCoordinator`` 125-305, ``shard_model_4d`` 307-330).  The rank layout is the
reference's ``[DP][TP][PP][EP]`` (EP innermost, so the ranks of one EP group are adjacent GPUs of
one NVSwitch domain), kept so that a launch configuration means the same thing in both
frameworks.

Differences from the reference:

* ``torch.distributed.new_group`` is collective over the whole world, so every rank creates every
  group of every dimension in the same order and keeps the one it belongs to (the reference
  creates only its own groups, which NCCL does not allow once groups differ between ranks).
* Two derived groups used by the data-parallel reductions: ``dense_dp`` (all ranks holding the
  same replicated non-expert shard: the DP x EP plane at fixed TP/PP) and ``expert_dp`` (ranks
  holding the same expert shard: the DP line at fixed TP/PP/EP).
"""

from __future__ import annotations

import itertools
import logging
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn

logger = logging.getLogger(__name__)

DIMS = ("dp", "tp", "pp", "ep")


@dataclass
class ParallelConfig:
    dp_size: int = 1
    tp_size: int = 1
    pp_size: int = 1
    ep_size: int = 1

    @property
    def world_size(self) -> int:
        return self.dp_size * self.tp_size * self.pp_size * self.ep_size

    def sizes(self) -> Dict[str, int]:
        return {"dp": self.dp_size, "tp": self.tp_size, "pp": self.pp_size, "ep": self.ep_size}

    def validate(self, world_size: Optional[int] = None) -> None:
        """Checks of ``coordinator.py:61-103``: positive sizes, TP within one node and a power of
        two, EP <= 64, product equal to the launched world size."""
        for k, v in self.sizes().items():
            if v < 1:
                raise ValueError(f"{k}_size must be >= 1, got {v}")
        if self.world_size == 1:
            return
        if self.tp_size > 8:
            raise ValueError(f"tp_size ({self.tp_size}) > 8 would cross the NVSwitch domain")
        if self.tp_size & (self.tp_size - 1):
            raise ValueError(f"tp_size ({self.tp_size}) must be a power of 2")
        if self.ep_size > 64:
            raise ValueError(f"ep_size ({self.ep_size}) > 64 leaves too few experts per rank")
        if world_size is None and dist.is_available() and dist.is_initialized():
            world_size = dist.get_world_size()
        if world_size is not None and world_size != self.world_size:
            raise ValueError(
                f"ParallelConfig world_size ({self.world_size}) does not match the launched world "
                f"({world_size}): DP={self.dp_size} * TP={self.tp_size} * PP={self.pp_size} * "
                f"EP={self.ep_size}")

    def get_4d_rank(self, global_rank: int) -> Tuple[int, int, int, int]:
        """global rank -> (dp, tp, pp, ep); EP varies fastest."""
        ep = global_rank % self.ep_size
        pp = (global_rank // self.ep_size) % self.pp_size
        tp = (global_rank // (self.ep_size * self.pp_size)) % self.tp_size
        dp = global_rank // (self.ep_size * self.pp_size * self.tp_size)
        return dp, tp, pp, ep

    def get_global_rank(self, dp: int, tp: int, pp: int, ep: int) -> int:
        return ((dp * self.tp_size + tp) * self.pp_size + pp) * self.ep_size + ep

    def group_members(self, dims: Tuple[str, ...]) -> List[List[int]]:
        """All groups spanned by ``dims`` (the other dimensions fixed), in a deterministic order."""
        sizes = self.sizes()
        fixed = [d for d in DIMS if d not in dims]
        out = []
        for fv in itertools.product(*[range(sizes[d]) for d in fixed]):
            base = dict(zip(fixed, fv))
            ranks = []
            for vv in itertools.product(*[range(sizes[d]) for d in dims]):
                c = dict(base)
                c.update(zip(dims, vv))
                ranks.append(self.get_global_rank(c["dp"], c["tp"], c["pp"], c["ep"]))
            out.append(sorted(ranks))
        return out


class DistributedCoordinator:
    """Creates the process groups of a :class:`ParallelConfig` and answers topology queries."""

    GROUP_DIMS = {"tp": ("tp",), "pp": ("pp",), "ep": ("ep",), "dp": ("dp",),
                  "dense_dp": ("dp", "ep"), "expert_dp": ("dp",)}

    def __init__(self, config: ParallelConfig, backend_timeout=None):
        self.config = config
        self._sizes = config.sizes()
        self._ranks = {d: 0 for d in DIMS}
        self._groups: Dict[str, Optional[dist.ProcessGroup]] = {k: None for k in self.GROUP_DIMS}
        self._members: Dict[str, List[int]] = {}
        self._initialized = False

    @property
    def is_initialized(self) -> bool:
        return dist.is_available() and dist.is_initialized()

    def initialize(self) -> "DistributedCoordinator":
        if not self.is_initialized:
            return self
        self.config.validate(dist.get_world_size())
        rank = dist.get_rank()
        self._ranks = dict(zip(DIMS, self.config.get_4d_rank(rank)))
        for name, dims in self.GROUP_DIMS.items():
            size = 1
            for d in dims:
                size *= self._sizes[d]
            if size <= 1:
                self._members[name] = [rank]
                continue
            for members in self.config.group_members(dims):   # every rank creates every group
                g = dist.new_group(members)
                if rank in members:
                    self._groups[name] = g
                    self._members[name] = members
        for d in DIMS:
            g = self._groups[d]
            if g is not None and dist.get_rank(g) != self._ranks[d]:
                raise RuntimeError(f"rank {rank}: position {dist.get_rank(g)} in the {d} group, "
                                   f"expected {self._ranks[d]}")
        if self._groups["tp"] is not None:
            from mamformer_b200.parallel import tensor_parallel
            tensor_parallel.set_tp_group(self._groups["tp"])
        self._initialized = True
        if rank == 0:
            logger.info("4D topology: world=%d DP=%d TP=%d PP=%d EP=%d", self.config.world_size,
                        *[self._sizes[d] for d in DIMS])
        return self

    def get_group(self, dim: str) -> Optional[dist.ProcessGroup]:
        return self._groups.get(dim)

    def get_members(self, dim: str) -> List[int]:
        return self._members.get(dim, [dist.get_rank() if self.is_initialized else 0])

    def get_rank(self, dim: str) -> int:
        return self._ranks.get(dim, 0)

    def get_size(self, dim: str) -> int:
        if dim in self._sizes:
            return self._sizes[dim]
        n = 1
        for d in self.GROUP_DIMS[dim]:
            n *= self._sizes[d]
        return n

    def shard_model(self, model: nn.Module) -> nn.Module:
        """Apply PP (layer slice), TP (shard projections) and EP (shard routed experts) in that
        order (``coordinator.py:263-293``; the reference applies only PP).  DP needs no model
        change: gradients are reduced by the optimizer over ``dense_dp`` / ``expert_dp``."""
        if self.config.world_size == 1 or not self.is_initialized:
            return model
        if self._sizes["pp"] > 1:
            from mamformer_b200.parallel.pipeline_parallel import shard_model_pp
            model = shard_model_pp(model, self._sizes["pp"], self._ranks["pp"], group=self._groups["pp"])
        if self._sizes["tp"] > 1:
            from mamformer_b200.parallel.tensor_parallel import shard_model_tp
            model = shard_model_tp(model, self._sizes["tp"], group=self._groups["tp"])
        if self._sizes["ep"] > 1:
            from mamformer_b200.parallel.expert_parallel import ExpertParallelGroup, shard_experts_ep
            model = shard_experts_ep(model, ExpertParallelGroup(group=self._groups["ep"]),
                                     dp_factor=self.get_size("dense_dp"), dense_dp_group=self._groups["dense_dp"])
        return model

    def get_4d_info(self) -> dict:
        return {
            "world_size": self.config.world_size,
            **{d: {"size": self._sizes[d], "rank": self._ranks[d]} for d in DIMS},
            "groups": {k: (v is not None) for k, v in self._groups.items()},
        }


def shard_model_4d(model: nn.Module, parallel_config: ParallelConfig) -> nn.Module:
    coord = DistributedCoordinator(parallel_config)
    if coord.is_initialized:
        coord.initialize()
    return coord.shard_model(model)
