"""4-D parallel runtime: data, tensor, pipeline and expert parallelism.

Public names follow the reference package ``mamformer.parallelism`` (``__init__.py``).
"""

from mamformer_b200.parallel.coordinator import DistributedCoordinator, ParallelConfig, shard_model_4d
from mamformer_b200.parallel.diagnostics import (CommMonitor, LoadBalanceAnalyzer, ParallelismMonitor,
                                                 PipelineBubbleAnalyzer)
from mamformer_b200.parallel.expert_parallel import (EPEngine, EPMoE, ExpertParallelGroup, expert_combine,
                                                     expert_dispatch, expert_parameters, shard_experts_ep)
from mamformer_b200.parallel.pipeline_parallel import PipelineScheduler1F1B, PipelineStage, shard_model_pp
from mamformer_b200.parallel.tensor_parallel import (ColumnParallelLinear, RowParallelLinear, TPAttention,
                                                     TPMamba2Block, TPSwiGLUFFN, shard_model_tp)

__all__ = [
    "ColumnParallelLinear", "RowParallelLinear", "TPAttention", "TPMamba2Block", "TPSwiGLUFFN", "shard_model_tp",
    "ExpertParallelGroup", "EPEngine", "EPMoE", "expert_dispatch", "expert_combine", "expert_parameters",
    "shard_experts_ep", "PipelineStage", "PipelineScheduler1F1B", "shard_model_pp", "DistributedCoordinator",
    "ParallelConfig", "shard_model_4d", "CommMonitor", "LoadBalanceAnalyzer", "PipelineBubbleAnalyzer",
    "ParallelismMonitor",
]
