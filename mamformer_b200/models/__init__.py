"""Model and layer modules (the reference's ``mamformer.layers`` + ``mamformer.model``)."""

from mamformer_b200.models.norm import RMSNorm, LayerNorm
from mamformer_b200.models.rope import RotaryEmbedding, CachedRotaryEmbedding, apply_rotary_emb
from mamformer_b200.models.attention import GroupedQueryAttention
from mamformer_b200.models.mamba2 import Mamba2Block, selective_scan
from mamformer_b200.models.ffn import SwiGLUFFN, GEGLUFFN, StandardFFN
from mamformer_b200.models.moe import DeepSeekMoE, MoERouter
from mamformer_b200.models.st_moe import SpaceTimeMoE
from mamformer_b200.models.communicative_moe import CommunicativeMoE, ExpertCommunicationLayer
from mamformer_b200.models.dsa import DifferentialStateAttention
from mamformer_b200.models.kda_diff import (KDADiffAttention, LinearDiffAttention, FullDiffAttention,
                                            DynamicInterleaveGate, kernel_feature_map)
from mamformer_b200.models.mtp import MultiTokenPredictor
from mamformer_b200.models.math_opt import (DynamicGate, EntropyRouter, AdaptiveLambda, DeepNorm,
                                            compute_moe_entropy_loss)
from mamformer_b200.models.hybrid import MamformerBlock
from mamformer_b200.models.model import MamformerModel, MamformerForCausalLM

__all__ = [
    "RMSNorm", "LayerNorm", "RotaryEmbedding", "CachedRotaryEmbedding", "apply_rotary_emb",
    "GroupedQueryAttention", "DifferentialStateAttention", "Mamba2Block", "selective_scan",
    "SwiGLUFFN", "GEGLUFFN", "StandardFFN", "DeepSeekMoE", "MoERouter", "SpaceTimeMoE",
    "CommunicativeMoE", "ExpertCommunicationLayer", "KDADiffAttention", "LinearDiffAttention",
    "FullDiffAttention", "DynamicInterleaveGate", "kernel_feature_map", "MultiTokenPredictor",
    "DynamicGate", "EntropyRouter", "AdaptiveLambda", "DeepNorm", "compute_moe_entropy_loss",
    "MamformerBlock", "MamformerModel", "MamformerForCausalLM",
]
