"""mamformer_b200: a B200-native hybrid Mamba/Transformer MoE training framework.

Public API mirrors the reference package ``mamformer`` (``mamformer/__init__.py:18-46``).
"""

from mamformer_b200.config import MamformerConfig
from mamformer_b200.models.model import MamformerModel, MamformerForCausalLM
from mamformer_b200.tokenizer import MamformerTokenizer
from mamformer_b200.generation import GenerationMixin, RuntimeGenerationConfig
from mamformer_b200.models.communicative_moe import CommunicativeMoE
from mamformer_b200.thinking import ThinkingConfig, ThinkingMode, MultiPathController
from mamformer_b200.thinking_data import (format_sequence_with_thinking, format_labels_with_thinking,
                                          format_batch_with_thinking)

__version__ = "0.1.0"


def __getattr__(name):
    # Lazily-imported optional pieces (avoid import cost / cycles at package import).
    if name in ("ReflectionModule", "SelfReflectiveGenerator", "add_reflection_to_model"):
        from mamformer_b200 import reflection
        return getattr(reflection, name)
    if name in ("StochasticGRPOConfig", "sample_token_mask"):
        from mamformer_b200 import sgrpo
        return getattr(sgrpo, name)
    raise AttributeError(name)


__all__ = [
    "MamformerConfig", "MamformerModel", "MamformerForCausalLM", "MamformerTokenizer",
    "GenerationMixin", "RuntimeGenerationConfig", "ReflectionModule", "SelfReflectiveGenerator",
    "add_reflection_to_model", "CommunicativeMoE", "ThinkingConfig", "ThinkingMode",
    "MultiPathController", "StochasticGRPOConfig", "sample_token_mask",
    "format_sequence_with_thinking", "format_labels_with_thinking", "format_batch_with_thinking",
]
