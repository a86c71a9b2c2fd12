#!/usr/bin/env python
"""Write ``configs/_1b_ultra.yaml``: a ~1B model with every Ultra feature switched on
(KDA-Diff with dynamic ratio, 32-expert DeepSeekMoE top-4, MTP depth 2, cross-layer
interleave with two fusion layers).  Reference: ``scripts/gen_1b_ultra_config.py``, whose
architecture values are kept so the config name means the same model in both frameworks.

    python scripts/gen_1b_ultra_config.py [--out configs/_1b_ultra.yaml]
"""
import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import _common  # noqa: E402

ARCH = {
    "name": "Mamformer-1B-Ultra", "d_model": 2048, "n_layers": 24, "n_heads": 16, "n_kv_heads": 4,
    "head_dim": 128, "d_ff": 5632, "vocab_size": 64000, "max_seq_len": 4096,
    "mamba": {"expand": 1, "d_state": 128, "d_conv": 4},
    "rope": {"theta": 10000.0},
    "moe": {"enabled": True, "n_shared_experts": 2, "shared_expert_intermediate_dim": 1024,
            "n_routed_experts": 32, "top_k": 4, "expert_intermediate_dim": 384,
            "aux_loss_free": True, "bias_update_speed": 0.001},
    "kda_diff": {"enabled": True, "linear_ratio": 3, "kernel_dim": 64, "latent_dim": 256,
                 "use_dynamic_ratio": True},
    "mtp": {"enabled": True, "depth": 2, "loss_weight": 0.3},
    "interleave": {"enabled": True, "pattern": "cross_layer", "attn_every_k": 4, "first_layer_attn": True,
                   "last_layers_dense": 2, "fusion_layers": [22, 23]},
    "generation": {"max_context": 4096, "max_output_tokens": 2048},
}


def build():
    from mamformer_b200.config import MamformerConfig
    return MamformerConfig.from_dict({"model": ARCH})


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--out", default=os.path.join(_common.ROOT, "configs", "_1b_ultra.yaml"))
    a = p.parse_args(argv)
    cfg = build()
    cfg.to_yaml(a.out)
    print(cfg.summary())
    return a.out


if __name__ == "__main__":
    main()
