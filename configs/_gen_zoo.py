"""Regenerate the YAML model zoo in this folder from the values below (nested schema).

The model values are those of the reference zoo (``configs/*.yaml`` of Mamformer), so a
config name means the same architecture in both frameworks.  ``training:`` holds the defaults
the training scripts read when the matching command-line flag is not given.
"""

import os
import sys

import yaml

HERE = os.path.dirname(os.path.abspath(__file__))

TRAIN = dict(batch_size=1, gradient_accumulation_steps=8, learning_rate=3.0e-4, weight_decay=0.1,
             warmup_steps=2000, max_steps=100000, lr_schedule="cosine", optimizer="adamw",
             adam_beta1=0.9, adam_beta2=0.95, adam_epsilon=1.0e-8, mixed_precision="bf16",
             gradient_checkpointing=True)

KDA = dict(enabled=True, linear_ratio=3, kernel_dim=128, latent_dim=512, use_dynamic_ratio=True)
DSA_OFF = dict(enabled=False, lambda_init=0.8, use_state_injection=True, state_injection_dim=64)
MTP = dict(enabled=True, depth=2, loss_weight=0.3)
GEN = lambda ctx, out: dict(max_context=ctx, max_output_tokens=out, default_temperature=0.7,  # noqa: E731
                             default_top_k=50, default_top_p=0.9)


def inter(fusion):
    return dict(enabled=True, pattern="cross_layer", attn_every_k=4, first_layer_attn=True,
                last_layers_dense=2, fusion_layers=fusion)


def moe(shared_dim, n_routed, routed_dim):
    return dict(enabled=True, n_shared_experts=2, shared_expert_intermediate_dim=shared_dim,
                n_routed_experts=n_routed, top_k=8, expert_intermediate_dim=routed_dim,
                router_temperature=1.0, aux_loss_free=True, bias_update_speed=0.001)


def mamba(expand):
    return dict(expand=expand, d_state=128, d_conv=4, dt_rank="auto")


ZOO = {
    "7b": dict(name="Mamformer-7b", d_model=4096, n_layers=32, n_heads=32, n_kv_heads=8, head_dim=128,
               d_ff=9216, vocab_size=128000, max_seq_len=8192, tie_word_embeddings=True, mamba=mamba(1),
               rope=dict(theta=10000.0, use_yarn=False), dropout=0.0, rms_norm_eps=1.0e-6,
               initializer_range=0.02),
    "pro-7b": dict(name="Mamformer-pro-7b", d_model=4096, n_layers=26, n_heads=32, n_kv_heads=8,
                   head_dim=128, d_ff=14336, vocab_size=32000, max_seq_len=8192, tie_word_embeddings=True,
                   sliding_window=4096, use_sliding_window=True, mamba=mamba(1), interleave=inter([24, 25]),
                   rope=dict(theta=1000000.0, use_yarn=True), dropout=0.0, rms_norm_eps=1.0e-6,
                   initializer_range=0.02),
    "ultra-7b": dict(name="Mamformer-Ultra-7b", d_model=4096, n_layers=32, n_heads=32, n_kv_heads=8,
                     head_dim=128, d_ff=9216, vocab_size=128000, max_seq_len=8192, tie_word_embeddings=True,
                     sliding_window=4096, use_sliding_window=True, mamba=mamba(2),
                     moe=moe(2304, 128, 576), dsa=DSA_OFF, kda_diff=KDA, mtp=MTP, interleave=inter([30, 31]),
                     rope=dict(theta=1000000.0, use_yarn=True), dropout=0.0, rms_norm_eps=1.0e-6,
                     initializer_range=0.02),
    "ultra-7b-dense": dict(name="Mamformer-Ultra-7b-Dense", d_model=4096, n_layers=32, n_heads=32,
                           n_kv_heads=8, head_dim=128, d_ff=14336, vocab_size=128000, max_seq_len=8192,
                           tie_word_embeddings=True, sliding_window=4096, use_sliding_window=True,
                           mamba=mamba(2), moe=dict(enabled=False), dsa=DSA_OFF, kda_diff=KDA, mtp=MTP,
                           interleave=inter([30, 31]), rope=dict(theta=1000000.0, use_yarn=True),
                           dropout=0.0, rms_norm_eps=1.0e-6, initializer_range=0.02),
    "ultra-37b": dict(name="Mamformer-Ultra-37B", description="~200B total / ~37B active | 128K context | 32K output",
                      d_model=6144, n_layers=40, n_heads=48, n_kv_heads=8, head_dim=128, d_ff=12288,
                      vocab_size=128000, max_seq_len=131072, tie_word_embeddings=True, use_sliding_window=True,
                      sliding_window=16384, mamba=mamba(1), moe=moe(3072, 256, 768), dsa=DSA_OFF,
                      kda_diff=KDA, mtp=MTP, interleave=inter([38, 39]),
                      rope=dict(theta=10000000.0, use_yarn=True, yarn_scale=16.0, yarn_original_max_seq_len=8192),
                      generation=GEN(131072, 32768), dropout=0.0, rms_norm_eps=1.0e-6, initializer_range=0.01),
    "ultra-371b": dict(name="Mamformer-Ultra-371B", description="371B total / 28B active | 256K context | 65K output",
                       d_model=7168, n_layers=46, n_heads=56, n_kv_heads=8, head_dim=128, d_ff=14336,
                       vocab_size=128000, max_seq_len=262144, tie_word_embeddings=True, use_sliding_window=True,
                       sliding_window=16384, mamba=mamba(1), moe=moe(3584, 384, 896), dsa=DSA_OFF,
                       kda_diff=KDA, mtp=MTP, interleave=inter([44, 45]),
                       rope=dict(theta=20000000.0, use_yarn=True, yarn_scale=32.0, yarn_original_max_seq_len=8192),
                       generation=GEN(262144, 65536), dropout=0.0, rms_norm_eps=1.0e-6, initializer_range=0.008),
    "ultra-671b-max": dict(name="Mamformer-Ultra-671B",
                           description="671B total / 37B active | 1M context | 163K output [MAX]",
                           d_model=7168, n_layers=52, n_heads=56, n_kv_heads=8, head_dim=128, d_ff=14336,
                           vocab_size=128000, max_seq_len=1048576, tie_word_embeddings=True,
                           use_sliding_window=True, sliding_window=32768, mamba=mamba(1),
                           moe=moe(3584, 640, 896), dsa=DSA_OFF, kda_diff=KDA, mtp=MTP,
                           interleave=inter([48, 49, 50, 51]),
                           rope=dict(theta=50000000.0, use_yarn=True, yarn_scale=128.0,
                                     yarn_original_max_seq_len=8192, yarn_beta_fast=32, yarn_beta_slow=1),
                           generation=GEN(1048576, 163800), dropout=0.0, rms_norm_eps=1.0e-6,
                           initializer_range=0.006),
}
TRAIN_OVERRIDES = {
    "ultra-7b": dict(learning_rate=2.0e-4),
    "ultra-37b": dict(gradient_accumulation_steps=12, learning_rate=2.0e-4, warmup_steps=3000, max_steps=150000),
    "ultra-371b": dict(gradient_accumulation_steps=12, learning_rate=1.8e-4, warmup_steps=3500, max_steps=150000),
    "ultra-671b-max": dict(gradient_accumulation_steps=16, learning_rate=1.5e-4, warmup_steps=4000,
                           max_steps=200000, max_grad_norm=0.5),
}


def arch_verify_config():
    """The small all-features model of ``_arch_verify.yaml`` (8 layers, KDA-Diff, 16-expert MoE,
    MTP, cross-layer interleave with one fusion layer) used by the parity tests."""
    sys.path.insert(0, os.path.dirname(HERE))
    from mamformer_b200.config import (DSAConfig, InterleaveConfig, KDADiffConfig, MambaConfig,
                                       MamformerConfig, MoEConfig, MTPConfig)
    arch = MamformerConfig(name="ArchVerify", d_model=512, n_layers=8, n_heads=8, n_kv_heads=2, head_dim=64,
                           d_ff=2048, vocab_size=8000, max_seq_len=512,
                           mamba=MambaConfig(expand=1, d_state=64, d_conv=4, dt_rank=32),
                           moe=MoEConfig(enabled=True, n_shared_experts=2, shared_expert_intermediate_dim=512,
                                         n_routed_experts=16, top_k=4, expert_intermediate_dim=256),
                           kda_diff=KDADiffConfig(enabled=True, kernel_dim=64, latent_dim=256),
                           mtp=MTPConfig(enabled=True), dsa=DSAConfig(enabled=False),
                           interleave=InterleaveConfig(enabled=True, pattern="cross_layer", attn_every_k=4,
                                                       last_layers_dense=1, fusion_layers=[7]))
    arch.generation.max_context, arch.generation.max_output_tokens = 512, 256
    return arch


def main():
    for name, model in ZOO.items():
        train = dict(TRAIN, max_seq_len=model["max_seq_len"], **TRAIN_OVERRIDES.get(name, {}))
        with open(os.path.join(HERE, f"{name}.yaml"), "w") as fh:
            fh.write(f"# {model['name']} - generated by configs/_gen_zoo.py\n")
            yaml.safe_dump({"model": model, "training": train}, fh, sort_keys=False, default_flow_style=None)
    sys.path.insert(0, os.path.dirname(HERE))
    from mamformer_b200.config import (DSAConfig, InterleaveConfig, KDADiffConfig, MambaConfig,
                                       MamformerConfig, MTPConfig)
    arch_verify_config().to_yaml(os.path.join(HERE, "_arch_verify.yaml"))
    dense = MamformerConfig(name="Mamformer-1b", d_model=2048, n_layers=24, n_heads=16, n_kv_heads=4,
                            head_dim=128, d_ff=5632, vocab_size=64000, max_seq_len=2048,
                            mamba=MambaConfig(expand=1, d_state=128, d_conv=4, dt_rank=128),
                            kda_diff=KDADiffConfig(enabled=True, kernel_dim=128, latent_dim=512),
                            mtp=MTPConfig(enabled=True), dsa=DSAConfig(enabled=False),
                            interleave=InterleaveConfig(enabled=True, pattern="cross_layer", attn_every_k=4,
                                                        last_layers_dense=2, fusion_layers=[22, 23]))
    dense.generation.max_context, dense.generation.max_output_tokens = 4096, 2048
    dense.to_yaml(os.path.join(HERE, "_1b_dense_kda.yaml"))
    os.makedirs(os.path.join(HERE, "distributed"), exist_ok=True)
    with open(os.path.join(HERE, "distributed", "ultra-671b-64gpu.yaml"), "w") as fh:
        yaml.safe_dump({"parallelism": {"dp": 2, "tp": 4, "pp": 4, "ep": 2},
                        "training": dict(TRAIN, gradient_accumulation_steps=16, learning_rate=1.5e-4,
                                         warmup_steps=4000, max_steps=200000, max_seq_len=1048576,
                                         max_grad_norm=0.5)}, fh, sort_keys=False)


if __name__ == "__main__":
    main()
