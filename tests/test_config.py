"""Config system: presets, both YAML layouts, numeric coercion, layer layouts, param counts."""

import os

import pytest
import yaml

from mamformer_b200.config import MamformerConfig, PRESETS

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CFG = os.path.join(ROOT, "configs")

# layouts and analytic sizes of the reference zoo (reference config formulas)
ZOO = {
    "ultra-7b": ("ASSSASSSASSSASSSASSSASSSASSSASFF", 38.59, 10.93),
    "7b": ("F" * 32, 8.23, 8.23),
    "ultra-37b": ("ASSS" * 9 + "ASFF", 162.19, 21.08),
    "_1b_dense_kda": ("ASSSASSSASSSASSSASSSASFF", 1.82, 1.74),
    "ultra-371b": ("ASSS" * 11 + "FF", 366.76, 32.57),
    "ultra-671b-max": ("ASSS" * 12 + "FFFF", 670.94, 36.80),
}


@pytest.mark.parametrize("name", sorted(ZOO))
def test_zoo_layouts_and_sizes(name):
    c = MamformerConfig.from_yaml(os.path.join(CFG, f"{name}.yaml"))
    layout, total, active = ZOO[name]
    assert c.layout_string() == layout
    assert round(c.num_parameters_billions, 2) == total
    assert round(c.num_active_parameters_billions, 2) == active


def test_string_eps_is_coerced(tmp_path):
    # PyYAML reads "1e-6" as a string; the reference then fails in RMSNorm.  Here it is a float.
    p = tmp_path / "c.yaml"
    p.write_text("model:\n  d_model: 256\n  n_layers: 2\n  n_heads: 4\n  n_kv_heads: 2\n  head_dim: 64\n"
                 "  rms_norm_eps: 1e-6\n  mamba:\n    d_state: '64'\n")
    c = MamformerConfig.from_yaml(str(p))
    assert isinstance(c.rms_norm_eps, float) and c.rms_norm_eps == 1e-6
    assert c.mamba.d_state == 64


def test_flat_and_nested_roundtrip(tmp_path):
    c = MamformerConfig.from_yaml(os.path.join(CFG, "ultra-7b.yaml"))
    flat = tmp_path / "flat.yaml"
    nested = tmp_path / "nested.yaml"
    c.to_yaml(str(flat))
    c.to_yaml(str(nested), nested=True)
    raw = yaml.safe_load(flat.read_text())
    assert "moe_n_routed_experts" in raw and "comm_moe_n_heads" in raw and "gen_max_context" in raw
    for p in (flat, nested):
        c2 = MamformerConfig.from_yaml(str(p))
        assert c2.to_dict() == c.to_dict()


@pytest.mark.parametrize("name", sorted(PRESETS))
def test_presets_build(name):
    c = MamformerConfig.from_preset(name)
    assert c.d_model % c.n_heads == 0
    assert c.summary()


def test_interleave_patterns():
    from mamformer_b200.config import InterleaveConfig
    i = InterleaveConfig(enabled=True, pattern="attn_every_k", attn_every_k=3, last_layers_dense=1)
    assert [t["is_fusion"] for t in i.resolve_layer_types(7)] == [True, False, False, True, False, False, True]
    i = InterleaveConfig(enabled=True, pattern="custom", attention_layers=[1, 5])
    assert i.resolve_attention_layers(6) == [1, 5]
    with pytest.raises(ValueError):
        InterleaveConfig(pattern="custom", attention_layers=[]).resolve_attention_layers(4)


def test_validation_errors():
    with pytest.raises(ValueError):
        MamformerConfig(d_model=100, n_heads=3)
    with pytest.raises(ValueError):
        MamformerConfig(d_model=256, n_heads=4, n_kv_heads=3, head_dim=64)


def test_kernels_namespace_cpu():
    """Reference-named kernel API on the CPU path (``mamformer.kernels`` names)."""
    import torch
    from mamformer_b200 import kernels
    from mamformer_b200.ops import reference as ref
    torch.manual_seed(0)
    B, H, S, hd = 1, 2, 16, 8
    q1, q2, k, v = (torch.randn(B, H, S, hd) for _ in range(4))
    o1, o2 = kernels.triton_linear_attn_scan(q1, q2, k, v, hd)
    assert o1.shape == (B, H, S, hd) and o2.shape == (B, H, S, hd)
    lam = torch.tensor([0.3, 0.5])
    want = ref.linear_diff_attention_fp32(q1.transpose(1, 2), q2.transpose(1, 2), k.transpose(1, 2),
                                          v.transpose(1, 2), lam, hd).transpose(1, 2)
    got = (o1 - lam.view(1, -1, 1, 1) * o2) / (1 - lam.view(1, -1, 1, 1) + 1e-8)
    assert torch.allclose(got, want, atol=3e-2, rtol=3e-2)
    a = kernels.flash_attn_gqa(q1, k, v, sliding_window=4)
    assert a.shape == q1.shape
    d = kernels.flash_attn_dsa(q1, q2, k, v, 0.2)
    assert d.shape == q1.shape
    x = torch.randn(1, 8, 4)
    y = kernels.triton_ssd_scan(x, torch.rand(1, 8, 4), torch.zeros(3), torch.randn(1, 8, 3), torch.randn(1, 8, 3),
                                torch.ones(4))
    assert y.shape == x.shape
    assert isinstance(kernels.is_triton_available(), bool)
