"""Model behaviour on CPU (fp32 reference path): shapes, losses, generation, checkpoints."""

import os
import sys

import pytest
import torch

from mamformer_b200 import MamformerConfig, MamformerForCausalLM, MamformerModel

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def debug_cfg():
    return MamformerConfig.from_preset("debug")


@pytest.fixture(scope="module")
def model(debug_cfg):
    torch.manual_seed(0)
    return MamformerForCausalLM(debug_cfg)


def test_hidden_shape(debug_cfg):
    m = MamformerModel(debug_cfg)
    out = m(torch.randint(0, 1000, (2, 32)))
    assert out["last_hidden_state"].shape == (2, 32, 256)
    assert torch.isfinite(out["last_hidden_state"]).all()


def test_logits_loss_and_grads(model):
    ids = torch.randint(0, 1000, (2, 16))
    out = model(ids, labels=ids)
    assert out["logits"].shape == (2, 16, 1000)
    assert out["loss"].ndim == 0 and out["loss"].item() > 0
    out["loss"].backward()
    for n, p in model.named_parameters():
        if p.grad is not None:
            assert torch.isfinite(p.grad).all(), n
    model.zero_grad()


def test_parameter_count_matches_reference(model):
    # measured with the reference implementation on the same preset
    assert model.num_parameters() == 3_492_224


def test_weight_tying(model):
    model.eval()
    ids = torch.randint(0, 1000, (1, 8))
    logits = model(ids)["logits"]
    h = model.model(ids)["last_hidden_state"]
    torch.testing.assert_close(logits, h @ model.model.embed_tokens.weight.t(), atol=1e-5, rtol=1e-5)
    model.train()


def test_overfit_fixed_batch(debug_cfg):
    torch.manual_seed(1)
    m = MamformerForCausalLM(debug_cfg)
    ids = torch.randint(0, 500, (4, 32))
    opt = torch.optim.AdamW(m.parameters(), lr=1e-3)
    losses = []
    for _ in range(15):
        opt.zero_grad()
        loss = m(ids, labels=ids)["loss"]
        loss.backward()
        torch.nn.utils.clip_grad_norm_(m.parameters(), 1.0)
        opt.step()
        losses.append(loss.item())
    assert losses[-1] < losses[0] - 0.5


def test_generation_greedy_deterministic(model):
    model.eval()
    ids = torch.randint(0, 500, (1, 4))
    with torch.no_grad():
        a = model.generate(ids, max_new_tokens=6, temperature=0)
        b = model.generate(ids, max_new_tokens=6, temperature=0)
        c = model.generate(ids, max_new_tokens=6, temperature=1.0, top_k=0, top_p=1.0)
    torch.testing.assert_close(a, b)
    assert a.shape == (1, 10) and c.shape == (1, 10) and int(c.max()) < 1000
    model.train()


def test_cache_structure(debug_cfg):
    m = MamformerModel(debug_cfg)
    out = m(torch.randint(0, 1000, (1, 8)), use_cache=True)
    assert len(out["cache"]) == len(m.layers)


def test_gradient_checkpointing(debug_cfg):
    m = MamformerForCausalLM(debug_cfg)
    m.model.enable_gradient_checkpointing()
    ids = torch.randint(0, 1000, (2, 16))
    m(ids, labels=ids)["loss"].backward()
    assert any(p.grad is not None for p in m.parameters())


def test_state_dict_roundtrip_moe():
    cfg = MamformerConfig.from_yaml(os.path.join(ROOT, "configs", "_arch_verify.yaml"))
    d = cfg.to_dict()
    d.update(d_model=128, n_heads=2, n_kv_heads=1, head_dim=64, vocab_size=300, d_ff=256,
             moe_shared_expert_intermediate_dim=64, moe_expert_intermediate_dim=32, kda_diff_latent_dim=64)
    cfg = MamformerConfig.from_dict(d)
    torch.manual_seed(0)
    a = MamformerForCausalLM(cfg)
    sd = a.state_dict()
    assert "model.layers.1.ffn.routed_experts.15.down_proj.weight" in sd
    assert not any("routed_gate_proj" in k for k in sd)
    torch.manual_seed(1)
    b = MamformerForCausalLM(cfg)
    b.load_state_dict(sd)
    for k, v in b.state_dict().items():
        torch.testing.assert_close(v, sd[k])


def test_mtp_loss_present_in_training():
    cfg = MamformerConfig.from_yaml(os.path.join(ROOT, "configs", "_arch_verify.yaml"))
    d = cfg.to_dict()
    d.update(d_model=128, n_heads=2, n_kv_heads=1, head_dim=64, vocab_size=300, d_ff=256, n_layers=4,
             interleave_fusion_layers=[3], moe_shared_expert_intermediate_dim=64,
             moe_expert_intermediate_dim=32, kda_diff_latent_dim=64)
    m = MamformerForCausalLM(MamformerConfig.from_dict(d))
    ids = torch.randint(0, 300, (2, 24))
    out = m(ids, labels=ids)
    assert "mtp_loss" in out and out["loss"].item() > out["main_loss"].item()
    m.eval()
    assert "mtp_loss" not in m(ids, labels=ids)


def _config1():
    from mamformer_b200.config import DSAConfig, InterleaveConfig, KDADiffConfig, MambaConfig
    return MamformerConfig(d_model=256, n_layers=4, n_heads=4, n_kv_heads=4, head_dim=64, d_ff=1024,
                           vocab_size=32000, max_seq_len=256, mamba=MambaConfig(expand=2, d_state=64, d_conv=4),
                           kda_diff=KDADiffConfig(enabled=True, kernel_dim=64, latent_dim=128, use_dynamic_ratio=True),
                           dsa=DSAConfig(enabled=False),
                           interleave=InterleaveConfig(enabled=True, pattern="cross_layer", attn_every_k=3,
                                                       first_layer_attn=True, last_layers_dense=0, fusion_layers=[3]))


def test_golden_loss_curve_config1():
    """Tiny hybrid benchmark config (fp32, seed 0, 10 AdamW steps): all ten losses the
    reference recorded for the same seed, batch and optimizer."""
    torch.manual_seed(0)
    m = MamformerForCausalLM(_config1())
    with torch.no_grad():
        m.model.layers[3].attention.interleave_gate.mlp[2].bias.fill_(10.0)
    ids = torch.randint(0, 32000, (2, 256), generator=torch.Generator().manual_seed(0))
    opt = torch.optim.AdamW(m.parameters(), lr=3e-4)
    golden = [10.4113, 10.1362, 9.9614, 9.8093, 9.6655, 9.5245, 9.3837, 9.2421, 9.0984, 8.9572]
    for want in golden:
        opt.zero_grad()
        loss = m(ids, labels=ids)["loss"]
        loss.backward()
        opt.step()
        assert abs(loss.item() - want) < 5e-4, (loss.item(), want)
    assert m.model.layers[3].attention.last_choice == "full"
    assert m.model.layers[0].attention.last_choice == "linear"


def _reference_root():
    """Directory holding the reference's ``mamformer`` package: the installed copy under
    baseline/_ref, else a source tree named by MAMF_REFERENCE_SRC (imported read-only, no
    bytecode written)."""
    for cand in (os.path.join(ROOT, "baseline", "_ref"), os.environ.get("MAMF_REFERENCE_SRC", "")):
        if cand and os.path.isdir(os.path.join(cand, "mamformer")):
            return cand
    return None


REF = _reference_root()


@pytest.mark.skipif(REF is None, reason="reference package not found (baseline/_ref or MAMF_REFERENCE_SRC)")
@pytest.mark.parametrize("which", ["debug", "arch_verify"])
def test_bit_parity_with_reference(which):
    """Same seed -> identical state dict (names, shapes, values) and identical loss."""
    sys.path.insert(0, REF)
    sys.dont_write_bytecode = True
    try:
        from mamformer.config import MamformerConfig as RC
        from mamformer.model import MamformerForCausalLM as RM
        import mamformer.layers.kda_diff as kd
        kd.triton_linear_attn_scan = None
    finally:
        sys.path.remove(REF)
    if which == "debug":
        c1, c2 = RC.from_preset("debug"), MamformerConfig.from_preset("debug")
    else:
        path = os.path.join(ROOT, "configs", "_arch_verify.yaml")
        c1, c2 = RC.from_yaml(path), MamformerConfig.from_yaml(path)
    torch.manual_seed(0)
    a = RM(c1)
    torch.manual_seed(0)
    b = MamformerForCausalLM(c2)
    sa, sb = a.state_dict(), b.state_dict()
    assert set(sa) == set(sb)
    for k in sa:
        assert torch.equal(sa[k], sb[k]), k
    ids = torch.randint(0, c1.vocab_size, (2, 32), generator=torch.Generator().manual_seed(1))
    assert a(ids, labels=ids)["loss"].item() == b(ids, labels=ids)["loss"].item()


@pytest.mark.parametrize("moe", [False, True])
def test_full_layer_checkpointing_matches_plain_backward(moe):
    """enable_gradient_checkpointing(all_layers=True): same loss, same gradients, and MoE routing
    statistics updated once per forward (the recomputation replays the stashed bias)."""
    d = MamformerConfig.from_yaml(os.path.join(ROOT, "configs", "ultra-7b.yaml")).to_dict()
    d.update(d_model=64, n_heads=2, n_kv_heads=1, head_dim=32, n_layers=4, vocab_size=128,
             interleave_fusion_layers=[3], interleave_last_layers_dense=1, moe_enabled=moe,
             moe_n_routed_experts=8, moe_top_k=2, moe_expert_intermediate_dim=32,
             moe_shared_expert_intermediate_dim=32, kda_diff_kernel_dim=32, kda_diff_latent_dim=32,
             d_ff=128, mamba_d_state=32, mtp_enabled=False)
    cfg = MamformerConfig.from_dict(d)
    ids = torch.randint(0, 128, (2, 48), generator=torch.Generator().manual_seed(3))
    res = []
    for ck in (False, True):
        torch.manual_seed(0)
        m = MamformerForCausalLM(cfg)
        if ck:
            m.model.enable_gradient_checkpointing(all_layers=True)
        for _ in range(2):                      # the second pass sees biases moved by the first
            m.zero_grad()
            loss = m(ids, labels=ids)["loss"]
            loss.backward()
        grads = {n: p.grad.clone() for n, p in m.named_parameters() if p.grad is not None}
        bufs = {n: b.clone() for n, b in m.named_buffers() if "expert_bias" in n or "_expert_counts" in n}
        res.append((loss.item(), grads, bufs))
    (l0, g0, b0), (l1, g1, b1) = res
    assert abs(l0 - l1) < 1e-6
    assert set(g0) == set(g1)
    for n in g0:
        assert torch.allclose(g0[n], g1[n], rtol=1e-5, atol=1e-7), n
    for n in b0:
        assert torch.equal(b0[n], b1[n]), n


def test_native_layer_switch_keeps_embedding_semantics_on_cpu(debug_cfg):
    """use_native_linear also switches nn.Embedding to FusedEmbedding; on CPU (no main_grad
    routing) the module behaves exactly like nn.Embedding and keeps its state-dict keys."""
    from mamformer_b200.ops.linear import FusedEmbedding, use_native_linear
    torch.manual_seed(0)
    m = MamformerForCausalLM(debug_cfg)
    keys = list(m.state_dict().keys())
    ids = torch.randint(0, debug_cfg.vocab_size, (2, 9))
    ref = m.model.embed_tokens.weight[ids].clone()
    use_native_linear(m)
    assert isinstance(m.model.embed_tokens, FusedEmbedding)
    assert list(m.state_dict().keys()) == keys
    y = m.model.embed_tokens(ids)
    assert torch.equal(y, ref)
    y.sum().backward()
    g = m.model.embed_tokens.weight.grad
    want = torch.zeros_like(g).index_add_(0, ids.reshape(-1), torch.ones(ids.numel(), g.shape[1]))
    assert torch.equal(g, want)
