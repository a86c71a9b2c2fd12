"""Command-line entry points run end to end (tiny config, synthetic tokens, a few steps)."""
import glob
import os
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(args, timeout=600, env=None):
    e = dict(os.environ)
    e["PYTHONPATH"] = ROOT + os.pathsep + e.get("PYTHONPATH", "")
    if env:
        e.update(env)
    r = subprocess.run([sys.executable] + args, cwd=ROOT, capture_output=True, text=True, timeout=timeout, env=e)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    return r


def _train_args(tmp_path, extra=()):
    return ["scripts/train.py", "--config", "debug", "--data", str(tmp_path / "nodata"),
            "--max_seq_len", "64", "--batch_size", "2", "--gradient_accumulation_steps", "2",
            "--max_steps", "3", "--warmup_steps", "1", "--save_every", "2", "--log_every", "1",
            "--output_dir", str(tmp_path / "ck")] + list(extra)


def test_train_script_cpu_writes_checkpoints_and_resumes(tmp_path):
    _run(_train_args(tmp_path))
    cks = sorted(glob.glob(str(tmp_path / "ck" / "checkpoint_*")))
    assert cks, "no checkpoint written"
    ck = torch.load(cks[-1], map_location="cpu", weights_only=False)
    assert "model" in ck and int(ck["step"]) >= 2
    # resume from the step-2 checkpoint and run to step 3
    step2 = str(tmp_path / "ck" / "checkpoint_step_2.pt")
    assert os.path.exists(step2)
    _run(_train_args(tmp_path, ["--resume", step2]))


def test_generate_script_cpu(tmp_path):
    r = _run(["scripts/generate.py", "--config", "debug", "--prompt", "hello", "--max_new_tokens", "8",
              "--temperature", "0"])
    assert r.stdout.strip() != ""


@pytest.mark.gpu
def test_train_script_gpu_bf16(tmp_path):
    """The pre-training entry point on one GPU in bf16: native kernels, native optimizer."""
    _run(_train_args(tmp_path, ["--bf16"]))
    assert glob.glob(str(tmp_path / "ck" / "checkpoint_*"))


def _torchrun(args, nproc=2, timeout=900):
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return _run(["-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
                 "--master-addr", "127.0.0.1", f"--master-port={port}"] + args, timeout=timeout,
                env={"CUDA_VISIBLE_DEVICES": "", "OMP_NUM_THREADS": "1"})


@pytest.mark.parametrize("layout", [["--tp", "2"], ["--pp", "2"], ["--dp", "2"]])
def test_train_distributed_script_cpu(tmp_path, layout):
    """The 4-D entry point under torchrun with two gloo ranks: runs a few steps and writes its
    per-rank checkpoint shards."""
    args = ["scripts/train_distributed.py", "--config", "debug", "--data", str(tmp_path / "nodata"),
            "--max_seq_len", "64", "--batch_size", "1", "--gradient_accumulation_steps", "2",
            "--max_steps", "2", "--warmup_steps", "1", "--save_every", "2", "--log_every", "1",
            "--no_gradient_checkpointing", "--output_dir", str(tmp_path / "ck")] + layout
    _torchrun(args)
    assert glob.glob(str(tmp_path / "ck" / "**" / "*.pt"), recursive=True), "no checkpoint written"


def test_train_script_expert_parallel_cpu(tmp_path):
    """scripts/train.py with --ep 2 on a small MoE config: routed experts sharded over two gloo
    ranks, a few steps, per-rank checkpoint shards."""
    import yaml
    from mamformer_b200 import MamformerConfig
    d = MamformerConfig.from_preset("debug").to_dict()
    d.update(moe_enabled=True, moe_n_routed_experts=8, moe_top_k=2, moe_expert_intermediate_dim=64,
             moe_n_shared_experts=1, moe_shared_expert_intermediate_dim=64)
    cfg_path = tmp_path / "moe.yaml"
    cfg_path.write_text(yaml.safe_dump(MamformerConfig.from_dict(d).to_dict()))
    args = ["scripts/train.py", "--config", str(cfg_path), "--data", str(tmp_path / "nodata"),
            "--max_seq_len", "64", "--batch_size", "1", "--gradient_accumulation_steps", "2",
            "--max_steps", "2", "--warmup_steps", "1", "--save_every", "2", "--log_every", "1",
            "--ep", "2", "--output_dir", str(tmp_path / "ck")]
    _torchrun(args)
    assert glob.glob(str(tmp_path / "ck" / "**" / "*.pt"), recursive=True), "no checkpoint written"


def test_grpo_script_cpu(tmp_path):
    """scripts/train_grpo.py: rollouts, rewards, group advantages and an update on CPU (random
    init, two prompts from a local JSONL file, S-GRPO selection on)."""
    import json
    data = tmp_path / "prompts.jsonl"
    data.write_text("\n".join(json.dumps({"prompt": f"Question {i}: 2+{i}?", "answer": str(2 + i),
                                          "reward_type": "math"}) for i in range(2)))
    _run(["scripts/train_grpo.py", "--config", "debug", "--checkpoint", "none", "--data", str(data),
          "--group_size", "2", "--gen_max_tokens", "8", "--batch_size", "2", "--max_steps", "1",
          "--warmup_steps", "1", "--save_every", "1", "--log_every", "1", "--num_workers", "0",
          "--sgrpo", "--output_dir", str(tmp_path / "ck")])


def test_evaluate_and_data_scripts_cpu(tmp_path):
    """scripts/evaluate.py on a local multiple-choice file; scripts/prepare_data.py writes
    .bin shards and metadata that scripts/train.py then trains on."""
    import json
    ev = tmp_path / "eval"
    ev.mkdir()
    (ev / "arc_easy.jsonl").write_text(json.dumps({"question": "1+1?", "choices": ["2", "3"], "answer": 0}))
    r = _run(["scripts/evaluate.py", "--config", "debug", "--benchmarks", "arc_easy",
              "--data_dir", str(ev), "--max_samples", "1"])
    assert "arc_easy" in r.stdout + r.stderr
    src = tmp_path / "docs.jsonl"
    src.write_text("\n".join(json.dumps({"text": "hello world " * 40}) for _ in range(8)))
    out = tmp_path / "shards"
    _run(["scripts/prepare_data.py", "--input", str(src), "--output", str(out), "--seq_len", "64",
          "--num_shards", "2"])
    assert glob.glob(str(out / "*.bin")) and os.path.exists(out / "metadata.json")
    _run(["scripts/train.py", "--config", "debug", "--data", str(out), "--max_seq_len", "64",
          "--batch_size", "1", "--gradient_accumulation_steps", "1", "--max_steps", "2",
          "--warmup_steps", "1", "--save_every", "100", "--output_dir", str(tmp_path / "ck")])


def test_profile_model_script_cpu():
    """scripts/profile_model.py: analytic memory budget of a parallel layout (no GPU needed)."""
    r = _run(["scripts/profile_model.py", "--config", "configs/ultra-7b.yaml", "--seq_len", "4096",
              "--ep", "8"])
    assert (r.stdout + r.stderr).strip() != ""


def test_data_pipeline_and_thinking_generation_cpu(tmp_path):
    """scripts/data_pipeline.py curates a small corpus; scripts/generate.py runs a thinking mode."""
    import json
    src = tmp_path / "raw"
    src.mkdir()
    (src / "a.jsonl").write_text("\n".join(json.dumps({"text": f"Document {i}. " + "Some prose here. " * 30})
                                           for i in range(6)))
    _run(["scripts/data_pipeline.py", "--input", str(src), "--output", str(tmp_path / "out")])
    assert any((tmp_path / "out").rglob("*")), "data pipeline wrote nothing"
    r = _run(["scripts/generate.py", "--config", "debug", "--prompt", "2+2?", "--max_new_tokens", "8",
              "--thinking", "FastThink", "--temperature", "0", "--show_thinking", "--seed", "0"])
    assert r.stdout.strip() != ""          # the control tokens of the thinking phases are shown


def test_profile_kda_ablations_change_the_layer_stack():
    """scripts/profile_kda.py: each ablation really changes the model (no_mamba leaves no SSM
    layer, no_kda_diff switches DSA on, no_interleave makes every layer a fusion layer)."""
    sys.path.insert(0, os.path.join(ROOT, "scripts"))
    try:
        import profile_kda
    finally:
        sys.path.remove(os.path.join(ROOT, "scripts"))
    from mamformer_b200.config import MamformerConfig
    base = lambda: MamformerConfig.from_yaml(os.path.join(ROOT, "configs", "_arch_verify.yaml"))  # noqa: E731
    assert any(t["has_ssm"] for t in base().layer_types())
    nm = profile_kda.ablate(base(), "no_mamba")
    assert all(t["has_attention"] and not t["has_ssm"] for t in nm.layer_types())
    nk = profile_kda.ablate(base(), "no_kda_diff")
    assert not nk.kda_diff.enabled and nk.dsa.enabled
    ni = profile_kda.ablate(base(), "no_interleave")
    assert ni.layout_string() == "F" * ni.n_layers


def test_gen_1b_ultra_config_writes_the_file(tmp_path):
    out = tmp_path / "_1b_ultra.yaml"
    _run(["scripts/gen_1b_ultra_config.py", "--out", str(out)])
    from mamformer_b200.config import MamformerConfig
    cfg = MamformerConfig.from_yaml(str(out))
    assert (cfg.d_model, cfg.n_layers, cfg.moe.n_routed_experts, cfg.moe.top_k) == (2048, 24, 32, 4)
    assert cfg.layout_string().endswith("FF") and cfg.mtp.depth == 2
    committed = MamformerConfig.from_yaml(os.path.join(ROOT, "configs", "_1b_ultra.yaml"))
    assert committed.to_dict() == cfg.to_dict()


def test_gen_arch_config_writes_the_committed_file(tmp_path):
    out = tmp_path / "_arch_verify.yaml"
    _run(["scripts/gen_arch_config.py", "--out", str(out)])
    import yaml
    assert yaml.safe_load(out.read_text()) == yaml.safe_load(open(os.path.join(ROOT, "configs", "_arch_verify.yaml")))
