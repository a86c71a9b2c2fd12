"""Shared helpers of the command-line entry points."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def init_distributed(timeout_s: int = 1800):
    """torchrun environment -> (rank, world, local_rank, device); NCCL on GPUs, gloo on CPU."""
    import datetime

    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
        device = torch.device("cuda", local)
    else:
        device = torch.device("cpu")
    if world > 1 and not dist.is_initialized():
        kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
        if device.type == "cuda":
            kw["device_id"] = device
        dist.init_process_group("nccl" if device.type == "cuda" else "gloo", **kw)
    return rank, world, local, device


def load_config(path_or_preset: str):
    from mamformer_b200.config import MamformerConfig
    if os.path.exists(path_or_preset):
        return MamformerConfig.from_yaml(path_or_preset)
    return MamformerConfig.from_preset(path_or_preset)


def load_model(config_path: str, checkpoint=None, device="cpu", dtype=None):
    import torch
    from mamformer_b200 import MamformerForCausalLM
    from mamformer_b200.checkpoint import load_model_state
    cfg = load_config(config_path)
    model = MamformerForCausalLM(cfg)
    if checkpoint:
        ck = torch.load(checkpoint, map_location="cpu", weights_only=False)
        load_model_state(model, ck["model"] if isinstance(ck, dict) and "model" in ck else ck)
    model = model.to(device)
    if dtype is not None and dtype != torch.float32:
        from mamformer_b200.utils.precision import to_compute_dtype
        to_compute_dtype(model, dtype)
    return model.eval(), cfg
