"""One tiny training micro-step of the flagship path on a CUDA device.

Teacher forward (GEMM, RMSNorm, conv1d+SiLU, GDN, attention pre-processing
kernels), one TimeMix student forward/backward (WKV7 kernels) and its fused
update, on a random-init hybrid with two full-attention blocks.
"""
import torch

from .config import DEFAULTS
from .models.hf_io import random_model
from .models.qwen35 import HybridConfig
from .models.runner import Capture, Runner, migration_order
from .stage import Student


def smoke_config():
    return HybridConfig(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=4,
                        num_attention_heads=4, num_key_value_heads=2, head_dim=64, linear_num_key_heads=2,
                        linear_num_value_heads=4, linear_key_head_dim=64, linear_value_head_dim=64,
                        linear_conv_kernel_dim=4, layer_types=["linear_attention", "full_attention"] * 2,
                        rope_theta=1e6, partial_rotary_factor=0.25)


class _Topo:
    def __init__(self, device):
        self.rank, self.world, self.leader, self.device = 0, 1, 0, device

    def grad_sync(self):
        return None


def run_smoke(device, tokens=40, steps=2):
    torch.manual_seed(0)
    cfg = smoke_config()
    model = random_model(cfg, device)
    order = migration_order(model, 2)
    runner = Runner(model)
    captures = {i: Capture(model.model.layers[i].self_attn) for i in order}
    train_cfg = DEFAULTS | {"head_size": 64, "backend": "cuda", "lr": 1e-3, "warmup_steps": 0}
    topo = _Topo(device)
    students = {i: Student(cfg, i, train_cfg, topo, total_steps=steps) for i in order}
    ids = torch.randint(0, cfg.vocab_size, (1, tokens), device=device)
    for _ in range(steps):
        runner.reset()
        runner.forward(ids)
        for i in order:
            students[i].state = None
            students[i].micro_step(captures[i].x, captures[i].y)
            students[i].update()
    reports = torch.stack([students[i].report for i in order]).cpu()
    if not torch.isfinite(reports).all() or reports[:, 4].any():
        raise RuntimeError(f"smoke step produced invalid statistics: {reports}")
    for c in captures.values():
        c.close()
    return reports
