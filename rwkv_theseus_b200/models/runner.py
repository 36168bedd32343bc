"""Teacher runner, capture points and student installation.

Public surface matches the reference adapter (``theseus/hf_model.py:71-252``):
``Runner`` (cursor-positioned cached forward, optional stop at a layer's
attention output, state save/restore), ``Capture`` (detached input after
``input_layernorm`` and attention output before the residual add),
``AttentionAdapter`` (a TimeMix in place of ``self_attn``), ``install``,
``migration_order`` and ``isolated_state``.
"""
from contextlib import contextmanager, nullcontext

import torch
from torch import nn

from .qwen35 import HybridCache
from .timemix import TimeMix, detach_state


def state_to_device(value, device):
    if torch.is_tensor(value):
        return value.to(device)
    if isinstance(value, dict):
        return {k: state_to_device(v, device) for k, v in value.items()}
    if isinstance(value, list):
        return [state_to_device(v, device) for v in value]
    if isinstance(value, tuple):
        return tuple(state_to_device(v, device) for v in value)
    return value


class AttentionAdapter(nn.Module):
    """Runs a TimeMix where the teacher's attention was; carries its state."""

    def __init__(self, core):
        super().__init__()
        self.core = core
        self.state = None
        self.teacher_input = None
        self.prediction = None
        self.debug_input = False
        self.teacher = None
        self.teacher_mode = False
        # A DDP wrapper must not be registered as a second child of the same core.
        self.__dict__["train_call"] = None
        # Fused CUDA inference forward for frozen bf16 cores (set by ``install``); not a submodule.
        self.__dict__["fast"] = None

    def forward(self, hidden_states, rope=None, cache=None, **_):
        if self.teacher_mode:
            return self.teacher(hidden_states, rope=rope, cache=cache)
        if self.teacher_input is not None:
            if self.debug_input:
                torch.testing.assert_close(hidden_states, self.teacher_input, atol=.04, rtol=.02)
            with torch.enable_grad():
                y, state = self.train_call(self.teacher_input.detach(), self.state)
            self.prediction = y
        elif self.fast is not None:
            y, state = self.fast(hidden_states, self.state)
        else:
            y, state = self.core(hidden_states, self.state)
        self.state = detach_state(state)
        return y.detach()


def migration_order(model, expected=16):
    order = [i for i, kind in enumerate(model.config.layer_types) if kind == "full_attention"]
    if len(order) != expected:
        raise ValueError(f"Expected {expected} full attention blocks, found {order}")
    return order


def make_timemix(model, layer, options, device=None):
    cfg = model.config
    with torch.device(device or "cpu"):
        return TimeMix(cfg.hidden_size, layer, cfg.num_hidden_layers, head_size=options["head_size"],
                       backend=options.get("backend", "cuda"), lora_rank=options.get("lora_rank"),
                       gate_lora_rank=options.get("gate_lora_rank"))


def install(model, layer, options, weights=None, trainable=False, retain_teacher=False, attach=True):
    device = next(model.parameters()).device
    core = make_timemix(model, layer, options, "meta" if weights is not None else device)
    if weights is not None:
        core.load_state_dict(weights, strict=True, assign=True)
    core.to(device=device, dtype=torch.float32 if trainable else torch.bfloat16)
    core.requires_grad_(trainable)
    adapter = AttentionAdapter(core)
    if not trainable and device.type == "cuda" and options.get("backend", "cuda") == "cuda":
        from .student_fused import FusedTimeMixInference
        adapter.__dict__["fast"] = FusedTimeMixInference(core)
    if retain_teacher:
        adapter.teacher = model.model.layers[layer].self_attn
        adapter.teacher.requires_grad_(False).eval()
    if attach:
        model.model.layers[layer].self_attn = adapter
    return adapter


class Capture:
    """Forward hooks recording a block's attention input and output (detached)."""

    def __init__(self, attention):
        self.x = self.y = None
        self.pre = attention.register_forward_pre_hook(self._pre, with_kwargs=True)
        self.post = attention.register_forward_hook(self._post)

    def _pre(self, module, args, kwargs):
        self.x = (kwargs["hidden_states"] if "hidden_states" in kwargs else args[0]).detach()

    def _post(self, module, args, output):
        self.y = (output[0] if isinstance(output, tuple) else output).detach()

    def close(self):
        self.pre.remove()
        self.post.remove()
        self.x = self.y = None


class _Boundary(Exception):
    pass


class Runner:
    def __init__(self, model):
        self.model = model
        self.cache = HybridCache(model.config)

    def reset(self):
        self.cache = HybridCache(self.model.config)
        for block in self.model.model.layers:
            if isinstance(getattr(block, "self_attn", None), AttentionAdapter):
                block.self_attn.state = None

    @torch.no_grad()
    def forward(self, ids, through_layer=None):
        """Cached forward of one chunk; returns final hidden states, or the
        attention output of ``through_layer`` (stopping there)."""
        T = ids.shape[1]
        hook = None
        found = []
        if through_layer is not None:
            if not 0 <= through_layer < self.model.config.num_hidden_layers:
                raise ValueError(f"Invalid decoder layer {through_layer}")
            block = self.model.model.layers[through_layer]
            target = block.self_attn if hasattr(block, "self_attn") else block.linear_attn

            def stop(module, args, output):
                found.append(output[0] if isinstance(output, tuple) else output)
                raise _Boundary()
            hook = target.register_forward_hook(stop)
        cast = torch.autocast(ids.device.type, dtype=torch.bfloat16) if ids.device.type == "cpu" else nullcontext()
        try:
            with cast:
                try:
                    hidden = self.model.model(ids, self.cache.cursor, self.cache)
                except _Boundary:
                    hidden = found.pop()
        finally:
            if hook is not None:
                hook.remove()
        self.cache.cursor += T
        return hidden

    def state_dict(self):
        return {"cursor": self.cache.cursor, "layers": self.cache.state_dict(),
                "timemix": {i: block.self_attn.state for i, block in enumerate(self.model.model.layers)
                            if isinstance(getattr(block, "self_attn", None), AttentionAdapter)}}

    def load_state_dict(self, state):
        self.reset()
        device = next(self.model.parameters()).device
        self.cache.cursor = state["cursor"]
        self.cache.load_state_dict(state["layers"], device)
        for i, s in state["timemix"].items():
            self.model.model.layers[int(i)].self_attn.state = (
                None if s is None else {k: v.to(device) for k, v in s.items()})


@contextmanager
def isolated_state(runner):
    """Run with a fresh cache and student states; restore the live ones after."""
    cache = runner.cache
    states = {i: b.self_attn.state for i, b in enumerate(runner.model.model.layers)
              if isinstance(getattr(b, "self_attn", None), AttentionAdapter)}
    runner.reset()
    try:
        yield
    finally:
        runner.cache = cache
        for i, state in states.items():
            runner.model.model.layers[i].self_attn.state = state
