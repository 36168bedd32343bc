"""Teacher runner, capture points and student installation.

Public surface of the reference adapter (``theseus/hf_model.py:71-252``):
``Runner`` (a cursor-positioned cached forward that can end at one block's
attention output, with save/restore of the cache and the students' recurrent
states), ``Capture`` (the detached input after ``input_layernorm`` and the
attention output before the residual add of one block), ``AttentionAdapter``
(a TimeMix in place of ``self_attn``), ``install``, ``migration_order`` and
``isolated_state``.

The teacher is this package's own Qwen3.5 hybrid (``models/qwen35.py``), so the
early stop is an argument of its forward (``stop_at``) instead of an exception
raised from a hook, and the runner's cache is ``qwen35.HybridCache``.
"""
from contextlib import contextmanager, nullcontext

import torch
from torch import nn
from torch.utils._pytree import tree_map

from .qwen35 import HybridCache
from .timemix import TimeMix, detach_state


def state_to_device(value, device):
    """`value` (a nest of dicts, lists and tuples) with every tensor moved to `device`."""
    return tree_map(lambda leaf: leaf.to(device) if torch.is_tensor(leaf) else leaf, value)


class AttentionAdapter(nn.Module):
    """A TimeMix student standing where a block's attention was, carrying its recurrent state between calls.

    Modes (checked in this order): ``teacher_mode`` runs the retained teacher attention; a set ``teacher_input``
    runs the training call on that input (legacy sequential stages; ``prediction`` keeps the graph); a fused
    inference forward (``fast``, set by ``install`` for frozen CUDA students); otherwise the module itself."""

    def __init__(self, core):
        super().__init__()
        self.core = core
        self.state = None
        self.teacher = None
        self.teacher_mode = False
        self.teacher_input = None
        self.prediction = None
        self.debug_input = False
        # Plain attributes, not submodules: a DDP wrapper or the fused path must not register the core twice.
        self.__dict__["train_call"] = None
        self.__dict__["fast"] = None

    def _student(self, hidden_states):
        if self.teacher_input is not None:
            if self.debug_input:
                torch.testing.assert_close(hidden_states, self.teacher_input, atol=.04, rtol=.02)
            with torch.enable_grad():
                out, state = self.train_call(self.teacher_input.detach(), self.state)
            self.prediction = out
            return out, state
        run = self.fast if self.fast is not None else self.core
        return run(hidden_states, self.state)

    def forward(self, hidden_states, rope=None, cache=None, **_):
        if self.teacher_mode:
            return self.teacher(hidden_states, rope=rope, cache=cache)
        out, state = self._student(hidden_states)
        self.state = detach_state(state)
        return out.detach()


def adapters(model):
    """{block index: AttentionAdapter} of the students installed in `model`."""
    return {index: block.self_attn for index, block in enumerate(model.model.layers)
            if isinstance(getattr(block, "self_attn", None), AttentionAdapter)}


def migration_order(model, expected=16):
    """Indices of the full-attention blocks (the layers to migrate); exactly `expected` of them."""
    order = [index for index, kind in enumerate(model.config.layer_types) if kind == "full_attention"]
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
    """Put a TimeMix (fp32 when trainable, else bf16) at block `layer`; `weights` load without initialisation."""
    device = next(model.parameters()).device
    core = make_timemix(model, layer, options, "meta" if weights is not None else device)
    if weights is not None:
        core.load_state_dict(weights, strict=True, assign=True)
    core.to(device=device, dtype=torch.float32 if trainable else torch.bfloat16).requires_grad_(trainable)
    adapter = AttentionAdapter(core)
    if device.type == "cuda" and not trainable and options.get("backend", "cuda") == "cuda":
        from .student_fused import FusedTimeMixInference
        adapter.__dict__["fast"] = FusedTimeMixInference(core)
    if retain_teacher:
        adapter.teacher = model.model.layers[layer].self_attn.requires_grad_(False).eval()
    if attach:
        model.model.layers[layer].self_attn = adapter
    return adapter


class Capture:
    """Records, detached, what one attention module receives (``x``) and returns (``y``) on each forward.

    With ``record_events`` set, a CUDA event is recorded on the forward's stream right after the module's work
    (``ready``): work on another stream that reads ``x`` and ``y`` waits on it instead of on the whole forward."""

    def __init__(self, attention):
        self.x = self.y = None
        self.ready = None
        self.record_events = False
        self._handles = [attention.register_forward_pre_hook(self._take_input, with_kwargs=True),
                         attention.register_forward_hook(self._take_output)]

    def _take_input(self, module, args, kwargs):
        self.x = (args[0] if args else kwargs["hidden_states"]).detach()

    def _take_output(self, module, args, output):
        self.y = (output[0] if isinstance(output, tuple) else output).detach()
        if self.record_events and self.y.is_cuda:
            self.ready = torch.cuda.Event()
            self.ready.record()

    def close(self):
        for handle in self._handles:
            handle.remove()
        self._handles = []
        self.x = self.y = None


class Runner:
    """Chunk-by-chunk teacher forward over one cache; ``cache.cursor`` is the absolute position of the next token."""

    def __init__(self, model):
        self.model = model
        self.cache = HybridCache(model.config)

    def reset(self):
        """New window: the cache restarts at position 0 with empty states (its buffers are reused)."""
        self.cache.reset()
        for adapter in adapters(self.model).values():
            adapter.state = None

    @torch.no_grad()
    def forward(self, ids, through_layer=None):
        """Forward of one chunk ``ids`` [B, T]: the final hidden states, or with ``through_layer`` the attention
        output of that block (the blocks after it, and its own MLP, are not run and their caches are unchanged)."""
        if through_layer is not None and not 0 <= through_layer < self.model.config.num_hidden_layers:
            raise ValueError(f"Invalid decoder layer {through_layer}")
        autocast = torch.autocast("cpu", dtype=torch.bfloat16) if ids.device.type == "cpu" else nullcontext()
        with autocast:
            hidden = self.model.model(ids, self.cache.cursor, self.cache, stop_at=through_layer)
        self.cache.cursor += ids.shape[1]
        return hidden

    def state_dict(self):
        return {"cursor": self.cache.cursor, "hf_layers": self.cache.state_dict(),
                "timemix": {index: adapter.state for index, adapter in adapters(self.model).items()}}

    def load_state_dict(self, state):
        self.reset()
        device = next(self.model.parameters()).device
        self.cache.cursor = state["cursor"]
        self.cache.load_state_dict(state.get("hf_layers", state.get("layers")), device)
        students = adapters(self.model)
        for index, saved in state["timemix"].items():
            students[int(index)].state = None if saved is None else state_to_device(saved, device)


@contextmanager
def isolated_state(runner):
    """Run the body on a fresh cache and fresh student states; the live ones are put back afterwards."""
    live_cache = runner.cache
    live_states = {index: adapter.state for index, adapter in adapters(runner.model).items()}
    runner.cache = HybridCache(runner.model.config)  # a separate cache (reset() would clear the live one)
    for adapter in adapters(runner.model).values():
        adapter.state = None
    try:
        yield runner
    finally:
        runner.cache = live_cache
        for index, adapter in adapters(runner.model).items():
            adapter.state = live_states.get(index)
