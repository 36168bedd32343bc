"""One trainable TimeMix student: flat fp32 buffers, fused update, state.

Reference semantics (``theseus/stage.py:27-44`` and ``train.py:170-211``)
kept exactly: fp32 parameters and Adam moments, AdamW with two groups
(decoupled weight decay only on the four 2-D ``*.weight`` matrices), the
LambdaLR schedule of ``schedule.lr_factor``, gradients summed over ranks and
divided by the global token count, ``clip_grad_norm_`` on the layer's 23
tensors (pre-clip norm reported, non-finite norm is an error).

B200 design: the 23 parameters live as views into ONE contiguous fp32 buffer
(decay group first), with matching flat gradient and moment buffers. The
per-layer gradient bucket is therefore a single range, reduced across ranks by
one collective (the peer-memory kernel of ``parallel.grad_sync`` or NCCL), and
norm + clip + AdamW + bf16 weight refresh are two fused kernels over the flat
range with no host synchronisation (count, norm and error flags stay on the
device until the step's metrics are read).
"""
import torch

from .models.timemix import TimeMix, PARAM_ORDER
from .schedule import lr_factor

DECAY_NAMES = ("receptance.weight", "key.weight", "value.weight", "output.weight")


def optimizer_order(core):
    """Parameter names in torch AdamW state_dict index order (decay group first)."""
    named = dict(core.named_parameters())
    decay = [n for n in named if n.endswith(".weight") and named[n].ndim == 2]
    rest = [n for n in named if n not in decay]
    return decay + rest, len(decay)


class FlatBuffers:
    """Params/grads/moments of one module as views into contiguous buffers."""

    def __init__(self, module, names, device):
        params = dict(module.named_parameters())
        self.names = list(names)
        self.shapes = [tuple(params[n].shape) for n in names]
        self.sizes = [params[n].numel() for n in names]
        self.offsets = [0]
        for size in self.sizes:
            self.offsets.append(self.offsets[-1] + size)
        total = self.offsets[-1]
        self.numel = total
        self.param = torch.empty(total, device=device, dtype=torch.float32)
        self.grad = torch.zeros(total, device=device, dtype=torch.float32)
        self.exp_avg = torch.zeros(total, device=device, dtype=torch.float32)
        self.exp_avg_sq = torch.zeros(total, device=device, dtype=torch.float32)
        with torch.no_grad():
            for name, start, size, shape in zip(names, self.offsets, self.sizes, self.shapes):
                p = params[name]
                self.param[start:start + size].copy_(p.detach().reshape(-1))
                p.data = self.param[start:start + size].view(shape)
                p.grad = self.grad[start:start + size].view(shape)

    def view(self, buffer, name):
        i = self.names.index(name)
        return buffer[self.offsets[i]:self.offsets[i + 1]].view(self.shapes[i])


_UPDATE_STREAMS = {}


def _update_stream(device):
    """Side stream of a device for the local fused optimizer updates."""
    if device.index not in _UPDATE_STREAMS:
        _UPDATE_STREAMS[device.index] = torch.cuda.Stream(device)
    return _UPDATE_STREAMS[device.index]


class Student:
    def __init__(self, model_cfg, layer, cfg, topo, weights=None, total_steps=1):
        self.layer, self.cfg, self.topo = layer, cfg, topo
        self.total_steps = total_steps
        device = topo.device
        with torch.device("meta" if weights is not None else device):
            core = TimeMix(model_cfg.hidden_size, layer, model_cfg.num_hidden_layers, head_size=cfg["head_size"],
                           backend=cfg["backend"], lora_rank=cfg.get("lora_rank"),
                           gate_lora_rank=cfg.get("gate_lora_rank"))
        if weights is not None:
            core.load_state_dict(weights, strict=True, assign=True)
        core.to(device=device, dtype=torch.float32)
        self.core = core
        names, n_decay = optimizer_order(core)
        self.flat = FlatBuffers(core, names, device)
        self.n_decay = n_decay
        self.decay_numel = self.flat.offsets[n_decay]
        self.steps_done = 0            # optimizer updates applied (LambdaLR last_epoch)
        self.state = None              # carried {shift, wkv} across chunks
        self.stats = torch.zeros(3, device=device)      # [sum nmse, sum cos, count] of the current update
        self.report = torch.zeros(5, device=device)     # [nmse, cos, count, grad_norm, error] of last update
        self.fused = None
        self.sharded = False           # fp32 masters / moments hold only this rank's shard (peer exchange)
        self.grads_live = False        # the flat gradient holds this update's micro-steps (fused path)
        self._update_done = None       # event of a local fused update still running on the update stream
        self.overlap_update = False    # run local fused updates on the side stream (set by the step engine)
        if device.type == "cuda" and cfg.get("fused_optimizer", True):
            from .models.student_fused import FusedStudent
            self.fused = FusedStudent(self)
        exchange = self._exchange()
        if exchange is not None:  # collective: every rank builds the same students in the same order
            exchange.register(self)

    # ---------------------------------------------------------------- forward/backward
    def join_update(self):
        """Make the current stream wait for this student's last update (local fused update or peer exchange):
        parameters, moments and report."""
        if self._update_done is not None:
            torch.cuda.current_stream(self.topo.device).wait_event(self._update_done)
            self._update_done = None

    def micro_step(self, x, target):
        """Forward + backward on one chunk; gradients accumulate into the flat buffer."""
        self.join_update()
        eps = self.cfg["loss_epsilon"]
        if self.fused is not None:  # the loss sums accumulate into self.stats on the device
            self.state = self.fused.forward_backward(x, target, self.state, eps, self.stats, first=not self.grads_live)
            self.grads_live = True
            return
        from .losses import statistics
        with torch.autocast(x.device.type, dtype=torch.bfloat16):
            prediction, state = self.core(x, self.state)
        self.state = {k: v.detach() for k, v in state.items()}
        stats = statistics(prediction, target, eps)
        stats[0].backward()
        self.stats += stats.detach()

    @torch.no_grad()
    def predict(self, x, state):
        """Inference forward (validation); returns (prediction, new state)."""
        self.join_update()
        if self.fused is not None:
            return self.fused.forward(x, state)
        with torch.autocast(x.device.type, dtype=torch.bfloat16):
            return self.core(x, state)

    # ---------------------------------------------------------------- update
    def current_lr(self):
        return self.cfg["lr"] * lr_factor(self.steps_done, self.cfg, self.total_steps)

    def _exchange(self):
        """The peer-memory exchange when it applies (CUDA, fused optimizer, one node, world > 1)."""
        if self.topo.world == 1 or self.fused is None or self.cfg.get("grad_sync", "peer") != "peer":
            return None
        return self.topo.grad_sync()

    def reduce(self):
        """Sum gradients and loss statistics over ranks (one bucket per layer).

        With the peer-memory exchange the reduction is part of ``update``."""
        self.join_update()
        if self.fused is not None and not self.grads_live:
            self.flat.grad.zero_()  # no micro-step this update (exhausted rank): contribute zeros
            self.grads_live = True
        topo = self.topo
        if topo.world == 1 or self._exchange() is not None:
            return
        import torch.distributed as dist
        dist.all_reduce(self.flat.grad, group=topo.student_group)
        dist.all_reduce(self.stats, group=topo.student_group)

    def update_stream(self):
        """The CUDA stream this student's updates run on (and write ``report`` on): the peer exchange's stream,
        the device's side update stream, or None for the current stream."""
        if self.topo.device.type != "cuda":
            return None
        exchange = self._exchange()
        if exchange is not None:
            return exchange.stream
        if self.fused is not None and self.overlap_update:
            return _update_stream(self.topo.device)
        return None

    @torch.no_grad()
    def update(self):
        """Scale by 1/count, clip, AdamW, clear gradients; stats go to ``report``."""
        lr = self.current_lr()
        self.steps_done += 1
        exchange = self._exchange()
        if exchange is not None:
            # Reduce-scatter, clip, AdamW on this rank's shard, all-gather; clears grad and stats on its stream.
            self._update_done = exchange.update(self, lr, self.steps_done)
            self.sharded = True
            self.grads_live = False
            return lr
        if self.fused is not None:
            # Memory-bound; it runs on a side stream under the next layer's compute-bound micro-step and is
            # joined where its results are next read (join_update).
            self.join_update()
            if not self.grads_live:
                self.flat.grad.zero_()
            if not self.overlap_update:
                self.fused.update(lr, self.steps_done)  # also clears stats for the next update
                self.grads_live = False
                return lr
            main = torch.cuda.current_stream(self.topo.device)
            side = _update_stream(self.topo.device)
            side.wait_stream(main)
            with torch.cuda.stream(side):
                self.fused.update(lr, self.steps_done)
            self._update_done = torch.cuda.Event()
            self._update_done.record(side)
            self.grads_live = False
            return lr
        self._update_reference(lr, self.steps_done)
        self.stats.zero_()
        return lr

    def sync_state(self):
        """Collective before a checkpoint or export: complete fp32 parameters and Adam moments on every rank.

        With the peer exchange each rank updates only its shard of the fp32 masters of the decay matrices and
        of the moments (compute reads the all-gathered bf16 copy)."""
        self.join_update()
        exchange = self._exchange()
        if exchange is not None and self.sharded:
            exchange.gather_state(self)
            self.sharded = False

    def _update_reference(self, lr, step):
        cfg, flat = self.cfg, self.flat
        count = self.stats[2]
        g = flat.grad
        g.div_(count.clamp_min(1e-30))
        norm = torch.linalg.vector_norm(g)
        bad = (~torch.isfinite(norm)) | (count <= 0)
        g.mul_(torch.clamp(cfg["clip_norm"] / (norm + 1e-6), max=1.0))
        beta1, beta2 = cfg["betas"]
        p, m, v = flat.param, flat.exp_avg, flat.exp_avg_sq
        p[:self.decay_numel].mul_(1 - lr * cfg["weight_decay"])
        m.lerp_(g, 1 - beta1)
        v.mul_(beta2).addcmul_(g, g, value=1 - beta2)
        bias1, bias2 = 1 - beta1 ** step, 1 - beta2 ** step
        denom = (v.sqrt() / bias2 ** 0.5).add_(cfg["adam_eps"])
        p.addcdiv_(m, denom, value=-lr / bias1)
        g.zero_()
        self.report.copy_(torch.stack([self.stats[0], self.stats[1], count, norm, bad.float()]))

    # ---------------------------------------------------------------- state/IO
    def weights(self):
        self.join_update()
        if self.sharded:
            raise RuntimeError("fp32 parameters are sharded across ranks; call sync_state() on every rank first")
        return {name: t.detach() for name, t in self.core.state_dict().items()}

    def optimizer_state_dict(self):
        """torch.optim.AdamW-compatible state_dict (same indices and groups)."""
        self.join_update()
        if self.sharded:
            raise RuntimeError("Adam moments are sharded across ranks; call sync_state() on every rank first")
        flat, cfg = self.flat, self.cfg
        state = {}
        if self.steps_done:
            for i, name in enumerate(flat.names):
                state[i] = {"step": torch.tensor(float(self.steps_done)),
                            "exp_avg": flat.view(flat.exp_avg, name).clone(),
                            "exp_avg_sq": flat.view(flat.exp_avg_sq, name).clone()}
        lr = self.current_lr()
        common = {"lr": lr, "betas": tuple(cfg["betas"]), "eps": cfg["adam_eps"], "amsgrad": False,
                  "foreach": None, "maximize": False, "capturable": False, "differentiable": False,
                  "fused": self.topo.device.type == "cuda", "decoupled_weight_decay": True, "initial_lr": cfg["lr"]}
        groups = [dict(common, weight_decay=cfg["weight_decay"], params=list(range(self.n_decay))),
                  dict(common, weight_decay=0.0, params=list(range(self.n_decay, len(flat.names))))]
        return {"state": state, "param_groups": groups}

    def scheduler_state_dict(self):
        lr = self.current_lr()
        return {"base_lrs": [self.cfg["lr"]] * 2, "last_epoch": self.steps_done, "_step_count": self.steps_done + 1,
                "_get_lr_called_within_step": False, "_last_lr": [lr, lr], "lr_lambdas": [None, None]}

    def load_optimizer_state(self, optimizer, scheduler):
        self.join_update()
        flat = self.flat
        with torch.no_grad():
            for i, name in enumerate(flat.names):
                entry = optimizer["state"].get(i)
                if entry is None:
                    continue
                flat.view(flat.exp_avg, name).copy_(entry["exp_avg"])
                flat.view(flat.exp_avg_sq, name).copy_(entry["exp_avg_sq"])
        self.steps_done = int(scheduler["last_epoch"])
        if self.fused is not None:
            self.fused.refresh_weights()


def promote(topo, model, layer, cfg):
    """Legacy sequential-stage handoff (reference ``theseus/stage.py:47-57``): the leader's trained student
    of ``layer`` is broadcast to every rank as bf16 and installed frozen in place of the attention block."""
    from .models.runner import install
    topo.barrier()
    weights = None
    if topo.rank == topo.leader:
        core = model.model.layers[layer].self_attn.core
        weights = {k: v.detach().cpu().to(torch.bfloat16) for k, v in core.state_dict().items()}
    weights = topo.broadcast_weights(weights)
    install(model, layer, cfg, weights=weights, trainable=False)
    topo.barrier()
