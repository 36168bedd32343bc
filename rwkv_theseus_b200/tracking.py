"""Optional Weights & Biases logging, on the leader rank only.

Observable contract kept from the reference (``theseus/tracking.py:7-54``):

* ``<output>/wandb_run.json`` records ``{project, entity, id, mode}``; a resumed
  online run with the same project and entity continues under the old id;
* ``progress/global_step`` is the x-axis of ``sum_loss``, ``mean_cos``,
  ``layer_*`` and ``val/*``;
* a ``train`` event logs ``sum_loss``, ``mean_cos`` and
  ``layer_XX/{nmse,cosine,rrms,grad_norm,lr}``; a ``validation`` event logs the
  same names under ``val/``; other events are not sent;
* with ``wandb_mode: disabled`` (or on any other rank) the SDK is never imported.
"""
import json
from pathlib import Path
from uuid import uuid4

TRACKED_LAYER_FIELDS = ("nmse", "cosine", "rrms", "grad_norm", "lr")
STEP_AXIS = "progress/global_step"


def flatten(event, fields):
    """The W&B payload of one emitted event (``None`` for events that are not tracked)."""
    prefix = {"train": "", "validation": "val/"}.get(event)
    if prefix is None:
        return None
    payload = {STEP_AXIS: fields["step"], prefix + "sum_loss": fields["sum_loss"],
               prefix + "mean_cos": fields["mean_cos"]}
    for layer, values in fields["layers"].items():
        payload.update({f"{prefix}{layer}/{name}": values[name] for name in TRACKED_LAYER_FIELDS if name in values})
    return payload


class RunIdentity:
    """The ``wandb_run.json`` record: which run id a (resumed) job logs to."""

    def __init__(self, output, cfg):
        self.path = Path(output) / "wandb_run.json"
        self.owner = {"project": cfg["wandb_project"], "entity": cfg["wandb_entity"]}
        self.mode = cfg["wandb_mode"]

    def resumable_id(self, resume):
        """The previous run's id when this job may continue it: an online resume of an online run of the same
        project and entity."""
        if not (resume and self.mode == "online" and self.path.exists()):
            return None
        old = json.loads(self.path.read_text())
        same_owner = all(old.get(key) == value for key, value in self.owner.items())
        return old.get("id") if old.get("mode") == "online" and same_owner else None

    def record(self, run_id):
        staging = self.path.with_suffix(".tmp")
        staging.write_text(json.dumps({**self.owner, "id": run_id, "mode": self.mode}))
        staging.replace(self.path)


class Tracker:
    """W&B run of the leader rank; every other rank (and ``wandb_mode: disabled``) logs nothing."""

    run = None
    cfg = None

    def start(self, cfg, topo, resume=False):
        logging_rank = topo.rank == topo.leader and cfg["wandb_mode"] != "disabled"
        if not logging_rank:
            return
        import wandb
        self.cfg = cfg
        output = Path(cfg["output"])
        output.mkdir(parents=True, exist_ok=True)
        identity = RunIdentity(output, cfg)
        continued = identity.resumable_id(resume)
        run_id = continued or uuid4().hex[:8]
        self.run = wandb.init(project=cfg["wandb_project"], entity=cfg["wandb_entity"], name=cfg["wandb_name"],
                              id=run_id, mode=cfg["wandb_mode"], resume="allow" if continued else None,
                              dir=str(output), save_code=False,
                              config={key: value for key, value in cfg.items() if not key.startswith("wandb_")},
                              settings=wandb.Settings(init_timeout=60, console="off"))
        identity.record(run_id)
        self.run.define_metric(STEP_AXIS)
        for series in ("sum_loss", "mean_cos", "layer_*", "val/*"):
            self.run.define_metric(series, step_metric=STEP_AXIS)

    def log(self, event, fields):
        if self.run is None:
            return
        payload = flatten(event, fields)
        if payload is not None:
            self.run.log(payload)

    def finish(self, exit_code=0):
        run, self.run = self.run, None
        if run is not None:
            run.finish(exit_code=exit_code)
