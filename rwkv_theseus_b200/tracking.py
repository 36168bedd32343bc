"""Optional Weights & Biases logging on the leader rank only.

Same observable contract as the reference ``theseus/tracking.py:7-54``:
``wandb_run.json`` keeps the run identity so an online run resumes under its
old id; metrics use ``progress/global_step`` as x-axis; ``train`` events log
``sum_loss``/``mean_cos`` and ``layer_XX/{nmse,cosine,rrms,grad_norm,lr}``;
``validation`` events log the same under ``val/``. Disabled mode never
imports the SDK.
"""
import json
from pathlib import Path
from uuid import uuid4

_LAYER_KEYS = {"nmse", "cosine", "rrms", "grad_norm", "lr"}


class Tracker:
    def __init__(self):
        self.run = None
        self.cfg = None

    def start(self, cfg, topo, resume=False):
        if topo.rank != topo.leader or cfg["wandb_mode"] == "disabled":
            return
        import wandb
        self.cfg = cfg
        root = Path(cfg["output"])
        root.mkdir(parents=True, exist_ok=True)
        identity_file = root / "wandb_run.json"
        identity = {"project": cfg["wandb_project"], "entity": cfg["wandb_entity"]}
        previous = None
        if resume and identity_file.exists():
            previous = json.loads(identity_file.read_text())
        reuse = (cfg["wandb_mode"] == "online" and previous is not None
                 and previous.get("mode") == "online"
                 and all(previous.get(key) == value for key, value in identity.items()))
        run_id = previous["id"] if reuse else uuid4().hex[:8]
        self.run = wandb.init(
            project=cfg["wandb_project"], entity=cfg["wandb_entity"], name=cfg["wandb_name"],
            id=run_id, mode=cfg["wandb_mode"], resume="allow" if reuse else None, dir=str(root),
            config={k: v for k, v in cfg.items() if not k.startswith("wandb_")}, save_code=False,
            settings=wandb.Settings(init_timeout=60, console="off"))
        tmp = identity_file.with_suffix(".tmp")
        tmp.write_text(json.dumps({**identity, "id": run_id, "mode": cfg["wandb_mode"]}))
        tmp.replace(identity_file)
        self.run.define_metric("progress/global_step")
        for pattern in ("sum_loss", "mean_cos", "layer_*", "val/*"):
            self.run.define_metric(pattern, step_metric="progress/global_step")

    def log(self, event, fields):
        if self.run is None or event not in ("train", "validation"):
            return
        prefix = "val/" if event == "validation" else ""
        values = {"progress/global_step": fields["step"]}
        for key in ("sum_loss", "mean_cos"):
            values[prefix + key] = fields[key]
        for layer, details in fields["layers"].items():
            for key, value in details.items():
                if key in _LAYER_KEYS:
                    values[f"{prefix}{layer}/{key}"] = value
        self.run.log(values)

    def finish(self, exit_code=0):
        if self.run is not None:
            self.run.finish(exit_code=exit_code)
            self.run = None
