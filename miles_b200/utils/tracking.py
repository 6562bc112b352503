"""Metric tracking fan-out: stdout/jsonl, TensorBoard, Prometheus, Weights & Biases.

Backends are optional: a backend whose package is missing is reported once and skipped. All
ranks may call `log`; only rank 0 writes (DP-averaged metrics are reduced by the caller).

Reference: miles/utils/tracking_utils.py:12-37, wandb_utils.py, tensorboard_utils.py,
prometheus_utils.py:19-109, logging_utils.py:15.
"""
from __future__ import annotations

import json
import logging
import os
import time

logger = logging.getLogger("miles_b200")


def configure_logger(level=logging.INFO):
    logging.basicConfig(level=level, format="[%(asctime)s %(name)s %(levelname)s] %(message)s")


class Tracker:
    def __init__(self, args, rank: int = 0):
        self.args = args
        self.rank = rank
        self.history: list[dict] = []
        self.tb = self.wandb = self.prom = None
        self.jsonl = None
        if rank != 0:
            return
        out = getattr(args, "save", None) or getattr(args, "tensorboard_dir", None)
        if out:
            os.makedirs(out, exist_ok=True)
            self.jsonl = open(os.path.join(out, "metrics.jsonl"), "a")
        if getattr(args, "use_tensorboard", False):
            try:
                from torch.utils.tensorboard import SummaryWriter

                d = args.tensorboard_dir or os.path.join(out or ".", "tb", getattr(args, "tb_project_name", None) or "",
                                                         args.tb_experiment_name or "run")
                self.tb = SummaryWriter(d)
            except Exception as e:
                logger.warning("tensorboard unavailable: %s", e)
        if getattr(args, "use_wandb", False):
            try:
                import wandb

                if getattr(args, "wandb_key", None) or getattr(args, "wandb_host", None):
                    wandb.login(key=args.wandb_key, host=args.wandb_host)
                name = args.wandb_group
                if name and not getattr(args, "disable_wandb_random_suffix", False):
                    import uuid

                    name = f"{name}_{uuid.uuid4().hex[:6]}"
                self.wandb = wandb.init(project=args.wandb_project, group=args.wandb_group, name=name,
                                        entity=args.wandb_team, dir=args.wandb_dir, mode=args.wandb_mode,
                                        id=args.wandb_run_id, resume="allow", config=vars(args))
                if getattr(args, "wandb_always_use_train_step", False):
                    # every metric on the train-step axis (the logged `step`)
                    self.wandb.define_metric("*", step_metric="train/step")
            except Exception as e:
                logger.warning("wandb unavailable: %s", e)
        if getattr(args, "use_prometheus", False):
            try:
                import prometheus_client as pc

                pc.start_http_server(args.prometheus_port)
                self.prom = {"pc": pc, "gauges": {}}
            except Exception as e:
                logger.warning("prometheus unavailable: %s", e)

    def log(self, metrics: dict, step: int):
        rec = {"step": step, "time": time.time(), **{k: v for k, v in metrics.items() if _scalar(v)}}
        self.history.append(rec)
        if self.rank != 0:
            return
        logger.info("step %d %s", step, {k: round(v, 5) if isinstance(v, float) else v for k, v in rec.items() if k not in ("time",)})
        if self.jsonl:
            self.jsonl.write(json.dumps(rec) + "\n")
            self.jsonl.flush()
        for k, v in rec.items():
            if k in ("step", "time"):
                continue
            if self.tb:
                self.tb.add_scalar(k, v, step)
            if self.prom:
                g = self.prom["gauges"].get(k)
                if g is None:
                    name = "miles_" + "".join(c if c.isalnum() else "_" for c in k)
                    g = self.prom["pc"].Gauge(name, k, ["run"])
                    self.prom["gauges"][k] = g
                g.labels(run=self.args.prometheus_run_name or "run").set(v)
        if self.wandb:
            if getattr(self.args, "wandb_always_use_train_step", False):
                self.wandb.log({**rec, "train/step": step})
            else:
                self.wandb.log(rec, step=step)

    def finish(self):
        if self.jsonl:
            self.jsonl.close()
        if self.tb:
            self.tb.close()
        if self.wandb:
            self.wandb.finish()


def _scalar(v) -> bool:
    return isinstance(v, (int, float)) and not isinstance(v, bool)
