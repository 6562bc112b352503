"""Rollout deployment YAML (`--sglang-config`): which models run on how many rollout GPUs, in
which server groups, with which engine overrides, and whether they take weight refits.

    sglang:
      - name: actor
        update_weights: true
        server_groups:
          - {worker_type: regular, num_gpus: 4}
      - name: ref
        model_path: /ckpt/ref
        update_weights: false
        server_groups:
          - {worker_type: regular, num_gpus: 2, overrides: {mem_fraction_static: 0.7}}

The schema is the reference's, so existing deployment files load unchanged (`engine_groups`
is accepted for `server_groups`). `plan()` turns it into concrete engine instances over the
rollout ranks: one engine per `num_gpus_per_engine` GPUs, in file order, `placeholder`
groups reserving GPUs without an engine. Engines here run one GPU each (tensor-parallel
engines are not built). `load_deployment` is what the drivers use: one deployed model (the
actor being trained), each engine's `overrides` applied as forwarded SGLang flags, and under
train_async.py the prefill / decode groups run disaggregated (`pd_pairs`: the i-th prefill
engine serves the i-th decode engine's prompts); `plan()` itself still reports prefill /
decode groups as regular engines for callers that do not pair them.

Reference: miles/backends/sglang_utils/sglang_config.py (ServerGroupConfig :11-36,
ModelConfig :39-100, SglangConfig.from_yaml / from_prefill_num_servers :103-190).
"""
from __future__ import annotations

from dataclasses import dataclass, field

WORKER_TYPES = ("regular", "prefill", "decode", "placeholder")


@dataclass
class ServerGroup:
    worker_type: str
    num_gpus: int
    num_gpus_per_engine: int | None = None
    overrides: dict = field(default_factory=dict)

    def __post_init__(self):
        if self.worker_type not in WORKER_TYPES:
            raise ValueError(f"worker_type {self.worker_type!r} not in {WORKER_TYPES}")
        if self.num_gpus <= 0:
            raise ValueError("num_gpus must be positive")


@dataclass
class ModelDeployment:
    name: str
    model_path: str | None = None
    num_gpus_per_engine: int | None = None
    server_groups: list[ServerGroup] = field(default_factory=list)
    update_weights: bool | None = None

    def resolve(self, args):
        per = self.num_gpus_per_engine or getattr(args, "rollout_num_gpus_per_engine", 1)
        path = self.model_path or getattr(args, "hf_checkpoint", None)
        for g in self.server_groups:
            g.num_gpus_per_engine = g.num_gpus_per_engine or per
            g.overrides.setdefault("model_path", path)
        paths = {g.overrides["model_path"] for g in self.server_groups} or {path}
        if len(paths) > 1:
            raise ValueError(f"model {self.name}: server groups disagree on model_path {paths}")
        if self.update_weights is None:  # refit only the model that is being trained
            self.update_weights = paths.pop() == getattr(args, "hf_checkpoint", None)

    @property
    def total_num_gpus(self) -> int:
        return sum(g.num_gpus for g in self.server_groups)

    @property
    def has_pd_disaggregation(self) -> bool:
        return any(g.worker_type in ("prefill", "decode") for g in self.server_groups)


@dataclass
class EngineInstance:
    model: str
    group: int
    worker_type: str
    ranks: list[int]
    update_weights: bool
    overrides: dict


@dataclass
class DeploymentConfig:
    models: list[ModelDeployment]

    @staticmethod
    def from_dict(data: dict) -> "DeploymentConfig":
        if "sglang" not in data:
            raise ValueError("deployment config needs a top-level 'sglang' list")
        models = []
        for m in data["sglang"]:
            groups = [ServerGroup(**g) for g in (m.get("server_groups") or m.get("engine_groups") or [])]
            models.append(ModelDeployment(name=m["name"], model_path=m.get("model_path"),
                                          num_gpus_per_engine=m.get("num_gpus_per_engine"),
                                          server_groups=groups,
                                          update_weights=m.get("update_weights")))
        return DeploymentConfig(models)

    @staticmethod
    def from_yaml(path: str) -> "DeploymentConfig":
        import yaml

        with open(path) as f:
            return DeploymentConfig.from_dict(yaml.safe_load(f))

    @staticmethod
    def from_prefill_num_servers(args) -> "DeploymentConfig":
        """Equivalent of the legacy --prefill-num-servers flag."""
        pre = args.prefill_num_servers * args.rollout_num_gpus_per_engine
        dec = args.rollout_num_gpus - pre
        if dec <= 0:
            raise ValueError(f"no decode GPUs left: {args.rollout_num_gpus} total, {pre} prefill")
        return DeploymentConfig([ModelDeployment("default", server_groups=[
            ServerGroup("prefill", pre), ServerGroup("decode", dec)])])

    @property
    def total_num_gpus(self) -> int:
        return sum(m.total_num_gpus for m in self.models)

    @property
    def has_pd_disaggregation(self) -> bool:
        return any(m.has_pd_disaggregation for m in self.models)

    def plan(self, args, rollout_ranks: list[int]) -> tuple[list[EngineInstance], list[str]]:
        """Assign rollout ranks to engine instances. Returns (engines, notes)."""
        for m in self.models:
            m.resolve(args)
        if self.total_num_gpus > len(rollout_ranks):
            raise ValueError(f"deployment needs {self.total_num_gpus} GPUs, "
                             f"{len(rollout_ranks)} rollout GPUs available")
        engines, notes, k = [], [], 0
        for m in self.models:
            for gi, g in enumerate(m.server_groups):
                ranks = rollout_ranks[k:k + g.num_gpus]
                k += g.num_gpus
                if g.worker_type == "placeholder":
                    continue
                if g.num_gpus_per_engine != 1:
                    notes.append(f"{m.name}/group{gi}: {g.num_gpus_per_engine}-GPU engines run as "
                                 f"{g.num_gpus} single-GPU engines (no tensor-parallel engine)")
                if g.worker_type in ("prefill", "decode"):
                    notes.append(f"{m.name}/group{gi}: {g.worker_type} group runs regular engines "
                                 f"(prefill and decode on the same engine)")
                for r in ranks:
                    engines.append(EngineInstance(m.name, gi, g.worker_type, [r],
                                                  bool(m.update_weights), dict(g.overrides)))
        return engines, notes


def load_deployment(args, rollout_ranks: list[int]) -> tuple[list[EngineInstance], list[str]]:
    """The `--sglang-config` deployment over `rollout_ranks`, as the drivers run it: exactly one
    model (the trained actor, refitted), no placeholder groups, GPUs matching the rollout ranks."""
    dep = DeploymentConfig.from_yaml(args.sglang_config)
    if len(dep.models) != 1:
        raise ValueError("--sglang-config: one deployed model (the trained actor) is supported; "
                         f"got {[m.name for m in dep.models]}")
    if any(g.worker_type == "placeholder" for g in dep.models[0].server_groups):
        raise ValueError("--sglang-config: placeholder groups are not supported by the drivers")
    if dep.total_num_gpus != len(rollout_ranks):
        raise ValueError(f"--sglang-config uses {dep.total_num_gpus} GPUs, the job has "
                         f"{len(rollout_ranks)} rollout GPUs")
    engines, notes = dep.plan(args, rollout_ranks)
    if dep.models[0].update_weights is False:
        raise ValueError("--sglang-config: the deployed actor must take weight updates")
    return engines, notes


def overrides_for(engines: list[EngineInstance], rank: int) -> dict:
    """The SGLang-flag overrides of the engine that runs on `rank` ({} if none)."""
    for e in engines:
        if rank in e.ranks:
            return {k: v for k, v in e.overrides.items() if k != "model_path"}
    return {}


def pd_pairs(engines: list[EngineInstance]) -> tuple[list[int], list[int]] | None:
    """(prefill ranks, decode ranks), paired by position, or None without prefill / decode
    groups."""
    pre = [e.ranks[0] for e in engines if e.worker_type == "prefill"]
    dec = [e.ranks[0] for e in engines if e.worker_type == "decode"]
    if not pre and not dec:
        return None
    if len(pre) != len(dec):
        raise ValueError(f"--sglang-config: {len(pre)} prefill and {len(dec)} decode engines; "
                         "each decode engine needs its own prefill engine")
    return pre, dec
