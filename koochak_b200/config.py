"""Structured configuration: schema, YAML layering, strict unknown-key checks.

Same schema and behaviour as the reference's OmegaConf-based config
(reference: koochak/config.py:34-309), implemented without OmegaConf:

* the schema is a tree of dataclasses (``RootConfig``); ``STRUCTURED_DEFAULTS``
  is its default tree and ``SCHEMA`` the plain-dict form;
* ``load_config(path, overrides)`` = defaults <- YAML <- overrides, keys not in
  the schema are rejected while merging (``ConfigKeyError``), then ``${a.b}``
  and ``${oc.env:VAR,default}`` interpolations are resolved;
* the result is a ``ConfigNode``: a ``dict`` with attribute access, so both
  ``cfg.train.max_steps`` and ``cfg["train"]["max_steps"]`` work and every
  helper that accepts a ``Mapping`` accepts it. OmegaConf ``DictConfig``
  objects are accepted wherever a config is read, when OmegaConf is installed.

Sections added for this runtime: ``kernels`` (native or torch oracle path),
``comm`` (gradient-sync transport and bucket size) and ``bench``.
"""

from __future__ import annotations

import copy
import os
import re
from dataclasses import asdict, dataclass, field, fields, is_dataclass
from typing import Any, Dict, Mapping, Optional, Set

from .core import dist as dist_lib

__all__ = [
    "TrainEMADualConfig", "TrainEMAConfig", "TrainOomRecoveryConfig", "TrainConfig", "DataConfig",
    "OptimizerConfig", "SchedulerConfig", "OptimConfig", "LoggingConfig", "WandbConfig", "EntryConfig",
    "KernelsConfig", "CommConfig", "BenchConfig", "RootConfig", "STRUCTURED_DEFAULTS", "SCHEMA", "ConfigNode",
    "ConfigKeyError", "load_config", "get_section", "validate_unknown_keys", "summarize", "as_dict", "get",
    "to_container", "merge",
]


@dataclass
class TrainEMADualConfig:
    enabled: bool = False
    gamma1: Optional[float] = None
    gamma2: Optional[float] = None
    srel1: Optional[float] = None
    srel2: Optional[float] = None


@dataclass
class TrainEMAConfig:
    enabled: Optional[bool] = None
    decay: Optional[float] = None
    decay_init: Optional[float] = None
    warmup_steps: int = 0
    schedule: str = "constant"
    profile: Optional[str] = None
    gamma: Optional[float] = None
    srel: Optional[float] = None
    offload_to_cpu: bool = True
    pin_memory: bool = True
    update_every: int = 1
    compensate_update_every: bool = True
    eval_with_ema: bool = False
    dual: TrainEMADualConfig = field(default_factory=TrainEMADualConfig)


@dataclass
class TrainOomRecoveryConfig:
    enabled: bool = False
    max_consecutive: int = 3
    max_skipped_steps: Optional[int] = None


@dataclass
class TrainConfig:
    max_steps: int = 100_000
    log_every: int = 100
    eval_every: int = 5_000
    eval_at_step_zero: bool = True
    ckpt_every: int = 5_000
    grad_accum: int = 1
    grad_clip_norm: Optional[float] = None
    nonfinite_grad_check_every: int = 0
    scheduler_step: str = "step"
    amp: str = "fp32"
    ddp: bool = False
    find_unused_parameters: bool = False
    ddp_static_graph: bool = False
    ddp_gradient_as_bucket_view: bool = False
    ddp_bucket_cap_mb: Optional[int] = None
    ddp_bucket_cap_mb_list: Optional[list] = None
    ddp_broadcast_buffers: bool = True
    seed: int = 42
    compile: Optional[Any] = None
    prefetch_batches: int = 0
    prefetch_pipeline: str = "single"
    device: Optional[str] = None
    out_dir: str = "./runs/exp0"
    keep_last_k: int = 3
    checkpoint_dir: Optional[str] = None
    checkpoint_async: bool = False
    shard_dataset: bool = False
    shard_dataset_mode: Optional[str] = None
    shard_eval_dataset: bool = False
    shard_eval_dataset_mode: Optional[str] = None
    warn_unsharded: bool = True
    strict_config: bool = True
    config_warn_unknown: bool = True
    prefetch_threaded: bool = False
    autocast_in_step_fn: bool = False
    scalarize_loss_every_step: bool = True
    resume: str = "none"
    evacuation_enabled: bool = False
    evacuation_signal: str = "USR1"
    oom_recovery: TrainOomRecoveryConfig = field(default_factory=TrainOomRecoveryConfig)
    ema: TrainEMAConfig = field(default_factory=TrainEMAConfig)
    ema_enabled: Optional[bool] = None
    ema_decay: Optional[float] = None
    ema_decay_init: Optional[float] = None
    ema_warmup_steps: Optional[int] = None
    ema_schedule: Optional[str] = None
    ema_profile: Optional[str] = None
    ema_gamma: Optional[float] = None
    ema_srel: Optional[float] = None
    ema_offload_to_cpu: Optional[bool] = None
    ema_pin_memory: Optional[bool] = None
    ema_update_every: Optional[int] = None
    ema_compensate_update_every: Optional[bool] = None
    ema_eval: Optional[bool] = None
    # Loop-only keys (read by the loop; accepted here so strict checks pass).
    intervals_use_completed_steps: bool = False
    rank_timing_every: int = 0
    rank_timing_keys: Optional[list] = None
    profile_step_fn_timing: bool = False
    profile_step_fn_cuda_sync: bool = True
    profile_nvtx: bool = False
    device_timing: bool = False
    comm_transport: str = "auto"


@dataclass
class DataConfig:
    data_dir: str = "./data"
    batch_size: int = 128
    num_workers: int = 4


@dataclass
class OptimizerConfig:
    name: str = "adamw"
    lr: float = 3e-4
    weight_decay: float = 0.0
    betas: tuple = (0.9, 0.999)
    eps: float = 1e-8
    momentum: float = 0.9
    nesterov: bool = False
    muon_lr: Optional[float] = None
    adam_lr: Optional[float] = None
    foreach_adam_update: Optional[bool] = None
    hyperball_eps: float = 1.0e-8
    hyperball_radius_scale: float = 1.0
    hyperball_projection: str = "sphere"
    fused: Optional[bool] = None


@dataclass
class SchedulerConfig:
    name: str = "none"
    T_max: Optional[int] = None
    t_max: Optional[int] = None
    eta_min: float = 0.0
    warmup_steps: int = 0
    step_size: int = 1_000
    gamma: float = 0.1
    mode: str = "min"
    factor: float = 0.1
    patience: int = 10


@dataclass
class OptimConfig:
    optimizer: OptimizerConfig = field(default_factory=OptimizerConfig)
    scheduler: SchedulerConfig = field(default_factory=SchedulerConfig)


@dataclass
class LoggingConfig:
    csv_path: Optional[str] = None
    jsonl_path: Optional[str] = None


@dataclass
class WandbConfig:
    enabled: bool = False
    project: Optional[str] = None
    entity: Optional[str] = None
    name: Optional[str] = None
    group: Optional[str] = None
    job_type: Optional[str] = None
    tags: Optional[list] = None
    notes: Optional[str] = None
    mode: Optional[str] = None
    dir: Optional[str] = None
    resume: Optional[str] = None
    id: Optional[str] = None
    log_artifacts: Optional[bool] = None
    artifact_name_prefix: Optional[str] = None
    artifact_name: Optional[str] = None
    artifact_type: Optional[str] = None
    watch_model: Optional[bool] = None
    watch_unwrap_ddp: Optional[bool] = None
    watch_log: Optional[str] = None
    watch_log_freq: Optional[int] = None
    watch_log_graph: Optional[bool] = None


@dataclass
class EntryConfig:
    model: Optional[str] = None
    dataset: Optional[str] = None
    step: Optional[str] = None
    eval_dataset: Optional[str] = None
    eval_fn: Optional[str] = None


@dataclass
class KernelsConfig:
    backend: str = "native"      # native | torch (oracle path)


@dataclass
class CommConfig:
    transport: str = "auto"      # auto | p2p | nccl
    bucket_mb: float = 64.0
    timeout_ms: int = 5000


@dataclass
class BenchConfig:
    model: Optional[str] = None
    steps: int = 20
    warmup: int = 5


@dataclass
class RootConfig:
    train: TrainConfig = field(default_factory=TrainConfig)
    data: DataConfig = field(default_factory=DataConfig)
    optim: OptimConfig = field(default_factory=OptimConfig)
    logging: LoggingConfig = field(default_factory=LoggingConfig)
    wandb: WandbConfig = field(default_factory=WandbConfig)
    entry: EntryConfig = field(default_factory=EntryConfig)
    kernels: KernelsConfig = field(default_factory=KernelsConfig)
    comm: CommConfig = field(default_factory=CommConfig)
    bench: BenchConfig = field(default_factory=BenchConfig)


class ConfigKeyError(KeyError):
    """A key that the schema does not define."""


class ConfigNode(dict):
    """``dict`` with attribute access; nested mappings become ConfigNodes."""

    def __init__(self, data: Optional[Mapping[str, Any]] = None) -> None:
        super().__init__()
        for k, v in (data or {}).items():
            self[k] = _wrap(v)

    def __getattr__(self, name: str) -> Any:
        try:
            return self[name]
        except KeyError:
            raise AttributeError(name) from None

    def __setattr__(self, name: str, value: Any) -> None:
        self[name] = _wrap(value)

    def __delattr__(self, name: str) -> None:
        del self[name]

    def __deepcopy__(self, memo):
        return ConfigNode(copy.deepcopy(dict(self), memo))


def _wrap(v: Any) -> Any:
    if isinstance(v, ConfigNode):
        return v
    if isinstance(v, Mapping):
        return ConfigNode(v)
    if isinstance(v, tuple):
        return list(v)
    return v


def _dataclass_tree(obj: Any) -> Dict[str, Any]:
    return {f.name: (_dataclass_tree(getattr(obj, f.name)) if is_dataclass(getattr(obj, f.name))
                     else copy.deepcopy(getattr(obj, f.name))) for f in fields(obj)}


STRUCTURED_DEFAULTS = ConfigNode(_dataclass_tree(RootConfig()))


def to_container(cfg: Any) -> Any:
    """Deep plain-Python copy (dicts and lists) of a config tree."""

    try:  # accept OmegaConf objects when OmegaConf is installed
        from omegaconf import DictConfig, ListConfig, OmegaConf  # type: ignore

        if isinstance(cfg, (DictConfig, ListConfig)):
            return OmegaConf.to_container(cfg, resolve=True)
    except ImportError:
        pass
    if is_dataclass(cfg) and not isinstance(cfg, type):
        return _dataclass_tree(cfg)
    if isinstance(cfg, Mapping):
        return {k: to_container(v) for k, v in cfg.items()}
    if isinstance(cfg, (list, tuple)):
        return [to_container(v) for v in cfg]
    return cfg


SCHEMA: Dict[str, Any] = to_container(STRUCTURED_DEFAULTS)


def get(cfg: Mapping[str, Any] | Any, key: str, default: Any = None) -> Any:
    if isinstance(cfg, Mapping):
        return cfg.get(key, default)
    return getattr(cfg, key, default)


def as_dict(cfg: Mapping[str, Any] | Any) -> Dict[str, Any]:
    if is_dataclass(cfg) and not isinstance(cfg, type):
        return asdict(cfg)
    try:
        from omegaconf import DictConfig, OmegaConf  # type: ignore

        if isinstance(cfg, DictConfig):
            return OmegaConf.to_container(cfg, resolve=True)  # type: ignore[return-value]
    except ImportError:
        pass
    if isinstance(cfg, Mapping):
        return dict(cfg)
    return {k: getattr(cfg, k) for k in dir(cfg) if not k.startswith("_")}


def _merge_into(dst: Dict[str, Any], src: Mapping[str, Any], schema: Optional[Mapping[str, Any]], path: str) -> None:
    for k, v in src.items():
        p = f"{path}.{k}" if path else str(k)
        if schema is not None and k not in schema:
            raise ConfigKeyError(f"Key '{p}' is not in the config schema")
        sub_schema = schema.get(k) if isinstance(schema, Mapping) else None
        if isinstance(v, Mapping) and isinstance(dst.get(k), Mapping):
            _merge_into(dst[k], v, sub_schema if isinstance(sub_schema, Mapping) else None, p)
        else:
            dst[k] = copy.deepcopy(to_container(v))


def merge(base: Mapping[str, Any], *others: Mapping[str, Any], strict: bool = False) -> ConfigNode:
    """Deep merge; with ``strict`` every key must already exist in ``base``."""

    out = to_container(base)
    for o in others:
        if o is None:
            continue
        _merge_into(out, to_container(o), out if strict else None, "")
    return ConfigNode(out)


_INTERP = re.compile(r"\$\{([^}]+)\}")


def _lookup(root: Mapping[str, Any], dotted: str) -> Any:
    node: Any = root
    for part in dotted.split("."):
        if isinstance(node, Mapping) and part in node:
            node = node[part]
        else:
            raise KeyError(f"interpolation key '{dotted}' not found")
    return node


def _resolve_value(v: Any, root: Mapping[str, Any], depth: int = 0) -> Any:
    if depth > 32:
        raise ValueError("config interpolation is too deep (cycle?)")
    if isinstance(v, str):
        def expr(e: str) -> Any:
            e = e.strip()
            if e.startswith("oc.env:"):
                name, _, default = e[len("oc.env:"):].partition(",")
                val = os.environ.get(name.strip())
                if val is None:
                    if not _:
                        raise KeyError(f"environment variable {name!r} is not set")
                    val = default.strip().strip("'\"")
                return val
            return _resolve_value(_lookup(root, e), root, depth + 1)

        whole = _INTERP.fullmatch(v)
        if whole:
            return expr(whole.group(1))
        return _INTERP.sub(lambda m: str(expr(m.group(1))), v)
    if isinstance(v, Mapping):
        return {k: _resolve_value(x, root, depth) for k, x in v.items()}
    if isinstance(v, list):
        return [_resolve_value(x, root, depth) for x in v]
    return v


def resolve(cfg: Mapping[str, Any]) -> ConfigNode:
    plain = to_container(cfg)
    return ConfigNode(_resolve_value(plain, plain))


def _dotlist(overrides: Any) -> Dict[str, Any]:
    if overrides is None:
        return {}
    if isinstance(overrides, Mapping):
        return to_container(overrides)
    import yaml

    out: Dict[str, Any] = {}
    for item in overrides:
        key, _, raw = str(item).partition("=")
        node = out
        parts = key.strip().split(".")
        for p in parts[:-1]:
            node = node.setdefault(p, {})
        node[parts[-1]] = yaml.safe_load(raw) if raw else None
    return out


def load_config(path: str, overrides: Optional[Mapping[str, Any]] = None) -> ConfigNode:
    """Defaults <- YAML file <- overrides (mapping or ``["a.b=1", ...]``), resolved."""

    import yaml

    with open(path, encoding="utf-8") as fh:
        data = yaml.safe_load(fh) or {}
    if not isinstance(data, Mapping):
        raise ValueError(f"{path}: top level of a config must be a mapping")
    cfg = merge(STRUCTURED_DEFAULTS, data, strict=True)
    if overrides:
        cfg = merge(cfg, _dotlist(overrides), strict=True)
    return resolve(cfg)


def get_section(cfg: Mapping[str, Any] | Any, name: str, *, required: bool = True) -> Any:
    section = get(cfg, name, None)
    if section is None and required:
        raise KeyError(f"Missing required config section: {name}")
    return section


def _unknown(cfg: Mapping[str, Any], schema: Mapping[str, Any], prefix: str = "") -> Set[str]:
    out: Set[str] = set()
    for k, v in (cfg or {}).items():
        p = f"{prefix}.{k}" if prefix else str(k)
        if k not in schema:
            out.add(p)
        elif isinstance(v, Mapping) and isinstance(schema.get(k), Mapping):
            out |= _unknown(v, schema[k], p)
    return out


def validate_unknown_keys(cfg: Mapping[str, Any] | Any, schema: Optional[Dict[str, Any]] = None) -> Set[str]:
    """Dotted paths of keys in ``cfg`` that the schema does not define."""

    return _unknown(to_container(as_dict(cfg)), schema or SCHEMA)


def summarize(cfg: Mapping[str, Any] | Any, *, schema: Optional[Dict[str, Any]] = None, strict: bool = True,
              warn_unknown: bool = True) -> Set[str]:
    """Print sections and unknown keys (rank 0); raise ValueError when strict and any are unknown."""

    schema = schema or SCHEMA
    payload = to_container(as_dict(cfg))
    unknown = _unknown(payload, schema)
    sections = ", ".join(sorted(payload.keys())) or "<none>"
    if strict and unknown:
        if dist_lib.rank0():
            print("[koochak][config] sections:", sections)
        raise ValueError("[koochak][config] unknown keys: " + ", ".join(sorted(unknown)))
    if (warn_unknown or not unknown) and dist_lib.rank0():
        print("[koochak][config] sections:", sections)
        print("[koochak][config] unknown keys: " + (", ".join(sorted(unknown)) if unknown else "<none>"))
        print(f"[koochak][config] strict: {'on' if strict else 'off'}")
    return unknown
