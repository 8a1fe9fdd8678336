"""Generic YAML-driven training entry point.

(reference: koochak/cli/train.py:38-118)

    python -m koochak_b200.cli.train --config run.yaml [--resume auto|none]

The config's ``entry`` section names no-argument callables as
``module:attr`` or ``module.attr``: ``model`` (returns the module),
``dataset`` (returns the training iterable), ``step`` (the ``step_fn``), and
optionally ``eval_dataset`` and ``eval_fn``. The optimizer and scheduler come
from the ``optim`` section, logging from ``logging`` (CSV and JSONL default to
``<out_dir>/log.csv`` and ``log.jsonl``) and ``wandb``. Inside a Scruffy
worker (``SCRUFFY_ROOT`` and ``SCRUFFY_JOB_ID`` set) the coordinator event
hooks are attached as well.

The optimizer is built from the model module rather than its parameter
iterator, so the Muon family (which needs the module to form its parameter
groups) works from the CLI too.
"""

from __future__ import annotations

import argparse
import importlib
import os
from typing import List, Optional

from .. import config as config_lib
from ..core import hooks as hooks_lib

__all__ = ["main", "import_object"]


def import_object(path: str):
    """Resolve ``module:attr`` or ``module.attr``."""

    if ":" in path:
        mod, name = path.split(":", 1)
    elif "." in path:
        mod, name = path.rsplit(".", 1)
    else:
        raise ValueError(f"Invalid import path: {path}")
    return getattr(importlib.import_module(mod), name)


def _build_hooks(cfg_train, cfg_logging, cfg_wandb):
    from ..logging import make_csv_hooks, make_jsonl_hooks, make_stdout_hooks

    out_dir = str(config_lib.get(cfg_train, "out_dir", "./runs/exp0"))
    hooks = make_stdout_hooks()
    csv_path = config_lib.get(cfg_logging, "csv_path", None) or os.path.join(out_dir, "log.csv")
    jsonl_path = config_lib.get(cfg_logging, "jsonl_path", None) or os.path.join(out_dir, "log.jsonl")
    hooks = hooks_lib.merge(hooks, make_csv_hooks(csv_path))
    hooks = hooks_lib.merge(hooks, make_jsonl_hooks(jsonl_path))
    if cfg_wandb is not None and bool(config_lib.get(cfg_wandb, "enabled", False)):
        from ..logging.wandb_logger import make_wandb_hooks

        hooks = hooks_lib.merge(hooks, make_wandb_hooks(cfg_wandb))
    if os.environ.get("SCRUFFY_ROOT") and os.environ.get("SCRUFFY_JOB_ID"):
        from ..logging.events import make_scruffy_hooks

        hooks = hooks_lib.merge(hooks, make_scruffy_hooks())
    return hooks


def main(argv: Optional[List[str]] = None):
    ap = argparse.ArgumentParser(description="koochak_b200 generic training CLI")
    ap.add_argument("--config", required=True, help="Path to YAML config")
    ap.add_argument("--resume", choices=("auto", "none"), default="auto",
                    help="Resume from the highest valid numbered checkpoint (default: auto)")
    args = ap.parse_args(argv)

    from ..loop import training_loop
    from ..optim.build import build_optimizer, build_scheduler
    from ..utils.seed import set_all_seeds

    cfg = config_lib.load_config(args.config)
    cfg_train = config_lib.get_section(cfg, "train")
    cfg_optim = config_lib.get_section(cfg, "optim")
    cfg_logging = config_lib.get_section(cfg, "logging", required=False)
    cfg_wandb = config_lib.get_section(cfg, "wandb", required=False)
    cfg_entry = config_lib.get_section(cfg, "entry")
    config_lib.summarize(cfg, strict=bool(config_lib.get(cfg_train, "strict_config", True)),
                         warn_unknown=bool(config_lib.get(cfg_train, "config_warn_unknown", True)))
    set_all_seeds(int(config_lib.get(cfg_train, "seed", 42)))

    entry = lambda key: config_lib.get(cfg_entry, key, None)  # noqa: E731
    if not entry("model"):
        raise ValueError("entry.model must be provided as 'module:callable' or 'module.Class'")
    if not entry("dataset") or not entry("step"):
        raise ValueError("entry.dataset and entry.step must be provided")
    model = import_object(entry("model"))()
    optimizer = build_optimizer(model, config_lib.get(cfg_optim, "optimizer", None))
    scheduler = build_scheduler(optimizer, config_lib.get(cfg_optim, "scheduler", None), cfg_train)
    dataset = import_object(entry("dataset"))()
    step_fn = import_object(entry("step"))
    eval_dataset = import_object(entry("eval_dataset"))() if entry("eval_dataset") else None
    eval_fn = import_object(entry("eval_fn")) if entry("eval_fn") else None
    return training_loop(model=model, dataset=dataset, step_fn=step_fn, optimizer=optimizer, scheduler=scheduler,
                         train_cfg=cfg_train, config_json=config_lib.as_dict(cfg), resume=args.resume,
                         eval_dataset=eval_dataset, eval_fn=eval_fn,
                         hooks=_build_hooks(cfg_train, cfg_logging, cfg_wandb))


if __name__ == "__main__":
    main()
