"""Weights & Biases hooks (reference: koochak/logging/wandb_logger.py:93-260).

``wandb`` is an optional dependency: it is imported when the hooks are built.
Behaviour kept from the reference because dashboards depend on it:

* run id: when only ``name`` is given, the id is the SHA-1 of the name
  lower-cased with runs of characters outside ``[A-Za-z0-9-_]`` replaced by
  ``-``, so a restarted job resumes the same run (auto-resume additionally
  requires ``resume: allow``);
* keys: train keys go to ``train/<k>``, bookkeeping keys (``step``,
  ``*_time_s``, ``*_count``, ``*_fraction``, ``profile_*``, ``sample_*``, ...)
  to ``stats/<k>``, eval keys to ``val/<k>`` (``val_loss`` -> ``val/loss``,
  ``val_seqctx_<context>_<metric>`` -> ``val/seqctx/<context>/<metric>``);
  keys that already contain ``/`` are kept;
* a train log is committed later when an eval will log at the same step;
* ``best/<k>`` summaries track the minimum of every eval metric; checkpoint
  artifacts (``log_artifacts``) get ``latest``, ``step-N`` and ``best-<k>``
  aliases.
"""

from __future__ import annotations

import hashlib
import re
from typing import Any, Dict, List, Mapping

from .. import config as config_lib
from ..core.hooks import rank0_only
from ..storage.naming import make_checkpoint_aliases

__all__ = ["make_wandb_hooks", "run_id_from_name", "wandb_key"]

_STATS_EXACT = {"step", "step_time_s", "run_iters", "node_count", "node_slot_count"}
_STATS_PREFIX = ("profile_", "sample_", "sequence_context_")
_STATS_SUFFIX = ("_skip_count", "_time_s", "_count", "_fraction")
_SEQCTX = ("replacement_failed_native", "sink_only", "no_sequence", "mismatched", "replacement", "replaced",
           "mismatch", "native", "full")


def run_id_from_name(name: str) -> str:
    if not isinstance(name, str) or not name:
        raise RuntimeError("W&B stable-id-by-name requires cfg.name to be a non-empty string.")
    canonical = re.sub(r"[^A-Za-z0-9-_]+", "-", name.strip().lower())
    return hashlib.sha1(canonical.encode("utf-8")).hexdigest()


def _is_stats(key: str) -> bool:
    return key in _STATS_EXACT or key.startswith(_STATS_PREFIX) or key.endswith(_STATS_SUFFIX)


def wandb_key(key: str, phase: str) -> str:
    """Dashboard name of a log key for ``phase`` ("train" or "val")."""

    if "/" in key:
        return key
    if phase != "val":
        return ("stats/" if _is_stats(key) else "train/") + key
    if key == "val_loss":
        return "val/loss"
    if key.startswith("val_seqctx_"):
        rest = key[len("val_seqctx_"):]
        for ctx in _SEQCTX:
            if rest.startswith(ctx + "_"):
                return f"val/seqctx/{ctx}/{rest[len(ctx) + 1:]}"
        head, _, tail = rest.partition("_")
        return f"val/seqctx/{head}/{tail}" if tail else f"val/seqctx/{head}"
    if key.startswith("val_"):
        metric = key[4:]
        return ("stats/val/" if _is_stats(metric) else "val/") + metric
    return ("stats/val/" if _is_stats(key) else "val/") + key


def _eval_due(ctx: Mapping[str, Any]) -> bool:
    cfg = ctx.get("train_cfg") or {}
    try:
        every = int(config_lib.get(cfg, "eval_every", 0) or 0)
    except (TypeError, ValueError):
        every = 0
    if every <= 0:
        return False
    step = int(ctx.get("step", 0)) + int(bool(config_lib.get(cfg, "intervals_use_completed_steps", False)))
    return step % every == 0 and (step != 0 or bool(config_lib.get(cfg, "eval_at_step_zero", True)))


def make_wandb_hooks(cfg) -> Dict[str, List]:
    import wandb  # type: ignore

    def opt(key: str, default: Any = None) -> Any:
        return config_lib.get(cfg, key, default)

    best_step: Dict[str, int] = {}

    def on_train_start(ctx):
        if opt("enabled", True) is False:
            return
        name, resume, run_id = opt("name"), opt("resume"), opt("id")
        if not run_id and name:
            run_id = run_id_from_name(name)
        if ctx.get("auto_resume_selected"):
            if resume != "allow":
                raise ValueError("W&B auto-resume requires wandb.resume='allow' on a restartable job")
            if not run_id:
                raise ValueError("W&B auto-resume requires a stable wandb.name or wandb.id")
        wandb.init(project=opt("project", "koochak"), entity=opt("entity"), name=name, group=opt("group"),
                   job_type=opt("job_type"), tags=opt("tags"), notes=opt("notes"), mode=opt("mode", "online"),
                   dir=opt("dir"), id=run_id, resume=resume, settings=wandb.Settings(),
                   config=ctx.get("config_json") or ctx.get("config"), allow_val_change=True)
        watch = opt("watch_model")
        if watch is None:
            comp = config_lib.get(ctx.get("train_cfg") or {}, "compile", None)
            compiled = bool(comp.get("enabled", True)) if isinstance(comp, Mapping) else bool(comp)
            watch = not compiled
        model = ctx.get("model")
        if not watch or model is None:
            return
        if opt("watch_unwrap_ddp", True):
            model = getattr(model, "module", model)
        kw = {"log": opt("watch_log", "all") or "all", "log_freq": int(opt("watch_log_freq", 100) or 100),
              "log_graph": bool(opt("watch_log_graph", False))}
        try:
            fn = getattr(wandb, "watch_model", None)
            if callable(fn):
                fn(model, criterion=None, **kw)
            else:
                wandb.watch(model, **kw)
        except (RuntimeError, TypeError, ValueError) as exc:
            msg = f"wandb.watch/watch_model failed; gradients/parameters won't be tracked. Error: {exc}"
            warn = getattr(wandb, "termwarn", None)
            warn(msg) if callable(warn) else print(f"[wandb] {msg}")

    def on_log(logs, ctx):
        wandb.log({wandb_key(str(k), "train"): v for k, v in logs.items()}, step=int(ctx.get("step", 0)),
                  commit=not _eval_due(ctx))

    def on_eval_end(metrics, ctx):
        wandb.log({wandb_key(str(k), "val"): v for k, v in metrics.items()}, step=ctx.get("step"), commit=True)
        run = wandb.run
        if run is None:
            return
        for k, v in metrics.items():
            try:
                prev, val = float(run.summary.get(f"best/{k}", float("inf"))), float(v)
            except (TypeError, ValueError):
                continue
            run.summary[f"best/{k}"] = min(prev, val)
            if val <= prev and int(ctx.get("step", -1)) >= 0:
                best_step[k] = int(ctx["step"])

    def on_checkpoint(path, ckpt, ctx):
        run = wandb.run
        if not opt("log_artifacts", False) or run is None:
            return
        prefix = opt("artifact_name_prefix") or opt("artifact_name") or "model"
        rid = getattr(run, "id", None) or getattr(run, "name", None) or "unknown"
        art = wandb.Artifact(name=f"{prefix}-{rid}", type=opt("artifact_type", "model"),
                             metadata={"step": ctx.get("step")})
        art.add_file(path)
        step = int(ctx.get("step", -1))
        best = [k for k, s in best_step.items() if s == step]
        wandb.log_artifact(art, aliases=make_checkpoint_aliases(step if step >= 0 else None, include_latest=True,
                                                                 best_keys=best or None))

    def on_train_end(ctx):
        fin = getattr(wandb, "finish", None)
        if callable(fin):
            try:
                fin()
            except RuntimeError:
                pass

    return {
        "on_train_start": [rank0_only(on_train_start)],
        "on_log": [rank0_only(on_log)],
        "on_eval_end": [rank0_only(on_eval_end)],
        "on_checkpoint": [rank0_only(on_checkpoint)],
        "on_train_end": [rank0_only(on_train_end)],
    }
