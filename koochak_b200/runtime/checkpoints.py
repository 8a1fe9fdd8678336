"""Checkpoints of a training run: what goes in, who writes, and how a run resumes from one.

(the checkpoint dict of reference koochak/loop.py:901-990 and the resume
rules of koochak/loop.py:726-897 -- the dict keys are the format shared with
the reference)

Collection is a step every rank takes (``collect``): the RNG states of all
ranks (gathered when the checkpoint must restore every rank exactly), and
the optimizer state gathered from its owners when the optimizer shards it
(``gathered_state_dict``: every Muon momentum and complete Adam moments, so
the dict a single process would write). Rank 0 then serializes and publishes
it (``publish``), synchronously or on the background publisher.

Resume (``restore``) loads model (``module.`` prefix matched either way),
optimizer, scheduler and scaler state, rebuilds the EMA / dual EMA from
their saved settings, restores this rank's RNG, and returns the next update
to run: ``next_step`` when present, else the cursor older checkpoints imply.
"""

from __future__ import annotations

import os
import time
import warnings
from typing import Any, Callable, Dict, List, Mapping, Optional, Sequence, Tuple

import torch
from torch.amp import GradScaler

from ..core import dist as dist_lib
from ..storage import checkpoint as checkpoint_lib
from ..utils.ema import EMA
from ..utils.seed import get_rng_state, set_rng_state
from .settings import EmaSettings

__all__ = ["CheckpointKeeper", "restore_ema", "resume_cursor"]


def _warn_restore(what: str, exc: BaseException) -> None:
    warnings.warn(f"Failed to restore {what} from checkpoint: {exc}", RuntimeWarning)


def resume_cursor(ckpt: Mapping[str, Any]) -> int:
    """First update to run after ``ckpt``: ``next_step``, else inferred from ``step`` and the saved max_steps."""

    try:
        if "next_step" in ckpt:
            return int(ckpt["next_step"])
        saved = int(ckpt.get("step", 0))
        cfg = ckpt.get("config", {})
        max_steps = int(cfg.get("train", cfg).get("max_steps", -1))
        # Older terminal checkpoints stored the completed count, periodic ones the last index.
        return saved if saved == max_steps else saved + 1
    except (AttributeError, TypeError, ValueError):
        return 0


def _one_ema(module: torch.nn.Module, state: Mapping[str, Any], settings: EmaSettings, profile: str,
             gamma: Any) -> EMA:
    decay = float(state.get("decay", settings.target_decay or 0.999))
    kind = str(state.get("profile", profile)).lower()
    gamma = state.get("gamma", gamma)
    ema = EMA(module, decay=decay, profile=kind, gamma=gamma, update_every=settings.update_every,
              offload_to_cpu=settings.offload_to_cpu, pin_memory=settings.pin_memory,
              compensate_update_every=settings.compensate_update_every)
    shadow = state.get("shadow", {})
    try:
        shadow = checkpoint_lib.match_state_dict_to_model(module, shadow)
    except (TypeError, AttributeError):
        pass
    ema.load_state_dict({
        "decay": decay, "profile": kind, "gamma": gamma, "shadow": shadow,
        "num_updates": state.get("num_updates", 0),
        "step_counter": state.get("step_counter", state.get("num_updates", 0)),
        "update_every": state.get("update_every", settings.update_every),
        "compensate_update_every": state.get("compensate_update_every", settings.compensate_update_every),
    })
    return ema


def restore_ema(module: torch.nn.Module, settings: EmaSettings, ema_state: Any,
                dual_state: Any) -> Tuple[Optional[EMA], List[EMA]]:
    """The EMA and dual EMAs of a resumed run (fresh ones when the checkpoint has none but the config asks)."""

    ema: Optional[EMA] = None
    if ema_state is not None:
        try:
            ema = _one_ema(module, ema_state, settings, settings.profile, settings.gamma)
        except (TypeError, ValueError, RuntimeError) as exc:
            _warn_restore("EMA", exc)
    elif settings.enabled:
        ema = EmaBuilder(settings).single(module)
    duals: List[EMA] = []
    if isinstance(dual_state, Sequence) and not isinstance(dual_state, (str, bytes)):
        for i, st in enumerate(dual_state):
            if not isinstance(st, Mapping):
                continue
            try:
                duals.append(_one_ema(module, st, settings, "power",
                                      settings.dual.gamma1 if i == 0 else settings.dual.gamma2))
            except (TypeError, ValueError, RuntimeError) as exc:
                _warn_restore(f"dual EMA #{i}", exc)
    elif settings.dual.enabled:
        duals = EmaBuilder(settings).pair(module)
    return ema, duals


class EmaBuilder:
    def __init__(self, settings: EmaSettings) -> None:
        self.s = settings

    def _make(self, module: torch.nn.Module, profile: str, gamma: Any, srel: Any) -> EMA:
        s = self.s
        return EMA(module, decay=float(s.target_decay or 0.999), profile=profile, gamma=gamma, srel=srel,
                   update_every=s.update_every, offload_to_cpu=s.offload_to_cpu, pin_memory=s.pin_memory,
                   compensate_update_every=s.compensate_update_every)

    def single(self, module: torch.nn.Module) -> EMA:
        return self._make(module, self.s.profile, self.s.gamma, self.s.srel)

    def pair(self, module: torch.nn.Module) -> List[EMA]:
        d = self.s.dual
        if not d.enabled:
            return []
        return [self._make(module, "power", d.gamma1, d.srel1), self._make(module, "power", d.gamma2, d.srel2)]


class CheckpointKeeper:
    """Builds, publishes and announces checkpoints for one run."""

    def __init__(self, *, location: str, keep_last_k: int, background: bool, is_rank0: bool, world_size: int,
                 emit: Callable[..., None], has_all_rank_hooks: bool) -> None:
        self.store = checkpoint_lib.checkpoint_store(location)
        self.keep_last_k = keep_last_k
        self.is_rank0 = is_rank0
        self.world_size = world_size
        self.emit = emit
        self.all_rank_hooks = has_all_rank_hooks
        self.publisher = (checkpoint_lib.BackgroundPublisher(self.store, keep_last_k=keep_last_k)
                          if background and is_rank0 else None)

    def path_of(self, step: int) -> str:
        return checkpoint_lib.checkpoint_path(self.store, f"step{step:09d}.pt")

    # ------------------------------------------------------------------ build (every rank)
    def _rng(self, gather: bool) -> Any:
        try:
            mine = get_rng_state()
            if gather and dist_lib.is_initialized() and self.world_size > 1:
                everyone: list = [None] * self.world_size
                torch.distributed.all_gather_object(everyone, mine)
                return {"per_rank": everyone}
            return mine
        except RuntimeError:
            if gather:
                raise
            return None

    @staticmethod
    def _optimizer_state(optimizer: Any) -> Dict[str, Any]:
        gathered = getattr(optimizer, "gathered_state_dict", None)
        return gathered() if callable(gathered) else optimizer.state_dict()

    def collect(self, *, step: int, next_step: int, module: torch.nn.Module, optimizer: Any, scheduler: Any,
                scaler: Any, config: Any, ema: Optional[EMA], dual: List[EMA], oom_skipped: Sequence[int],
                metrics: Optional[Mapping[str, Any]] = None, gather_rng: bool = False) -> Dict[str, Any]:
        """The checkpoint dict (a collective when the optimizer state or RNG must be gathered)."""

        ckpt: Dict[str, Any] = {
            "step": step, "next_step": next_step, "model": module.state_dict(),
            "optimizer": self._optimizer_state(optimizer),
            "scheduler": None if scheduler is None else scheduler.state_dict(),
            "scaler": scaler.state_dict() if isinstance(scaler, GradScaler) else None,
            "config": config, "rng": self._rng(gather_rng), "wall_time": time.time(), "metrics": dict(metrics or {}),
        }
        if ema is not None:
            ckpt["ema"] = ema.state_dict()
        if dual:
            ckpt["ema_dual"] = [e.state_dict() for e in dual]
        skipped = sorted(s for s in oom_skipped if s < next_step)
        if skipped:
            ckpt["oom_skipped_steps"] = skipped
        return ckpt

    # ------------------------------------------------------------------ publish (rank 0)
    def publish(self, step: int, ckpt: Dict[str, Any], *, announce: Optional[Callable[[str], None]] = None,
                background: bool = False) -> str:
        """Serialize and publish ``ckpt`` as ``step<N>.pt``; ``announce(path)`` once it is committed."""

        os.makedirs(os.path.dirname(self.path_of(step)), exist_ok=True)
        payload = checkpoint_lib.serialize(ckpt)
        self.drain()
        name = f"step{step:09d}.pt"
        if background and self.publisher is not None:
            return self.publisher.submit(name, payload, announce)
        path = checkpoint_lib.publish(self.store, name, payload, keep_last_k=self.keep_last_k)
        if announce is not None:
            announce(path)
        return path

    def _announce_finished(self, finished: Optional[Tuple[str, Any]]) -> None:
        if finished is not None and finished[1] is not None:
            path, announce = finished
            announce(path)

    def poll(self) -> None:
        if self.publisher is not None:
            self._announce_finished(self.publisher.poll())

    def drain(self) -> None:
        if self.publisher is not None:
            self._announce_finished(self.publisher.wait())

    def close(self) -> None:
        if self.publisher is not None:
            self.publisher.close()

    def all_rank_hooks_run(self, path: str, ckpt: Dict[str, Any], ctx: Mapping[str, Any]) -> None:
        """``on_checkpoint_all_ranks`` between barriers (every rank sees a published checkpoint)."""

        if self.all_rank_hooks:
            dist_lib.barrier()
            self.emit("on_checkpoint_all_ranks", path, ckpt, ctx, suppress_exceptions=False)
            dist_lib.barrier()


def restore_training_state(ckpt: Mapping[str, Any], *, model: torch.nn.Module, optimizer: Any, scheduler: Any,
                           scaler: Any, rank: int) -> int:
    """Load model / optimizer / scheduler / scaler / RNG from ``ckpt``; returns the first update to run."""

    state = ckpt.get("model")
    if state is not None:
        model.load_state_dict(checkpoint_lib.match_state_dict_to_model(model, state), strict=True)
    for key, target in (("optimizer", optimizer), ("scheduler", scheduler)):
        saved = ckpt.get(key)
        if target is None or saved is None:
            continue
        try:
            target.load_state_dict(saved)
        except (ValueError, RuntimeError, KeyError) as exc:
            _warn_restore(f"{key} state", exc)
    saved_scaler = ckpt.get("scaler")
    if saved_scaler is not None and isinstance(scaler, GradScaler):
        try:
            scaler.load_state_dict(saved_scaler)
        except (ValueError, RuntimeError, KeyError) as exc:
            _warn_restore("grad-scaler state", exc)
    rng = ckpt.get("rng")
    if isinstance(rng, Mapping) and isinstance(rng.get("per_rank"), Sequence):
        per_rank = rng["per_rank"]
        rng = per_rank[rank] if rank < len(per_rank) else rng
    if isinstance(rng, Mapping) and "per_rank" not in rng:
        try:
            set_rng_state(dict(rng))
        except (RuntimeError, TypeError, ValueError, KeyError) as exc:
            _warn_restore("RNG state", exc)
    return resume_cursor(ckpt)
