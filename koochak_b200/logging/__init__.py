"""Rank-0 metric sinks and coordinator events, wired in as hook dicts.

(reference: koochak/logging/{stdout,csv,jsonl,wandb_logger,events}.py)
"""

from .csv import CSVLogger, make_csv_hooks
from .jsonl import JSONLLogger, make_jsonl_hooks
from .stdout import StdoutLogger, log_step_tsv, make_stdout_hooks

__all__ = [
    "CSVLogger", "JSONLLogger", "StdoutLogger", "log_step_tsv", "make_csv_hooks", "make_jsonl_hooks",
    "make_stdout_hooks", "make_wandb_hooks", "make_event_hooks", "make_scruffy_hooks",
]


def __getattr__(name):  # optional integrations import lazily
    if name == "make_wandb_hooks":
        from .wandb_logger import make_wandb_hooks

        return make_wandb_hooks
    if name in ("make_event_hooks", "make_scruffy_hooks"):
        from . import events

        return getattr(events, name)
    raise AttributeError(name)
